"""Host-side checks of the fused-projection helpers (CPU tensors, no kernels)."""
import pytest
import torch

import mlx_server_runtime_b200 as mxq
from mlx_server_runtime_b200 import nn as mnn


def _q(N, K, gs=64, bits=4, dtype=torch.bfloat16, seed=0):
    g = torch.Generator().manual_seed(seed)
    w = torch.randint(0, 2**31 - 1, (N, K * bits // 32), generator=g, dtype=torch.int64)
    w = w.to(torch.int32).view(torch.uint32)
    s = torch.randn(N, K // gs, generator=g).to(dtype)
    b = torch.randn(N, K // gs, generator=g).to(dtype)
    return w, s, b


def test_concat_keeps_rows_bit_for_bit():
    parts = [_q(8, 256, seed=1), _q(3, 256, seed=2), _q(5, 256, seed=3)]
    w, s, b = mxq.concat_quantized(parts, 64, 4)
    assert w.shape == (16, 32) and s.shape == (16, 4) and b.shape == (16, 4)
    off = 0
    for pw, ps, pb in parts:
        n = pw.shape[0]
        assert torch.equal(w[off:off + n].view(torch.int32), pw.view(torch.int32))
        assert torch.equal(s[off:off + n].view(torch.int16), ps.view(torch.int16))
        assert torch.equal(b[off:off + n].view(torch.int16), pb.view(torch.int16))
        off += n


def test_concat_rejects_mismatched_parts():
    with pytest.raises(ValueError):
        mxq.concat_quantized([], 64, 4)
    with pytest.raises(ValueError):
        mxq.concat_quantized([_q(4, 256), _q(4, 512)], 64, 4)
    with pytest.raises(ValueError):
        mxq.concat_quantized([_q(4, 256), _q(4, 256, dtype=torch.float16)], 64, 4)
    w, s, b = _q(4, 256)
    with pytest.raises(ValueError):
        mxq.concat_quantized([(w, s, b[:, :2])], 64, 4)


def _layer(N, K, bias, seed):
    q = mnn.QuantizedLinear.__new__(mnn.QuantizedLinear)
    q.group_size, q.bits, q.mode = 64, 4, "affine"
    q.weight, q.scales, q.biases = _q(N, K, seed=seed)
    if bias:
        q.bias = torch.randn(N).to(torch.bfloat16)
    return q


def test_fused_module_layout():
    a, b, c = _layer(8, 256, True, 1), _layer(4, 256, False, 2), _layer(4, 256, True, 3)
    f = mnn.FusedQuantizedLinear([a, b, c])
    assert f.splits == [8, 4, 4] and f.output_dims == 16 and f.input_dims == 256
    assert torch.equal(f.bias[:8], a.bias) and torch.equal(f.bias[12:], c.bias)
    assert torch.count_nonzero(f.bias[8:12]) == 0  # a part without bias adds zeros
    with pytest.raises(ValueError):
        mnn.FusedQuantizedLinear([a, _layer(4, 512, False, 4)])
    g = _layer(4, 256, False, 5)
    g.bits = 8
    with pytest.raises(ValueError):
        mnn.FusedQuantizedLinear([a, g])


def test_interleave_gate_up_layout():
    g = _q(24, 256, seed=4)
    u = _q(24, 256, seed=5)
    w, s, b = mxq.interleave_gate_up(g, u, 64, 4)
    assert w.shape == (48, 32) and s.shape == (48, 4)
    for j in range(3):
        for src, dst in ((g, slice(16 * j, 16 * j + 8)), (u, slice(16 * j + 8, 16 * j + 16))):
            rows = slice(8 * j, 8 * j + 8)
            assert torch.equal(w[dst].view(torch.int32), src[0][rows].view(torch.int32))
            assert torch.equal(s[dst].view(torch.int16), src[1][rows].view(torch.int16))
            assert torch.equal(b[dst].view(torch.int16), src[2][rows].view(torch.int16))
    with pytest.raises(ValueError):
        mxq.interleave_gate_up(_q(20, 256), _q(20, 256), 64, 4)   # rows not a multiple of 8
    with pytest.raises(ValueError):
        mxq.interleave_gate_up(_q(24, 256), _q(16, 256), 64, 4)


def test_fused_gate_up_rejects_bias_and_mismatch():
    a, b = _layer(16, 256, False, 1), _layer(16, 256, True, 2)
    with pytest.raises(ValueError):
        mnn.FusedGateUp(a, b)
    c = _layer(16, 256, False, 3)
    c.bits = 8
    with pytest.raises(ValueError):
        mnn.FusedGateUp(a, c)
    f = mnn.FusedGateUp(a, _layer(16, 256, False, 4))
    assert f.weight.shape == (32, 32)
