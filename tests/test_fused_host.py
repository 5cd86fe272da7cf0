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


def _bank(E, N, K, seed):
    w, s, b = _q(E * N, K, seed=seed)
    return w.reshape(E, N, -1), s.reshape(E, N, -1), b.reshape(E, N, -1)


def test_interleave_expert_banks_per_expert():
    """3-D banks interleave within each expert: expert e of the result is the 2-D
    interleave of expert e's gate and up."""
    E, I, K = 3, 24, 256
    gate, up = _bank(E, I, K, 11), _bank(E, I, K, 12)
    w, s, b = mxq.interleave_gate_up(gate, up, 64, 4)
    assert w.shape == (E, 2 * I, K // 8) and s.shape == (E, 2 * I, K // 64)
    for e in range(E):
        w2, s2, b2 = mxq.interleave_gate_up(tuple(t[e] for t in gate), tuple(t[e] for t in up),
                                            64, 4)
        assert torch.equal(w[e].view(torch.int32), w2.view(torch.int32))
        assert torch.equal(s[e].view(torch.int16), s2.view(torch.int16))
        assert torch.equal(b[e].view(torch.int16), b2.view(torch.int16))
    # tile j of expert 1: gate rows 8j..8j+7, then up rows 8j..8j+7
    assert torch.equal(w[1, 16:24].view(torch.int32), gate[0][1, 8:16].view(torch.int32))
    assert torch.equal(w[1, 24:32].view(torch.int32), up[0][1, 8:16].view(torch.int32))


def _switch(E, N, K, seed, bias=False):
    q = mnn.QuantizedSwitchLinear.__new__(mnn.QuantizedSwitchLinear)
    q.group_size, q.bits, q.mode = 64, 4, "affine"
    q.weight, q.scales, q.biases = _bank(E, N, K, seed)
    if bias:
        q.bias = torch.zeros(E, N, dtype=torch.bfloat16)
    return q


def test_fuse_switch_gate_up_replaces_the_pair():
    sw = mnn.SwitchGLU.__new__(mnn.SwitchGLU)
    sw.gate_proj, sw.up_proj = _switch(4, 16, 128, 1), _switch(4, 16, 128, 2)
    sw.down_proj = _switch(4, 128, 16 * 4, 3)
    sw.fuse_gate_up()
    f = sw.gate_up_proj
    assert not hasattr(sw, "gate_proj") and not hasattr(sw, "up_proj")
    assert f.weight.shape == (4, 32, 16) and f.num_experts == 4
    with pytest.raises(ValueError):   # a bank with bias cannot fuse
        mnn.FusedSwitchGateUp.from_pair(_switch(4, 16, 128, 4, bias=True), _switch(4, 16, 128, 5))
    with pytest.raises(ValueError):
        mxq.interleave_gate_up(_bank(4, 12, 128, 6), _bank(4, 12, 128, 7), 64, 4)  # 12 % 8
