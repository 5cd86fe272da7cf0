"""Fused projections (concat_quantized / nn.FusedQuantizedLinear): q/k/v and
gate/up stacked along N run as one launch; every part must match the oracle
and its own unfused call."""
import numpy as np
import pytest
import torch

import mlx_server_runtime_b200 as mxq
from mlx_server_runtime_b200 import nn as mnn
from oracle import coracle

from gpu_util import close, rand_weights, rand_x, to_dev, to_np

pytestmark = pytest.mark.gpu


def _parts(rng, dt, gs, bits, Ns, K, bias):
    parts = []
    for N in Ns:
        w = rand_weights(rng, (N, K), dt)
        wq, s, b = coracle.quantize(w, dt, gs, bits)
        bv = rand_x(rng, (N,), dt) if bias else None
        parts.append((wq, s, b, bv))
    return parts


@pytest.mark.parametrize("Ns,K", [((3584, 512, 512), 3584), ((18944, 18944), 3584),
                                  ((200, 17, 64), 1024)])
@pytest.mark.parametrize("M", [1, 5, 64])
def test_fused_parts_match_oracle_and_unfused(Ns, K, M):
    dt, gs, bits = "bfloat16", 64, 4
    rng = np.random.default_rng(sum(Ns) + K + M)
    parts = _parts(rng, dt, gs, bits, Ns, K, bias=True)
    x = rand_x(rng, (M, K), dt)
    xd = to_dev(x, dt)
    dev = [(to_dev(wq), to_dev(s, dt), to_dev(b, dt), to_dev(bv, dt)) for wq, s, b, bv in parts]
    wf, sf, bf = mxq.concat_quantized([d[:3] for d in dev], gs, bits)
    assert wf.shape[0] == sum(Ns)
    bias = torch.cat([d[3] for d in dev])
    y = mxq.quantized_matmul(xd, wf, sf, bf, group_size=gs, bits=bits, bias=bias)
    outs = torch.split(y, list(Ns), dim=-1)
    for (wq, s, b, bv), d, yo in zip(parts, dev, outs):
        ref = coracle.quantized_matmul(x, wq, s, b, dt, gs, bits, bias=bv)
        close(to_np(yo.contiguous()), ref, dt)
        sep = mxq.quantized_matmul(xd, *d[:3], group_size=gs, bits=bits, bias=d[3])
        close(to_np(yo.contiguous()), to_np(sep), dt)


def test_fused_module_qkv_with_and_without_bias():
    torch.manual_seed(0)
    K = 1024
    q = mnn.QuantizedLinear(K, 512, bias=True)
    k = mnn.QuantizedLinear(K, 128, bias=False)
    v = mnn.QuantizedLinear(K, 128, bias=True)
    q.bias.normal_()
    v.bias.normal_()
    fused = mnn.FusedQuantizedLinear([q, k, v])
    x = torch.randn(3, K, device="cuda").to(torch.bfloat16)
    yq, yk, yv = fused(x)
    for layer, y in ((q, yq), (k, yk), (v, yv)):
        ref = layer(x)
        assert y.shape == ref.shape
        close(to_np(y.contiguous()), to_np(ref), "bfloat16")


def _swiglu_ref(x, gate, up, dt, gs, bits):
    from oracle import oracle_np as O
    g = O.to_f32(coracle.quantized_matmul(x, *gate, dt, gs, bits), dt)
    u = O.to_f32(coracle.quantized_matmul(x, *up, dt, gs, bits), dt)
    return O.from_f32((g / (1.0 + np.exp(-g)) * u).astype(np.float32), dt)


# (intermediate I, K): k/v-like (16-row CTAs), gate-like, down-like K (split row blocks)
@pytest.mark.parametrize("I,K", [(256, 3584), (18944, 3584), (1792, 18944), (200, 1024)])
@pytest.mark.parametrize("M", [1, 3, 8, 11, 16, 40])
def test_swiglu_matches_oracle(I, K, M):
    dt, gs, bits = "bfloat16", 64, 4
    rng = np.random.default_rng(I + K + M)
    gate = coracle.quantize(rand_weights(rng, (I, K), dt), dt, gs, bits)
    up = coracle.quantize(rand_weights(rng, (I, K), dt), dt, gs, bits)
    x = rand_x(rng, (M, K), dt)
    ref = _swiglu_ref(x, gate, up, dt, gs, bits)
    dev = lambda t: (to_dev(t[0]), to_dev(t[1], dt), to_dev(t[2], dt))
    w, s, b = mxq.interleave_gate_up(dev(gate), dev(up), gs, bits)
    y = mxq.quantized_matmul_swiglu(to_dev(x, dt), w, s, b, gs, bits)
    torch.cuda.synchronize()
    assert y.shape == (M, I)
    close(to_np(y), ref, dt)


@pytest.mark.parametrize("dt", ["bfloat16", "float16"])
@pytest.mark.parametrize("bits,gs", [(4, 32), (4, 128), (8, 64)])
def test_swiglu_types(dt, bits, gs):
    rng = np.random.default_rng(bits + gs)
    I, K, M = 512, 8 * gs * 4, 2
    gate = coracle.quantize(rand_weights(rng, (I, K), dt), dt, gs, bits)
    up = coracle.quantize(rand_weights(rng, (I, K), dt), dt, gs, bits)
    x = rand_x(rng, (M, K), dt)
    ref = _swiglu_ref(x, gate, up, dt, gs, bits)
    dev = lambda t: (to_dev(t[0]), to_dev(t[1], dt), to_dev(t[2], dt))
    w, s, b = mxq.interleave_gate_up(dev(gate), dev(up), gs, bits)
    y = mxq.quantized_matmul_swiglu(to_dev(x, dt), w, s, b, gs, bits)
    torch.cuda.synchronize()
    close(to_np(y), ref, dt)


def test_fused_gate_up_module_repeat():
    torch.manual_seed(1)
    gate, up = mnn.QuantizedLinear(1024, 768, bias=False), mnn.QuantizedLinear(1024, 768, bias=False)
    f = mnn.FusedGateUp(gate, up)
    x = torch.randn(4, 1024, device="cuda").to(torch.bfloat16)
    ref = (torch.nn.functional.silu(gate(x).float()) * up(x).float()).to(torch.bfloat16)
    outs = [f(x) for _ in range(3)]
    assert torch.equal(outs[0], outs[1]) and torch.equal(outs[1], outs[2])
    close(to_np(outs[0]), to_np(ref), "bfloat16")


@pytest.mark.parametrize("bits,gs,dt", [(4, 64, "bfloat16"), (8, 32, "float16"),
                                        (4, 128, "bfloat16")])
@pytest.mark.parametrize("M", [33, 333])
def test_swiglu_prefill_epilogue(bits, gs, dt, M):
    """More than 32 rows: the tensor-core kernel's SwiGLU epilogue (gate lane and up
    lane of each 16-row tile paired in the epilogue warp); I = 520 leaves a partial
    last weight block."""
    rng = np.random.default_rng(M + bits + gs)
    I, K = 520, 2048
    gate = coracle.quantize(rand_weights(rng, (I, K), dt), dt, gs, bits)
    up = coracle.quantize(rand_weights(rng, (I, K), dt), dt, gs, bits)
    x = rand_x(rng, (M, K), dt)
    ref = _swiglu_ref(x, gate, up, dt, gs, bits)
    dev = lambda t: (to_dev(t[0]), to_dev(t[1], dt), to_dev(t[2], dt))
    w, s, b = mxq.interleave_gate_up(dev(gate), dev(up), gs, bits)
    y = mxq.quantized_matmul_swiglu(to_dev(x, dt), w, s, b, gs, bits)
    torch.cuda.synchronize()
    assert y.shape == (M, I)
    close(to_np(y), ref, dt)
