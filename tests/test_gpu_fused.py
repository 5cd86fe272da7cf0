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
