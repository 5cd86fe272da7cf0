"""The MoE router kernel (core.moe_route / nn.route_topk) against a numpy
restatement of lfm2.py:366-375: softmax of the logits in float64, plus the optional
expert bias, top-k, optional renormalisation. The chosen experts must be the same
set (the reference's argpartition leaves their order open; the kernel returns them
in descending gate order), scores within bf16/f32 rounding of the reference."""
import numpy as np
import pytest
import torch

from mlx_server_runtime_b200 import nn

pytestmark = pytest.mark.gpu


def _ref(logits, k, norm, bias):
    x = logits.astype(np.float64)
    e = np.exp(x - x.max(-1, keepdims=True))
    p = e / e.sum(-1, keepdims=True)
    if bias is not None:
        p = p + bias
    top = np.argsort(-p, axis=-1, kind="stable")[:, :k]
    sc = np.take_along_axis(p, top, -1)
    if norm:
        sc = sc / (sc.sum(-1, keepdims=True) + 1e-20)
    return top, sc, p


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
@pytest.mark.parametrize("T,E,k", [(1, 128, 8), (64, 128, 8), (4096, 128, 8), (7, 32, 4),
                                   (3, 1000, 32), (5, 8, 8)])
@pytest.mark.parametrize("norm", [True, False])
def test_router_matches_reference(dtype, T, E, k, norm):
    g = torch.Generator(device="cuda").manual_seed(T + E + k)
    logits = (torch.randn(T, E, device="cuda", generator=g) * 2).to(dtype)
    bias = (torch.randn(E, device="cuda", generator=g) * 0.01) if E == 128 else None
    idx, sc = nn.route_topk(logits, k, norm, bias)
    assert idx.dtype == torch.int32 and sc.dtype == dtype and idx.shape == (T, k)
    lf = logits.float().cpu().numpy()
    top, ref, p = _ref(lf, k, norm, None if bias is None else bias.cpu().numpy())
    got_i, got_s = idx.cpu().numpy(), sc.float().cpu().numpy()
    tol = 1e-5 if dtype == torch.float32 else 8e-3
    for t in range(T):
        kth = np.sort(p[t])[-k]
        # same experts, except where the k-th and (k+1)-th gates tie to rounding
        if set(got_i[t]) != set(top[t]):
            near = np.abs(p[t] - kth) <= 1e-6
            assert set(got_i[t]) ^ set(top[t]) <= set(np.nonzero(near)[0])
        ref_t = p[t, got_i[t]]
        if norm:
            ref_t = ref_t / (ref_t.sum() + 1e-20)
        np.testing.assert_allclose(got_s[t], ref_t, rtol=tol, atol=1e-6)
        assert np.all(np.diff(p[t, got_i[t]]) <= 1e-6)   # descending gates
