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


@pytest.mark.parametrize("n,E", [(1, 1), (8, 128), (512, 128), (4096, 128), (16384, 1024),
                                 (333, 7)])
def test_moe_sort_matches_stable_argsort(n, E):
    """core.moe_sort against numpy's stable argsort (order, sorted indices, inverse)."""
    from mlx_server_runtime_b200 import core
    rng = np.random.default_rng(n + E)
    idx = rng.integers(0, E, n).astype(np.int32)
    order, srt, inv = (t.cpu().numpy() for t in core.moe_sort(torch.from_numpy(idx).cuda(), E))
    ref = np.argsort(idx, kind="stable")
    assert np.array_equal(order, ref)
    assert np.array_equal(srt, idx[ref])
    assert np.array_equal(inv, np.argsort(ref, kind="stable"))


def test_moe_sort_out_of_range_groups():
    from mlx_server_runtime_b200 import core
    idx = np.array([3, -2, 9, 0, -1, 3, 12, 1], np.int32)     # E = 4
    order, srt, inv = (t.cpu().numpy() for t in core.moe_sort(torch.from_numpy(idx).cuda(), 4))
    # negatives first (entry order), then experts 0..3 (stable), then values >= 4
    assert order.tolist() == [1, 4, 3, 7, 0, 5, 2, 6]
    assert srt.tolist() == idx[order].tolist()
    assert np.array_equal(inv[order], np.arange(8))


def test_switch_glu_sorted_path_uses_device_sort():
    """SwitchGLU at 64 entries sorts on the device; the result equals the unsorted
    form (each entry through its expert) for the same routing."""
    E, D, H = 16, 256, 128
    g = torch.Generator(device="cuda").manual_seed(3)
    sw = nn.SwitchGLU(D, H, E, generator=g)
    nn.quantize(sw, 64, 4)
    x = (torch.randn(8, D, device="cuda", generator=g)).to(torch.bfloat16)
    idx = torch.stack([torch.randperm(E, device="cuda", generator=g)[:8] for _ in range(8)]).int()
    y_sorted = sw(x, idx)                                   # 64 entries: sorted path
    y_rows = torch.cat([sw(x[t:t + 1], idx[t:t + 1]) for t in range(8)])  # 8 entries each
    assert torch.equal(y_sorted, y_rows)
