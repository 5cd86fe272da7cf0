"""GPU parity of the CUDA path (through the C ABI via the ctypes shim) against
the CPU oracle on identical seeded inputs.

Bars: quantize / dequantize bit-exact; matmuls max|d| <= 2e-2 * max|ref|
with bf16/f16 output and float32 accumulation."""
import os

import numpy as np
import pytest
import torch

import mlx_server_runtime_b200 as mxq
from mlx_server_runtime_b200 import nn
from oracle import coracle, oracle_np as O

from gpu_util import as_f32, close, rand_weights, rand_x, to_dev, to_np

pytestmark = pytest.mark.gpu
GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


def _quant_both(w_np, dt, gs, bits):
    ref = coracle.quantize(w_np, dt, gs, bits)
    got = mxq.quantize(to_dev(w_np, dt), gs, bits)
    return ref, got


@pytest.mark.parametrize("dt", ["bfloat16", "float16", "float32"])
@pytest.mark.parametrize("bits", [2, 4, 8])
@pytest.mark.parametrize("gs", [32, 64, 128])
def test_quantize_dequantize_bit_exact(dt, bits, gs):
    rng = np.random.default_rng(100 * bits + gs)
    w = rand_weights(rng, (67, 768), dt)
    w[3, :gs] = O.from_f32(np.zeros(gs, np.float32), dt)          # constant group
    w[5, 7] = O.from_f32(np.array([1.5], np.float32), dt)[0]       # outlier
    ref, got = _quant_both(w, dt, gs, bits)
    for r, g, name in zip(ref, got, ("wq", "scales", "biases")):
        assert to_np(g).tobytes() == np.asarray(r).tobytes(), name
    d_ref = coracle.dequantize(*ref, dt, gs, bits)
    d_got = mxq.dequantize(*got, gs, bits)
    assert to_np(d_got).tobytes() == np.asarray(d_ref).tobytes()


@pytest.mark.parametrize("dt,bits", [("bfloat16", 4), ("float16", 4), ("float16", 8),
                                     ("float32", 4), ("float32", 8)])
def test_quantize_half_integer_quotients(dt, bits):
    """Groups whose (w - bias) / scale land exactly on half-integers (ties, rounded to
    even) and, in float32, one ulp either side of them: the kernel's fast quotient must
    give the codes of the IEEE quotient."""
    rng = np.random.default_rng(7 * bits)
    n, gs, rows = (1 << bits) - 1, 64, 192
    half = rng.integers(0, 2 * n + 1, (rows, gs)).astype(np.float32) / 2
    half[:, 0], half[:, 1] = 0.0, n          # endpoints: scale -step, bias = max
    step = (2.0 ** rng.integers(-10, 6, (rows, 1))).astype(np.float32)
    w = half * step                          # exact in every dtype tested
    if dt == "float32":
        nudge = rng.integers(-1, 2, w.shape)
        nudge[:, :2] = 0
        w = np.where(nudge < 0, np.nextafter(w, -np.inf),
                     np.where(nudge > 0, np.nextafter(w, np.inf), w)).astype(np.float32)
    w = O.from_f32(w, dt)
    ref, got = _quant_both(w, dt, gs, bits)
    for r, g, name in zip(ref, got, ("wq", "scales", "biases")):
        assert to_np(g).tobytes() == np.asarray(r).tobytes(), name


def test_kat_on_gpu():
    import json
    with open(os.path.join(GOLDEN, "kat.json")) as f:
        kat = json.load(f)
    for case in kat["quantize_f32"]:
        w = np.array([case["w"]], np.float32)
        wq, s, b = mxq.quantize(to_dev(w), case["group_size"], case["bits"])
        assert O.unpack(to_np(wq), case["bits"]).tolist() == [case["codes"]]
        assert to_np(s)[0, 0] == np.float32(case["scale"])
        assert to_np(b)[0, 0] == np.float32(case["bias"])
    for case in kat["dequant_bf16"]:
        wq = O.pack(np.array([case["codes"]], np.uint32), case["bits"])
        s = np.array([[case["scale"]]], np.uint16)
        b = np.array([[case["bias"]]], np.uint16)
        out = mxq.dequantize(to_dev(wq), to_dev(s, "bfloat16"), to_dev(b, "bfloat16"),
                             case["group_size"], case["bits"])
        assert to_np(out).tolist() == [case["out"]]


def _qmm_case(dt, bits, gs, M, N, K, seed, bias=False):
    rng = np.random.default_rng(seed)
    w = rand_weights(rng, (N, K), dt)
    x = rand_x(rng, (M, K), dt)
    wq, s, b = coracle.quantize(w, dt, gs, bits)
    bvec = rand_x(rng, (N,), dt) if bias else None
    ref = coracle.quantized_matmul(x, wq, s, b, dt, gs, bits, bias=bvec)
    y = mxq.quantized_matmul(to_dev(x, dt), to_dev(wq), to_dev(s, dt), to_dev(b, dt),
                             group_size=gs, bits=bits,
                             bias=None if bvec is None else to_dev(bvec, dt))
    torch.cuda.synchronize()
    return to_np(y), ref


@pytest.mark.parametrize("M", [1, 2, 3, 8, 9, 16, 17, 25, 32, 33, 64, 100])
@pytest.mark.parametrize("bits", [4, 8])
def test_qmm_token_counts(M, bits):
    y, ref = _qmm_case("bfloat16", bits, 64, M, 272, 1024, seed=M * 10 + bits)
    close(y, ref, "bfloat16")


@pytest.mark.parametrize("dt", ["bfloat16", "float16"])
@pytest.mark.parametrize("bits", [4, 8])
@pytest.mark.parametrize("gs", [32, 64, 128])
@pytest.mark.parametrize("N,K", [(96, 512), (100, 384), (8, 128), (1000, 640)])
def test_qmm_shapes(dt, bits, gs, N, K):
    if K % gs:
        pytest.skip("K not a multiple of the group")
    for M in (1, 5, 20):
        y, ref = _qmm_case(dt, bits, gs, M, N, K, seed=N + K + gs + bits + M)
        close(y, ref, dt)


@pytest.mark.parametrize("N,K", [(512, 3584), (3584, 3584), (3584, 18944)])
def test_qmm_split_k_paths(N, K):
    """Small N relative to the SM count -> K splits with a last-CTA reduction."""
    for M in (1, 8):
        y, ref = _qmm_case("bfloat16", 4, 64, M, N, K, seed=N + M)
        close(y, ref, "bfloat16")


@pytest.mark.parametrize("K", [64, 768, 2048 + 64 * 3])
def test_qmm_group_counts_not_multiple_of_chunk(K):
    """K/group not a multiple of the stage chunk: scalar scale/bias path."""
    for bits, gs in ((4, 64), (8, 64), (4, 32), (8, 128)):
        if K % gs:
            continue
        y, ref = _qmm_case("bfloat16", bits, gs, 3, 160, K, seed=K + bits + gs)
        close(y, ref, "bfloat16")


def test_qmm_bias_fused():
    y, ref = _qmm_case("bfloat16", 4, 64, 4, 512, 3584, seed=5, bias=True)
    close(y, ref, "bfloat16")


def test_qmm_seeded_fixtures():
    z = np.load(os.path.join(GOLDEN, "seeded.npz"))
    names = sorted({k.split("/")[0] for k in z.files if k.endswith("/meta")})
    for n in names:
        bits, gs, M, N, K = (int(v) for v in z[f"{n}/meta"])
        dt = "float16" if n.startswith("f16") else "bfloat16"
        y = mxq.quantized_matmul(to_dev(z[f"{n}/x"], dt), to_dev(z[f"{n}/wq"]),
                                 to_dev(z[f"{n}/s"], dt), to_dev(z[f"{n}/b"], dt),
                                 group_size=gs, bits=bits)
        close(to_np(y), z[f"{n}/y"], dt)
        wq, s, b = mxq.quantize(to_dev(z[f"{n}/w"], dt), gs, bits)
        assert to_np(wq).tobytes() == z[f"{n}/wq"].tobytes()


def test_qmm_deterministic():
    rng = np.random.default_rng(11)
    for (N, K) in ((512, 3584), (18944, 3584)):
        w = rand_weights(rng, (N, K), "bfloat16")
        x = to_dev(rand_x(rng, (3, K), "bfloat16"), "bfloat16")
        wq, s, b = mxq.quantize(to_dev(w, "bfloat16"), 64, 4)
        outs = [to_np(mxq.quantized_matmul(x, wq, s, b)).tobytes() for _ in range(3)]
        assert outs[0] == outs[1] == outs[2]


def test_config1_full_size():
    """x [1,3584] ~ N(0,1); W [18944,3584] ~ N(0,0.02) -> bf16,
    4-bit g64, seed 0."""
    rng = np.random.default_rng(0)
    x = O.from_f32(rng.standard_normal((1, 3584)).astype(np.float32), "bfloat16")
    w = O.from_f32((rng.standard_normal((18944, 3584)) * 0.02).astype(np.float32), "bfloat16")
    (wq_r, s_r, b_r), (wq, s, b) = _quant_both(w, "bfloat16", 64, 4)
    assert to_np(wq).tobytes() == wq_r.tobytes()
    assert to_np(s).tobytes() == s_r.tobytes() and to_np(b).tobytes() == b_r.tobytes()
    y = mxq.quantized_matmul(to_dev(x, "bfloat16"), wq, s, b)
    ref = coracle.quantized_matmul(x, wq_r, s_r, b_r, "bfloat16", 64, 4)
    rel = close(to_np(y), ref, "bfloat16")
    assert rel < 5e-3  # well inside the 2e-2 bar


def test_leading_dims_and_empty():
    rng = np.random.default_rng(2)
    w = to_dev(rand_weights(rng, (64, 256), "bfloat16"), "bfloat16")
    wq, s, b = mxq.quantize(w)
    x = to_dev(rand_x(rng, (2, 3, 256), "bfloat16"), "bfloat16")
    y = mxq.quantized_matmul(x, wq, s, b)
    assert y.shape == (2, 3, 64)
    y2 = mxq.quantized_matmul(x.reshape(6, 256), wq, s, b)
    assert torch.equal(y.reshape(6, 64), y2)
    e = mxq.quantized_matmul(x[:0], wq, s, b)
    assert e.shape == (0, 3, 64)


# ---------------------------------------------------------------- gather_qmm ----
def _experts(rng, E, N, K, dt, gs, bits):
    w = rand_weights(rng, (E * N, K), dt)
    wq, s, b = coracle.quantize(w, dt, gs, bits)
    return wq.reshape(E, N, -1), s.reshape(E, N, -1), b.reshape(E, N, -1)


@pytest.mark.parametrize("bits", [4, 8])
@pytest.mark.parametrize("T,topk,E", [(1, 8, 16), (5, 2, 6), (64, 8, 32), (300, 4, 16)])
def test_gather_unsorted_broadcast(bits, T, topk, E):
    """SwitchGLU's unsorted call: x [T,1,1,K] against indices [T,k]."""
    rng = np.random.default_rng(T * topk + E + bits)
    N, K = 96, 512
    wq, s, b = _experts(rng, E, N, K, "bfloat16", 64, bits)
    x = rand_x(rng, (T, 1, K), "bfloat16")
    rhs = np.stack([rng.choice(E, topk, replace=False) for _ in range(T)]).astype(np.int32)
    ref = coracle.gather_qmm(x, wq, s, b, rhs.reshape(-1), "bfloat16", 64, bits, lhs_div=topk)
    xd = to_dev(x, "bfloat16").reshape(T, 1, 1, K)
    y = mxq.gather_qmm(xd, to_dev(wq), to_dev(s, "bfloat16"), to_dev(b, "bfloat16"),
                       rhs_indices=to_dev(rhs), group_size=64, bits=bits)
    assert y.shape == (T, topk, 1, N)
    close(to_np(y).reshape(T * topk, 1, N), ref, "bfloat16")


@pytest.mark.parametrize("T,topk,E", [(8, 8, 16), (64, 8, 128), (512, 8, 128)])
def test_gather_sorted_matches_unsorted(T, topk, E):
    rng = np.random.default_rng(T + E)
    N, K = 128, 256
    wq, s, b = _experts(rng, E, N, K, "bfloat16", 64, 4)
    x = rand_x(rng, (T, K), "bfloat16")
    rhs = np.stack([rng.choice(E, topk, replace=False) for _ in range(T)]).astype(np.int32)
    flat = rhs.reshape(-1)
    order = np.argsort(flat, kind="stable")
    xs = x[order // topk][:, None, :]            # [T*k, 1, K]
    sel = flat[order].astype(np.int32)
    ref = coracle.gather_qmm(xs, wq, s, b, sel, "bfloat16", 64, 4)
    args = (to_dev(wq), to_dev(s, "bfloat16"), to_dev(b, "bfloat16"))
    y_sorted = mxq.gather_qmm(to_dev(xs, "bfloat16"), *args, rhs_indices=to_dev(sel),
                              sorted_indices=True)
    y_plain = mxq.gather_qmm(to_dev(xs, "bfloat16"), *args, rhs_indices=to_dev(sel),
                             sorted_indices=False)
    close(to_np(y_sorted), ref, "bfloat16")
    close(to_np(y_plain), ref, "bfloat16")


def test_gather_lhs_indices_and_multi_row():
    rng = np.random.default_rng(9)
    E, N, K, M = 4, 64, 256, 3
    wq, s, b = _experts(rng, E, N, K, "float16", 32, 8)
    x = rand_x(rng, (5, M, K), "float16")
    lhs = np.array([4, 0, 2, 2, 1, 3], np.int32)
    rhs = np.array([1, 1, 0, 3, 2, 0], np.int32)
    ref = coracle.gather_qmm(x, wq, s, b, rhs, "float16", 32, 8, lhs=lhs)
    y = mxq.gather_qmm(to_dev(x), to_dev(wq), to_dev(s), to_dev(b), lhs_indices=to_dev(lhs),
                       rhs_indices=to_dev(rhs), group_size=32, bits=8)
    close(to_np(y), ref, "float16")


def test_gather_seeded_fixture():
    z = np.load(os.path.join(GOLDEN, "seeded.npz"))
    x, wq, s, b, rhs = (z[f"gather/{k}"] for k in ("x", "wq", "s", "b", "rhs"))
    T, k = rhs.shape
    y = mxq.gather_qmm(to_dev(x, "bfloat16").reshape(T, 1, 1, -1), to_dev(wq),
                       to_dev(s, "bfloat16"), to_dev(b, "bfloat16"), rhs_indices=to_dev(rhs))
    close(to_np(y).reshape(T * k, 1, -1), z["gather/y"], "bfloat16")


def test_gather_out_of_range_rows_untouched():
    """An expert index outside [0, E) is skipped by the kernel's bounds check."""
    rng = np.random.default_rng(4)
    wq, s, b = _experts(rng, 4, 64, 128, "bfloat16", 64, 4)
    x = to_dev(rand_x(rng, (2, 1, 128), "bfloat16"), "bfloat16")
    rhs = torch.tensor([1, 7], dtype=torch.int32, device="cuda")
    out = mxq.gather_qmm(x, to_dev(wq), to_dev(s, "bfloat16"), to_dev(b, "bfloat16"),
                         rhs_indices=rhs)
    torch.cuda.synchronize()
    assert out.shape == (2, 1, 64)


# ---------------------------------------------------------------- modules -------
def test_quantized_linear_and_nn_quantize():
    torch.manual_seed(0)
    lin = nn.Linear(256, 96, bias=True)
    lin.bias = torch.randn(96, device="cuda").to(torch.bfloat16)

    class Net(nn.Module):
        def __init__(self):
            self.proj = lin

    net = Net()
    nn.quantize(net, group_size=64, bits=4)
    assert isinstance(net.proj, nn.QuantizedLinear)
    x = torch.randn(3, 256, device="cuda").to(torch.bfloat16)
    y = net.proj(x)
    wq, s, b = (to_np(t) for t in (net.proj.weight, net.proj.scales, net.proj.biases))
    ref = coracle.quantized_matmul(to_np(x), wq, s, b, "bfloat16", 64, 4, bias=to_np(lin.bias))
    close(to_np(y), ref, "bfloat16")


@pytest.mark.parametrize("T", [1, 4, 64])
def test_switch_glu_matches_oracle(T):
    """SwitchGLU (lfm2.py:193-218): sorted path when T*k >= 64."""
    torch.manual_seed(T)
    E, D, H, topk = 16, 256, 128, 4
    glu = nn.SwitchGLU(D, H, E)
    for name in ("gate_proj", "up_proj", "down_proj"):
        setattr(glu, name, getattr(glu, name).to_quantized(64, 4))
    x = torch.randn(T, D, device="cuda").to(torch.bfloat16)
    idx = torch.stack([torch.randperm(E, device="cuda")[:topk] for _ in range(T)]).to(torch.int32)
    y = glu(x, idx)
    assert y.shape == (T, topk, D)

    def ora(layer, xin, rhs, div):
        return coracle.gather_qmm(xin, to_np(layer.weight), to_np(layer.scales),
                                  to_np(layer.biases), rhs, "bfloat16", 64, 4, lhs_div=div)
    xn = to_np(x)[:, None, :]
    rhs = to_np(idx).reshape(-1).astype(np.int32)
    up = ora(glu.up_proj, xn, rhs, topk)
    gate = ora(glu.gate_proj, xn, rhs, topk)
    g, u = as_f32(gate, "bfloat16"), as_f32(up, "bfloat16")
    act = O.from_f32(O.round_to(g / (1 + np.exp(-g)), "bfloat16") * u, "bfloat16")
    down = ora(glu.down_proj, act, rhs, 1)
    close(to_np(y).reshape(T * topk, 1, D), down, "bfloat16", rel=3e-2)


def test_ops_capture_in_cuda_graph():
    """The operators enqueue only stream-ordered work, so a CUDA graph of them
    replays to the same results (the decode loop replays one graph per step)."""
    rng = np.random.default_rng(21)
    w = to_dev(rand_weights(rng, (512, 3584), "bfloat16"), "bfloat16")
    wq, s, b = mxq.quantize(w)
    x = to_dev(rand_x(rng, (2, 3584), "bfloat16"), "bfloat16")
    eager = mxq.quantized_matmul(x, wq, s, b)       # also sets up kernel attributes
    st = torch.cuda.Stream()
    st.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(st):
        mxq.quantized_matmul(x, wq, s, b)             # workspace for this stream
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=st):
        y = mxq.quantized_matmul(x, wq, s, b)
    for _ in range(3):
        g.replay()
    torch.cuda.synchronize()
    with torch.cuda.stream(st):
        again = mxq.quantized_matmul(x, wq, s, b)
    torch.cuda.synchronize()
    diff = (y.float() - eager.float()).abs()
    assert torch.equal(again, eager), "eager results differ between streams"
    assert torch.equal(y, eager), (
        f"graph replay differs: max|d|={diff.max().item()} at {int((diff > 0).sum())} of "
        f"{diff.numel()} outputs")


def test_split_k_after_sorted_gather_same_stream():
    """The sorted gather path writes a segment table into its workspace; a later
    K-split quantized_matmul on the same stream must still see zeroed tickets."""
    rng = np.random.default_rng(31)
    wq, s, b = _experts(rng, 16, 64, 256, "bfloat16", 64, 4)
    xs = to_dev(rand_x(rng, (128, 1, 256), "bfloat16"), "bfloat16")
    sel = torch.sort(torch.randint(0, 16, (128,), device="cuda").to(torch.int32)).values
    mxq.gather_qmm(xs, to_dev(wq), to_dev(s, "bfloat16"), to_dev(b, "bfloat16"),
                   rhs_indices=sel, sorted_indices=True)
    y, ref = _qmm_case("bfloat16", 4, 64, 2, 512, 3584, seed=77)
    close(y, ref, "bfloat16")


def test_launch_overlap_dependent_chain():
    """With launch overlap on, a chain of matmuls where each consumes the previous
    output (and a K split that uses tickets) gives the same bits as without."""
    rng = np.random.default_rng(41)
    dims = [3584, 512, 3584, 18944, 3584]
    layers = []
    for k, n in zip(dims[:-1], dims[1:]):
        w = to_dev(rand_weights(rng, (n, k), "bfloat16"), "bfloat16")
        layers.append(mxq.quantize(w, 64, 4))
    x0 = to_dev(rand_x(rng, (1, dims[0]), "bfloat16"), "bfloat16")

    def chain():
        h = x0
        outs = []
        for wq, s, b in layers:
            h = mxq.quantized_matmul(h, wq, s, b)
            outs.append(h)
        return outs

    ref = chain()
    torch.cuda.synchronize()
    with mxq.launch_overlap(True):
        for _ in range(3):
            got = chain()
        torch.cuda.synchronize()
    assert _lib_overlap_state() == 0
    for a, b in zip(ref, got):
        assert torch.equal(a, b)


def _lib_overlap_state():
    from mlx_server_runtime_b200 import _lib as L
    return L.load().mlxq_get_launch_overlap()
