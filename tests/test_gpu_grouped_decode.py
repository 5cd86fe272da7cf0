"""gather_qmm at decode sizes on the TMA-fed grouped kernel (qmv_grouped.cuh): an
expert's sorted rows taken TM at a time (experts with more rows than one chunk, empty
experts), unsorted entries one at a time (several chunks per entry when an entry has
more rows than the token slots), weight rows past N in the last row block, K whose
group count is not a multiple of 8 (a zero-padded last stage; scales copied in 4- or
8-byte pieces), and shapes the kernel does not take (an odd group count) on the
cp.async kernel. Every case against the C oracle.

Tolerance: max|d| <= 2e-2 * max|ref| (bf16/f16 outputs, fp32 accumulation)."""
import numpy as np
import pytest
import torch

import mlx_server_runtime_b200 as mxq
from oracle import coracle, oracle_np as O

from gpu_util import close, rand_weights, rand_x, to_dev, to_np

pytestmark = pytest.mark.gpu


def _experts(rng, E, N, K, dt, gs, bits):
    w = rand_weights(rng, (E * N, K), dt)
    wq, s, b = coracle.quantize(w, dt, gs, bits)
    return wq.reshape(E, N, -1), s.reshape(E, N, -1), b.reshape(E, N, -1)


def _sorted_case(E, N, K, counts, dt="bfloat16", bits=4, gs=64, M=1, seed=0):
    rng = np.random.default_rng(seed)
    wq, s, b = _experts(rng, E, N, K, dt, gs, bits)
    sel = np.repeat(np.arange(E, dtype=np.int32), counts)
    x = rand_x(rng, (sel.size, M, K), dt)
    ref = coracle.gather_qmm(x, wq, s, b, sel, dt, gs, bits)
    y = mxq.gather_qmm(to_dev(x, dt), to_dev(wq), to_dev(s, dt), to_dev(b, dt),
                       rhs_indices=to_dev(sel), group_size=gs, bits=bits, sorted_indices=True)
    torch.cuda.synchronize()
    close(to_np(y), ref, dt)


@pytest.mark.parametrize("K", [768, 1024, 2048])
def test_sorted_chunks(K):
    # mean 6.5 rows per expert: 8-slot chunks; experts of 0, 1, 8, 9, 17 and 30 rows
    counts = [0, 1, 8, 9, 17, 30, 3, 0, 5, 6, 4, 7, 2, 5, 6, 1]
    _sorted_case(16, 200, K, counts, seed=K)


@pytest.mark.parametrize("dt", ["bfloat16", "float16"])
@pytest.mark.parametrize("bits,gs", [(4, 32), (4, 64), (4, 128), (8, 32), (8, 64)])
def test_sorted_types(dt, bits, gs):
    rng = np.random.default_rng(bits * gs)
    counts = rng.integers(0, 6, size=24)
    _sorted_case(24, 96, 768, counts, dt=dt, bits=bits, gs=gs, seed=bits + gs)


def test_sorted_few_rows_per_expert():
    # 64 entries over 128 experts (mean 0.5 rows): single-slot chunks
    rng = np.random.default_rng(5)
    counts = rng.multinomial(64, np.ones(128) / 128)
    _sorted_case(128, 768, 2048, counts, seed=6)


def test_sorted_two_rows_per_entry():
    _sorted_case(6, 130, 512, [3, 0, 5, 1, 2, 4], M=2, seed=7)


@pytest.mark.parametrize("M", [1, 3, 9])
def test_unsorted_entries(M):
    """Entries one at a time: lhs indices, repeated experts, M rows per entry (9 rows
    take two chunks of 8 slots)."""
    rng = np.random.default_rng(M)
    E, N, K = 12, 80, 640
    wq, s, b = _experts(rng, E, N, K, "bfloat16", 64, 4)
    x = rand_x(rng, (7, M, K), "bfloat16")
    lhs = rng.integers(0, 7, 10).astype(np.int32)
    rhs = rng.integers(0, E, 10).astype(np.int32)
    rhs[3] = rhs[4]
    ref = coracle.gather_qmm(x, wq, s, b, rhs, "bfloat16", 64, 4, lhs=lhs)
    y = mxq.gather_qmm(to_dev(x, "bfloat16"), to_dev(wq), to_dev(s, "bfloat16"),
                       to_dev(b, "bfloat16"), lhs_indices=to_dev(lhs), rhs_indices=to_dev(rhs))
    close(to_np(y), ref, "bfloat16")


def test_odd_group_count_takes_cp_async_kernel():
    # K = 192 at group 64: three groups (scale rows of 6 bytes) -> the cp.async kernel
    _sorted_case(8, 64, 192, [2, 0, 3, 1, 4, 0, 2, 5], seed=11)


def test_repeated_calls_and_graph_replay():
    """The chunk table lives in shared memory: back-to-back calls with different
    routings, and a CUDA graph replayed after its index array changed."""
    rng = np.random.default_rng(13)
    E, N, K = 32, 256, 1024
    wq, s, b = _experts(rng, E, N, K, "bfloat16", 64, 4)
    args = (to_dev(wq), to_dev(s, "bfloat16"), to_dev(b, "bfloat16"))
    x = to_dev(rand_x(rng, (40, 1, K), "bfloat16"), "bfloat16")
    sel = torch.zeros(40, dtype=torch.int32, device="cuda")
    out = {}

    def run():
        out["y"] = mxq.gather_qmm(x, *args, rhs_indices=sel, sorted_indices=True)

    for trial in range(3):
        routing = np.sort(rng.integers(0, E, 40)).astype(np.int32)
        sel.copy_(torch.from_numpy(routing))
        run()
        ref = coracle.gather_qmm(to_np(x), wq, s, b, routing, "bfloat16", 64, 4)
        close(to_np(out["y"]), ref, "bfloat16")
    g = torch.cuda.CUDAGraph()
    st = torch.cuda.Stream()
    st.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(st):
        run()
        with torch.cuda.graph(g, stream=st):
            run()
    torch.cuda.synchronize()
    routing = np.sort(rng.integers(0, E, 40)).astype(np.int32)
    sel.copy_(torch.from_numpy(routing))
    g.replay()
    torch.cuda.synchronize()
    ref = coracle.gather_qmm(to_np(x), wq, s, b, routing, "bfloat16", 64, 4)
    close(to_np(out["y"]), ref, "bfloat16")
    del g


# ------------------------------------------------------------ SwiGLU epilogue ----
def _swiglu_ref(g, u, dt):
    """silu(g) * u from the two projections as the oracle writes them (rounded to dt)."""
    gf, uf = O.to_f32(g, dt).astype(np.float64), O.to_f32(u, dt).astype(np.float64)
    return O.from_f32((gf / (1.0 + np.exp(-gf)) * uf).astype(np.float32), dt)


@pytest.mark.parametrize("sorted_rows", [True, False])
@pytest.mark.parametrize("K", [768, 2048, 192])
def test_gather_qmm_swiglu(sorted_rows, K):
    """Gate and up banks interleaved per expert; K=192 (three groups) takes the
    gather_qmm + element-wise form."""
    dt, gs, bits = "bfloat16", 64, 4
    rng = np.random.default_rng(K + sorted_rows)
    E, I, T, k = 16, 96, 12, 4
    gate, up = _experts(rng, E, I, K, dt, gs, bits), _experts(rng, E, I, K, dt, gs, bits)
    idx = np.stack([rng.choice(E, k, replace=False) for _ in range(T)]).astype(np.int32)
    x = rand_x(rng, (T, K), dt)
    if sorted_rows:
        flat = idx.reshape(-1)
        order = np.argsort(flat, kind="stable")
        xs, sel, lhs = x[order // k][:, None, :], flat[order].astype(np.int32), None
    else:
        xs, sel, lhs = x[:, None, :], idx.reshape(-1), np.repeat(np.arange(T, dtype=np.int32), k)
    g = coracle.gather_qmm(xs, *gate, sel, dt, gs, bits, lhs=lhs)
    u = coracle.gather_qmm(xs, *up, sel, dt, gs, bits, lhs=lhs)
    ref = _swiglu_ref(g, u, dt)
    dev = lambda t: tuple(to_dev(a, dt) if a.dtype != np.uint32 else to_dev(a) for a in t)
    w, s, b = mxq.interleave_gate_up(dev(gate), dev(up), gs, bits)
    y = mxq.gather_qmm_swiglu(to_dev(xs, dt), w, s, b,
                              lhs_indices=None if lhs is None else to_dev(lhs),
                              rhs_indices=to_dev(sel), sorted_indices=sorted_rows)
    assert y.shape == (len(sel), 1, I)
    close(to_np(y), ref, dt)


@pytest.mark.parametrize("T", [1, 64, 512])
def test_fused_switch_glu_matches_unfused(T):
    # 512 tokens x 8 = 4096 rows over 32 experts: the grouped tensor-core kernel's epilogue
    from mlx_server_runtime_b200 import nn
    E, D, H = 32, 512, 256
    g = torch.Generator(device="cuda").manual_seed(T)
    sw = nn.SwitchGLU(D, H, E, generator=g)
    nn.quantize(sw, 64, 4)
    x = torch.randn(T, D, device="cuda", generator=g).to(torch.bfloat16)
    idx = torch.stack([torch.randperm(E, device="cuda", generator=g)[:8] for _ in range(T)]).int()
    y_ref = sw(x, idx)
    sw.fuse_gate_up()
    assert not hasattr(sw, "gate_proj") and hasattr(sw, "gate_up_proj")
    y = sw(x, idx)
    close(to_np(y), to_np(y_ref), "bfloat16")


def test_gather_qmm_swiglu_grouped_prefill():
    """Sorted rows with enough per expert (>= 24 on average) take the grouped tensor-core
    kernel with the SwiGLU epilogue; an empty expert and a ragged one included."""
    dt, gs, bits = "bfloat16", 64, 4
    rng = np.random.default_rng(99)
    E, I, K = 8, 200, 1024
    counts = [50, 0, 131, 64, 1, 70, 90, 40]
    gate, up = _experts(rng, E, I, K, dt, gs, bits), _experts(rng, E, I, K, dt, gs, bits)
    sel = np.repeat(np.arange(E, dtype=np.int32), counts)
    xs = rand_x(rng, (sel.size, 1, K), dt)
    g = coracle.gather_qmm(xs, *gate, sel, dt, gs, bits)
    u = coracle.gather_qmm(xs, *up, sel, dt, gs, bits)
    ref = _swiglu_ref(g, u, dt)
    dev = lambda t: tuple(to_dev(a, dt) if a.dtype != np.uint32 else to_dev(a) for a in t)
    w, s, b = mxq.interleave_gate_up(dev(gate), dev(up), gs, bits)
    y = mxq.gather_qmm_swiglu(to_dev(xs, dt), w, s, b, rhs_indices=to_dev(sel),
                              sorted_indices=True)
    assert y.shape == (sel.size, 1, I)
    close(to_np(y), ref, dt)
