"""Parity at the benchmark configurations' real shapes, against the C oracle.

  config 2  decode: M in {1,2,4,8,16,32} x the Qwen2.5-7B projections (q/o 3584x3584,
            k/v 512x3584, gate/up 18944x3584, down 3584x18944) x bits {4, 8}, g64
  config 3  prefill: M in {512, 2048, 8192} x the same shapes, 4-bit g64, through the
            plan's own form (whole tiles or stream-K) and, for stream-K shapes, through
            whole tiles too (no workspace)
  config 5  MoE: 128 experts, top-8 routing from a softmax over N(0,1) logits, hidden
            2048, expert intermediate 768, T in {1, 64, 4096}: gather_qmm sorted and
            unsorted, and the SwitchGLU block end to end
plus the QuantizedEmbedding lookup (bit-exact rows) and its tied as_linear head.

Weights are N(0, 0.02) bf16, x ~ N(0, 1) bf16 (seeded numpy). The oracle computes
every output at decode sizes; at prefill and MoE sizes it computes a sample of rows
(the first and last rows, rows on tile boundaries and random rows) and the GPU's
rows at those positions are compared. Tolerance: max|d| <= 2e-2 * max|ref|
(bf16 output, fp32 accumulation)."""
import ctypes
import functools

import numpy as np
import pytest
import torch

import mlx_server_runtime_b200 as mxq
from mlx_server_runtime_b200 import _lib, nn
from oracle import coracle, oracle_np as O

from gpu_util import close, rand_x, to_dev, to_np

pytestmark = pytest.mark.gpu

SHAPES = {"q_o": (3584, 3584), "k_v": (512, 3584), "gate_up": (18944, 3584),
          "down": (3584, 18944)}
SEEDS = {"q_o": 101, "k_v": 102, "gate_up": 103, "down": 104}
DT = "bfloat16"


@functools.lru_cache(maxsize=None)
def _host_weights(name: str):
    N, K = SHAPES[name]
    rng = np.random.default_rng(SEEDS[name])
    w = O.from_f32((rng.standard_normal((N, K), dtype=np.float32) * 0.02), DT)
    return w


@functools.lru_cache(maxsize=4)
def _quantized(name: str, bits: int):
    wq, s, b = coracle.quantize(_host_weights(name), DT, 64, bits)
    return wq, s, b


def _dev(wq, s, b):
    return to_dev(wq), to_dev(s, DT), to_dev(b, DT)


@pytest.mark.parametrize("bits", [4, 8])
@pytest.mark.parametrize("name", sorted(SHAPES))
def test_config2_decode_sweep(name, bits):
    N, K = SHAPES[name]
    wq, s, b = _quantized(name, bits)
    wd = _dev(wq, s, b)
    rng = np.random.default_rng(N + K + bits)
    bias = rand_x(rng, (N,), DT) if name in ("q_o", "k_v") else None
    for M in (1, 2, 4, 8, 16, 32):
        x = rand_x(rng, (M, K), DT)
        ref = coracle.quantized_matmul(x, wq, s, b, DT, 64, bits, bias=bias)
        y = mxq.quantized_matmul(to_dev(x, DT), *wd, group_size=64, bits=bits,
                                 bias=None if bias is None else to_dev(bias, DT))
        close(to_np(y), ref, DT)


def _sample_rows(M, rng, n_random=40):
    rows = set(range(8)) | set(range(M - 8, M))
    for t in (128, 192, 384, 1024):  # token-tile boundaries of both tile widths
        if t < M:
            rows |= {t - 1, t}
    rows |= set(int(r) for r in rng.choice(M, n_random, replace=False))
    return np.array(sorted(rows), dtype=np.int64)


def _qmm_abi(x, w, s, b, out, M, N, K, workspace):
    ws_ptr = None if workspace is None else workspace.data_ptr()
    ws_len = 0 if workspace is None else workspace.numel()
    return _lib.load().mlxq_quantized_matmul(
        x.data_ptr(), w.data_ptr(), s.data_ptr(), b.data_ptr(), None, out.data_ptr(), M, N, K,
        64, 4, _lib.BF16, ws_ptr, ws_len, ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))


@pytest.mark.parametrize("M", [512, 2048, 8192])
@pytest.mark.parametrize("name", sorted(SHAPES))
def test_config3_prefill(name, M):
    N, K = SHAPES[name]
    wq, s, b = _quantized(name, 4)
    wd = _dev(wq, s, b)
    rng = np.random.default_rng(M + N)
    x = rand_x(rng, (M, K), DT)
    rows = _sample_rows(M, rng)
    ref = coracle.quantized_matmul(np.ascontiguousarray(x[rows]), wq, s, b, DT, 64, 4)
    xd = to_dev(x, DT)
    y = to_np(mxq.quantized_matmul(xd, *wd, group_size=64, bits=4))
    close(y[rows], ref, DT)
    if _lib.load().mlxq_qmm_workspace_size(M, N, K, 64, 4, _lib.BF16) > 0:
        # the plan runs stream-K here; without a workspace the kernel runs whole tiles
        out = torch.empty(M, N, dtype=torch.bfloat16, device="cuda")
        assert _qmm_abi(xd, *wd, out, M, N, K, None) == 0, _lib.last_error()
        close(to_np(out)[rows], ref, DT)


# ------------------------------------------------------------------ config 5: MoE ----
E, TOPK, HID, INTER = 128, 8, 2048, 768


@functools.lru_cache(maxsize=1)
def _moe_weights():
    """gate/up [E, 768, 2048] and down [E, 2048, 768], N(0, 0.02) bf16, quantized
    4-bit g64 (on the device; the packing is bit-exact to the oracle's, tested
    elsewhere), with host copies for the oracle."""
    g = torch.Generator(device="cuda").manual_seed(5)
    out = {}
    for name, (n, k) in (("gate", (INTER, HID)), ("up", (INTER, HID)), ("down", (HID, INTER))):
        w = (torch.randn(E, n, k, device="cuda", generator=g) * 0.02).to(torch.bfloat16)
        dev = mxq.quantize(w, 64, 4)
        out[name] = (dev, tuple(to_np(t) for t in dev))
    return out


def _route(T, rng):
    logits = rng.standard_normal((T, E)).astype(np.float32)
    p = np.exp(logits - logits.max(-1, keepdims=True))
    p /= p.sum(-1, keepdims=True)
    return np.argsort(-p, axis=-1, kind="stable")[:, :TOPK].astype(np.int32)


def _oracle_switch_glu(x, idx, host):
    """SwitchGLU for the given tokens: per (token, expert) row, silu(gate) * up with
    each projection and the activation rounded to bf16 as the module computes them,
    then the down projection (lfm2.py:193-218)."""
    T = x.shape[0]
    flat = idx.reshape(-1)
    lhs = np.repeat(np.arange(T, dtype=np.int32), TOPK)
    xs = x.reshape(T, 1, HID)
    g = O.to_f32(coracle.gather_qmm(xs, *host["gate"], flat, DT, 64, 4, lhs=lhs), DT)
    u = O.to_f32(coracle.gather_qmm(xs, *host["up"], flat, DT, 64, 4, lhs=lhs), DT)
    act = O.round_to(g / (1.0 + np.exp(-g)), DT)
    h = O.from_f32(act * u, DT)                                       # [T*k, 1, 768]
    y = coracle.gather_qmm(h, *host["down"], flat, DT, 64, 4)          # [T*k, 1, 2048]
    return y.reshape(T, TOPK, HID)


@pytest.mark.parametrize("T", [1, 64, 4096])
def test_config5_moe(T):
    W = _moe_weights()
    host = {k: v[1] for k, v in W.items()}
    rng = np.random.default_rng(T)
    x = rand_x(rng, (T, HID), DT)
    idx = _route(T, rng)
    toks = np.arange(T) if T <= 64 else _sample_rows(T, rng)
    ref = _oracle_switch_glu(np.ascontiguousarray(x[toks]), np.ascontiguousarray(idx[toks]), host)

    # the SwitchGLU block as the model graphs call it (sorted by expert from 64 rows)
    sw = nn.SwitchGLU.__new__(nn.SwitchGLU)
    for name, attr in (("gate", "gate_proj"), ("up", "up_proj"), ("down", "down_proj")):
        q = nn.QuantizedSwitchLinear.__new__(nn.QuantizedSwitchLinear)
        q.group_size, q.bits, q.mode = 64, 4, "affine"
        q.weight, q.scales, q.biases = W[name][0]
        setattr(sw, attr, q)
    xd, idd = to_dev(x, DT), to_dev(idx)
    y = to_np(sw(xd, idd))                                             # [T, k, 2048]
    close(y[toks], ref, DT)

    # gather_qmm of the gate projection, both forms, on the same rows
    flat = idx.reshape(-1)
    order = np.argsort(flat, kind="stable")
    xs = x[order // TOPK][:, None, :]
    sel = flat[order].astype(np.int32)
    gdev = W["gate"][0]
    y_sorted = to_np(mxq.gather_qmm(to_dev(xs, DT), *gdev, rhs_indices=to_dev(sel),
                                    sorted_indices=True))
    y_plain = to_np(mxq.gather_qmm(to_dev(xs, DT), *gdev, rhs_indices=to_dev(sel),
                                   sorted_indices=False))
    pick = np.arange(len(sel)) if len(sel) <= 512 else _sample_rows(len(sel), rng, 120)
    ref_g = coracle.gather_qmm(np.ascontiguousarray(xs[pick]), *host["gate"], sel[pick], DT, 64, 4)
    close(y_sorted[pick], ref_g, DT)
    close(y_plain[pick], ref_g, DT)


# ------------------------------------------------------- QuantizedEmbedding (a2) ----
def test_quantized_embedding_lookup_and_tied_head():
    rng = np.random.default_rng(21)
    V, D = 4096, 3584
    w = O.from_f32(rng.standard_normal((V, D), dtype=np.float32) * 0.02, DT)
    wq, s, b = coracle.quantize(w, DT, 64, 4)
    emb = nn.QuantizedEmbedding.__new__(nn.QuantizedEmbedding)
    emb.group_size, emb.bits, emb.mode = 64, 4, "affine"
    emb.weight, emb.scales, emb.biases = _dev(wq, s, b)
    ids = rng.integers(0, V, size=(3, 7)).astype(np.int64)
    ids[0, :3] = [0, V - 1, 17]
    rows = to_np(emb(torch.from_numpy(ids).cuda()))                     # [3, 7, D]
    table = coracle.dequantize(wq, s, b, DT, 64, 4)
    assert rows.tobytes() == table[ids].tobytes()                      # bit-exact
    x = rand_x(rng, (5, D), DT)
    ref = coracle.quantized_matmul(x, wq, s, b, DT, 64, 4)
    close(to_np(emb.as_linear(to_dev(x, DT))), ref, DT)
    tok = to_np(emb.greedy_tokens(to_dev(x, DT)))
    ref_f = O.to_f32(ref, DT)
    assert np.array_equal(ref_f[np.arange(5), tok], ref_f.max(-1))
