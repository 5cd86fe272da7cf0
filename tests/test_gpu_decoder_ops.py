"""The decoder-layer operators against the numpy restatement (oracle/decoder_np.py):
RMSNorm with the fused residual add, RoPE with the paged KV append, paged attention
(decode with several key splits, and prefill including a chunk over an existing
cache), the quantized embedding lookup (bit-exact) and the decode-state advance.

Floating-point tolerance: max|d| <= 2e-2 * max|ref| (bf16/f16 outputs; the oracle
computes angles, norms and softmax in float64, the kernels in float32)."""
import numpy as np
import pytest
import torch

import mlx_server_runtime_b200 as mxq
from mlx_server_runtime_b200 import _lib, attention as A
from oracle import coracle, decoder_np as D, oracle_np as O

from gpu_util import close, rand_weights, rand_x, to_dev, to_np

pytestmark = pytest.mark.gpu


def _f32(t, dt):
    return O.to_f32(to_np(t), dt)


@pytest.mark.parametrize("dt", ["bfloat16", "float16"])
@pytest.mark.parametrize("rows,dim", [(1, 3584), (7, 3584), (33, 896), (5, 128)])
def test_rms_norm(dt, rows, dim):
    rng = np.random.default_rng(rows * dim)
    x, r = rand_x(rng, (rows, dim), dt), rand_x(rng, (rows, dim), dt)
    w = O.from_f32((1.0 + 0.1 * rng.standard_normal(dim)).astype(np.float32), dt)
    y = A.rms_norm(to_dev(x, dt), to_dev(w, dt), 1e-6)
    ref, _ = D.rms_norm(O.to_f32(x, dt), O.to_f32(w, dt), 1e-6, dt)
    close(to_np(y), O.from_f32(ref, dt), dt)
    y2, h = A.rms_norm(to_dev(x, dt), to_dev(w, dt), 1e-6, residual=to_dev(r, dt),
                       residual_out=True)
    ref2, href = D.rms_norm(O.to_f32(x, dt), O.to_f32(w, dt), 1e-6, dt, residual=O.to_f32(r, dt))
    assert to_np(h).tobytes() == O.from_f32(href, dt).tobytes()   # the add is exact
    close(to_np(y2), O.from_f32(ref2, dt), dt)


@pytest.mark.parametrize("hq,hkv,hd,base", [(28, 4, 128, 1e6), (8, 2, 64, 1e4)])
def test_rope_kv_append(hq, hkv, hd, base):
    dt = "bfloat16"
    rng = np.random.default_rng(hq + hd)
    T, pages, page = 9, 12, 16
    qkv = rand_x(rng, (T, (hq + 2 * hkv) * hd), dt)
    positions = rng.integers(0, 3000, T).astype(np.int32)
    slots = rng.choice(pages * page, T, replace=False).astype(np.int32)
    slots[4] = -1  # not appended
    kc = torch.zeros(pages, page, hkv, hd, dtype=torch.bfloat16, device="cuda")
    vc = torch.zeros_like(kc)
    q = A.rope_kv_append(to_dev(qkv, dt), to_dev(positions), to_dev(slots), kc, vc, hq, hkv, hd,
                         base)
    xf = O.to_f32(qkv, dt)
    qref = D.rope(xf[:, :hq * hd].reshape(T, hq, hd), positions, base, dt)
    kref = D.rope(xf[:, hq * hd:(hq + hkv) * hd].reshape(T, hkv, hd), positions, base, dt)
    vref = xf[:, (hq + hkv) * hd:].reshape(T, hkv, hd)
    close(to_np(q), O.from_f32(qref, dt), dt)
    kflat = _f32(kc, dt).reshape(pages * page, hkv, hd)
    vflat = _f32(vc, dt).reshape(pages * page, hkv, hd)
    for t in range(T):
        if slots[t] < 0:
            continue
        close(O.from_f32(kflat[slots[t]], dt), O.from_f32(kref[t], dt), dt)
        assert np.array_equal(vflat[slots[t]], vref[t])
    untouched = np.setdiff1d(np.arange(pages * page), slots[slots >= 0])
    assert not kflat[untouched].any() and not vflat[untouched].any()


def _paged_problem(rng, B, hkv, hd, kv_lens, page=16, dt="bfloat16"):
    """Random K/V for each sequence written to shuffled pages of a pool."""
    max_blocks = max((n + page - 1) // page for n in kv_lens)
    pages = B * max_blocks + 3
    perm = rng.permutation(pages).astype(np.int32)
    bt = perm[:B * max_blocks].reshape(B, max_blocks)
    kpool = rand_x(rng, (pages, page, hkv, hd), dt)
    vpool = rand_x(rng, (pages, page, hkv, hd), dt)
    return bt, kpool, vpool


@pytest.mark.parametrize("hq,hkv,hd,long", [(28, 4, 128, False), (8, 2, 64, False),
                                            (4, 4, 128, False), (28, 4, 128, True)])
def test_paged_attention_decode(hq, hkv, hd, long):
    dt = "bfloat16"
    rng = np.random.default_rng(hq * hd + long)
    kv_lens = np.array([1, 17, 128, 129, 300, 640, 511, 64], np.int32)
    if long:  # more than 64 tiles of 64 keys: several tiles per split
        kv_lens = np.array([5000, 4097, 1, 300], np.int32)
    B = len(kv_lens)
    bt, kpool, vpool = _paged_problem(rng, B, hkv, hd, kv_lens)
    q = rand_x(rng, (B, hq, hd), dt)
    kc, vc = to_dev(kpool, dt), to_dev(vpool, dt)
    scale = hd ** -0.5
    for _ in range(2):  # a second call reuses the workspace (tickets left at zero)
        out = A.paged_attention_decode(to_dev(q, dt), kc, vc, to_dev(bt), to_dev(kv_lens),
                                       int(kv_lens.max()), scale)
        got = to_np(out)
        for b in range(B):
            k = D.gather_pages(O.to_f32(kpool, dt), bt[b], kv_lens[b])
            v = D.gather_pages(O.to_f32(vpool, dt), bt[b], kv_lens[b])
            ref = D.attention(O.to_f32(q, dt)[b:b + 1], k, v, np.array([kv_lens[b] - 1]),
                              scale, dt)
            close(got[b:b + 1], O.from_f32(ref, dt), dt)


@pytest.mark.parametrize("hq,hkv,hd", [(28, 4, 128), (8, 2, 64)])
def test_paged_attention_prefill(hq, hkv, hd):
    dt = "bfloat16"
    rng = np.random.default_rng(hq + hkv + hd)
    q_lens = np.array([64, 100, 1, 200], np.int32)
    kv_lens = np.array([64, 300, 77, 200], np.int32)   # chunks over existing caches
    B = len(q_lens)
    bt, kpool, vpool = _paged_problem(rng, B, hkv, hd, kv_lens)
    cu = np.concatenate([[0], np.cumsum(q_lens)]).astype(np.int32)
    q = rand_x(rng, (int(cu[-1]), hq, hd), dt)
    out = A.paged_attention_prefill(to_dev(q, dt), to_dev(cu), int(q_lens.max()),
                                    to_dev(kpool, dt), to_dev(vpool, dt), to_dev(bt),
                                    to_dev(kv_lens), hd ** -0.5)
    got = to_np(out)
    for b in range(B):
        k = D.gather_pages(O.to_f32(kpool, dt), bt[b], kv_lens[b])
        v = D.gather_pages(O.to_f32(vpool, dt), bt[b], kv_lens[b])
        pos = kv_lens[b] - q_lens[b] + np.arange(q_lens[b])
        ref = D.attention(O.to_f32(q, dt)[cu[b]:cu[b + 1]], k, v, pos, hd ** -0.5, dt)
        close(got[cu[b]:cu[b + 1]], O.from_f32(ref, dt), dt)


@pytest.mark.parametrize("bits,gs,dt", [(4, 64, "bfloat16"), (8, 32, "float16")])
def test_quantized_embedding_bit_exact(bits, gs, dt):
    rng = np.random.default_rng(bits + gs)
    V, Dm = 1000, 768
    w = rand_weights(rng, (V, Dm), dt)
    wq, s, b = coracle.quantize(w, dt, gs, bits)
    ids = rng.integers(0, V, 37).astype(np.int32)
    ids[:3] = [0, V - 1, 5]
    out = A.quantized_embedding(to_dev(ids), to_dev(wq), to_dev(s, dt), to_dev(b, dt), gs, bits)
    table = coracle.dequantize(wq, s, b, dt, gs, bits)
    assert to_np(out).tobytes() == np.ascontiguousarray(table[ids]).tobytes()
    bad = to_dev(np.array([-1, V], np.int32))
    z = A.quantized_embedding(bad, to_dev(wq), to_dev(s, dt), to_dev(b, dt), gs, bits)
    assert not O.to_f32(to_np(z), dt).any()


def test_decode_advance():
    page = 16
    bt = torch.tensor([[5, 9, 2], [7, 1, 0]], dtype=torch.int32, device="cuda")
    pos = torch.tensor([14, 30], dtype=torch.int32, device="cuda")
    kv = pos + 1
    slots = torch.zeros(2, dtype=torch.int32, device="cuda")
    A.decode_advance(pos, kv, slots, bt, page)
    assert pos.tolist() == [15, 31] and kv.tolist() == [16, 32]
    assert slots.tolist() == [5 * 16 + 15, 1 * 16 + 15]
    A.decode_advance(pos, kv, slots, bt, page)
    assert pos.tolist() == [16, 32] and slots.tolist() == [9 * 16 + 0, 0 * 16 + 0]
    pos.fill_(47)
    A.decode_advance(pos, kv, slots, bt, page)  # position 48 is past 3 pages of 16
    assert slots.tolist() == [-1, -1]
