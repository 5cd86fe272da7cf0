"""Numpy restatement of the decoder-layer operators around the quantized projections,
and of a whole Qwen2-architecture forward pass, for the parity tests.

TEST INFRASTRUCTURE ONLY: imported by tests/ (and nothing in the product package).
It follows the reference's graph (python/mlx_worker/native_mlx/ of the reference):
  rms_norm   nn.RMSNorm / mx.fast.rms_norm (models/qwen2.py:144-147): the normalized
             value rounded to the activation dtype, then the weight product rounded
  rope       mx.fast.rope, traditional=False (models/qwen2.py:91-105): pairs (i, i+hd/2)
             rotated by position * base^(-2i/hd)
  attention  append_and_attend (attention.py:215-298): SDPA over the sequence's keys
             gathered from its pages (_dense_kv_rows) with the causal mask of
             _dense_causal_mask (attention.py:404-427), softmax in float
  forward    Qwen2ForCausalLM (models/qwen2.py:46-227) with every projection through
             the C oracle's quantized_matmul and op-by-op rounding as MLX evaluates
             the graph (silu rounded, then the product rounded)
Angles, norms and softmax are computed in float64 here (the kernels use float32), so
agreement is to the tolerance the tests state, not bit for bit.

Parity status: unpinned against the reference (MLX is neither vendored nor
installable here), like the rest of oracle/.
"""
from __future__ import annotations

import numpy as np

from . import coracle
from .oracle_np import from_f32, round_to, to_f32


def rms_norm(x, w, eps, dtype, residual=None):
    """Returns (normed, h) as float32 values already rounded to dtype; x, w,
    residual are float32 arrays holding dtype values."""
    h = x if residual is None else round_to(x + residual, dtype)
    h64 = h.astype(np.float64)
    r = 1.0 / np.sqrt((h64 * h64).mean(axis=-1, keepdims=True) + eps)
    y = round_to(round_to((h64 * r).astype(np.float32), dtype) * w, dtype)
    return y, h


def rope(x, positions, base, dtype):
    """x [T, H, hd] float32, positions [T] -> rotated, rounded to dtype."""
    T, H, hd = x.shape
    half = hd // 2
    inv = base ** (-(2.0 * np.arange(half, dtype=np.float64)) / hd)
    ang = positions.astype(np.float64)[:, None] * inv[None, :]          # [T, half]
    c, s = np.cos(ang)[:, None, :], np.sin(ang)[:, None, :]
    a, b = x[..., :half].astype(np.float64), x[..., half:].astype(np.float64)
    out = np.concatenate([a * c - b * s, a * s + b * c], axis=-1)
    return round_to(out.astype(np.float32), dtype)


def attention(q, k, v, q_positions, scale, dtype):
    """q [Tq, Hq, hd] of one sequence at q_positions, k/v [L, Hkv, hd] its cached keys
    and values (dense rows): causal SDPA, heads grouped Hq / Hkv per kv head."""
    Tq, Hq, hd = q.shape
    L, Hkv, _ = k.shape
    G = Hq // Hkv
    kk = np.repeat(k.astype(np.float64), G, axis=1)                     # [L, Hq, hd]
    vv = np.repeat(v.astype(np.float64), G, axis=1)
    s = np.einsum("thd,lhd->htl", q.astype(np.float64), kk) * scale      # [Hq, Tq, L]
    mask = np.arange(L)[None, :] <= q_positions[:, None]                 # [Tq, L]
    s = np.where(mask[None], s, -np.inf)
    s -= s.max(axis=-1, keepdims=True)
    p = np.exp(s)
    p /= p.sum(axis=-1, keepdims=True)
    o = np.einsum("htl,lhd->thd", p, vv)
    return round_to(o.astype(np.float32), dtype)


def gather_pages(pool, block_table_row, length):
    """Dense rows [length, ...] of one sequence from a [pages, page, ...] pool."""
    page = pool.shape[1]
    nb = (length + page - 1) // page
    return pool[block_table_row[:nb]].reshape(-1, *pool.shape[2:])[:length]


def dequant_rows(wq, s, b, ids, dtype, group_size, bits):
    table = coracle.dequantize(np.ascontiguousarray(wq[ids]), np.ascontiguousarray(s[ids]),
                               np.ascontiguousarray(b[ids]), dtype, group_size, bits)
    return to_f32(table, dtype)


def qmm(x, w, dtype, group_size, bits, bias=None):
    """x float32 [M, K] of dtype values; w = (wq, s, b) in storage form; returns float32."""
    y = coracle.quantized_matmul(from_f32(x, dtype), *w, dtype, group_size, bits,
                                 bias=None if bias is None else bias)
    return to_f32(y, dtype)


def forward(P, cfg, ids, dtype="bfloat16"):
    """Qwen2 forward over one whole sequence ids [L] (positions 0..L-1, no cache):
    returns (final normed hidden [L, D], logits [L, vocab]) as float32 values.
    P holds the model's parameters in storage form (see tests)."""
    gs, bits = cfg["group_size"], cfg["bits"]
    Hq, Hkv, hd = cfg["heads"], cfg["kv_heads"], cfg["head_dim"]
    eps, base = cfg["eps"], cfg["rope_theta"]
    L = len(ids)
    pos = np.arange(L)
    h = dequant_rows(*P["embed"], np.asarray(ids), dtype, gs, bits)
    for lp in P["layers"]:
        x, _ = rms_norm(h, lp["in_norm"], eps, dtype)
        qkv = qmm(x, lp["qkv"], dtype, gs, bits, bias=lp["qkv_bias"])
        q = qkv[:, :Hq * hd].reshape(L, Hq, hd)
        k = qkv[:, Hq * hd:(Hq + Hkv) * hd].reshape(L, Hkv, hd)
        v = qkv[:, (Hq + Hkv) * hd:].reshape(L, Hkv, hd)
        q, k = rope(q, pos, base, dtype), rope(k, pos, base, dtype)
        a = attention(q, k, v, pos, hd ** -0.5, dtype).reshape(L, Hq * hd)
        o = qmm(a, lp["o"], dtype, gs, bits)
        h = round_to(h + o, dtype)
        x, _ = rms_norm(h, lp["post_norm"], eps, dtype)
        gu = qmm(x, lp["gate_up"], dtype, gs, bits)          # rows interleaved by 8
        gu = gu.reshape(L, -1, 2, 8)
        g, u = gu[:, :, 0, :].reshape(L, -1), gu[:, :, 1, :].reshape(L, -1)
        act = round_to((g.astype(np.float64) / (1.0 + np.exp(-g.astype(np.float64))))
                       .astype(np.float32), dtype)
        m = qmm(round_to(act * u, dtype), lp["down"], dtype, gs, bits)
        h = round_to(h + m, dtype)
    x, _ = rms_norm(h, P["norm"], eps, dtype)
    logits = qmm(x, P["head"], dtype, gs, bits)
    return x, logits
