"""Independent numpy restatement of MLX's affine quantization family.

TEST INFRASTRUCTURE ONLY: used by tests/ to cross-check the C oracle
(oracle/qmm_oracle.c) and to build golden fixtures. The product path never
imports it.

Parity status: UNPINNED against the reference (mlx 0.31.2, pinned at
python/uv.lock:939-940 of the reference tree, is neither vendored nor
installable here, and the reference's tests hold no quantized vectors).
This module restates MLX's published semantics a second time, in vectorized
numpy, so that the C oracle is checked by an implementation that shares no
code with it.

Arrays of bf16/f16 values are carried as numpy ``uint16`` bit patterns
(bf16) or ``float16`` (f16); ``dtype`` strings are "float32", "bfloat16",
"float16".
"""
from __future__ import annotations

import numpy as np

DTYPES = ("float32", "bfloat16", "float16")


# ---- bit-exact conversions -------------------------------------------------------------
def bf16_bits_to_f32(bits: np.ndarray) -> np.ndarray:
    return (bits.astype(np.uint32) << 16).view(np.float32)


def f32_to_bf16_bits(x: np.ndarray) -> np.ndarray:
    """Round-to-nearest-even float32 -> bfloat16 bit pattern (NaNs stay quiet NaNs).

    In uint32: the rounding add cannot wrap for a non-NaN pattern (the largest,
    -inf = 0xFF800000, plus 0x8000 stays below 2^32); NaN lanes are replaced."""
    u = np.ascontiguousarray(x, dtype=np.float32).view(np.uint32)
    r = (u >> 16) & 1
    r += 0x7FFF
    r += u
    r >>= 16
    out = r.astype(np.uint16)
    nan = (u & 0x7FFFFFFF) > 0x7F800000
    if nan.any():
        out[nan] = ((u[nan] >> 16) | 0x40).astype(np.uint16)
    return out


def to_f32(a: np.ndarray, dtype: str) -> np.ndarray:
    if dtype == "bfloat16":
        return bf16_bits_to_f32(a)
    return np.asarray(a).astype(np.float32)


def from_f32(a: np.ndarray, dtype: str) -> np.ndarray:
    if dtype == "bfloat16":
        return f32_to_bf16_bits(a)
    if dtype == "float16":
        return np.asarray(a, dtype=np.float32).astype(np.float16)
    return np.asarray(a, dtype=np.float32)


def round_to(a: np.ndarray, dtype: str) -> np.ndarray:
    """Round float32 values to the storage precision of ``dtype`` (result float32)."""
    return to_f32(from_f32(a, dtype), dtype)


# ---- the operators ---------------------------------------------------------------------
def quantize(w, dtype: str, group_size: int = 64, bits: int = 4):
    """MLX affine quantize of the last axis. Returns (w_q uint32, scales, biases)."""
    wf = to_f32(w, dtype)
    rows, K = wf.shape
    assert K % group_size == 0
    n_bins = np.float32((1 << bits) - 1)
    g = wf.reshape(rows, K // group_size, group_size)
    w_max = g.max(axis=-1)
    w_min = g.min(axis=-1)
    mask = np.abs(w_min) > np.abs(w_max)
    scale = np.maximum((w_max - w_min) / n_bins, np.float32(1e-7)).astype(np.float32)
    scale = np.where(mask, scale, -scale).astype(np.float32)
    edge = np.where(mask, w_min, w_max).astype(np.float32)
    with np.errstate(divide="ignore", invalid="ignore"):
        q0 = np.rint(edge / scale).astype(np.float32)
        nz = q0 != 0
        scale = np.where(nz, edge / np.where(nz, q0, np.float32(1)), scale).astype(np.float32)
    bias = np.where(nz, edge, np.float32(0)).astype(np.float32)
    q = np.rint((g - bias[..., None]) / scale[..., None]).astype(np.float32)
    q = np.clip(q, np.float32(0), n_bins).astype(np.uint32)
    epw = 32 // bits
    q = q.reshape(rows, K // epw, epw)
    shifts = (np.arange(epw, dtype=np.uint32) * bits).astype(np.uint32)
    wq = np.bitwise_or.reduce(q << shifts, axis=-1).astype(np.uint32)
    return wq, from_f32(scale, dtype), from_f32(bias, dtype)


def unpack(wq: np.ndarray, bits: int) -> np.ndarray:
    """uint32 [rows, K*bits/32] -> integer codes [rows, K] (little-endian within a word)."""
    epw = 32 // bits
    shifts = (np.arange(epw, dtype=np.uint32) * bits).astype(np.uint32)
    codes = (wq[..., None] >> shifts) & np.uint32((1 << bits) - 1)
    return codes.reshape(*wq.shape[:-1], wq.shape[-1] * epw)


def pack(codes: np.ndarray, bits: int) -> np.ndarray:
    epw = 32 // bits
    c = codes.astype(np.uint32).reshape(*codes.shape[:-1], codes.shape[-1] // epw, epw)
    shifts = (np.arange(epw, dtype=np.uint32) * bits).astype(np.uint32)
    return np.bitwise_or.reduce(c << shifts, axis=-1).astype(np.uint32)


def dequantize(wq, scales, biases, dtype: str, group_size: int = 64, bits: int = 4):
    """out = round(round(scale*q) + bias) in ``dtype`` (one rounding per operation)."""
    q = unpack(wq, bits).astype(np.float32)
    rows, K = q.shape
    s = np.repeat(to_f32(scales, dtype), group_size, axis=-1).reshape(rows, K)
    b = np.repeat(to_f32(biases, dtype), group_size, axis=-1).reshape(rows, K)
    t = round_to((s * q).astype(np.float32), dtype)
    return from_f32((t + b).astype(np.float32), dtype)


def dequantize_f32(wq, scales, biases, dtype: str, group_size: int = 64, bits: int = 4):
    """scale*q + bias computed in float32 (the weight value the matmul oracle uses)."""
    q = unpack(wq, bits).astype(np.float32)
    rows, K = q.shape
    s = np.repeat(to_f32(scales, dtype), group_size, axis=-1).reshape(rows, K)
    b = np.repeat(to_f32(biases, dtype), group_size, axis=-1).reshape(rows, K)
    return (s * q + b).astype(np.float32)


def quantized_matmul(x, wq, scales, biases, dtype: str, group_size=64, bits=4, bias=None):
    """x [M,K] @ dequant(w)^T, float accumulation (float64 here), rounded to ``dtype``."""
    wf = dequantize_f32(wq, scales, biases, dtype, group_size, bits).astype(np.float64)
    xf = to_f32(x, dtype).astype(np.float64)
    y = round_to((xf @ wf.T).astype(np.float32), dtype)
    if bias is not None:
        y = round_to(y + to_f32(bias, dtype)[None, :], dtype)
    return from_f32(y, dtype)


def gather_qmm(x, wq, scales, biases, rhs, dtype: str, group_size=64, bits=4, lhs=None,
               lhs_div=1):
    """x [Xb, M, K]; w [E, N, Kw]; out [B, M, N] with out[b] = x[xi(b)] @ W[rhs[b]]^T."""
    B = rhs.shape[0]
    E, N, _ = wq.shape
    outs = []
    for b in range(B):
        xi = int(lhs[b]) if lhs is not None else b // lhs_div
        e = int(rhs[b])
        outs.append(quantized_matmul(x[xi], wq[e], scales[e], biases[e], dtype, group_size,
                                     bits))
    return np.stack(outs, axis=0)
