"""Decoder-layer operators around the quantized projections, over torch CUDA tensors.

The reference's Qwen2-style graphs (python/mlx_worker/native_mlx/ of the reference)
run, on either side of every projection:
  * RMSNorm (models/qwen2.py:144-147,161-165; mx.fast.rms_norm),
  * RoPE on queries and keys (models/qwen2.py:91-105; mx.fast.rope, traditional=False),
  * the paged KV append and attention over the cached pages
    (attention.py:215-298 append_and_attend, cache.py:485-520 stage_layer, with the
    [pages, page_size, kv_heads, head_dim] pools of cache.py:651-700),
  * the embedding lookup (models/qwen2.py:185).
Each function here is one call into libmlxq_b200.so on the tensors' device and
current stream; misuse raises ValueError, device failures RuntimeError.
"""
from __future__ import annotations

import math
import threading
from dataclasses import dataclass

import torch

from . import _lib
from .core import Workspace

__all__ = ["rms_norm", "rope_kv_append", "paged_attention_decode", "paged_attention_prefill",
           "quantized_embedding", "decode_advance", "PagedKVCache", "PagedBatch"]

_DT = {torch.bfloat16: _lib.BF16, torch.float16: _lib.F16}


def _code(t: torch.Tensor, what: str) -> int:
    if t.dtype not in _DT:
        raise ValueError(f"{what} must be bfloat16 or float16, got {t.dtype}")
    return _DT[t.dtype]


def _stream(dev: torch.device):
    return torch.cuda.current_stream(dev).cuda_stream


def _p(t):
    return None if t is None else t.data_ptr()


def _i32(t: torch.Tensor, what: str) -> torch.Tensor:
    if t.dtype != torch.int32:
        raise ValueError(f"{what} must be int32, got {t.dtype}")
    return t.contiguous()


def rms_norm(x: torch.Tensor, weight: torch.Tensor, eps: float = 1e-6,
             residual: torch.Tensor | None = None, residual_out: bool = False):
    """RMSNorm of the last axis (nn.RMSNorm): round(round(h * rsqrt(mean(h^2) + eps))
    * weight) with h = x, or h = round(x + residual). With residual_out, returns
    (normed, h): the decoder block's `hidden = x + attn_out` and its norm in one
    launch (qwen2.py:161-165)."""
    dt = _code(x, "x")
    D = x.shape[-1]
    if weight.shape != (D,) or weight.dtype != x.dtype:
        raise ValueError(f"weight must be [{D}] of dtype {x.dtype}")
    if residual is not None and (residual.shape != x.shape or residual.dtype != x.dtype):
        raise ValueError("residual must match x")
    if residual_out and residual is None:
        raise ValueError("residual_out needs a residual")
    x = x.contiguous()
    rows = x.numel() // D if D else 0
    out = torch.empty_like(x)
    h = torch.empty_like(x) if residual_out else None
    with torch.cuda.device(x.device):
        rc = _lib.load().mlxq_rms_norm(_p(x), _p(None if residual is None else residual.contiguous()),
                                       _p(weight.contiguous()), _p(out), _p(h), rows, D,
                                       float(eps), dt, _stream(x.device))
    _lib.check(rc, "rms_norm")
    return (out, h) if residual_out else out


def rope_kv_append(qkv: torch.Tensor, positions: torch.Tensor, slots: torch.Tensor,
                   k_cache: torch.Tensor, v_cache: torch.Tensor, n_heads: int, n_kv_heads: int,
                   head_dim: int, base: float = 10000.0) -> torch.Tensor:
    """RoPE of the queries and keys in `qkv` [T, (n_heads + 2 n_kv_heads) * head_dim]
    (the fused q/k/v projection's output) at `positions` [T], keys and values written
    to cache rows `slots` [T] (page * page_size + offset, -1 = skip) of
    k_cache / v_cache [pages, page_size, n_kv_heads, head_dim]. Returns the rotated
    queries [T, n_heads, head_dim]."""
    dt = _code(qkv, "qkv")
    if qkv.ndim != 2 or qkv.stride(1) != 1:
        raise ValueError("qkv must be a 2-D tensor with contiguous rows")
    T = qkv.shape[0]
    for c in (k_cache, v_cache):
        if c.dtype != qkv.dtype or c.shape[-2:] != (n_kv_heads, head_dim) or not c.is_contiguous():
            raise ValueError("caches must be contiguous [pages, page_size, n_kv_heads, head_dim] "
                             "of qkv's dtype")
    positions, slots = _i32(positions, "positions"), _i32(slots, "slots")
    if positions.shape != (T,) or slots.shape != (T,):
        raise ValueError(f"positions and slots must be [{T}]")
    q = torch.empty(T, n_heads, head_dim, dtype=qkv.dtype, device=qkv.device)
    with torch.cuda.device(qkv.device):
        rc = _lib.load().mlxq_rope_kv_append(_p(qkv), qkv.stride(0), _p(q), _p(k_cache),
                                             _p(v_cache), _p(positions), _p(slots), T, n_heads,
                                             n_kv_heads, head_dim, float(base), dt,
                                             _stream(qkv.device))
    _lib.check(rc, "rope_kv_append")
    return q


def _cache_geometry(k_cache, v_cache, q):
    if k_cache.shape != v_cache.shape or k_cache.dtype != q.dtype or v_cache.dtype != q.dtype:
        raise ValueError("k_cache and v_cache must share shape and q's dtype")
    if k_cache.ndim != 4 or not k_cache.is_contiguous() or not v_cache.is_contiguous():
        raise ValueError("caches must be contiguous [pages, page_size, n_kv_heads, head_dim]")
    _, page, hkv, hd = k_cache.shape
    return page, hkv, hd


def paged_attention_decode(q: torch.Tensor, k_cache: torch.Tensor, v_cache: torch.Tensor,
                           block_table: torch.Tensor, kv_lens: torch.Tensor, max_kv_len: int,
                           scale: float) -> torch.Tensor:
    """One query per sequence: q [B, n_heads, head_dim] at position kv_lens[b] - 1
    attends all kv_lens[b] cached keys of sequence b (pages block_table[b])."""
    dt = _code(q, "q")
    page, hkv, hd = _cache_geometry(k_cache, v_cache, q)
    B, H, _ = q.shape
    block_table, kv_lens = _i32(block_table, "block_table"), _i32(kv_lens, "kv_lens")
    out = torch.empty_like(q)
    dev = q.device
    L = _lib.load()
    need = L.mlxq_paged_attention_workspace_size(B, hkv, max_kv_len, hd)
    with torch.cuda.device(dev):
        st = torch.cuda.current_stream(dev)
        ws = Workspace.get(dev, st, need, "attention") if need else None
        rc = L.mlxq_paged_attention_decode(_p(q.contiguous()), _p(k_cache), _p(v_cache),
                                           _p(block_table), block_table.shape[1], _p(kv_lens),
                                           int(max_kv_len), _p(out), B, H, hkv, hd, page,
                                           float(scale), dt, _p(ws),
                                           0 if ws is None else ws.numel(), st.cuda_stream)
    _lib.check(rc, "paged_attention_decode")
    return out


def paged_attention_prefill(q: torch.Tensor, cu_q: torch.Tensor, max_q_len: int,
                            k_cache: torch.Tensor, v_cache: torch.Tensor,
                            block_table: torch.Tensor, kv_lens: torch.Tensor,
                            scale: float) -> torch.Tensor:
    """New tokens of every sequence: q [total, n_heads, head_dim], sequence b's rows
    [cu_q[b], cu_q[b+1]) at the last positions of its kv_lens[b] cached keys, causal."""
    dt = _code(q, "q")
    page, hkv, hd = _cache_geometry(k_cache, v_cache, q)
    _, H, _ = q.shape
    block_table, kv_lens = _i32(block_table, "block_table"), _i32(kv_lens, "kv_lens")
    cu_q = _i32(cu_q, "cu_q")
    B = block_table.shape[0]
    if cu_q.shape != (B + 1,):
        raise ValueError(f"cu_q must be [{B + 1}] (one offset per sequence, then the total)")
    out = torch.empty_like(q)
    with torch.cuda.device(q.device):
        rc = _lib.load().mlxq_paged_attention_prefill(
            _p(q.contiguous()), _p(cu_q), int(max_q_len), _p(k_cache), _p(v_cache),
            _p(block_table), block_table.shape[1], _p(kv_lens), _p(out), B, H, hkv, hd, page,
            float(scale), dt, _stream(q.device))
    _lib.check(rc, "paged_attention_prefill")
    return out


def quantized_embedding(ids: torch.Tensor, wq: torch.Tensor, scales: torch.Tensor,
                        biases: torch.Tensor, group_size: int = 64, bits: int = 4,
                        out: torch.Tensor | None = None) -> torch.Tensor:
    """Rows ids of a quantized table, dequantized (QuantizedEmbedding lookup):
    bit-identical to dequantize() of those rows; [..., dim]."""
    dt = _code(scales, "scales")
    ids = _i32(ids, "ids")
    vocab, dim = wq.shape[0], scales.shape[-1] * group_size
    if wq.ndim != 2 or wq.shape[1] * 32 // bits != dim or scales.shape != biases.shape or \
            scales.shape[0] != vocab:
        raise ValueError("wq [vocab, dim*bits/32], scales/biases [vocab, dim/group_size] expected")
    flat = ids.reshape(-1)
    if out is None:
        out = torch.empty(*ids.shape, dim, dtype=scales.dtype, device=wq.device)
    with torch.cuda.device(wq.device):
        rc = _lib.load().mlxq_quantized_embedding(_p(flat), flat.numel(), _p(wq), _p(scales),
                                                  _p(biases), _p(out), vocab, dim, group_size,
                                                  bits, dt, _stream(wq.device))
    _lib.check(rc, "quantized_embedding")
    return out


def decode_advance(positions: torch.Tensor, kv_lens: torch.Tensor, slots: torch.Tensor,
                   block_table: torch.Tensor, page_size: int) -> None:
    """In place on the device: every sequence one token further (positions += 1,
    kv_lens = positions + 1, slots = the new position's cache row)."""
    with torch.cuda.device(positions.device):
        rc = _lib.load().mlxq_decode_advance(_p(positions), _p(kv_lens), _p(slots),
                                             _p(block_table), block_table.shape[1],
                                             positions.numel(), page_size,
                                             _stream(positions.device))
    _lib.check(rc, "decode_advance")


@dataclass
class PagedBatch:
    """Where one forward step's tokens go (the reference's ForwardBatch and
    PagedBatchReservation, interfaces.py:95-109, cache.py:420-520): per new token its
    position and cache slot; per sequence its page ids, cached length after the
    append, and (prefill) the offsets of its tokens in the flat batch."""
    block_table: torch.Tensor      # [B, max_blocks] int32
    kv_lens: torch.Tensor          # [B] int32, keys cached after this step
    positions: torch.Tensor        # [T] int32
    slots: torch.Tensor            # [T] int32
    max_kv_len: int
    cu_q: torch.Tensor | None = None   # [B + 1] int32 (prefill); None = one token each
    max_q_len: int = 1


class PagedKVCache:
    """Fixed-size page pools per layer, [num_pages, page_size, n_kv_heads, head_dim]
    for keys and for values (cache.py:651-700), and a free list of page ids handed
    out to sequences in any order (the pages of a sequence need not be contiguous)."""

    def __init__(self, num_layers: int, n_kv_heads: int, head_dim: int, num_pages: int,
                 page_size: int = 16, dtype=torch.bfloat16, device="cuda"):
        if page_size not in (8, 16, 32):
            raise ValueError("page_size must be 8, 16 or 32")
        self.page_size, self.n_kv_heads, self.head_dim = page_size, n_kv_heads, head_dim
        shape = (num_pages, page_size, n_kv_heads, head_dim)
        self.keys = [torch.zeros(shape, dtype=dtype, device=device) for _ in range(num_layers)]
        self.values = [torch.zeros(shape, dtype=dtype, device=device) for _ in range(num_layers)]
        self._free = list(range(num_pages))
        self._lock = threading.Lock()

    @property
    def num_free_pages(self) -> int:
        return len(self._free)

    def allocate(self, lengths, generator=None) -> torch.Tensor:
        """Pages for sequences of the given maximum lengths: block table [B, max_blocks]
        int32 (unused entries 0). With a generator the free pages are handed out in
        a shuffled order."""
        blocks = [math.ceil(n / self.page_size) for n in lengths]
        with self._lock:
            if sum(blocks) > len(self._free):
                raise RuntimeError(f"KV cache full: {sum(blocks)} pages asked, "
                                   f"{len(self._free)} free")
            if generator is not None:
                perm = torch.randperm(len(self._free), generator=generator).tolist()
                self._free = [self._free[i] for i in perm]
            table = torch.zeros(len(lengths), max(1, max(blocks, default=1)), dtype=torch.int32)
            for b, nb in enumerate(blocks):
                for j in range(nb):
                    table[b, j] = self._free.pop()
        return table.to(self.keys[0].device)

    def release(self, block_table: torch.Tensor, lengths) -> None:
        with self._lock:
            for b, n in enumerate(lengths):
                self._free.extend(block_table[b, :math.ceil(n / self.page_size)].tolist())

    def slots(self, block_table: torch.Tensor, positions_per_seq) -> torch.Tensor:
        """Cache rows of the given positions of each sequence (host-computed), int32."""
        bt = block_table.cpu()
        out = []
        for b, poss in enumerate(positions_per_seq):
            for p in poss:
                out.append(int(bt[b, p // self.page_size]) * self.page_size + p % self.page_size)
        return torch.tensor(out, dtype=torch.int32, device=block_table.device)
