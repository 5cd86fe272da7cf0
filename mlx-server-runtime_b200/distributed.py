"""Multi-GPU forms of the quantized matmul path (one process per GPU).

Neither form exists in the reference (it runs one process on one Apple GPU); they
are how the path shards on a B200 box:

  * ShardedQuantizedLinear: a QuantizedLinear split by output rows (N). Rank r
    keeps rows [r*P, (r+1)*P) of the packed weight, scales and biases (P =
    ceil(N / world)); a forward is the local quantized_matmul followed by one
    all-gather of the outputs along N. x is replicated.
  * ExpertParallelSwitchGLU: a SwitchGLU (lfm2.py:193-218) whose experts are
    split across ranks (E / world each). Each rank routes its own tokens, sends
    every (token, expert) row to the rank owning the expert (an all-to-all of
    hidden rows after an all-to-all of counts), runs its local experts with
    gather_qmm, and sends the results back with the reverse all-to-all.

Collectives go through torch.distributed (NCCL on GPUs). The per-rank compute
is an injectable callable so the host logic runs under gloo on CPU in tests;
by default it is this package's CUDA operators.
"""
from __future__ import annotations

from typing import Callable

import torch
import torch.distributed as dist

from . import core

__all__ = ["shard_rows", "ShardedQuantizedLinear", "ExpertParallelSwitchGLU"]


def shard_rows(n: int, world: int, rank: int) -> tuple[int, int]:
    """[lo, hi) of the rows rank `rank` owns when n rows are split in ceil(n/world) blocks."""
    per = (n + world - 1) // world
    lo = min(n, rank * per)
    return lo, min(n, lo + per)


def _default_qmm(x, w, s, b, group_size, bits, bias=None):
    return core.quantized_matmul(x, w, s, b, group_size=group_size, bits=bits, bias=bias)


class ShardedQuantizedLinear:
    def __init__(self, weight, scales, biases, bias=None, *, out_features: int, group_size=64,
                 bits=4, group=None, local_qmm: Callable | None = None):
        self.weight, self.scales, self.biases, self.bias = weight, scales, biases, bias
        self.out_features = out_features
        self.group_size, self.bits = group_size, bits
        self.group = group
        self.local_qmm = local_qmm or _default_qmm
        self.world = dist.get_world_size(group)
        self.per = (out_features + self.world - 1) // self.world

    @classmethod
    def from_full(cls, weight, scales, biases, bias=None, *, group_size=64, bits=4, group=None,
                  local_qmm=None):
        """Slice this rank's rows out of full (unsharded) tensors."""
        world, rank = dist.get_world_size(group), dist.get_rank(group)
        n = weight.shape[0]
        lo, hi = shard_rows(n, world, rank)
        sl = slice(lo, hi)
        return cls(weight[sl].contiguous(), scales[sl].contiguous(), biases[sl].contiguous(),
                   None if bias is None else bias[sl].contiguous(), out_features=n,
                   group_size=group_size, bits=bits, group=group, local_qmm=local_qmm)

    def __call__(self, x: torch.Tensor) -> torch.Tensor:
        lead = x.shape[:-1]
        x2 = x.reshape(-1, x.shape[-1])
        m = x2.shape[0]
        # every rank contributes `per` columns (the last shard is zero-padded; a rank
        # past the end of N owns no rows and sends zeros only)
        padded = x2.new_zeros(m, self.per)
        if self.weight.shape[0]:
            local = self.local_qmm(x2, self.weight, self.scales, self.biases, self.group_size,
                                   self.bits, self.bias)
            padded[:, :local.shape[1]] = local
        gathered = [torch.empty_like(padded) for _ in range(self.world)]
        dist.all_gather(gathered, padded.contiguous(), group=self.group)
        out = torch.cat(gathered, dim=1)[:, :self.out_features]
        return out.reshape(*lead, self.out_features)


def _default_gather(x, w, s, b, rhs, group_size, bits, sorted_indices):
    return core.gather_qmm(x, w, s, b, rhs_indices=rhs, group_size=group_size, bits=bits,
                           sorted_indices=sorted_indices)


class ExpertParallelSwitchGLU:
    """SwitchGLU with experts split across ranks; rank r owns experts
    [r*E_local, (r+1)*E_local). `gate`, `up`, `down` are this rank's (w_q,
    scales, biases) triples with a leading local-expert dimension."""

    def __init__(self, gate, up, down, *, num_experts: int, group_size=64, bits=4, group=None,
                 local_gather: Callable | None = None, act: Callable | None = None,
                 capacity: int | None = None):
        self.gate, self.up, self.down = gate, up, down
        self.num_experts = num_experts
        self.group_size, self.bits = group_size, bits
        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        if num_experts % self.world:
            raise ValueError(f"{num_experts} experts do not split over {self.world} ranks")
        self.e_local = num_experts // self.world
        self.local_gather = local_gather or _default_gather
        self.act = act or (lambda g, u: torch.nn.functional.silu(g) * u)
        if capacity is not None and capacity < 1:
            raise ValueError(f"capacity={capacity} must be >= 1 routed rows")
        self.capacity = capacity

    def __call__(self, x: torch.Tensor, indices: torch.Tensor) -> torch.Tensor:
        """x [T, D], indices [T, k] (global expert ids) -> [T, k, D] expert outputs.

        With a `capacity` (routed rows per rank, the same on every rank; decode sizes)
        every rank sends every rank a buffer of `capacity` rows, so the split sizes
        are fixed: the call reads nothing back to the host and can be captured in a
        CUDA graph, at the cost of sending world x capacity rows. Without one, the
        ranks exchange their per-destination counts first (read back to the host) and
        send only the routed rows. Every rank must use the same form."""
        T, D = x.shape
        k = indices.shape[1]
        if self.capacity is not None:
            if T * k > self.capacity:
                raise ValueError(f"{T * k} routed rows exceed the capacity {self.capacity}")
            return self._call_fixed(x, indices)
        k = indices.shape[1]
        flat = indices.reshape(-1).to(torch.int64)
        dest = flat // self.e_local                              # owning rank per row
        order = torch.argsort(dest * self.num_experts + flat, stable=True)
        send_rows = x[order // k]                                # [T*k, D], grouped by rank
        send_experts = flat[order]
        send_counts = torch.bincount(dest, minlength=self.world)
        recv_counts = torch.empty_like(send_counts)
        dist.all_to_all_single(recv_counts, send_counts, group=self.group)
        sc, rc = send_counts.tolist(), recv_counts.tolist()
        recv_rows = x.new_empty(sum(rc), D)
        dist.all_to_all_single(recv_rows, send_rows.contiguous(), rc, sc, group=self.group)
        recv_exp = flat.new_empty(sum(rc))
        dist.all_to_all_single(recv_exp, send_experts.contiguous(), rc, sc, group=self.group)

        # local experts on the received rows, sorted by expert
        local_e = (recv_exp - self.rank * self.e_local)
        lorder = torch.argsort(local_e, stable=True)
        rows = recv_rows[lorder].unsqueeze(1)                     # [R, 1, D]
        sel = local_e[lorder].to(torch.int32)
        if rows.shape[0]:
            y = self._local_experts(rows, sel)
        else:
            y = x.new_empty(0, D)
        back = torch.empty_like(y)
        back[lorder] = y
        # reverse all-to-all, then undo the send permutation
        out_rows = x.new_empty(T * k, D)
        dist.all_to_all_single(out_rows, back.contiguous(), sc, rc, group=self.group)
        out = torch.empty_like(out_rows)
        out[order] = out_rows
        return out.reshape(T, k, D)

    def _local_experts(self, rows, sel):
        """The rank's experts on rows [R, D] sorted by local expert sel (entries with
        sel < 0 first: padding, which the gathers leave unwritten)."""
        g = self.local_gather(rows, *self.gate, sel, self.group_size, self.bits, True)
        u = self.local_gather(rows, *self.up, sel, self.group_size, self.bits, True)
        h = self.act(g, u)
        y = self.local_gather(h, *self.down, sel, self.group_size, self.bits, True)
        return y.reshape(rows.shape[0], -1)

    def _call_fixed(self, x, indices):
        T, D = x.shape
        k = indices.shape[1]
        W, C = self.world, self.capacity
        dev = x.device
        flat = indices.reshape(-1).to(torch.int64)
        dest = flat // self.e_local
        order = torch.argsort(dest * self.num_experts + flat, stable=True)
        # slot of each routed row in the [W, C] send buffer: its destination's block,
        # then its place among the rows for that destination (scatter_add: no host sync)
        counts = torch.zeros(W, dtype=torch.int64, device=dev).scatter_add_(
            0, dest, torch.ones_like(dest))
        starts = torch.cumsum(counts, 0) - counts
        sdest = dest[order]
        slot = sdest * C + (torch.arange(T * k, device=dev) - starts[sdest])
        send = x.new_zeros(W * C, D)
        send[slot] = x[order // k]
        send_e = torch.full((W * C,), -1, dtype=torch.int64, device=dev)
        send_e[slot] = flat[order]
        recv = torch.empty_like(send)
        dist.all_to_all_single(recv, send, group=self.group)
        recv_e = torch.empty_like(send_e)
        dist.all_to_all_single(recv_e, send_e, group=self.group)
        local_e = torch.where(recv_e >= 0, recv_e - self.rank * self.e_local,
                              torch.full_like(recv_e, -1))
        lorder = torch.argsort(local_e, stable=True)
        y = self._local_experts(recv[lorder].unsqueeze(1), local_e[lorder].to(torch.int32))
        back = torch.empty_like(y)
        back[lorder] = y
        ret = torch.empty_like(back)
        dist.all_to_all_single(ret, back, group=self.group)
        out = torch.empty(T * k, D, dtype=x.dtype, device=dev)
        out[order] = ret[slot]
        return out.reshape(T, k, D)
