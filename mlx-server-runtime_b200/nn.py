"""MLX-style quantized modules over the B200 operators.

The reference's model graphs swap dense layers for quantized twins through a
module protocol (reference tree, python/mlx_worker/native_mlx/models/):
  * ``to_quantized(group_size, bits, mode)`` on a layer returns its quantized
    twin (``SwitchLinear.to_quantized``, lfm2.py:97-121);
  * ``quantize(model, group_size, bits, mode, class_predicate)`` walks the
    module tree and replaces every layer the predicate accepts; the predicate
    may return a per-layer dict of quantization parameters (qwen2.py:315-323,
    lfm2.py:579-591).
The classes here follow that protocol with the same constructor arguments
and call signatures, so a graph written like qwen2.py / lfm2.py runs on them
unchanged; parameters are torch CUDA tensors.
"""
from __future__ import annotations

import math
from typing import Any, Callable, Iterator

import torch

from . import core

__all__ = [
    "Module", "Linear", "QuantizedLinear", "FusedQuantizedLinear", "FusedGateUp", "Embedding",
    "QuantizedEmbedding", "SwitchLinear", "QuantizedSwitchLinear", "SwitchGLU", "MoEBlock",
    "route_topk", "quantize", "silu",
]


def silu(x: torch.Tensor) -> torch.Tensor:
    return torch.nn.functional.silu(x)


class Module:
    """Minimal module tree: child modules are attributes (or lists of them)."""

    def children(self) -> Iterator[tuple[str, Any]]:
        for name, v in vars(self).items():
            if isinstance(v, Module):
                yield name, v
            elif isinstance(v, (list, tuple)):
                for i, m in enumerate(v):
                    if isinstance(m, Module):
                        yield f"{name}.{i}", m

    def named_modules(self, prefix: str = "") -> Iterator[tuple[str, "Module"]]:
        yield prefix, self
        for name, child in self.children():
            yield from child.named_modules(f"{prefix}.{name}" if prefix else name)

    def _set_child(self, name: str, value: "Module") -> None:
        if "." in name:
            attr, idx = name.split(".", 1)
            getattr(self, attr)[int(idx)] = value
        else:
            setattr(self, name, value)

    def __call__(self, *a, **k):  # pragma: no cover - subclasses define the call
        raise NotImplementedError


def _uniform(shape, scale, device, dtype, generator=None):
    t = torch.empty(*shape, device=device, dtype=torch.float32)
    t.uniform_(-scale, scale, generator=generator)
    return t.to(dtype)


class Linear(Module):
    """Dense linear layer y = x W^T (+ b), convertible with to_quantized."""

    def __init__(self, input_dims: int, output_dims: int, bias: bool = True, *,
                 device="cuda", dtype=torch.bfloat16, generator=None):
        scale = math.sqrt(1.0 / input_dims)
        self.weight = _uniform((output_dims, input_dims), scale, device, dtype, generator)
        if bias:
            self.bias = torch.zeros(output_dims, device=device, dtype=dtype)

    def __call__(self, x):
        y = x @ self.weight.t()
        return y + self.bias if hasattr(self, "bias") else y

    def to_quantized(self, group_size: int = 64, bits: int = 4, mode: str = "affine"):
        return QuantizedLinear.from_linear(self, group_size, bits, mode)


class QuantizedLinear(Module):
    """Linear layer over packed affine-quantized weights (MLX QuantizedLinear).

    Called for every projection of the reference graphs: q/k/v/o
    (qwen2.py:58-61, q/k/v with bias), gate/up/down (qwen2.py:123-134) and
    the untied lm_head (qwen2.py:227). The bias add is fused into the same
    kernel launch.
    """

    def __init__(self, input_dims: int, output_dims: int, bias: bool = True,
                 group_size: int = 64, bits: int = 4, mode: str = "affine", *,
                 device="cuda", dtype=torch.bfloat16, generator=None):
        self.group_size, self.bits, self.mode = group_size, bits, mode
        scale = math.sqrt(1.0 / input_dims)
        w = _uniform((output_dims, input_dims), scale, device, dtype, generator)
        self.weight, self.scales, self.biases = core.quantize(w, group_size, bits, mode)
        if bias:
            self.bias = torch.zeros(output_dims, device=device, dtype=dtype)

    @classmethod
    def from_linear(cls, linear: Linear, group_size: int = 64, bits: int = 4,
                    mode: str = "affine") -> "QuantizedLinear":
        q = cls.__new__(cls)
        q.group_size, q.bits, q.mode = group_size, bits, mode
        q.weight, q.scales, q.biases = core.quantize(linear.weight, group_size, bits, mode)
        if hasattr(linear, "bias"):
            q.bias = linear.bias
        return q

    @property
    def input_dims(self) -> int:
        return self.scales.shape[-1] * self.group_size

    @property
    def output_dims(self) -> int:
        return self.weight.shape[0]

    def __call__(self, x):
        return core.quantized_matmul(x, self.weight, self.scales, self.biases, transpose=True,
                                     group_size=self.group_size, bits=self.bits, mode=self.mode,
                                     bias=getattr(self, "bias", None))

    def greedy_tokens(self, x):
        """argmax over this layer's outputs (an lm_head's greedy next token), int32,
        without writing the logits at decode (core.quantized_matmul_argmax)."""
        return core.quantized_matmul_argmax(x, self.weight, self.scales, self.biases,
                                            self.group_size, self.bits, self.mode,
                                            bias=getattr(self, "bias", None))


class FusedQuantizedLinear(Module):
    """QuantizedLinear layers that read the same input, computed in one launch.

    A decoder layer's q/k/v projections (qwen2.py:58-60, with bias) and its
    gate/up projections (qwen2.py:133-134) each take the same activations; their
    packed weights, scales, biases (and bias, zeros for a part without one) are
    stacked along the output features once, and a call returns one output per
    part, split from a single quantized_matmul. Each part's outputs equal its
    own layer's up to the fp32 summation order.
    """

    def __init__(self, layers):
        layers = list(layers)
        if not layers or not all(isinstance(m, QuantizedLinear) for m in layers):
            raise ValueError("FusedQuantizedLinear takes one or more QuantizedLinear layers")
        q0 = layers[0]
        for m in layers:
            if (m.group_size, m.bits, m.mode) != (q0.group_size, q0.bits, q0.mode):
                raise ValueError("fused layers must share group_size, bits and mode")
            if m.input_dims != q0.input_dims:
                raise ValueError("fused layers must share input_dims")
        self.group_size, self.bits, self.mode = q0.group_size, q0.bits, q0.mode
        self.weight, self.scales, self.biases = core.concat_quantized(
            [(m.weight, m.scales, m.biases) for m in layers], q0.group_size, q0.bits)
        self.splits = [m.output_dims for m in layers]
        if any(hasattr(m, "bias") for m in layers):
            self.bias = torch.cat([
                m.bias if hasattr(m, "bias") else
                torch.zeros(m.output_dims, dtype=q0.scales.dtype, device=q0.scales.device)
                for m in layers])

    @property
    def input_dims(self) -> int:
        return self.scales.shape[-1] * self.group_size

    @property
    def output_dims(self) -> int:
        return self.weight.shape[0]

    def __call__(self, x):
        y = core.quantized_matmul(x, self.weight, self.scales, self.biases, transpose=True,
                                  group_size=self.group_size, bits=self.bits, mode=self.mode,
                                  bias=getattr(self, "bias", None))
        return tuple(torch.split(y, self.splits, dim=-1))


class FusedGateUp(Module):
    """silu(gate_proj(x)) * up_proj(x) of a SwiGLU MLP (qwen2.py:133-134,
    lfm2.py:212) from two bias-free QuantizedLinear layers, in one launch at decode:
    their rows are interleaved once (core.interleave_gate_up) and the activation
    runs in the matmul's epilogue (core.quantized_matmul_swiglu)."""

    def __init__(self, gate: "QuantizedLinear", up: "QuantizedLinear"):
        if not isinstance(gate, QuantizedLinear) or not isinstance(up, QuantizedLinear):
            raise ValueError("FusedGateUp takes two QuantizedLinear layers")
        if hasattr(gate, "bias") or hasattr(up, "bias"):
            raise ValueError("FusedGateUp takes layers without bias")
        if (gate.group_size, gate.bits, gate.mode) != (up.group_size, up.bits, up.mode):
            raise ValueError("gate and up must share group_size, bits and mode")
        self.group_size, self.bits, self.mode = gate.group_size, gate.bits, gate.mode
        self.weight, self.scales, self.biases = core.interleave_gate_up(
            (gate.weight, gate.scales, gate.biases), (up.weight, up.scales, up.biases),
            gate.group_size, gate.bits)

    def __call__(self, x):
        return core.quantized_matmul_swiglu(x, self.weight, self.scales, self.biases,
                                            self.group_size, self.bits, self.mode)


class Embedding(Module):
    def __init__(self, num_embeddings: int, dims: int, *, device="cuda", dtype=torch.bfloat16,
                 generator=None):
        scale = math.sqrt(1.0 / dims)
        self.weight = _uniform((num_embeddings, dims), scale, device, dtype, generator)

    def __call__(self, ids):
        return self.weight[ids]

    def as_linear(self, x):
        return x @ self.weight.t()

    def to_quantized(self, group_size: int = 64, bits: int = 4, mode: str = "affine"):
        return QuantizedEmbedding.from_embedding(self, group_size, bits, mode)


class QuantizedEmbedding(Module):
    """Quantized embedding table; ``as_linear`` is the tied vocabulary head
    (qwen2.py:225-226, lfm2.py:457)."""

    @classmethod
    def from_embedding(cls, emb: Embedding, group_size=64, bits=4, mode="affine"):
        q = cls.__new__(cls)
        q.group_size, q.bits, q.mode = group_size, bits, mode
        q.weight, q.scales, q.biases = core.quantize(emb.weight, group_size, bits, mode)
        return q

    def __call__(self, ids):
        flat = ids.reshape(-1)
        # (torch gathers no uint32 rows on CUDA: gather the packed words as int32)
        wq = self.weight.view(torch.int32)[flat].view(torch.uint32)
        rows = core.dequantize(wq, self.scales[flat], self.biases[flat],
                               self.group_size, self.bits, self.mode)
        return rows.reshape(*ids.shape, rows.shape[-1])

    def as_linear(self, x):
        return core.quantized_matmul(x, self.weight, self.scales, self.biases, True,
                                     self.group_size, self.bits, self.mode)

    def greedy_tokens(self, x):
        """argmax of as_linear(x) per row (tied-head greedy decoding), int32."""
        return core.quantized_matmul_argmax(x, self.weight, self.scales, self.biases,
                                            self.group_size, self.bits, self.mode)


class SwitchLinear(Module):
    """Expert-indexed dense linear layer (lfm2.py:59-121)."""

    def __init__(self, input_dims: int, output_dims: int, num_experts: int, *, bias=False,
                 device="cuda", dtype=torch.bfloat16, generator=None):
        scale = math.sqrt(1.0 / input_dims)
        self.weight = _uniform((num_experts, output_dims, input_dims), scale, device, dtype,
                               generator)
        if bias:
            self.bias = torch.zeros(num_experts, output_dims, device=device, dtype=dtype)

    def to_quantized(self, group_size: int = 64, bits: int = 4, mode: str = "affine"):
        q = QuantizedSwitchLinear.__new__(QuantizedSwitchLinear)
        q.group_size, q.bits, q.mode = group_size, bits, mode
        q.weight, q.scales, q.biases = core.quantize(self.weight, group_size, bits, mode)
        if hasattr(self, "bias"):
            q.bias = self.bias
        return q


class QuantizedSwitchLinear(Module):
    """Quantized expert bank: gather_qmm over rows routed to experts (lfm2.py:124-190)."""

    def __init__(self, input_dims: int, output_dims: int, num_experts: int, *, bias: bool,
                 group_size: int, bits: int, mode: str, device="cuda", dtype=torch.bfloat16,
                 generator=None):
        self.group_size, self.bits, self.mode = group_size, bits, mode
        scale = math.sqrt(1.0 / input_dims)
        w = _uniform((num_experts, output_dims, input_dims), scale, device, dtype, generator)
        self.weight, self.scales, self.biases = core.quantize(w, group_size, bits, mode)
        if bias:
            self.bias = torch.zeros(num_experts, output_dims, device=device, dtype=dtype)

    @property
    def input_dims(self) -> int:
        return self.scales.shape[-1] * self.group_size

    @property
    def output_dims(self) -> int:
        return self.weight.shape[1]

    @property
    def num_experts(self) -> int:
        return self.weight.shape[0]

    def __call__(self, x, indices, *, sorted_indices: bool = False):
        out = core.gather_qmm(x, self.weight, self.scales, self.biases, rhs_indices=indices,
                              transpose=True, group_size=self.group_size, bits=self.bits,
                              mode=self.mode, sorted_indices=sorted_indices)
        if hasattr(self, "bias"):
            out = out + self.bias[indices].unsqueeze(-2)
        return out


def _gather_sort(x, indices, num_experts=None):
    """Rows sorted by expert (lfm2.py:613-618): the rows of x for the routing entries
    in expert order (stable), the sorted indices and the inverse permutation. With the
    expert count known and at most 16384 entries, one device kernel (core.moe_sort)
    gives both permutations; otherwise torch's stable argsort."""
    width = indices.shape[-1]
    flat = indices.reshape(-1)
    xs = x.reshape(-1, *x.shape[-2:])
    if num_experts is not None and 0 < flat.numel() <= 16384 and num_experts <= 1024:
        order, srt, inverse = core.moe_sort(flat.to(torch.int32), num_experts)
        rows = torch.div(order, width, rounding_mode="floor")
        return xs.index_select(0, rows), srt, inverse
    order = torch.argsort(flat, stable=True)
    inverse = torch.argsort(order)
    return xs[order // width], flat[order], inverse


def _scatter_unsort(x, inverse, shape):
    """Inverse of _gather_sort (lfm2.py:621-622)."""
    return x.index_select(0, inverse).reshape(*shape, *x.shape[1:])


class FusedSwitchGateUp(Module):
    """An expert bank's gate and up projections in interleave_gate_up's layout (each
    expert's rows interleaved by 16-row tiles): silu(gate) * up per routed entry from
    one gather_qmm_swiglu call (one launch at decode sizes)."""

    def __init__(self, weight, scales, biases, group_size: int, bits: int, mode: str):
        self.weight, self.scales, self.biases = weight, scales, biases
        self.group_size, self.bits, self.mode = group_size, bits, mode

    @classmethod
    def from_pair(cls, gate: "QuantizedSwitchLinear", up: "QuantizedSwitchLinear"):
        for a in (gate, up):
            if not isinstance(a, QuantizedSwitchLinear) or hasattr(a, "bias"):
                raise ValueError("gate and up must be quantized expert banks without bias")
        if (gate.group_size, gate.bits, gate.mode) != (up.group_size, up.bits, up.mode):
            raise ValueError("gate and up must share group_size, bits and mode")
        w, s, b = core.interleave_gate_up((gate.weight, gate.scales, gate.biases),
                                          (up.weight, up.scales, up.biases),
                                          gate.group_size, gate.bits)
        return cls(w, s, b, gate.group_size, gate.bits, gate.mode)

    @property
    def num_experts(self) -> int:
        return self.weight.shape[0]

    def __call__(self, x, indices, *, sorted_indices: bool = False):
        return core.gather_qmm_swiglu(x, self.weight, self.scales, self.biases,
                                      rhs_indices=indices, group_size=self.group_size,
                                      bits=self.bits, mode=self.mode,
                                      sorted_indices=sorted_indices)


class SwitchGLU(Module):
    """SwiGLU expert bank with top-k routing (lfm2.py:193-218)."""

    def __init__(self, input_dims: int, hidden_dims: int, num_experts: int, **kw):
        self.gate_proj = SwitchLinear(input_dims, hidden_dims, num_experts, **kw)
        self.up_proj = SwitchLinear(input_dims, hidden_dims, num_experts, **kw)
        self.down_proj = SwitchLinear(hidden_dims, input_dims, num_experts, **kw)

    def fuse_gate_up(self) -> None:
        """Replace the quantized gate_proj and up_proj by one FusedSwitchGateUp (rows
        copied bit for bit, no extra memory kept): up, gate and the activation then run
        as one launch at decode sizes."""
        self.gate_up_proj = FusedSwitchGateUp.from_pair(self.gate_proj, self.up_proj)
        del self.gate_proj, self.up_proj

    def __call__(self, x, indices):
        x = x.unsqueeze(-2).unsqueeze(-3)
        do_sort = indices.numel() >= 64
        selected, inverse = indices, None
        fused = getattr(self, "gate_up_proj", None)
        if do_sort:
            experts = (fused or self.gate_proj).weight.shape[0]
            x, selected, inverse = _gather_sort(x, indices, experts)
        if fused is not None:
            act = fused(x, selected, sorted_indices=do_sort)
        else:
            up = self.up_proj(x, selected, sorted_indices=do_sort)
            gate = self.gate_proj(x, selected, sorted_indices=do_sort)
            act = silu(gate) * up
        out = self.down_proj(act, selected, sorted_indices=do_sort)
        if do_sort:
            out = _scatter_unsort(out, inverse, indices.shape)
        return out.squeeze(-2)


def route_topk(logits: torch.Tensor, top_k: int, norm_topk_prob: bool = True,
               expert_bias: torch.Tensor | None = None):
    """Top-k expert routing of an MoE layer (lfm2.py:366-373 of the reference), one
    device kernel (core.moe_route): softmax over the experts in float32, plus the
    optional per-expert bias, the top_k experts per token (their order is not part of
    the contract: the reference takes an argpartition), their gate values,
    renormalised to sum to one when `norm_topk_prob` (with the reference's 1e-20
    guard), cast back to the logits' dtype. Returns (indices [.., top_k] int32,
    scores [.., top_k])."""
    return core.moe_route(logits, top_k, norm_topk_prob, expert_bias)


class MoEBlock(Module):
    """Sparse MoE feed-forward (lfm2.py:345-375): a dense router, top-k routing,
    the SwitchGLU expert bank (gather_qmm), outputs weighted by the gate scores
    and summed over the k experts."""

    def __init__(self, hidden: int, moe_inter: int, num_experts: int, top_k: int, *,
                 norm_topk_prob: bool = True, use_expert_bias: bool = False, device="cuda",
                 dtype=torch.bfloat16, generator=None):
        self.top_k, self.norm_topk_prob = top_k, norm_topk_prob
        self.gate = Linear(hidden, num_experts, bias=False, device=device, dtype=dtype,
                           generator=generator)
        self.switch_mlp = SwitchGLU(hidden, moe_inter, num_experts, device=device, dtype=dtype,
                                    generator=generator)
        if use_expert_bias:
            self.expert_bias = torch.zeros(num_experts, device=device, dtype=torch.float32)

    def __call__(self, x):
        indices, scores = route_topk(self.gate(x), self.top_k, self.norm_topk_prob,
                                     getattr(self, "expert_bias", None))
        y = self.switch_mlp(x, indices)
        return (y * scores.unsqueeze(-1)).sum(dim=-2)


def quantize(model: Module, group_size: int = 64, bits: int = 4, mode: str = "affine",
             class_predicate: Callable[[str, Module], bool | dict] | None = None) -> None:
    """Replace, in place, every layer that has ``to_quantized`` and that the
    predicate accepts; a dict returned by the predicate overrides
    group_size/bits/mode for that layer (MLX nn.quantize)."""
    pred = class_predicate or (lambda path, m: hasattr(m, "to_quantized"))
    replacements = []
    for path, m in model.named_modules():
        if not path or not hasattr(m, "to_quantized"):
            continue
        verdict = pred(path, m)
        if verdict is False or verdict is None:
            continue
        params = dict(group_size=group_size, bits=bits, mode=mode)
        if isinstance(verdict, dict):
            params.update(verdict)
        replacements.append((path, m.to_quantized(**params)))
    for path, q in replacements:
        parent_path, _, leaf = path.rpartition(".")
        parent = model
        if parent_path:
            for part in parent_path.split("."):
                parent = getattr(parent, part) if not part.isdigit() else parent[int(part)]
        if leaf.isdigit():
            parent[int(leaf)] = q
        else:
            setattr(parent, leaf, q)
