"""MLX-named quantized operators over torch CUDA tensors.

Mirrors the MLX operator surface the reference's model graphs call
(mlx 0.31.2, python/uv.lock:939-940 of the reference):

  quantize(w, group_size=64, bits=4, mode="affine") -> (w_q, scales, biases)
      mx.quantize, reference call sites lfm2.py:112-117,142-151
  dequantize(w_q, scales, biases, group_size=64, bits=4, mode="affine")
      mx.dequantize (north_star API)
  quantized_matmul(x, w, scales, biases, transpose=True, group_size=64, bits=4, mode="affine")
      mx.quantized_matmul via nn.QuantizedLinear, qwen2.py:58-61,123-134,227
  gather_qmm(x, w, scales, biases, lhs_indices=None, rhs_indices=None, transpose=True,
             group_size=64, bits=4, mode="affine", sorted_indices=False)
      mx.gather_qmm via QuantizedSwitchLinear, lfm2.py:176-187

Torch tensors are only device buffers here: every operator is one call into
libmlxq_b200.so on the tensor's device and current stream. Misuse raises
ValueError, as MLX does; device failures raise RuntimeError.
"""
from __future__ import annotations

import math
import threading

import torch

from . import _lib

_DT = {torch.float32: _lib.F32, torch.bfloat16: _lib.BF16, torch.float16: _lib.F16}

__all__ = ["quantize", "dequantize", "quantized_matmul", "gather_qmm", "gather_qmm_swiglu",
           "concat_quantized", "moe_route", "moe_sort",
           "interleave_gate_up", "quantized_matmul_swiglu", "quantized_matmul_argmax",
           "Workspace", "launch_overlap"]


def _dtype_code(t: torch.Tensor, what: str, allowed=(torch.bfloat16, torch.float16)) -> int:
    if t.dtype not in allowed:
        names = ", ".join(str(a).replace("torch.", "") for a in allowed)
        raise ValueError(f"{what} must have dtype in ({names}), got {t.dtype}")
    return _DT[t.dtype]


def _cuda(*ts: torch.Tensor) -> torch.device:
    dev = None
    for t in ts:
        if t is None:
            continue
        if t.device.type != "cuda":
            raise ValueError(f"expected CUDA tensors, got a tensor on {t.device}")
        if dev is None:
            dev = t.device
        elif t.device != dev:
            raise ValueError(f"tensors are on different devices ({dev} and {t.device})")
    return dev


def _mode(mode: str) -> None:
    if mode != "affine":
        raise ValueError(f"mode={mode!r} is not supported (only 'affine')")


def _ptr(t):
    return None if t is None else t.data_ptr()


class Workspace:
    """Per-(device, stream, operator) scratch buffers for the kernels that need them.

    The quantized_matmul workspace holds K-split partial sums and tickets that
    the kernel resets to zero on exit; it is zero-filled once when it is
    (re)allocated and is never shared with another operator (gather_qmm writes
    its expert segment table into its own buffer). Work enqueued on different
    streams never shares a buffer.
    """

    _lock = threading.Lock()
    _bufs: dict = {}

    @classmethod
    def get(cls, device: torch.device, stream: torch.cuda.Stream, nbytes: int,
            kind: str = "qmm") -> torch.Tensor:
        key = (device.index, stream.cuda_stream, kind)
        with cls._lock:
            buf = cls._bufs.get(key)
            if buf is None or buf.numel() < nbytes:
                size = max(nbytes, 1 << 20)
                size = 1 << int(math.ceil(math.log2(size)))
                with torch.cuda.stream(stream):
                    buf = torch.zeros(size, dtype=torch.uint8, device=device)
                cls._bufs[key] = buf
            return buf

    @classmethod
    def clear(cls) -> None:
        with cls._lock:
            cls._bufs.clear()

    @classmethod
    def reset(cls) -> None:
        """Zero-fill every cached buffer on its own stream (after a kernel gave
        up on a bounded wait and may have left tickets nonzero)."""
        with cls._lock:
            for (dev, stream_ptr, _kind), buf in cls._bufs.items():
                st = torch.cuda.ExternalStream(stream_ptr, device=torch.device("cuda", dev))
                with torch.cuda.stream(st):
                    buf.zero_()


class launch_overlap:
    """Context manager (or plain call) enabling launch overlap for quantized_matmul.

    While enabled, each quantized_matmul may begin streaming its packed weights,
    scales and biases before the previous kernel on the stream has finished; it
    waits for that kernel before touching activations or outputs. Use it for
    decode loops over weights that were loaded earlier and are not being written
    by in-flight work.
    """

    def __init__(self, enable: bool = True):
        self._prev = _lib.load().mlxq_set_launch_overlap(int(bool(enable)))

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        _lib.load().mlxq_set_launch_overlap(self._prev)
        return False


def quantize(w: torch.Tensor, group_size: int = 64, bits: int = 4, mode: str = "affine"):
    """Affine group quantization of the last axis: returns (w_q uint32, scales, biases)."""
    _mode(mode)
    dev = _cuda(w)
    dt = _dtype_code(w, "w", (torch.float32, torch.bfloat16, torch.float16))
    if w.ndim < 2:
        raise ValueError(f"quantize expects a matrix (ndim >= 2), got shape {tuple(w.shape)}")
    K = w.shape[-1]
    if bits not in (2, 4, 8):
        raise ValueError(f"bits={bits} is not supported (2, 4 or 8)")
    if group_size not in (32, 64, 128):
        raise ValueError(f"group_size={group_size} is not one of 32, 64, 128")
    if K % group_size:
        raise ValueError(f"the last dimension ({K}) must be divisible by group_size={group_size}")
    w = w.contiguous()
    lead = w.shape[:-1]
    rows = w.numel() // K
    wq = torch.empty(*lead, K * bits // 32, dtype=torch.uint32, device=dev)
    s = torch.empty(*lead, K // group_size, dtype=w.dtype, device=dev)
    b = torch.empty_like(s)
    with torch.cuda.device(dev):
        st = torch.cuda.current_stream(dev)
        rc = _lib.load().mlxq_quantize(_ptr(w), dt, _ptr(wq), _ptr(s), _ptr(b), rows, K,
                                       group_size, bits, st.cuda_stream)
    _lib.check(rc, "quantize")
    return wq, s, b


def dequantize(w: torch.Tensor, scales: torch.Tensor, biases: torch.Tensor, group_size: int = 64,
               bits: int = 4, mode: str = "affine") -> torch.Tensor:
    """w_hat = scale*q + bias in the dtype of scales (one rounding per operation)."""
    _mode(mode)
    dev = _cuda(w, scales, biases)
    if w.dtype != torch.uint32:
        raise ValueError(f"w must be uint32 packed codes, got {w.dtype}")
    dt = _dtype_code(scales, "scales", (torch.float32, torch.bfloat16, torch.float16))
    if biases.dtype != scales.dtype:
        raise ValueError("scales and biases must have the same dtype")
    if bits not in (2, 4, 8):
        raise ValueError(f"bits={bits} is not supported (2, 4 or 8)")
    K = w.shape[-1] * 32 // bits
    if scales.shape != (*w.shape[:-1], K // group_size) or biases.shape != scales.shape:
        raise ValueError(
            f"scales/biases shape {tuple(scales.shape)} does not match w {tuple(w.shape)} "
            f"with group_size={group_size}, bits={bits}")
    w, scales, biases = w.contiguous(), scales.contiguous(), biases.contiguous()
    rows = w.numel() // w.shape[-1]
    out = torch.empty(*w.shape[:-1], K, dtype=scales.dtype, device=dev)
    with torch.cuda.device(dev):
        st = torch.cuda.current_stream(dev)
        rc = _lib.load().mlxq_dequantize(_ptr(w), _ptr(scales), _ptr(biases), dt, _ptr(out),
                                         rows, K, group_size, bits, st.cuda_stream)
    _lib.check(rc, "dequantize")
    return out


def _check_qweights(w, scales, biases, group_size, bits, x_dtype):
    if w.dtype != torch.uint32:
        raise ValueError(f"w must be uint32 packed codes, got {w.dtype}")
    if bits not in (4, 8):
        raise ValueError(f"bits={bits} is not supported by the matmul (4 or 8)")
    if group_size not in (32, 64, 128):
        raise ValueError(f"group_size={group_size} is not one of 32, 64, 128")
    if biases is None:
        raise ValueError("affine quantization requires biases")
    if scales.dtype != x_dtype or biases.dtype != x_dtype:
        raise ValueError(
            f"scales/biases dtype ({scales.dtype}) must match the activations ({x_dtype})")
    K = w.shape[-1] * 32 // bits
    if scales.shape[-1] * group_size != K or scales.shape != biases.shape or \
            scales.shape[:-1] != w.shape[:-1]:
        raise ValueError(
            f"shapes of w {tuple(w.shape)}, scales {tuple(scales.shape)}, biases "
            f"{tuple(biases.shape)} are inconsistent with group_size={group_size}, bits={bits}")
    return K


def quantized_matmul(x: torch.Tensor, w: torch.Tensor, scales: torch.Tensor,
                     biases: torch.Tensor | None = None, transpose: bool = True,
                     group_size: int = 64, bits: int = 4, mode: str = "affine",
                     bias: torch.Tensor | None = None) -> torch.Tensor:
    """x[..., K] @ dequantize(w)^T -> [..., N] (float32 accumulation).

    ``bias`` (not an MLX argument) fuses QuantizedLinear's bias add into the
    same launch; the result equals ``quantized_matmul(...) + bias``.
    """
    _mode(mode)
    if not transpose:
        raise ValueError("transpose=False is not supported; the model graphs use transpose=True")
    dev = _cuda(x, w, scales, biases, bias)
    dt = _dtype_code(x, "x")
    if w.ndim != 2:
        raise ValueError(f"w must be 2-D [N, K*bits/32], got shape {tuple(w.shape)}")
    K = _check_qweights(w, scales, biases, group_size, bits, x.dtype)
    if x.shape[-1] != K:
        raise ValueError(f"x has {x.shape[-1]} features but w expects K={K}")
    N = w.shape[0]
    if bias is not None and (bias.shape != (N,) or bias.dtype != x.dtype):
        raise ValueError(f"bias must be [{N}] of dtype {x.dtype}")
    lead = x.shape[:-1]
    x2 = x.contiguous()
    M = x2.numel() // K
    out = torch.empty(*lead, N, dtype=x.dtype, device=dev)
    if M == 0:
        return out
    L = _lib.load()
    w, scales, biases = w.contiguous(), scales.contiguous(), biases.contiguous()
    with torch.cuda.device(dev):
        st = torch.cuda.current_stream(dev)
        need = L.mlxq_qmm_workspace_size(M, N, K, group_size, bits, dt)
        ws = Workspace.get(dev, st, need) if need else None
        rc = L.mlxq_quantized_matmul(_ptr(x2), _ptr(w), _ptr(scales), _ptr(biases), _ptr(bias),
                                     _ptr(out), M, N, K, group_size, bits, dt, _ptr(ws),
                                     0 if ws is None else ws.numel(), st.cuda_stream)
    _lib.check(rc, "quantized_matmul")
    return out


def concat_quantized(parts, group_size: int = 64, bits: int = 4):
    """Stack quantized matrices that share K, group_size and bits along their
    output features: returns (w, scales, biases) holding every part's rows
    unchanged, in order.

    One quantized_matmul over the result computes the outputs of all parts in a
    single launch; split its last dimension at the parts' N to get each one.
    This is the fused q/k/v and gate/up projection of a decoder layer, whose
    layers read the same input (qwen2.py:58-60,133-134 of the reference). The
    packed words, scales and biases are copied bit for bit, so each part's
    outputs equal its own quantized_matmul up to the fp32 summation order.
    """
    parts = list(parts)
    if not parts:
        raise ValueError("concat_quantized needs at least one (w, scales, biases)")
    w0, s0, b0 = parts[0]
    for w, s, b in parts:
        if w.ndim != 2 or s.ndim != 2 or b.ndim != 2:
            raise ValueError("every part must be 2-D (w [N, K*bits/32], scales/biases [N, K/g])")
        if w.shape[1] != w0.shape[1] or s.shape[1] != s0.shape[1] or b.shape != s.shape:
            raise ValueError("parts must share K, group_size and bits")
        if w.dtype != w0.dtype or s.dtype != s0.dtype or b.dtype != b0.dtype:
            raise ValueError("parts must share dtypes")
        if w.shape[0] != s.shape[0]:
            raise ValueError("w and scales disagree on N")
    _check_qweights(w0, s0, b0, group_size, bits, s0.dtype)
    return (torch.cat([p[0] for p in parts], 0), torch.cat([p[1] for p in parts], 0),
            torch.cat([p[2] for p in parts], 0))


def interleave_gate_up(gate, up, group_size: int = 64, bits: int = 4):
    """The weight layout quantized_matmul_swiglu (2-D, one matrix) and
    gather_qmm_swiglu (3-D, [experts, rows, ...]) read: the (w, scales, biases) of a
    SwiGLU MLP's gate and up projections (same shape [..., I, ...], I a multiple of 8)
    interleaved by 16-row tiles within each matrix, tile j = gate rows 8j..8j+7 then up
    rows 8j..8j+7. Rows are copied bit for bit (a load-time permutation, nothing is
    requantized)."""
    (wg, sg, bg), (wu, su, bu) = gate, up
    for a, c in ((wg, wu), (sg, su), (bg, bu)):
        if a.shape != c.shape or a.dtype != c.dtype or a.ndim not in (2, 3):
            raise ValueError("gate and up must be 2-D (or 3-D expert banks of) quantized "
                             "matrices of the same shape")
    _check_qweights(wg, sg, bg, group_size, bits, sg.dtype)
    lead, inter = tuple(wg.shape[:-2]), wg.shape[-2]
    if inter % 8:
        raise ValueError(f"gate/up rows ({inter}) must be a multiple of 8")

    def mix(a, c):
        return torch.stack([a.reshape(*lead, inter // 8, 8, a.shape[-1]),
                            c.reshape(*lead, inter // 8, 8, c.shape[-1])],
                           dim=-3).reshape(*lead, 2 * inter, a.shape[-1]).contiguous()
    if wg.dtype == torch.uint32:  # (torch has no uint32 stack on every device: move as int32)
        w = mix(wg.view(torch.int32), wu.view(torch.int32)).view(torch.uint32)
    else:
        w = mix(wg, wu)
    return w, mix(sg, su), mix(bg, bu)


def quantized_matmul_swiglu(x: torch.Tensor, w: torch.Tensor, scales: torch.Tensor,
                            biases: torch.Tensor, group_size: int = 64, bits: int = 4,
                            mode: str = "affine") -> torch.Tensor:
    """silu(x @ gate^T) * (x @ up^T) from interleave_gate_up's layout: [..., N/2].

    Decode shapes (up to 16 rows, K/group_size a multiple of 8) and prefill shapes
    (more than 32 rows, K a multiple of 64) run as one launch with the activation in
    the matmul's epilogue; other shapes run quantized_matmul and then the activation
    as torch element-wise ops. Either way each projection is rounded to x's dtype
    before silu(g) * u is formed in float32 and rounded once more.
    """
    _mode(mode)
    dev = _cuda(x, w, scales, biases)
    dt = _dtype_code(x, "x")
    if w.ndim != 2:
        raise ValueError(f"w must be 2-D [N, K*bits/32], got shape {tuple(w.shape)}")
    K = _check_qweights(w, scales, biases, group_size, bits, x.dtype)
    if x.shape[-1] != K:
        raise ValueError(f"x has {x.shape[-1]} features but w expects K={K}")
    N = w.shape[0]
    if N % 16:
        raise ValueError(f"w must hold gate/up 16-row tiles (N={N} is not a multiple of 16)")
    lead = x.shape[:-1]
    x2 = x.contiguous()
    M = x2.numel() // K
    L = _lib.load()
    if M == 0 or not L.mlxq_swiglu_supported(M, N, K, group_size, bits, dt):
        y = quantized_matmul(x, w, scales, biases, True, group_size, bits, mode)
        y = y.reshape(*lead, N // 16, 2, 8).float()
        g, u = y[..., 0, :], y[..., 1, :]
        return (torch.nn.functional.silu(g) * u).to(x.dtype).reshape(*lead, N // 2)
    out = torch.empty(*lead, N // 2, dtype=x.dtype, device=dev)
    w, scales, biases = w.contiguous(), scales.contiguous(), biases.contiguous()
    with torch.cuda.device(dev):
        st = torch.cuda.current_stream(dev)
        need = L.mlxq_qmm_workspace_size(M, N, K, group_size, bits, dt)
        ws = Workspace.get(dev, st, need) if need else None
        rc = L.mlxq_quantized_matmul_swiglu(_ptr(x2), _ptr(w), _ptr(scales), _ptr(biases),
                                            _ptr(out), M, N, K, group_size, bits, dt, _ptr(ws),
                                            0 if ws is None else ws.numel(), st.cuda_stream)
    _lib.check(rc, "quantized_matmul_swiglu")
    return out


def quantized_matmul_argmax(x: torch.Tensor, w: torch.Tensor, scales: torch.Tensor,
                            biases: torch.Tensor, group_size: int = 64, bits: int = 4,
                            mode: str = "affine", bias: torch.Tensor | None = None,
                            out: torch.Tensor | None = None) -> torch.Tensor:
    """Greedy next tokens: argmax over N of quantized_matmul(x, w, ...) (+ bias),
    int32 [...], the first index on ties, without writing the logits.

    Decode shapes (up to 16 rows, K/group_size a multiple of 8) run as one launch
    with the argmax in the matmul's epilogue; other shapes compute the logits and
    take torch.argmax. The logits compared are the ones quantized_matmul returns
    (rounded to x's dtype), so both forms pick the same token. `out` (int32, the
    leading shape of x) receives the ids when given.
    """
    _mode(mode)
    dev = _cuda(x, w, scales, biases, bias)
    dt = _dtype_code(x, "x")
    if w.ndim != 2:
        raise ValueError(f"w must be 2-D [N, K*bits/32], got shape {tuple(w.shape)}")
    K = _check_qweights(w, scales, biases, group_size, bits, x.dtype)
    if x.shape[-1] != K:
        raise ValueError(f"x has {x.shape[-1]} features but w expects K={K}")
    N = w.shape[0]
    if bias is not None and (bias.shape != (N,) or bias.dtype != x.dtype):
        raise ValueError(f"bias must be [{N}] of dtype {x.dtype}")
    lead = x.shape[:-1]
    x2 = x.contiguous()
    M = x2.numel() // K
    L = _lib.load()
    if out is not None and (out.dtype != torch.int32 or out.shape != lead or
                            not out.is_contiguous()):
        raise ValueError(f"out must be a contiguous int32 tensor of shape {tuple(lead)}")
    need = L.mlxq_argmax_workspace_size(M, N, K, group_size, bits, dt) if M else 0
    if need == 0:
        y = quantized_matmul(x, w, scales, biases, True, group_size, bits, mode, bias=bias)
        ids = y.argmax(dim=-1).to(torch.int32)
        if out is not None:
            out.copy_(ids)
            return out
        return ids
    ids = out if out is not None else torch.empty(*lead, dtype=torch.int32, device=dev)
    w, scales, biases = w.contiguous(), scales.contiguous(), biases.contiguous()
    with torch.cuda.device(dev):
        st = torch.cuda.current_stream(dev)
        ws = Workspace.get(dev, st, need)
        rc = L.mlxq_quantized_matmul_argmax(_ptr(x2), _ptr(w), _ptr(scales), _ptr(biases),
                                            _ptr(bias), _ptr(ids), M, N, K, group_size, bits, dt,
                                            _ptr(ws), ws.numel(), st.cuda_stream)
    _lib.check(rc, "quantized_matmul_argmax")
    return ids


def _broadcast_shape(a, b):
    return tuple(torch.broadcast_shapes(torch.Size(a), torch.Size(b)))


def broadcast_divisor(bx: tuple, bshape: tuple) -> int | None:
    """When x's batch dims ``bx`` broadcast to ``bshape`` only by trailing
    size-1 dims, output batch entry b reads x batch b // d: return d.
    Otherwise return None (an explicit index tensor is needed).

    SwitchGLU's unsorted call (x [T,1,1,K] against indices [T,k],
    lfm2.py:202-214) gives d = k; the sorted call gives d = 1.
    """
    pad = (1,) * (len(bshape) - len(bx)) + tuple(bx)
    tail, k = 1, len(bshape)
    while k > 0 and pad[k - 1] == 1:
        tail *= bshape[k - 1]
        k -= 1
    return tail if tuple(pad[:k]) == tuple(bshape[:k]) else None


def _gather_args(x, w, scales, biases, lhs_indices, rhs_indices, group_size, bits):
    """Checks and flattens gather_qmm's operands (shared by the gather entry points)."""
    dev = _cuda(x, w, scales, biases, lhs_indices, rhs_indices)
    dt = _dtype_code(x, "x")
    if x.ndim < 2 or w.ndim < 2:
        raise ValueError("gather_qmm expects x [..., M, K] and w [..., N, K*bits/32]")
    K = _check_qweights(w, scales, biases, group_size, bits, x.dtype)
    if x.shape[-1] != K:
        raise ValueError(f"x has {x.shape[-1]} features but w expects K={K}")
    M, N = x.shape[-2], w.shape[-2]
    bx, bw = tuple(x.shape[:-2]), tuple(w.shape[:-2])
    x_batches = math.prod(bx)
    E = math.prod(bw)
    for name, idx in (("lhs_indices", lhs_indices), ("rhs_indices", rhs_indices)):
        if idx is not None and idx.dtype not in (torch.int32, torch.int64, torch.uint32):
            raise ValueError(f"{name} must be an integer tensor, got {idx.dtype}")
    lhs_shape = bx if lhs_indices is None else tuple(lhs_indices.shape)
    rhs_shape = bw if rhs_indices is None else tuple(rhs_indices.shape)
    try:
        bshape = _broadcast_shape(lhs_shape, rhs_shape)
    except RuntimeError as e:
        raise ValueError(f"cannot broadcast index shapes {lhs_shape} and {rhs_shape}") from e
    batch = math.prod(bshape)

    def _flat(idx, natural):
        if idx is None:
            idx = torch.arange(math.prod(natural), device=dev, dtype=torch.int32).reshape(natural)
        return idx.to(torch.int32).expand(bshape).contiguous().reshape(-1)

    rhs = lhs = None
    lhs_div = 1
    if batch and M:
        rhs = _flat(rhs_indices, bw)
        if lhs_indices is None:
            lhs_div = broadcast_divisor(bx, bshape)
            if lhs_div is None:
                lhs, lhs_div = _flat(None, bx), 1
        else:
            lhs = _flat(lhs_indices, bx)
    return dict(dev=dev, dt=dt, K=K, M=M, N=N, E=E, x_batches=x_batches, bshape=bshape,
                batch=batch, lhs=lhs, lhs_div=lhs_div, rhs=rhs, x=x.contiguous(),
                w=w.contiguous(), scales=scales.contiguous(), biases=biases.contiguous())


def gather_qmm(x: torch.Tensor, w: torch.Tensor, scales: torch.Tensor,
               biases: torch.Tensor | None = None, lhs_indices: torch.Tensor | None = None,
               rhs_indices: torch.Tensor | None = None, transpose: bool = True,
               group_size: int = 64, bits: int = 4, mode: str = "affine",
               sorted_indices: bool = False) -> torch.Tensor:
    """Batched quantized matmul with index-selected operands (MLX gather_qmm).

    x [..., M, K] with batch dims Bx; w [..., N, K*bits/32] with batch dims Bw.
    lhs_indices index flattened Bx, rhs_indices flattened Bw; both broadcast to
    a common shape S and the result is [*S, M, N].
    """
    _mode(mode)
    if not transpose:
        raise ValueError("transpose=False is not supported; the model graphs use transpose=True")
    a = _gather_args(x, w, scales, biases, lhs_indices, rhs_indices, group_size, bits)
    dev, batch, M, N, K = a["dev"], a["batch"], a["M"], a["N"], a["K"]
    out = torch.empty(*a["bshape"], M, N, dtype=x.dtype, device=dev)
    if batch == 0 or M == 0:
        return out
    L = _lib.load()
    with torch.cuda.device(dev):
        st = torch.cuda.current_stream(dev)
        need = L.mlxq_gather_qmm_workspace_size(batch, M, N, K, a["E"], group_size, bits, a["dt"],
                                                int(bool(sorted_indices)))
        ws = Workspace.get(dev, st, need, "gather") if need else None
        rc = L.mlxq_gather_qmm(_ptr(a["x"]), _ptr(a["w"]), _ptr(a["scales"]), _ptr(a["biases"]),
                               _ptr(a["lhs"]), a["lhs_div"], _ptr(a["rhs"]), _ptr(out), batch, M,
                               N, K, a["E"], a["x_batches"], group_size, bits, a["dt"],
                               int(bool(sorted_indices)), _ptr(ws),
                               0 if ws is None else ws.numel(), st.cuda_stream)
    _lib.check(rc, "gather_qmm")
    return out


def gather_qmm_swiglu(x: torch.Tensor, w: torch.Tensor, scales: torch.Tensor,
                      biases: torch.Tensor, lhs_indices: torch.Tensor | None = None,
                      rhs_indices: torch.Tensor | None = None, group_size: int = 64,
                      bits: int = 4, mode: str = "affine",
                      sorted_indices: bool = False) -> torch.Tensor:
    """silu(x @ gate_e^T) * (x @ up_e^T) per routed entry, from an expert bank in
    interleave_gate_up's layout ([E, N, ...], N = 2 * hidden): [*S, M, N/2].

    Decode sizes and sorted batches with enough rows per expert run as one launch with
    the activation in the grouped (decode or tensor-core) kernel's epilogue (each
    projection rounded to x's dtype, silu(g) * u formed in float32 and rounded once);
    other sizes run gather_qmm and then torch's silu and multiply in x's dtype on the
    de-interleaved halves, as SwitchGLU's separate projections do."""
    _mode(mode)
    a = _gather_args(x, w, scales, biases, lhs_indices, rhs_indices, group_size, bits)
    dev, batch, M, N, K = a["dev"], a["batch"], a["M"], a["N"], a["K"]
    if N % 16:
        raise ValueError(f"w must hold gate/up 16-row tiles (N={N} is not a multiple of 16)")
    L = _lib.load()
    if batch == 0 or M == 0 or not L.mlxq_gather_swiglu_supported(
            batch, M, N, K, a["E"], a["x_batches"], group_size, bits, a["dt"],
            int(a["lhs"] is not None), int(bool(sorted_indices))):
        y = gather_qmm(x, w, scales, biases, lhs_indices, rhs_indices, True, group_size, bits,
                       mode, sorted_indices)
        y = y.reshape(*a["bshape"], M, N // 16, 2, 8)
        g, u = y[..., 0, :], y[..., 1, :]
        return (torch.nn.functional.silu(g) * u).reshape(*a["bshape"], M, N // 2)
    out = torch.empty(*a["bshape"], M, N // 2, dtype=x.dtype, device=dev)
    with torch.cuda.device(dev):
        st = torch.cuda.current_stream(dev)
        need = L.mlxq_gather_qmm_workspace_size(batch, M, N, K, a["E"], group_size, bits, a["dt"],
                                                int(bool(sorted_indices)))
        ws = Workspace.get(dev, st, need, "gather") if need else None
        rc = L.mlxq_gather_qmm_swiglu(_ptr(a["x"]), _ptr(a["w"]), _ptr(a["scales"]),
                                      _ptr(a["biases"]), _ptr(a["lhs"]), a["lhs_div"],
                                      _ptr(a["rhs"]), _ptr(out), batch, M, N, K, a["E"],
                                      a["x_batches"], group_size, bits, a["dt"],
                                      int(bool(sorted_indices)), _ptr(ws),
                                      0 if ws is None else ws.numel(), st.cuda_stream)
    _lib.check(rc, "gather_qmm_swiglu")
    return out


def moe_sort(indices: torch.Tensor, num_experts: int):
    """Stable sort of routing entries by expert on the device, the argsort pair of the
    sorted SwitchGLU path (_gather_sort, lfm2.py:613-618 of the reference): for the
    flattened int32 `indices` (n <= 16384 entries), returns int32 tensors (order,
    sorted_indices, inverse) with order[p] the entry at sorted position p (equal
    experts in entry order), sorted_indices[p] = indices[order[p]] and inverse[i] the
    position of entry i. Values outside [0, num_experts) form a group before
    (negative) or after (too large) every expert, in entry order."""
    dev = _cuda(indices)
    if indices.dtype != torch.int32:
        raise ValueError(f"indices must be int32, got {indices.dtype}")
    flat = indices.contiguous().reshape(-1)
    n = flat.numel()
    if not 1 <= num_experts <= 1024 or n > 16384:
        raise ValueError(f"moe_sort takes n <= 16384 entries and 1 <= num_experts <= 1024 "
                         f"(got n={n}, num_experts={num_experts})")
    order = torch.empty(n, dtype=torch.int32, device=dev)
    srt = torch.empty_like(order)
    inv = torch.empty_like(order)
    if n:
        with torch.cuda.device(dev):
            st = torch.cuda.current_stream(dev)
            rc = _lib.load().mlxq_moe_sort(_ptr(flat), n, num_experts, _ptr(order), _ptr(srt),
                                           _ptr(inv), st.cuda_stream)
        _lib.check(rc, "moe_sort")
    return order, srt, inv


def moe_route(logits: torch.Tensor, top_k: int, norm_topk_prob: bool = True,
              expert_bias: torch.Tensor | None = None):
    """Top-k expert routing of an MoE layer on the device (the router of
    Lfm2MoE.__call__, lfm2.py:366-375): softmax of the logits in float32 (+ the
    optional float32 per-expert bias), the top_k experts per token and their gates,
    renormalised to sum to one (with the reference's 1e-20 guard) when
    norm_topk_prob, in the logits' dtype. Experts come in descending gate order (the
    reference's argpartition leaves the order unspecified). Returns (indices int32
    [..., top_k], scores [..., top_k])."""
    dev = _cuda(logits, expert_bias)
    dt = _dtype_code(logits, "logits", (torch.float32, torch.bfloat16, torch.float16))
    E = logits.shape[-1]
    if not 1 <= top_k <= min(32, E) or E > 1024:
        raise ValueError(f"top_k={top_k} must be in [1, min(32, {E})] and experts <= 1024")
    if expert_bias is not None:
        if expert_bias.shape != (E,):
            raise ValueError(f"expert_bias must be [{E}]")
        expert_bias = expert_bias.float().contiguous()
    lead = logits.shape[:-1]
    x = logits.contiguous()
    T = x.numel() // E
    idx = torch.empty(*lead, top_k, dtype=torch.int32, device=dev)
    sc = torch.empty(*lead, top_k, dtype=logits.dtype, device=dev)
    with torch.cuda.device(dev):
        st = torch.cuda.current_stream(dev)
        rc = _lib.load().mlxq_moe_route(_ptr(x), dt, _ptr(expert_bias), _ptr(idx), _ptr(sc), dt,
                                        T, E, top_k, int(bool(norm_topk_prob)), st.cuda_stream)
    _lib.check(rc, "moe_route")
    return idx, sc
