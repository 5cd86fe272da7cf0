"""ctypes binding of libmlxq_b200.so (the C ABI declared in include/mlxq_b200.h).

The library is required: there is no CPU or pure-PyTorch fallback, and
loading fails loudly when the shared object is missing or was built for a
different ABI version.
"""
from __future__ import annotations

import ctypes
import os
import threading

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libmlxq_b200.so")
ABI_VERSION = 1

# dtype codes of the C ABI
F32, BF16, F16 = 0, 1, 2

OK = 0
ERR_SHAPE, ERR_DTYPE, ERR_ALIGN, ERR_BITS, ERR_GROUP = -1, -2, -3, -4, -5
ERR_CUDA, ERR_WORKSPACE, ERR_NULL, ERR_INDEX = -6, -7, -8, -9

EXPORTED = (
    "mlxq_abi_version",
    "mlxq_last_error",
    "mlxq_quantize",
    "mlxq_dequantize",
    "mlxq_qmm_workspace_size",
    "mlxq_quantized_matmul",
    "mlxq_gather_qmm",
    "mlxq_gather_qmm_workspace_size",
    "mlxq_set_launch_overlap",
    "mlxq_get_launch_overlap",
    "mlxq_quantized_matmul_noalloc",
    "mlxq_device_error",
    "mlxq_swiglu_supported",
    "mlxq_quantized_matmul_swiglu",
    "mlxq_argmax_workspace_size",
    "mlxq_quantized_matmul_argmax",
    "mlxq_check_bounded_wait",
    "mlxq_rms_norm",
    "mlxq_rope_kv_append",
    "mlxq_paged_attention_workspace_size",
    "mlxq_paged_attention_decode",
    "mlxq_paged_attention_prefill",
    "mlxq_quantized_embedding",
    "mlxq_decode_advance",
    "mlxq_moe_route",
    "mlxq_moe_sort",
    "mlxq_gather_swiglu_supported",
    "mlxq_gather_qmm_swiglu",
)

_lock = threading.Lock()
_lib = None


class LibraryError(RuntimeError):
    pass


def load(path: str | None = None):
    """Load (once) and return the ctypes handle of libmlxq_b200.so."""
    global _lib
    if _lib is not None and path is None:
        return _lib
    with _lock:
        if _lib is not None and path is None:
            return _lib
        p = path or LIB_PATH
        if not os.path.exists(p):
            raise LibraryError(
                f"{p} not found: build it with `python mlx-server-runtime_b200/build.py` "
                "(there is no fallback implementation)")
        L = ctypes.CDLL(p)
        vp, i64, i32, sz = ctypes.c_void_p, ctypes.c_int64, ctypes.c_int, ctypes.c_size_t
        L.mlxq_abi_version.restype = i32
        L.mlxq_last_error.restype = ctypes.c_char_p
        L.mlxq_quantize.argtypes = [vp, i32, vp, vp, vp, i64, i64, i32, i32, vp]
        L.mlxq_quantize.restype = i32
        L.mlxq_dequantize.argtypes = [vp, vp, vp, i32, vp, i64, i64, i32, i32, vp]
        L.mlxq_dequantize.restype = i32
        L.mlxq_qmm_workspace_size.argtypes = [i64, i64, i64, i32, i32, i32]
        L.mlxq_qmm_workspace_size.restype = sz
        L.mlxq_quantized_matmul.argtypes = [vp, vp, vp, vp, vp, vp, i64, i64, i64, i32, i32, i32,
                                            vp, sz, vp]
        L.mlxq_quantized_matmul.restype = i32
        L.mlxq_gather_qmm.argtypes = [vp, vp, vp, vp, vp, i64, vp, vp, i64, i64, i64, i64, i64,
                                      i64, i32, i32, i32, i32, vp, sz, vp]
        L.mlxq_gather_qmm.restype = i32
        L.mlxq_gather_qmm_workspace_size.argtypes = [i64, i64, i64, i64, i64, i32, i32, i32, i32]
        L.mlxq_gather_qmm_workspace_size.restype = sz
        L.mlxq_set_launch_overlap.argtypes = [i32]
        L.mlxq_set_launch_overlap.restype = i32
        L.mlxq_get_launch_overlap.restype = i32
        L.mlxq_quantized_matmul_noalloc.argtypes = [vp, vp, vp, vp, vp, vp, i64, i64, i64, i32,
                                                    i32, i32, vp]
        L.mlxq_quantized_matmul_noalloc.restype = i32
        L.mlxq_device_error.argtypes = [ctypes.POINTER(ctypes.c_int)]
        L.mlxq_device_error.restype = i32
        L.mlxq_swiglu_supported.argtypes = [i64, i64, i64, i32, i32, i32]
        L.mlxq_swiglu_supported.restype = i32
        L.mlxq_quantized_matmul_swiglu.argtypes = [vp, vp, vp, vp, vp, i64, i64, i64, i32, i32,
                                                   i32, vp, sz, vp]
        L.mlxq_quantized_matmul_swiglu.restype = i32
        L.mlxq_argmax_workspace_size.argtypes = [i64, i64, i64, i32, i32, i32]
        L.mlxq_argmax_workspace_size.restype = sz
        L.mlxq_quantized_matmul_argmax.argtypes = [vp, vp, vp, vp, vp, vp, i64, i64, i64, i32,
                                                   i32, i32, vp, sz, vp]
        L.mlxq_quantized_matmul_argmax.restype = i32
        L.mlxq_check_bounded_wait.argtypes = [ctypes.c_uint32, vp]
        L.mlxq_check_bounded_wait.restype = i32
        f32 = ctypes.c_float
        L.mlxq_rms_norm.argtypes = [vp, vp, vp, vp, vp, i64, i64, f32, i32, vp]
        L.mlxq_rms_norm.restype = i32
        L.mlxq_rope_kv_append.argtypes = [vp, i64, vp, vp, vp, vp, vp, i64, i32, i32, i32, f32,
                                          i32, vp]
        L.mlxq_rope_kv_append.restype = i32
        L.mlxq_paged_attention_workspace_size.argtypes = [i64, i32, i64, i32]
        L.mlxq_paged_attention_workspace_size.restype = sz
        L.mlxq_paged_attention_decode.argtypes = [vp, vp, vp, vp, i64, vp, i64, vp, i64, i32, i32,
                                                  i32, i32, f32, i32, vp, sz, vp]
        L.mlxq_paged_attention_decode.restype = i32
        L.mlxq_paged_attention_prefill.argtypes = [vp, vp, i64, vp, vp, vp, i64, vp, vp, i64, i32,
                                                   i32, i32, i32, f32, i32, vp]
        L.mlxq_paged_attention_prefill.restype = i32
        L.mlxq_quantized_embedding.argtypes = [vp, i64, vp, vp, vp, vp, i64, i64, i32, i32, i32,
                                               vp]
        L.mlxq_quantized_embedding.restype = i32
        L.mlxq_decode_advance.argtypes = [vp, vp, vp, vp, i64, i64, i32, vp]
        L.mlxq_decode_advance.restype = i32
        L.mlxq_moe_route.argtypes = [vp, i32, vp, vp, vp, i32, i64, i32, i32, i32, vp]
        L.mlxq_moe_route.restype = i32
        L.mlxq_moe_sort.argtypes = [vp, i64, i32, vp, vp, vp, vp]
        L.mlxq_moe_sort.restype = i32
        L.mlxq_gather_swiglu_supported.argtypes = [i64, i64, i64, i64, i64, i64, i32, i32, i32,
                                                   i32, i32]
        L.mlxq_gather_swiglu_supported.restype = i32
        L.mlxq_gather_qmm_swiglu.argtypes = [vp, vp, vp, vp, vp, i64, vp, vp, i64, i64, i64, i64,
                                             i64, i64, i32, i32, i32, i32, vp, sz, vp]
        L.mlxq_gather_qmm_swiglu.restype = i32
        v = L.mlxq_abi_version()
        if v != ABI_VERSION:
            raise LibraryError(f"{p} has ABI version {v}, expected {ABI_VERSION}; rebuild it")
        if path is None:
            _lib = L
        return L


def device_error() -> int:
    """Read and clear the current device's kernel error code (0 = none).

    A kernel that gave up on a bounded wait may have left workspace tickets
    nonzero, so after a nonzero code every cached workspace is zero-filled again
    (core.Workspace.reset) before later calls reuse it."""
    code = ctypes.c_int(0)
    check(load().mlxq_device_error(ctypes.byref(code)), "device_error")
    if code.value:
        from .core import Workspace
        Workspace.reset()
    return code.value


def last_error() -> str:
    return load().mlxq_last_error().decode(errors="replace")


def check(rc: int, what: str) -> None:
    """Map a C ABI status to the exception MLX would raise for the same misuse."""
    if rc == OK:
        return
    msg = f"{what}: {last_error()} (code {rc})"
    if rc in (ERR_SHAPE, ERR_DTYPE, ERR_ALIGN, ERR_BITS, ERR_GROUP, ERR_NULL, ERR_INDEX):
        raise ValueError(msg)
    raise RuntimeError(msg)
