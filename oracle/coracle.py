"""ctypes binding of the C oracle (oracle/libqmm_oracle.so).

TEST INFRASTRUCTURE ONLY: imported by tests/, __graft_entry__.smoke() and
bench.py's CPU-baseline leg, never by the product package. Arrays are numpy;
bf16 arrays are uint16 bit patterns (see oracle_np).
"""
from __future__ import annotations

import ctypes
import os
import subprocess

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
_LIB_PATH = os.path.join(_HERE, "libqmm_oracle.so")
_DT = {"float32": 0, "bfloat16": 1, "float16": 2}
_lib = None


def build(force: bool = False) -> str:
    if force or not os.path.exists(_LIB_PATH) or (
        os.path.getmtime(_LIB_PATH) < os.path.getmtime(os.path.join(_HERE, "qmm_oracle.c"))
    ):
        subprocess.run(["make", "-C", _HERE, "-s", "libqmm_oracle.so"], check=True)
    return _LIB_PATH


def lib():
    global _lib
    if _lib is None:
        build()
        L = ctypes.CDLL(_LIB_PATH)
        vp, i64, i32 = ctypes.c_void_p, ctypes.c_int64, ctypes.c_int
        L.oq_quantize.argtypes = [vp, i32, vp, vp, vp, i64, i64, i32, i32]
        L.oq_dequantize.argtypes = [vp, vp, vp, i32, vp, i64, i64, i32, i32]
        L.oq_quantized_matmul.argtypes = [vp, vp, vp, vp, vp, i32, vp, i64, i64, i64, i32, i32]
        L.oq_gather_qmm.argtypes = [vp, vp, vp, vp, vp, i64, vp, i32, vp, i64, i64, i64, i64,
                                    i64, i64, i32, i32]
        L.oq_num_threads.restype = i32
        L.oq_set_num_threads.argtypes = [i32]
        _lib = L
    return _lib


def _p(a):
    return None if a is None else a.ctypes.data_as(ctypes.c_void_p)


def _store_dtype(dtype):
    return {"float32": np.float32, "bfloat16": np.uint16, "float16": np.float16}[dtype]


def _chk(rc, what):
    if rc != 0:
        raise ValueError(f"oracle {what} failed with code {rc}")


def quantize(w, dtype, group_size=64, bits=4):
    w = np.ascontiguousarray(w)
    rows, K = w.shape
    wq = np.empty((rows, K * bits // 32), np.uint32)
    s = np.empty((rows, K // group_size), _store_dtype(dtype))
    b = np.empty_like(s)
    _chk(lib().oq_quantize(_p(w), _DT[dtype], _p(wq), _p(s), _p(b), rows, K, group_size, bits),
         "quantize")
    return wq, s, b


def dequantize(wq, s, b, dtype, group_size=64, bits=4):
    rows = wq.shape[0]
    K = wq.shape[1] * 32 // bits
    out = np.empty((rows, K), _store_dtype(dtype))
    _chk(lib().oq_dequantize(_p(np.ascontiguousarray(wq)), _p(np.ascontiguousarray(s)),
                             _p(np.ascontiguousarray(b)), _DT[dtype], _p(out), rows, K,
                             group_size, bits), "dequantize")
    return out


def quantized_matmul(x, wq, s, b, dtype, group_size=64, bits=4, bias=None):
    x = np.ascontiguousarray(x)
    M, K = x.shape
    N = wq.shape[0]
    out = np.empty((M, N), _store_dtype(dtype))
    bias = None if bias is None else np.ascontiguousarray(bias)
    _chk(lib().oq_quantized_matmul(_p(x), _p(np.ascontiguousarray(wq)),
                                   _p(np.ascontiguousarray(s)), _p(np.ascontiguousarray(b)),
                                   _p(bias), _DT[dtype], _p(out), M, N, K, group_size, bits),
         "quantized_matmul")
    return out


def gather_qmm(x, wq, s, b, rhs, dtype, group_size=64, bits=4, lhs=None, lhs_div=1):
    """x [Xb, M, K]; wq [E, N, Kw]; rhs/lhs int32 [B] -> out [B, M, N]."""
    x = np.ascontiguousarray(x)
    Xb, M, K = x.shape
    E, N, _ = wq.shape
    rhs = np.ascontiguousarray(rhs, dtype=np.int32)
    lhs = None if lhs is None else np.ascontiguousarray(lhs, dtype=np.int32)
    B = rhs.shape[0]
    out = np.empty((B, M, N), _store_dtype(dtype))
    _chk(lib().oq_gather_qmm(_p(x), _p(np.ascontiguousarray(wq)), _p(np.ascontiguousarray(s)),
                             _p(np.ascontiguousarray(b)), _p(lhs), lhs_div, _p(rhs), _DT[dtype],
                             _p(out), B, M, N, K, E, Xb, group_size, bits), "gather_qmm")
    return out


def num_threads() -> int:
    return lib().oq_num_threads()


def set_num_threads(n: int) -> None:
    lib().oq_set_num_threads(n)
