"""B200-native group-wise affine quantized matmul (MLX layout) for the
mlx-server-runtime model graphs.

The directory name contains dashes, so callers register it under the module
name ``mlx_server_runtime_b200`` with importlib (``spec_from_file_location``
on this file with ``submodule_search_locations`` set to this directory), as
tests/conftest.py, bench.py and __graft_entry__.py do. Operators live in
``core`` under MLX's names, MLX-style modules in ``nn``.
"""
from __future__ import annotations

from . import _lib
from .core import (Workspace, concat_quantized, dequantize, gather_qmm, gather_qmm_swiglu,
                   interleave_gate_up, launch_overlap, quantize, quantized_matmul,
                   quantized_matmul_argmax, quantized_matmul_swiglu)

__all__ = ["quantize", "dequantize", "quantized_matmul", "gather_qmm", "gather_qmm_swiglu",
           "concat_quantized",
           "interleave_gate_up", "quantized_matmul_swiglu", "quantized_matmul_argmax",
           "Workspace", "launch_overlap",
           "library_path", "load_library"]


def library_path() -> str:
    return _lib.LIB_PATH


def load_library():
    """Load libmlxq_b200.so now (raises if it is missing)."""
    return _lib.load()
