"""CPU tests of the C ABI boundary: the library loads, exports every symbol the
header declares, and rejects bad arguments on the host before touching the
device (no compute runs without a GPU)."""
import ctypes
import os
import re

import pytest

import mlx_server_runtime_b200 as pkg
from mlx_server_runtime_b200 import _lib

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "mlxq_b200.h")


def header_symbols():
    with open(HEADER) as f:
        text = f.read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(mlxq_[a-z0-9_]+)\s*\(", text)))


def test_library_loads_and_version():
    L = _lib.load()
    assert L.mlxq_abi_version() == _lib.ABI_VERSION


def test_every_header_symbol_is_exported():
    L = _lib.load()
    syms = header_symbols()
    assert len(syms) >= 8
    for s in syms:
        assert hasattr(L, s), f"{s} declared in mlxq_b200.h but not exported"
    assert set(syms) == set(_lib.EXPORTED)


def test_library_is_in_tree():
    assert os.path.dirname(pkg.library_path()) == os.path.join(ROOT, "mlx-server-runtime_b200")


FAKE = ctypes.c_void_p(0x1000)  # aligned, never dereferenced: validation fails first


@pytest.mark.parametrize("bits,gs,code", [(3, 64, _lib.ERR_BITS), (4, 48, _lib.ERR_GROUP),
                                          (16, 64, _lib.ERR_BITS)])
def test_quantize_rejects_bits_group(bits, gs, code):
    L = _lib.load()
    rc = L.mlxq_quantize(FAKE, 1, FAKE, FAKE, FAKE, 4, 128, gs, bits, None)
    assert rc == code
    assert _lib.last_error()


def test_quantize_rejects_k_not_multiple():
    L = _lib.load()
    assert L.mlxq_quantize(FAKE, 1, FAKE, FAKE, FAKE, 4, 100, 64, 4, None) == _lib.ERR_SHAPE


def test_quantize_rejects_dtype_null_align():
    L = _lib.load()
    assert L.mlxq_quantize(FAKE, 7, FAKE, FAKE, FAKE, 4, 128, 64, 4, None) == _lib.ERR_DTYPE
    assert L.mlxq_quantize(None, 1, FAKE, FAKE, FAKE, 4, 128, 64, 4, None) == _lib.ERR_NULL
    odd = ctypes.c_void_p(0x1002)
    assert L.mlxq_quantize(odd, 1, FAKE, FAKE, FAKE, 4, 128, 64, 4, None) == _lib.ERR_ALIGN


def test_quantize_zero_rows_is_noop():
    L = _lib.load()
    assert L.mlxq_quantize(FAKE, 1, FAKE, FAKE, FAKE, 0, 128, 64, 4, None) == _lib.OK


def test_matmul_rejects_2bit_and_f32():
    L = _lib.load()
    args = (FAKE, FAKE, FAKE, FAKE, None, FAKE, 1, 64, 128)
    assert L.mlxq_quantized_matmul(*args, 64, 2, 1, None, 0, None) == _lib.ERR_BITS
    assert L.mlxq_quantized_matmul(*args, 64, 4, 0, None, 0, None) == _lib.ERR_DTYPE
    assert L.mlxq_quantized_matmul(FAKE, FAKE, FAKE, FAKE, None, FAKE, 1, 0, 128, 64, 4, 1, None,
                                   0, None) == _lib.ERR_SHAPE
    assert L.mlxq_quantized_matmul(FAKE, FAKE, FAKE, FAKE, None, FAKE, 0, 64, 128, 64, 4, 1,
                                   None, 0, None) == _lib.OK


def test_gather_rejects_bad_index_args():
    L = _lib.load()
    base = dict(batch=4, M=1, N=64, K=128, E=8, xb=4)
    rc = L.mlxq_gather_qmm(FAKE, FAKE, FAKE, FAKE, None, 0, FAKE, FAKE, base["batch"], base["M"],
                           base["N"], base["K"], base["E"], base["xb"], 64, 4, 1, 0, None, 0, None)
    assert rc == _lib.ERR_INDEX
    rc = L.mlxq_gather_qmm(FAKE, FAKE, FAKE, FAKE, None, 1, None, FAKE, 4, 1, 64, 128, 8, 4, 64,
                           4, 1, 0, None, 0, None)
    assert rc == _lib.ERR_NULL
    rc = L.mlxq_gather_qmm(FAKE, FAKE, FAKE, FAKE, None, 1, FAKE, FAKE, 4, 1, 64, 128, 0, 4, 64,
                           4, 1, 0, None, 0, None)
    assert rc == _lib.ERR_SHAPE


def test_gather_workspace_size():
    L = _lib.load()
    assert L.mlxq_gather_qmm_workspace_size(64, 1, 768, 2048, 128, 64, 4, 1, 0) == 0
    n = L.mlxq_gather_qmm_workspace_size(64, 1, 768, 2048, 128, 64, 4, 1, 1)
    assert n >= 129 * 4 and n % 256 == 0


def test_check_maps_errors():
    with pytest.raises(ValueError):
        _lib.check(_lib.ERR_SHAPE, "x")
    with pytest.raises(RuntimeError):
        _lib.check(_lib.ERR_CUDA, "x")
