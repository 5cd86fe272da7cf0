"""GPU tests of mlxq_quantized_matmul_noalloc, the entry point for callers that
cannot allocate device memory: a host that binds the C ABI without a device
allocator of its own, or a plugin inside a serving engine whose memory manager
owns all device memory (and where a cudaMalloc in the middle of a decode step
could synchronize the device). It runs the decode kernel's K-split path with the
library's built-in 2 MiB scratch instead of a caller workspace.

Each case calls the entry point twice in a row (the scratch keeps the last
call's contents, so the second call checks that the tickets are cleared) and
checks both results against the C oracle and against mlxq_quantized_matmul,
within the path's tolerance max|d| <= 2e-2 * max|ref|.

This file is collected last on purpose, so a stop-at-first-failure run has
already run every other test before it."""
import ctypes

import numpy as np
import pytest
import torch

import mlx_server_runtime_b200 as mxq
from mlx_server_runtime_b200 import _lib
from oracle import coracle

from gpu_util import close, rand_weights, rand_x, to_dev, to_np

pytestmark = pytest.mark.gpu

_CODE = {"bfloat16": _lib.BF16, "float16": _lib.F16}


def _noalloc(x, wq, s, b, bias, group_size, bits, dt):
    M, K = x.shape
    N = wq.shape[0]
    out = torch.empty(M, N, dtype=x.dtype, device=x.device)
    rc = _lib.load().mlxq_quantized_matmul_noalloc(
        x.data_ptr(), wq.data_ptr(), s.data_ptr(), b.data_ptr(),
        None if bias is None else bias.data_ptr(), out.data_ptr(), M, N, K, group_size, bits,
        _CODE[dt], ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
    return rc, out


# (M, N, K, bits, group_size, dtype, bias): every shape splits K over CTAs (few
# 128-row blocks or a long K), so every call uses the built-in scratch.
CASES = [
    (4, 512, 3584, 4, 64, "bfloat16", False),
    (1, 3584, 18944, 8, 64, "bfloat16", True),
    (2, 640, 2048, 4, 32, "float16", True),
    (3, 512, 4096, 4, 128, "float16", False),
    (8, 256, 8192, 8, 128, "bfloat16", True),
    (17, 384, 3072, 8, 32, "float16", True),
]


@pytest.mark.parametrize("M,N,K,bits,gs,dt,with_bias", CASES)
def test_noalloc_matches_oracle_and_workspace_entry_point(M, N, K, bits, gs, dt, with_bias):
    rng = np.random.default_rng(M * 1000 + N + K + bits + gs)
    w = rand_weights(rng, (N, K), dt)
    wq, s, b = coracle.quantize(w, dt, gs, bits)
    x = rand_x(rng, (M, K), dt)
    bias = rand_x(rng, (N,), dt) if with_bias else None
    ref = coracle.quantized_matmul(x, wq, s, b, dt, gs, bits, bias=bias)
    xd, wd, sd, bd = to_dev(x, dt), to_dev(wq), to_dev(s, dt), to_dev(b, dt)
    biasd = to_dev(bias, dt) if with_bias else None
    with_ws = to_np(mxq.quantized_matmul(xd, wd, sd, bd, group_size=gs, bits=bits, bias=biasd))
    close(with_ws, ref, dt)
    for _ in range(2):
        rc, got = _noalloc(xd, wd, sd, bd, biasd, gs, bits, dt)
        assert rc == 0, _lib.last_error()
        torch.cuda.synchronize()
        got = to_np(got)
        close(got, ref, dt)
        close(got, with_ws, dt)


def test_noalloc_rejects_shapes_beyond_its_scratch():
    # 32 tokens against a 3584x3584 projection split five ways needs ~2.3 MB of
    # partial sums, more than the 2 MiB the library holds.
    rng = np.random.default_rng(7)
    w = rand_weights(rng, (3584, 3584), "bfloat16")
    wq, s, b = coracle.quantize(w, "bfloat16", 64, 4)
    x = rand_x(rng, (32, 3584), "bfloat16")
    rc, _ = _noalloc(to_dev(x, "bfloat16"), to_dev(wq), to_dev(s, "bfloat16"),
                     to_dev(b, "bfloat16"), None, 64, 4, "bfloat16")
    assert rc == _lib.ERR_WORKSPACE
    assert "scratch" in _lib.last_error()
