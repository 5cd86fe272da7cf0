"""GPU test of mlxq_quantized_matmul_noalloc, the entry point for callers that
cannot allocate device memory (a host binding the C ABI without an allocator of
its own, or a plugin whose engine owns all device memory). It runs the decode
kernel's K-split path with the library's built-in 2 MiB scratch instead of a
caller workspace; its results must match mlxq_quantized_matmul's.

This file is collected last on purpose, so a stop-at-first-failure run has
already run every other test before it."""
import ctypes

import numpy as np
import pytest
import torch

import mlx_server_runtime_b200 as mxq
from mlx_server_runtime_b200 import _lib

from gpu_util import close, rand_weights, rand_x, to_dev, to_np

pytestmark = pytest.mark.gpu


def _noalloc(x, wq, s, b, bias=None, group_size=64, bits=4):
    M, K = x.shape
    N = wq.shape[0]
    out = torch.empty(M, N, dtype=x.dtype, device=x.device)
    rc = _lib.load().mlxq_quantized_matmul_noalloc(
        x.data_ptr(), wq.data_ptr(), s.data_ptr(), b.data_ptr(),
        None if bias is None else bias.data_ptr(), out.data_ptr(), M, N, K, group_size, bits,
        _lib.BF16, ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
    return rc, out


def _problem(seed, M, N, K, bits=4):
    rng = np.random.default_rng(seed)
    w = to_dev(rand_weights(rng, (N, K), "bfloat16"), "bfloat16")
    wq, s, b = mxq.quantize(w, 64, bits)
    x = to_dev(rand_x(rng, (M, K), "bfloat16"), "bfloat16")
    return x, wq, s, b


def test_noalloc_matches_workspace_entry_point_twice():
    # The no-alloc entry point runs the skinny kernel, whose plan splits K when the
    # rows are few (N=512) or K is long (the down projection): it then needs its
    # scratch (partial sums + tickets) for every call.
    for call, (M, N, K, bits) in enumerate([(4, 512, 3584, 4), (4, 512, 3584, 4),
                                            (1, 3584, 18944, 8)]):
        x, wq, s, b = _problem(100 + call, M, N, K, bits)
        ref = mxq.quantized_matmul(x, wq, s, b, group_size=64, bits=bits)
        rc, got = _noalloc(x, wq, s, b, bits=bits)
        assert rc == 0, _lib.last_error()
        torch.cuda.synchronize()
        close(to_np(got), to_np(ref), "bfloat16")
        rc2, again = _noalloc(x, wq, s, b, bits=bits)
        assert rc2 == 0, _lib.last_error()
        torch.cuda.synchronize()
        close(to_np(again), to_np(ref), "bfloat16")


def test_noalloc_rejects_shapes_beyond_its_scratch():
    # 32 tokens against a 3584x3584 projection split five ways needs ~2.3 MB > 2 MiB.
    x, wq, s, b = _problem(7, 32, 3584, 3584)
    need = _lib.load().mlxq_qmm_workspace_size(32, 3584, 3584, 64, 4, _lib.BF16)
    assert need > 2 * 1024 * 1024
    rc, _ = _noalloc(x, wq, s, b)
    assert rc == _lib.ERR_WORKSPACE
    assert "scratch" in _lib.last_error()
