"""Failure path of the kernels' bounded waits, exercised without any device fault.

Every mbarrier wait in the kernels gives up after a bounded number of polls,
records a code in the device error word and lets the kernel exit. Here a wait
that nothing completes (mlxq_check_bounded_wait: a barrier that expects one
arrival that never comes, with no copy or tensor-core operation in flight) runs
out; the host must read the timeout code through mlxq_device_error, the code
must clear on read, cached workspaces must be zero-filled again, and the context
must stay usable for the next matmul."""
import ctypes

import numpy as np
import pytest
import torch

import mlx_server_runtime_b200 as mxq
from mlx_server_runtime_b200 import _lib
from oracle import coracle

from gpu_util import close, rand_weights, rand_x, to_dev, to_np

pytestmark = pytest.mark.gpu

TIMEOUT_CODE = 2


def _stream():
    return ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)


def test_bounded_wait_runs_out_and_reports():
    assert _lib.device_error() == 0
    rc = _lib.load().mlxq_check_bounded_wait(64, _stream())
    assert rc == 0, _lib.last_error()
    torch.cuda.synchronize()
    assert _lib.device_error() == TIMEOUT_CODE
    assert _lib.device_error() == 0  # cleared by the read


def test_bounded_wait_rejects_bad_poll_count():
    assert _lib.load().mlxq_check_bounded_wait(0, _stream()) == _lib.ERR_SHAPE
    assert _lib.load().mlxq_check_bounded_wait((1 << 22) + 1, _stream()) == _lib.ERR_SHAPE


def test_context_usable_after_timeout_and_workspace_rezeroed():
    rng = np.random.default_rng(5)
    N, K = 3584, 18944  # split row blocks: the workspace tickets are in use
    w = rand_weights(rng, (N, K), "bfloat16")
    wq, s, b = coracle.quantize(w, "bfloat16", 64, 4)
    x = rand_x(rng, (1, K), "bfloat16")
    ref = coracle.quantized_matmul(x, wq, s, b, "bfloat16", 64, 4)
    args = (to_dev(x, "bfloat16"), to_dev(wq), to_dev(s, "bfloat16"), to_dev(b, "bfloat16"))
    close(to_np(mxq.quantized_matmul(*args)), ref, "bfloat16")
    # plant nonzero tickets in the cached workspace, as a kernel that gave up might
    for (_dev, _st, kind), buf in list(mxq.Workspace._bufs.items()):
        if kind == "qmm":
            buf[:4096].fill_(3)
    assert _lib.load().mlxq_check_bounded_wait(64, _stream()) == 0
    torch.cuda.synchronize()
    assert _lib.device_error() == TIMEOUT_CODE  # also zero-fills the cached workspaces
    torch.cuda.synchronize()
    for (_dev, _st, kind), buf in list(mxq.Workspace._bufs.items()):
        assert int(buf.count_nonzero()) == 0
    close(to_np(mxq.quantized_matmul(*args)), ref, "bfloat16")
    assert _lib.device_error() == 0
