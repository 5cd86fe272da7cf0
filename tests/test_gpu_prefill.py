"""GPU parity of the tcgen05 prefill kernel (M > 32 rows, K a multiple of 64)
against the CPU oracle: max|d| <= 2e-2 * max|ref| with bf16/f16 output; the
dequantized weight is rounded once to the activation dtype inside the kernel,
so results are not bit-identical to the oracle's float32 weights."""
import numpy as np
import pytest
import torch

import mlx_server_runtime_b200 as mxq
from mlx_server_runtime_b200 import _lib
from oracle import coracle

from gpu_util import close, rand_weights, rand_x, to_dev, to_np

pytestmark = pytest.mark.gpu


def _case(dt, bits, gs, M, N, K, seed, bias=False):
    rng = np.random.default_rng(seed)
    w = rand_weights(rng, (N, K), dt)
    x = rand_x(rng, (M, K), dt)
    wq, s, b = coracle.quantize(w, dt, gs, bits)
    bvec = rand_x(rng, (N,), dt) if bias else None
    ref = coracle.quantized_matmul(x, wq, s, b, dt, gs, bits, bias=bvec)
    y = mxq.quantized_matmul(to_dev(x, dt), to_dev(wq), to_dev(s, dt), to_dev(b, dt),
                             group_size=gs, bits=bits,
                             bias=None if bvec is None else to_dev(bvec, dt))
    torch.cuda.synchronize()
    assert _lib.device_error() == 0
    return to_np(y), ref


@pytest.mark.parametrize("M,N,K", [(33, 256, 64), (128, 256, 256), (129, 300, 512),
                                   (200, 520, 1024), (512, 3584, 3584)])
def test_prefill_shapes_bf16_4bit(M, N, K):
    y, ref = _case("bfloat16", 4, 64, M, N, K, seed=M + N + K)
    close(y, ref, "bfloat16")


@pytest.mark.parametrize("dt", ["bfloat16", "float16"])
@pytest.mark.parametrize("bits", [4, 8])
@pytest.mark.parametrize("gs", [32, 64, 128])
def test_prefill_dtype_bits_groups(dt, bits, gs):
    y, ref = _case(dt, bits, gs, 160, 384, 768, seed=bits * 7 + gs)
    close(y, ref, dt)


def test_prefill_bias_and_leading_dims():
    y, ref = _case("bfloat16", 4, 64, 96, 512, 1024, seed=3, bias=True)
    close(y, ref, "bfloat16")
    rng = np.random.default_rng(5)
    w = to_dev(rand_weights(rng, (256, 512), "bfloat16"), "bfloat16")
    wq, s, b = mxq.quantize(w)
    x = to_dev(rand_x(rng, (4, 40, 512), "bfloat16"), "bfloat16")
    y3 = mxq.quantized_matmul(x, wq, s, b)
    y2 = mxq.quantized_matmul(x.reshape(160, 512), wq, s, b)
    assert torch.equal(y3.reshape(160, 256), y2)


def test_prefill_deterministic():
    rng = np.random.default_rng(8)
    w = to_dev(rand_weights(rng, (1024, 2048), "bfloat16"), "bfloat16")
    wq, s, b = mxq.quantize(w)
    x = to_dev(rand_x(rng, (300, 2048), "bfloat16"), "bfloat16")
    outs = [mxq.quantized_matmul(x, wq, s, b) for _ in range(3)]
    assert torch.equal(outs[0], outs[1]) and torch.equal(outs[1], outs[2])
    assert _lib.device_error() == 0


# Stream-K: shapes whose whole tiles fill few SMs' worth of waves (here 52-84 tiles on
# 148 SMs) split tiles x K blocks evenly over the CTAs; a tile shared by several CTAs
# is finished by the last of them from fp32 partials in the workspace.
@pytest.mark.parametrize("dt", ["bfloat16", "float16"])
@pytest.mark.parametrize("bits,gs", [(4, 32), (4, 64), (4, 128), (8, 32), (8, 64)])
def test_prefill_stream_k_types(dt, bits, gs):
    y, ref = _case(dt, bits, gs, 200, 3584, 2048, seed=bits * 11 + gs, bias=True)
    close(y, ref, dt)


@pytest.mark.parametrize("M,N,K", [(450, 3328, 1024), (1000, 1280, 2048), (257, 3584, 8192),
                                   (300, 3584, 4096)])
def test_prefill_stream_k_shapes(M, N, K):
    y, ref = _case("bfloat16", 4, 64, M, N, K, seed=M + N + K, bias=(M % 2 == 0))
    close(y, ref, "bfloat16")


def test_prefill_stream_k_repeat_and_whole_tiles_agree():
    """Three stream-K calls in a row (the tickets must be back at zero) give the
    same bits; the whole-tile form (no workspace passed) agrees within tolerance."""
    import ctypes
    rng = np.random.default_rng(21)
    M, N, K = 600, 1664, 2048
    w = to_dev(rand_weights(rng, (N, K), "bfloat16"), "bfloat16")
    wq, s, b = mxq.quantize(w)
    x = to_dev(rand_x(rng, (M, K), "bfloat16"), "bfloat16")
    L = _lib.load()
    assert L.mlxq_qmm_workspace_size(M, N, K, 64, 4, _lib.BF16) > 0
    outs = [mxq.quantized_matmul(x, wq, s, b) for _ in range(3)]
    assert torch.equal(outs[0], outs[1]) and torch.equal(outs[1], outs[2])
    whole = torch.empty(M, N, dtype=torch.bfloat16, device="cuda")
    rc = L.mlxq_quantized_matmul(x.data_ptr(), wq.data_ptr(), s.data_ptr(), b.data_ptr(), None,
                                 whole.data_ptr(), M, N, K, 64, 4, _lib.BF16, None, 0,
                                 ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
    assert rc == 0, _lib.last_error()
    torch.cuda.synchronize()
    assert _lib.device_error() == 0
    close(to_np(outs[0]), to_np(whole), "bfloat16")


def test_prefill_stream_k_reduced_grid_and_fallback():
    """A short-K shape with few tiles (k/v at 512 tokens: 12 tiles of 56 K blocks) runs
    stream-K on fewer CTAs than SMs: matches the oracle, repeats bit for bit, and the
    form without a workspace (128-token whole tiles) agrees within tolerance."""
    import ctypes
    rng = np.random.default_rng(31)
    M, N, K = 512, 512, 3584
    w = rand_weights(rng, (N, K), "bfloat16")
    xh = rand_x(rng, (M, K), "bfloat16")
    wq, s, b = coracle.quantize(w, "bfloat16", 64, 4)
    ref = coracle.quantized_matmul(xh, wq, s, b, "bfloat16", 64, 4)
    x, wd, sd, bd = to_dev(xh, "bfloat16"), to_dev(wq), to_dev(s, "bfloat16"), to_dev(b, "bfloat16")
    outs = [mxq.quantized_matmul(x, wd, sd, bd) for _ in range(2)]
    torch.cuda.synchronize()
    assert _lib.device_error() == 0
    assert torch.equal(outs[0], outs[1])
    close(to_np(outs[0]), ref, "bfloat16")
    L = _lib.load()
    whole = torch.empty(M, N, dtype=torch.bfloat16, device="cuda")
    rc = L.mlxq_quantized_matmul(x.data_ptr(), wd.data_ptr(), sd.data_ptr(), bd.data_ptr(), None,
                                 whole.data_ptr(), M, N, K, 64, 4, _lib.BF16, None, 0,
                                 ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
    assert rc == 0, _lib.last_error()
    torch.cuda.synchronize()
    assert _lib.device_error() == 0
    close(to_np(whole), ref, "bfloat16")


@pytest.mark.parametrize("dt", ["bfloat16", "float16"])
@pytest.mark.parametrize("bits,gs", [(4, 32), (8, 64), (4, 128)])
@pytest.mark.parametrize("M", [512, 2048])
def test_prefill_stream_k_reduced_grid_types(dt, bits, gs, M):
    # k/v-shaped (N=512, K=3584): stream-K on 36 (M=512) or 132 (M=2048) CTAs, with bias
    y, ref = _case(dt, bits, gs, M, 512, 3584, seed=M + bits * 13 + gs, bias=True)
    close(y, ref, dt)
