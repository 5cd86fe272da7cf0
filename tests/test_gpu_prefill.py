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
