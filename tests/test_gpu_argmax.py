"""Greedy next token with the argmax in the decode kernel's epilogue
(quantized_matmul_argmax): the ids must be exactly the argmax of the logits
quantized_matmul returns for the same inputs (first index on ties), whatever
plan the shape gets (16-row CTAs, whole 64-row blocks, split row blocks with
tickets, the ticket warp), call after call."""
import numpy as np
import pytest
import torch

import mlx_server_runtime_b200 as mxq
from mlx_server_runtime_b200 import _lib
from oracle import coracle

from gpu_util import rand_weights, rand_x, to_dev, to_np

pytestmark = pytest.mark.gpu


def _weights(rng, N, K, dt="bfloat16", gs=64, bits=4):
    w = to_dev(rand_weights(rng, (N, K), dt), dt)
    return mxq.quantize(w, gs, bits)


@pytest.mark.parametrize("N,K,M", [(152064, 3584, 1), (152064, 3584, 8), (9473, 3584, 3),
                                   (512, 3584, 2), (3584, 18944, 1), (1000, 1536, 5),
                                   (152064, 3584, 16), (9473, 3584, 11)])
def test_argmax_equals_argmax_of_logits(N, K, M):
    rng = np.random.default_rng(N + K + M)
    wq, s, b = _weights(rng, N, K)
    x = to_dev(rand_x(rng, (M, K), "bfloat16"), "bfloat16")
    logits = mxq.quantized_matmul(x, wq, s, b)
    want = logits.float().argmax(dim=-1).to(torch.int32)
    for _ in range(3):  # the keys and the done counter must be re-armed every call
        ids = mxq.quantized_matmul_argmax(x, wq, s, b)
        torch.cuda.synchronize()
        assert _lib.device_error() == 0
        assert torch.equal(ids, want)


@pytest.mark.parametrize("dt", ["bfloat16", "float16"])
def test_argmax_bias_dtypes_and_oracle(dt):
    rng = np.random.default_rng(9)
    N, K, M = 4096, 2048, 4
    w = rand_weights(rng, (N, K), dt)
    wq, s, b = coracle.quantize(w, dt, 64, 4)
    x = rand_x(rng, (M, K), dt)
    bias = rand_x(rng, (N,), dt)
    args = (to_dev(x, dt), to_dev(wq), to_dev(s, dt), to_dev(b, dt))
    ids = mxq.quantized_matmul_argmax(*args, bias=to_dev(bias, dt))
    logits = mxq.quantized_matmul(*args, bias=to_dev(bias, dt))
    assert torch.equal(ids, logits.float().argmax(dim=-1).to(torch.int32))
    # the chosen logit is the oracle's maximum up to the path's tolerance
    from oracle import oracle_np as O
    ref = O.to_f32(coracle.quantized_matmul(x, wq, s, b, dt, 64, 4, bias=bias), dt)
    got = ref[np.arange(M), to_np(ids)]
    assert np.all(ref.max(axis=1) - got <= 2e-2 * np.abs(ref).max())


def test_argmax_ties_take_the_first_index():
    rng = np.random.default_rng(4)
    K = 1024
    row = rand_weights(rng, (1, K), "bfloat16")
    w = to_dev(np.repeat(row, 3000, axis=0), "bfloat16")   # every logit identical
    wq, s, b = mxq.quantize(w)
    x = to_dev(rand_x(rng, (2, K), "bfloat16"), "bfloat16")
    ids = mxq.quantized_matmul_argmax(x, wq, s, b)
    assert ids.tolist() == [0, 0]


def test_argmax_other_shapes_fall_back_to_logits():
    rng = np.random.default_rng(6)
    wq, s, b = _weights(rng, 2000, 1024)
    x = to_dev(rand_x(rng, (40, 1024), "bfloat16"), "bfloat16")  # prefill rows
    ids = mxq.quantized_matmul_argmax(x, wq, s, b)
    assert torch.equal(ids, mxq.quantized_matmul(x, wq, s, b).float().argmax(-1).to(torch.int32))
