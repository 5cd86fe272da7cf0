"""Parity of the TMA-fed decode kernel (M <= 8 tokens, K/group_size a multiple
of 8) against the C oracle: every token count, both activation types, 4- and
8-bit codes, all group sizes, row counts that leave partial 64-row blocks, and
shapes whose 64-row blocks are shared by several CTAs (stream-K tickets)."""
import numpy as np
import pytest
import torch

import mlx_server_runtime_b200 as mxq
from oracle import coracle

from gpu_util import close, rand_weights, rand_x, to_dev, to_np

pytestmark = pytest.mark.gpu


def _case(dt, bits, gs, M, N, K, seed, bias=False, calls=1):
    rng = np.random.default_rng(seed)
    w = rand_weights(rng, (N, K), dt)
    x = rand_x(rng, (M, K), dt)
    wq, s, b = coracle.quantize(w, dt, gs, bits)
    bvec = rand_x(rng, (N,), dt) if bias else None
    ref = coracle.quantized_matmul(x, wq, s, b, dt, gs, bits, bias=bvec)
    args = (to_dev(x, dt), to_dev(wq), to_dev(s, dt), to_dev(b, dt))
    kw = dict(group_size=gs, bits=bits, bias=None if bvec is None else to_dev(bvec, dt))
    outs = [mxq.quantized_matmul(*args, **kw) for _ in range(calls)]
    torch.cuda.synchronize()
    for y in outs:
        close(to_np(y), ref, dt)
    return [to_np(y) for y in outs]


@pytest.mark.parametrize("M", [1, 2, 3, 4, 5, 6, 7, 8, 9, 12, 16, 17, 24, 31, 32])
def test_decode_token_counts(M):
    _case("bfloat16", 4, 64, M, 3584, 3584, seed=100 + M)


@pytest.mark.parametrize("bits", [4, 8])
@pytest.mark.parametrize("M", [17, 24, 31, 32])
def test_decode_two_launches(M, bits):
    # small matrices at 17-32 rows: two launches of the 16-slot kernel
    _case("bfloat16", bits, 64, M, 512, 3584, seed=300 + M + bits, bias=(M == 24))


@pytest.mark.parametrize("dt", ["bfloat16", "float16"])
@pytest.mark.parametrize("bits,gs", [(4, 32), (4, 64), (4, 128), (8, 32), (8, 64)])
@pytest.mark.parametrize("M", [1, 3, 8, 13, 16])
def test_decode_types_and_groups(dt, bits, gs, M):
    _case(dt, bits, gs, M, 1000, 8 * gs * 3, seed=bits * 1000 + gs + M)


@pytest.mark.parametrize("N", [1, 17, 64, 65, 200, 9473])
def test_decode_ragged_rows(N):
    _case("bfloat16", 4, 64, 2, N, 1024, seed=N)


@pytest.mark.parametrize("N,K", [(512, 3584), (3584, 3584), (3584, 18944), (4096, 2048),
                                 (768, 2048)])
def test_decode_shared_row_blocks_repeat(N, K):
    """Row blocks split over CTAs: three calls in a row also check that the
    tickets are left at zero; the results are bit-identical across calls."""
    outs = _case("bfloat16", 4, 64, 1, N, K, seed=N + K, bias=True, calls=3)
    assert outs[0].tobytes() == outs[1].tobytes() == outs[2].tobytes()


def test_decode_lm_head_size():
    _case("bfloat16", 4, 64, 1, 152064, 3584, seed=7)


def test_decode_device_error_clear():
    _case("bfloat16", 4, 64, 1, 3584, 3584, seed=9)
    from mlx_server_runtime_b200 import _lib
    assert _lib.device_error() == 0


def test_workspace_shared_by_plans_of_different_sizes():
    """Calls with different row-block counts, on both decode kernels, share one
    workspace on the stream: partial sums of one call must never sit where a
    later call keeps its tickets."""
    for M, N, K in ((20, 512, 3584), (2, 200, 512), (1, 9473, 1024), (20, 640, 3584),
                    (1, 512, 3584), (3, 3584, 18944), (2, 9473, 1024)):
        _case("bfloat16", 4, 64, M, N, K, seed=M * 7 + N)


@pytest.mark.parametrize("dt", ["bfloat16", "float16"])
def test_decode_activation_magnitudes(dt):
    """Activations far from 1 (every group slice is rescaled by its own power of
    two inside the kernel): huge, tiny, mixed per group, and all zero."""
    from oracle import oracle_np as O
    rng = np.random.default_rng(3)
    N, K, gs = 640, 2048, 64
    w = rand_weights(rng, (N, K), dt)
    wq, s, b = coracle.quantize(w, dt, gs, 4)
    big, tiny = (1e20, 1e-20) if dt == "bfloat16" else (60.0, 1e-3)
    xf = rng.standard_normal((4, K)).astype(np.float32)
    xf[0] *= big
    xf[1] *= tiny
    xf[2] *= np.repeat(np.where(np.arange(K // gs) % 2 == 0, big, tiny), gs).astype(np.float32)
    xf[3] = 0.0
    x = O.from_f32(xf, dt)
    ref = coracle.quantized_matmul(x, wq, s, b, dt, gs, 4)
    y = to_np(mxq.quantized_matmul(to_dev(x, dt), to_dev(wq), to_dev(s, dt), to_dev(b, dt),
                                   group_size=gs, bits=4))
    for t in range(4):
        close(y[t:t + 1], ref[t:t + 1], dt)
    assert not np.any(O.to_f32(y[3:4], dt))


def test_decode_nonfinite_activations_propagate():
    """An infinite activation makes the outputs non-finite, as in float arithmetic."""
    from oracle import oracle_np as O
    rng = np.random.default_rng(4)
    N, K = 128, 512
    w = rand_weights(rng, (N, K), "bfloat16")
    wq, s, b = coracle.quantize(w, "bfloat16", 64, 4)
    xf = rng.standard_normal((2, K)).astype(np.float32)
    xf[0, 5] = np.inf
    x = O.from_f32(xf, "bfloat16")
    y = O.to_f32(to_np(mxq.quantized_matmul(to_dev(x, "bfloat16"), to_dev(wq),
                                            to_dev(s, "bfloat16"), to_dev(b, "bfloat16"))),
                 "bfloat16")
    assert not np.isfinite(y[0]).any()
    assert np.isfinite(y[1]).all()
