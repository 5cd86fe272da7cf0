"""Sorted gather_qmm on the grouped tensor-core kernel (many rows per expert):
rows sorted by expert, each expert's contiguous rows multiplied by its own
weights. Checked against the C oracle."""
import numpy as np
import pytest
import torch

import mlx_server_runtime_b200 as mxq
from oracle import coracle

from gpu_util import close, rand_weights, rand_x, to_dev, to_np

pytestmark = pytest.mark.gpu


def _experts(rng, E, N, K, dt, gs, bits):
    w = rand_weights(rng, (E * N, K), dt)
    wq, s, b = coracle.quantize(w, dt, gs, bits)
    return wq.reshape(E, N, -1), s.reshape(E, N, -1), b.reshape(E, N, -1)


def _run(E, N, K, counts, M=1, dt="bfloat16", bits=4, gs=64, seed=0):
    rng = np.random.default_rng(seed)
    wq, s, b = _experts(rng, E, N, K, dt, gs, bits)
    sel = np.repeat(np.arange(E, dtype=np.int32), counts)
    batch = sel.size
    x = rand_x(rng, (batch, M, K), dt)
    ref = coracle.gather_qmm(x, wq, s, b, sel, dt, gs, bits)
    y = mxq.gather_qmm(to_dev(x, dt), to_dev(wq), to_dev(s, dt), to_dev(b, dt),
                       rhs_indices=to_dev(sel), group_size=gs, bits=bits, sorted_indices=True)
    torch.cuda.synchronize()
    close(to_np(y), ref, dt)


def test_grouped_uneven_segments():
    # empty experts, one exactly one tile (128), one spanning three tiles, ragged rest
    counts = [0, 128, 300, 1, 0, 77, 40, 129]
    _run(8, 320, 512, counts, seed=1)


@pytest.mark.parametrize("dt", ["bfloat16", "float16"])
@pytest.mark.parametrize("bits,gs", [(4, 64), (8, 64), (4, 32), (4, 128)])
def test_grouped_types(dt, bits, gs):
    rng = np.random.default_rng(bits + gs)
    counts = rng.integers(0, 90, size=16)
    _run(16, 256, 768, counts, dt=dt, bits=bits, gs=gs, seed=bits * gs)


def test_grouped_two_rows_per_entry():
    _run(4, 192, 256, [40, 0, 70, 25], M=2, seed=3)


def test_grouped_moe_shapes():
    """Qwen3-30B-A3B-like expert projections (2048 -> 768 and 768 -> 2048), 32 experts."""
    rng = np.random.default_rng(9)
    counts = rng.multinomial(32 * 48, np.ones(32) / 32)
    _run(32, 768, 2048, counts, seed=10)
    _run(32, 2048, 768, counts, seed=11)
