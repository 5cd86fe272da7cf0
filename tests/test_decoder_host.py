"""CPU tests of the decoder-layer operators: host-side argument checks of their C
entry points (nothing reaches a device), and the numpy restatement's own
consistency (attention over gathered pages equals attention over dense rows;
the half-rotation RoPE equals multiplication by e^{i angle})."""
import numpy as np

from mlx_server_runtime_b200 import _lib
from oracle import decoder_np as D

FAKE = 0x1000  # aligned, never dereferenced: validation fails first


def test_rejections_before_any_launch():
    L = _lib.load()
    assert L.mlxq_rms_norm(FAKE, None, FAKE, FAKE, None, 4, 100, 1e-6, _lib.BF16,
                           None) == _lib.ERR_SHAPE                    # dim % 8
    assert L.mlxq_rms_norm(FAKE, None, FAKE, FAKE, FAKE, 4, 128, 1e-6, _lib.BF16,
                           None) == _lib.ERR_NULL                     # residual_out alone
    assert L.mlxq_rms_norm(FAKE, None, FAKE, FAKE, None, 4, 128, 1e-6, _lib.F32,
                           None) == _lib.ERR_DTYPE
    assert L.mlxq_paged_attention_decode(FAKE, FAKE, FAKE, FAKE, 4, FAKE, 65, FAKE, 2, 28, 4,
                                         128, 16, 0.1, _lib.BF16, None, 0,
                                         None) == _lib.ERR_SHAPE      # 65 keys > 4 pages of 16
    assert L.mlxq_paged_attention_decode(FAKE, FAKE, FAKE, FAKE, 4, FAKE, 64, FAKE, 2, 28, 5,
                                         128, 16, 0.1, _lib.BF16, None, 0,
                                         None) == _lib.ERR_SHAPE      # 28 heads over 5
    assert L.mlxq_paged_attention_decode(FAKE, FAKE, FAKE, FAKE, 4, FAKE, 64, FAKE, 2, 28, 4,
                                         96, 16, 0.1, _lib.BF16, None, 0,
                                         None) == _lib.ERR_SHAPE      # head_dim 96
    assert L.mlxq_paged_attention_prefill(FAKE, FAKE, 65, FAKE, FAKE, FAKE, 4, FAKE, FAKE, 2,
                                          28, 4, 128, 16, 0.1, _lib.BF16,
                                          None) == _lib.ERR_SHAPE
    assert L.mlxq_rope_kv_append(FAKE, 100, FAKE, FAKE, FAKE, FAKE, FAKE, 1, 28, 4, 128,
                                 1e6, _lib.BF16, None) == _lib.ERR_SHAPE  # ld too small
    assert L.mlxq_quantized_embedding(FAKE, 3, FAKE, FAKE, FAKE, FAKE, 10, 100, 64, 4,
                                      _lib.BF16, None) == _lib.ERR_SHAPE  # dim % group
    assert L.mlxq_paged_attention_workspace_size(8, 4, 64, 128) == 0      # one split of 64 keys
    assert L.mlxq_paged_attention_workspace_size(8, 4, 640, 128) > 0
    assert _lib.last_error()


def test_paged_gather_equals_dense():
    rng = np.random.default_rng(0)
    L, hkv, hd, page = 45, 2, 64, 16
    k = rng.standard_normal((L, hkv, hd)).astype(np.float32)
    bt = np.array([6, 2, 4], np.int32)
    pool = np.zeros((8, page, hkv, hd), np.float32)
    for j in range(L):
        pool[bt[j // page], j % page] = k[j]
    assert np.array_equal(D.gather_pages(pool, bt, L), k)


def test_rope_is_complex_rotation():
    rng = np.random.default_rng(1)
    x = rng.standard_normal((5, 3, 64)).astype(np.float32)
    pos = np.array([0, 1, 7, 100, 4095])
    y = D.rope(x, pos, 1e4, "float32")
    half = 32
    z = x[..., :half] + 1j * x[..., half:]
    ang = pos[:, None] * 1e4 ** (-2.0 * np.arange(half) / 64)
    zr = z * np.exp(1j * ang)[:, None, :]
    ref = np.concatenate([zr.real, zr.imag], axis=-1)
    assert np.abs(y - ref).max() < 1e-5
    assert np.array_equal(y[0], x[0])  # position 0 is the identity


def test_attention_causal_and_softmax():
    rng = np.random.default_rng(2)
    q = rng.standard_normal((4, 2, 8)).astype(np.float32)
    k = rng.standard_normal((6, 1, 8)).astype(np.float32)
    v = rng.standard_normal((6, 1, 8)).astype(np.float32)
    o = D.attention(q, k, v, np.array([0, 2, 4, 5]), 0.5, "float32")
    assert np.allclose(o[0, 0], v[0, 0], atol=1e-6)   # only key 0 is visible at position 0
    s = (q[3, 1] @ k[:, 0].T) * 0.5
    p = np.exp(s - s.max())
    p /= p.sum()
    assert np.allclose(o[3, 1], p @ v[:, 0], atol=1e-5)
