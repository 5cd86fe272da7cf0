"""CPU tests of the oracle itself: hand-derived known answers, agreement of the
two independent restatements (C and numpy), round-trip bounds, and the
committed seeded fixtures."""
import json
import os

import numpy as np
import pytest

from oracle import coracle, oracle_np as O

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


@pytest.fixture(scope="module")
def kat():
    with open(os.path.join(GOLDEN, "kat.json")) as f:
        return json.load(f)


@pytest.fixture(scope="module")
def seeded():
    return np.load(os.path.join(GOLDEN, "seeded.npz"))


def test_pack_kat(kat):
    for case in kat["pack"]:
        codes = np.array([case["codes"]], np.uint32)
        words = O.pack(codes, case["bits"])
        assert words.tolist() == [case["words"]]
        assert O.unpack(words, case["bits"]).tolist() == [case["codes"]]


@pytest.mark.parametrize("impl", ["c", "np"])
def test_dequant_kat(kat, impl):
    for case in kat["dequant_bf16"]:
        bits, gs = case["bits"], case["group_size"]
        wq = O.pack(np.array([case["codes"]], np.uint32), bits)
        s = np.array([[case["scale"]]], np.uint16)
        b = np.array([[case["bias"]]], np.uint16)
        f = coracle.dequantize if impl == "c" else O.dequantize
        out = f(wq, s, b, "bfloat16", gs, bits)
        assert out.tolist() == [case["out"]], case


@pytest.mark.parametrize("impl", ["c", "np"])
def test_quantize_kat(kat, impl):
    for case in kat["quantize_f32"]:
        bits, gs = case["bits"], case["group_size"]
        w = np.array([case["w"]], np.float32)
        f = coracle.quantize if impl == "c" else O.quantize
        wq, s, b = f(w, "float32", gs, bits)
        assert O.unpack(wq, bits).tolist() == [case["codes"]], case
        assert s[0, 0] == np.float32(case["scale"])
        assert b[0, 0] == np.float32(case["bias"])


@pytest.mark.parametrize("dt", O.DTYPES)
@pytest.mark.parametrize("bits", [2, 4, 8])
@pytest.mark.parametrize("gs", [32, 64, 128])
def test_c_matches_numpy(dt, bits, gs):
    rng = np.random.default_rng(bits * 1000 + gs)
    w = O.from_f32((rng.standard_normal((23, 384)) * 0.02).astype(np.float32), dt)
    a = coracle.quantize(w, dt, gs, bits)
    b = O.quantize(w, dt, gs, bits)
    for x, y in zip(a, b):
        assert np.asarray(x).tobytes() == np.asarray(y).tobytes()
    d1 = coracle.dequantize(*a, dt, gs, bits)
    d2 = O.dequantize(*b, dt, gs, bits)
    assert np.asarray(d1).tobytes() == np.asarray(d2).tobytes()
    if bits in (4, 8) and dt != "float32":
        x = O.from_f32(rng.standard_normal((3, 384)).astype(np.float32), dt)
        y1 = O.to_f32(coracle.quantized_matmul(x, *a, dt, gs, bits), dt)
        y2 = O.to_f32(O.quantized_matmul(x, *b, dt, gs, bits), dt)
        assert np.abs(y1 - y2).max() <= 2e-2 * np.abs(y2).max()


@pytest.mark.parametrize("bits", [2, 4, 8])
def test_round_trip_bound(bits):
    """Elements inside the represented range are within |scale|/2; the far end of
    a group can be clipped by up to range/(2|q0|) because MLX re-derives the
    scale from the dominant endpoint, so the per-group bound is one step."""
    rng = np.random.default_rng(7)
    w = (rng.standard_normal((16, 256)) * 0.02).astype(np.float32)
    wq, s, b = coracle.quantize(w, "float32", 64, bits)
    d = coracle.dequantize(wq, s, b, "float32", 64, bits)
    err = np.abs(d - w).reshape(16, 4, 64).max(-1)
    bound = np.abs(s) * 1.0 + 1e-6
    assert (err <= bound).all()


def test_edge_groups():
    """Constant groups, a single outlier and negative-dominated groups quantize
    without NaN and reproduce their extreme exactly."""
    w = np.zeros((4, 64), np.float32)
    w[1] = 0.25
    w[2, 5] = -3.0
    w[3] = np.linspace(-0.1, 0.4, 64, dtype=np.float32)
    for f in (coracle.quantize, O.quantize):
        wq, s, b = f(w, "float32", 64, 4)
        d = coracle.dequantize(wq, s, b, "float32", 64, 4)
        assert np.isfinite(d).all()
        assert d[1, 0] == np.float32(0.25)      # constant group: edge stored exactly
        assert d[2, 5] == np.float32(-3.0)      # dominant endpoint exact
        assert d[3, -1] == np.float32(0.4)


def test_seeded_fixtures_reproduce(seeded):
    names = sorted({k.split("/")[0] for k in seeded.files if k.endswith("/meta")})
    assert names
    for n in names:
        bits, gs, M, N, K = (int(v) for v in seeded[f"{n}/meta"])
        dt = "float16" if n.startswith("f16") else "bfloat16"
        wq, s, b = coracle.quantize(seeded[f"{n}/w"], dt, gs, bits)
        assert wq.tobytes() == seeded[f"{n}/wq"].tobytes()
        assert s.tobytes() == seeded[f"{n}/s"].tobytes()
        assert b.tobytes() == seeded[f"{n}/b"].tobytes()
        y = coracle.quantized_matmul(seeded[f"{n}/x"], wq, s, b, dt, gs, bits)
        assert y.tobytes() == seeded[f"{n}/y"].tobytes()
        y_np = O.to_f32(O.quantized_matmul(seeded[f"{n}/x"], wq, s, b, dt, gs, bits), dt)
        ref = O.to_f32(seeded[f"{n}/y"], dt)
        assert np.abs(y_np - ref).max() <= 2e-2 * np.abs(ref).max()


def test_gather_fixture(seeded):
    x, wq, s, b = (seeded[f"gather/{k}"] for k in ("x", "wq", "s", "b"))
    rhs = seeded["gather/rhs"]
    y = coracle.gather_qmm(x, wq, s, b, rhs.reshape(-1), "bfloat16", 64, 4, lhs_div=rhs.shape[1])
    assert y.tobytes() == seeded["gather/y"].tobytes()
    y_np = O.gather_qmm(x, wq, s, b, rhs.reshape(-1), "bfloat16", 64, 4, lhs_div=rhs.shape[1])
    ref = O.to_f32(seeded["gather/y"], "bfloat16")
    assert np.abs(O.to_f32(y_np, "bfloat16") - ref).max() <= 2e-2 * np.abs(ref).max()


def test_bias_add_is_second_rounding():
    rng = np.random.default_rng(3)
    w = O.from_f32((rng.standard_normal((8, 64)) * 0.02).astype(np.float32), "bfloat16")
    x = O.from_f32(rng.standard_normal((2, 64)).astype(np.float32), "bfloat16")
    bias = O.from_f32(rng.standard_normal(8).astype(np.float32), "bfloat16")
    wq, s, b = coracle.quantize(w, "bfloat16", 64, 4)
    y0 = O.to_f32(coracle.quantized_matmul(x, wq, s, b, "bfloat16", 64, 4), "bfloat16")
    y1 = coracle.quantized_matmul(x, wq, s, b, "bfloat16", 64, 4, bias=bias)
    expect = O.round_to(y0 + O.to_f32(bias, "bfloat16")[None], "bfloat16")
    assert np.array_equal(O.to_f32(y1, "bfloat16"), expect)
