"""Generates the golden fixtures in this directory.

  kat.json     hand-derived known answers. Every expected value is written as
               a literal below and derived in the comment beside it from the
               layout / algorithm statement alone (no oracle is run to make it).
  seeded.npz   seeded random cases (numpy default_rng) with the C oracle's
               outputs, used as regression vectors for the oracle and as
               parity inputs for the GPU tests.

No golden vectors exist in the reference for this path (its tests build no
quantized layer, and MLX itself cannot be installed here), so these pin the
oracle to the stated MLX algorithm; they do not pin it to MLX's binaries.

Run: python tests/golden/make_golden.py
"""
from __future__ import annotations

import json
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, ROOT)

from oracle import coracle, oracle_np  # noqa: E402


def kat():
    k = {}
    # ---- packing: code k of a row at bits [bits*(k%(32/bits)), +bits) of word k/(32/bits)
    k["pack"] = [
        # codes 0..15 (4-bit): nibble j of word 0 holds code j -> 0x76543210, word 1 0xFEDCBA98
        {"bits": 4, "codes": list(range(16)), "words": [0x76543210, 0xFEDCBA98]},
        # bytes, lowest index in the least-significant byte
        {"bits": 8, "codes": [0x01, 0x02, 0x03, 0x04, 0xFF, 0x00, 0x80, 0x7F],
         "words": [0x04030201, 0x7F8000FF]},
        # 2-bit: codes 0,1,2,3 repeated -> each byte 0b11100100 = 0xE4
        {"bits": 2, "codes": [0, 1, 2, 3] * 4, "words": [0xE4E4E4E4]},
        # a single high code in the last slot
        {"bits": 4, "codes": [0] * 7 + [15], "words": [0xF0000000]},
    ]
    # ---- dequantize with exactly representable bf16 scale/bias: out = s*q + b exactly
    k["dequant_bf16"] = [
        # s = 0.5 (0x3F00), b = -1.0 (0xBF80), codes 0..7 -> -1, -0.5, 0, 0.5, 1, 1.5, 2, 2.5
        {"bits": 4, "group_size": 32, "scale": 0x3F00, "bias": 0xBF80,
         "codes": list(range(8)) + [0] * 24,
         "out": [0xBF80, 0xBF00, 0x0000, 0x3F00, 0x3F80, 0x3FC0, 0x4000, 0x4020] + [0xBF80] * 24},
        # negative scale (MLX stores a negative scale when max|w| is the maximum):
        # s = -1.0 (0xBF80), b = 15.0 (0x4170): q=0 -> 15, q=15 -> 0, q=5 -> 10 (0x4120)
        {"bits": 4, "group_size": 32, "scale": 0xBF80, "bias": 0x4170,
         "codes": [0, 15, 5] + [0] * 29,
         "out": [0x4170, 0x0000, 0x4120] + [0x4170] * 29},
        # 8-bit: s = 2^-7 (0x3C00), b = 0: q = 255 -> 255/128 = 1.9921875 (0x3FFF exactly)
        {"bits": 8, "group_size": 32, "scale": 0x3C00, "bias": 0x0000,
         "codes": [255, 128, 1] + [0] * 29,
         "out": [0x3FFF, 0x3F80, 0x3C00] + [0x0000] * 29},
        # one rounding per operation: s = 1.0078125 (0x3F81), q = 3, b = -2^-7 (0xBC00).
        # s*q = 3.0234375 is halfway between bf16 3.015625 (mantissa 65) and 3.03125 (66);
        # RNE gives 3.03125, then + b = 3.0234375 is again a tie and rounds to 3.03125
        # (0x4042). A fused s*q+b would give 3.015625 (0x4041). q = 0 -> b = 0xBC00.
        {"bits": 4, "group_size": 32, "scale": 0x3F81, "bias": 0xBC00,
         "codes": [3] + [0] * 31, "out": [0x4042] + [0xBC00] * 31},
    ]
    # ---- quantize (MLX affine): groups chosen so the answer follows by hand
    k["quantize_f32"] = [
        # values 0..15 then 15s: w_max=15 dominates -> scale=-(15-0)/15=-1, edge=15,
        # q0=rint(15/-1)=-15, scale=15/-15=-1, bias=15; code = rint((v-15)/-1) = 15-v
        {"bits": 4, "group_size": 32, "w": [float(v) for v in range(16)] + [15.0] * 16,
         "codes": [15 - v for v in range(16)] + [0] * 16, "scale": -1.0, "bias": 15.0},
        # values -8..7 twice: |w_min|=8 > 7 -> scale=15/15=1, edge=-8, q0=-8, scale=1, bias=-8;
        # code = v + 8
        {"bits": 4, "group_size": 32, "w": [float(v) for v in range(-8, 8)] * 2,
         "codes": [v + 8 for v in range(-8, 8)] * 2, "scale": 1.0, "bias": -8.0},
        # all zero: scale=max(0,1e-7) negated (w_max not dominated) = -1e-7, edge=0 -> q0=0,
        # bias=0; codes 0; stored scale = float32(-1e-7)
        {"bits": 4, "group_size": 32, "w": [0.0] * 32, "codes": [0] * 32,
         "scale": float(np.float32(-1e-7)), "bias": 0.0},
        # 8-bit, values 0..255 step 2 then 254s... use 0,2,...,62 (32 values): w_max=62 ->
        # scale=-(62/255), edge=62, q0=rint(62/-(62/255))=-255, scale=62/-255, bias=62;
        # code(v) = rint((v-62)/(62/-255)) = rint((62-v)*255/62)
        {"bits": 8, "group_size": 32, "w": [float(2 * i) for i in range(32)],
         "codes": [int(np.rint(np.float32(np.float32(2 * i) - np.float32(62.0)) /
                               np.float32(np.float32(62.0) / np.float32(-255.0))))
                   for i in range(32)],
         "scale": float(np.float32(62.0) / np.float32(-255.0)), "bias": 62.0},
    ]
    return k


def seeded():
    rng = np.random.default_rng(0)
    out = {}
    cases = [
        ("bf16_b4_g64", "bfloat16", 4, 64, 5, 96, 512),
        ("bf16_b8_g64", "bfloat16", 8, 64, 3, 80, 256),
        ("bf16_b4_g32", "bfloat16", 4, 32, 9, 40, 128),
        ("bf16_b4_g128", "bfloat16", 4, 128, 2, 64, 384),
        ("f16_b4_g64", "float16", 4, 64, 4, 48, 192),
        ("f16_b8_g128", "float16", 8, 128, 17, 33, 256),
    ]
    for name, dt, bits, gs, M, N, K in cases:
        w = (rng.standard_normal((N, K)) * 0.02).astype(np.float32)
        x = rng.standard_normal((M, K)).astype(np.float32)
        wd = oracle_np.from_f32(w, dt)
        xd = oracle_np.from_f32(x, dt)
        wq, s, b = coracle.quantize(wd, dt, gs, bits)
        y = coracle.quantized_matmul(xd, wq, s, b, dt, gs, bits)
        dq = coracle.dequantize(wq, s, b, dt, gs, bits)
        for key, val in (("w", wd), ("x", xd), ("wq", wq), ("s", s), ("b", b), ("y", y),
                         ("dq", dq)):
            out[f"{name}/{key}"] = val
        out[f"{name}/meta"] = np.array([bits, gs, M, N, K], np.int64)
    # one gather_qmm case: E=6 experts, N=64, K=256, 5 tokens routed top-2
    E, N, K, T, topk = 6, 64, 256, 5, 2
    w = (rng.standard_normal((E * N, K)) * 0.02).astype(np.float32)
    wq, s, b = coracle.quantize(oracle_np.from_f32(w, "bfloat16"), "bfloat16", 64, 4)
    wq, s, b = wq.reshape(E, N, -1), s.reshape(E, N, -1), b.reshape(E, N, -1)
    x = oracle_np.from_f32(rng.standard_normal((T, 1, K)).astype(np.float32), "bfloat16")
    rhs = np.stack([rng.choice(E, topk, replace=False) for _ in range(T)]).astype(np.int32)
    y = coracle.gather_qmm(x, wq, s, b, rhs.reshape(-1), "bfloat16", 64, 4, lhs=None,
                           lhs_div=topk)
    out.update({"gather/x": x, "gather/wq": wq, "gather/s": s, "gather/b": b,
                "gather/rhs": rhs, "gather/y": y})
    return out


def main():
    with open(os.path.join(HERE, "kat.json"), "w") as f:
        json.dump(kat(), f, indent=1)
    np.savez_compressed(os.path.join(HERE, "seeded.npz"), **seeded())
    print("wrote kat.json and seeded.npz")


if __name__ == "__main__":
    main()
