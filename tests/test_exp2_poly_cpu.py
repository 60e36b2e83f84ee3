"""Error bound of the FMA-pipe 2^x used for part of the softmax exponentials.

Re-evaluates, in numpy float32, the exact steps of exp2_poly2 in
techjam-2026-track3_b200/csrc/common.cuh (constants read from that file):
round with the 1.5*2^23 trick, degree-4 polynomial for 2^r on [-1/2, 1/2],
integer add into the exponent field; and checks it against float64 exp2 over
the range the softmax feeds it (x <= 8 after the running-max subtraction).
"""
from __future__ import annotations

import re
from pathlib import Path

import numpy as np

SRC = Path(__file__).resolve().parents[1] / "techjam-2026-track3_b200" / "csrc" / "common.cuh"


def _coefficients():
    body = SRC.read_text()
    body = body[body.index("float2 exp2_poly2(float2 x)"):]
    body = body[: body.index("\n}\n")]
    body = body[body.index("float2 p = "):]
    consts = [float(c) for c in re.findall(r"make_float2\(([0-9.e-]+)f, \1f\)", body)]
    # p = c4; p = p*r + c3; ... ; p = p*r + c0
    assert len(consts) == 5, consts
    return [np.float32(c) for c in consts]


def _exp2_poly(x: np.ndarray) -> np.ndarray:
    c4, c3, c2, c1, c0 = _coefficients()
    x = np.maximum(x.astype(np.float32), np.float32(-126.0))
    k = np.float32(12582912.0)
    t = (x + k).astype(np.float32)
    nj = (t * np.float32(-1.0) + k).astype(np.float32)
    r = (x + nj).astype(np.float32)
    p = c4
    for c in (c3, c2, c1, c0):
        p = (p * r + c).astype(np.float32)
    bits = p.view(np.int32) + (t.view(np.int32) << 23)
    return bits.astype(np.int32).view(np.float32)


def test_exp2_poly_relative_error():
    x = np.concatenate([np.linspace(-125.0, 8.0, 2_000_001, dtype=np.float32),
                        np.float32(np.random.default_rng(0).uniform(-30, 8, 1_000_000))])
    got = _exp2_poly(x).astype(np.float64)
    ref = np.exp2(x.astype(np.float64))
    rel = np.abs(got - ref) / ref
    assert rel.max() < 4e-6, rel.max()


def test_exp2_poly_masked_and_tiny_inputs():
    x = np.array([-np.inf, -1e30, -200.0, -126.0], dtype=np.float32)
    got = _exp2_poly(x)
    assert np.all(np.isfinite(got)) and np.all(got >= 0) and np.all(got < 1.2e-38)
