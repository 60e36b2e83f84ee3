"""Error bound of the erf-GELU used by the FFN-in GEMM epilogue.

Re-evaluates, in numpy float32, the steps of gelu2 in
techjam-2026-track3_b200/csrc/gemm_tcgen05.cu (constants read from that
file): erf from Abramowitz & Stegun 7.1.26, Phi(x) = 1 - erfc/2 or erfc/2 by
sign, GELU = x * Phi(x); and checks it against float64 x * (1 + erf(x/sqrt 2)) / 2
(the reference's exact GELU, torch.nn.functional.gelu(approximate="none")).
"""
from __future__ import annotations

import math
import re
from pathlib import Path

import numpy as np

SRC = Path(__file__).resolve().parents[1] / "techjam-2026-track3_b200" / "csrc" / "gemm_tcgen05.cu"


def _constants():
    body = SRC.read_text()
    body = body[body.index("float2 gelu2(float2 x)"):]
    body = body[: body.index("\n}\n")]
    vals = dict(re.findall(r"(k(?:P|A[1-5]))\s*=\s*(-?[0-9.]+)f", body))
    assert set(vals) == {"kP", "kA1", "kA2", "kA3", "kA4", "kA5"}, vals
    return {k: np.float32(float(v)) for k, v in vals.items()}


def _gelu_kernel_steps(x: np.ndarray) -> np.ndarray:
    c = _constants()
    f = np.float32
    x = x.astype(f)
    z = (np.abs(x) * f(0.70710678118654752)).astype(f)
    t = (f(1) / (z * c["kP"] + f(1)).astype(f)).astype(f)
    q = c["kA5"]
    for k in ("kA4", "kA3", "kA2", "kA1"):
        q = (q * t + c[k]).astype(f)
    q = (q * t).astype(f)
    e = np.exp2(((z * z).astype(f) * f(-1.4426950408889634)).astype(f)).astype(f)
    hc = ((q * e).astype(f) * f(0.5)).astype(f)
    phi = np.where(x >= 0, f(1) - hc, hc).astype(f)
    return (x * phi).astype(f)


def _gelu_exact(x: np.ndarray) -> np.ndarray:
    erf = np.vectorize(math.erf)
    xd = x.astype(np.float64)
    return 0.5 * xd * (1.0 + erf(xd / math.sqrt(2.0)))


def test_gelu_absolute_error_below_fp16_resolution():
    x = np.concatenate([np.linspace(-12.0, 12.0, 200_001, dtype=np.float32),
                        np.random.default_rng(0).standard_normal(100_000).astype(np.float32) * 3])
    got = _gelu_kernel_steps(x).astype(np.float64)
    ref = _gelu_exact(x)
    err = np.abs(got - ref)
    assert err.max() < 1e-6, err.max()
    big = np.abs(ref) > 1e-3
    # fp16 output rounding alone is up to 2^-11 relative.
    assert (err[big] / np.abs(ref[big])).max() < 2.5e-4


def test_gelu_limits():
    x = np.array([0.0, -0.0, 40.0, -40.0, 1e-30], dtype=np.float32)
    got = _gelu_kernel_steps(x)
    assert got[0] == 0 and got[1] == 0 and got[2] == 40.0 and got[3] == 0 and abs(got[4]) < 1e-29
