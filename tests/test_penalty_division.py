"""The row kernel divides penalised logits by the repetition penalty through
fp64 (``div_by_row_const`` in ``csrc/ns_device.cuh``): q0 = RN64(x * inv),
q1 = RN64(q0 + RN64(x - q0 * rp) * inv) with each line one fused
multiply-add, inv = RN64(1 / rp), and the result RN32(q1) -- or RN32(q0) when
q0 is zero or not finite.  This restates that arithmetic exactly (fused
multiply-adds through rationals, each rounded once to fp64) and checks it
against IEEE fp32 division (the reference's ``logits / penalty``,
nanoserve/scheduler/sampler.py:37) bit for bit."""
from fractions import Fraction

import numpy as np


def _rn64(q: Fraction) -> float:
    return float(q)  # Python rounds a Fraction to the nearest double, ties to even


def _fma(a: float, b: float, c: float) -> float:
    return _rn64(Fraction(a) * Fraction(b) + Fraction(c))


def div_by_row_const(x: np.float32, rp: np.float32) -> np.float32:
    xd, rd = float(x), float(rp)
    inv = float("inf") if rd == 0.0 else (0.0 if np.isinf(rd) else _rn64(Fraction(1) / Fraction(rd)))
    if rd == 0.0 and np.signbit(rd):
        inv = float("-inf")
    if np.isnan(xd) or np.isnan(rd):
        return np.float32(np.nan)
    q0 = xd * inv  # a product of two doubles, rounded once
    if q0 == 0.0 or not np.isfinite(q0):
        return np.float32(q0)
    q1 = _fma(_fma(-q0, rd, xd), inv, q0)
    return np.float32(q1)


def _check(xs, rps):
    with np.errstate(divide="ignore", invalid="ignore", over="ignore", under="ignore"):
        for rp in rps:
            want = (xs / np.float32(rp)).astype(np.float32)
            for x, w in zip(xs, want):
                got = div_by_row_const(np.float32(x), np.float32(rp))
                assert got.view(np.uint32) == w.view(np.uint32) or (np.isnan(got) and np.isnan(w)), (x, rp, got, w)


def test_random_logits_and_penalties():
    rng = np.random.default_rng(7)
    xs = np.concatenate([
        rng.standard_normal(600).astype(np.float32) * np.float32(8),
        rng.uniform(0, 40, 300).astype(np.float32),
    ])
    rps = [1.1, 1.2, 1.3, 1.05, 0.9, 2.0, 1.7999999523162842, 3.141592653589793]
    _check(xs, [np.float32(r) for r in rps])


def test_every_exponent_and_edge_operands():
    rng = np.random.default_rng(11)
    bits = rng.integers(0, 2**23, 400, dtype=np.uint32) | (rng.integers(0, 255, 400, dtype=np.uint32) << 23)
    xs = np.concatenate([
        bits.view(np.float32),                                    # every exponent, normal and subnormal
        np.array([0.0, -0.0, np.inf, -np.inf, np.nan, 1e-45, 3e38, -3e38, 1.0, 2.0], dtype=np.float32),
    ])
    rps = [np.float32(v) for v in (1.1, 1e-30, 1e30, 3e-39, 0.0, -0.0, np.inf, -1.25, 1.0)]
    _check(xs, rps)
