"""The INT4 quantiser's scale = absmax / 7 without a division (int4.cuh,
int4_quant8): q0 = m * fp32(1/7), q = fma(fma(-q0, 7, m), fp32(1/7), q0) must
equal the IEEE fp32 quotient for every value m it can see, i.e. every positive
finite fp16 value (m is the max of |fp16| inputs).  Checked exhaustively here
with exact rational arithmetic for the fma roundings."""
from __future__ import annotations

from fractions import Fraction

import numpy as np


def _rn32(x: Fraction) -> np.float32:
    """Correctly rounded (ties to even) float32 of a rational."""
    g = np.float32(float(x))
    best = None
    for c in (np.nextafter(g, np.float32(-np.inf)), g, np.nextafter(g, np.float32(np.inf))):
        d = abs(Fraction(float(c)) - x)
        even = (int(np.float32(c).view(np.uint32)) & 1) == 0
        if best is None or d < best[0] or (d == best[0] and even):
            best = (d, np.float32(c))
    return best[1]


def _fma32(a, b, c) -> np.float32:
    return _rn32(Fraction(float(a)) * Fraction(float(b)) + Fraction(float(c)))


def test_scale_without_division_matches_ieee_for_all_fp16():
    r7 = np.float32(1.0) / np.float32(7.0)
    assert r7 == np.float32(0.142857149)
    m = np.arange(1, 0x7C00, dtype=np.uint16).view(np.float16).astype(np.float32)
    ref = m / np.float32(7.0)
    q0 = (m * r7).astype(np.float32)
    bad = []
    for i in range(m.size):
        res = _fma32(-q0[i], np.float32(7.0), m[i])
        q = _fma32(res, r7, q0[i])
        if q != ref[i]:
            bad.append(float(m[i]))
    assert not bad, bad[:5]
