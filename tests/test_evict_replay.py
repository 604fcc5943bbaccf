"""The evict_tokens threshold as a function of one order statistic, on CPU.

The reference's threshold (kv_cache.cu:714-870, restated by the oracle) is 32
bisection steps ``mid = fma(hi - lo, 0.5, lo)``; ``count(s >= mid) >= keep``
moves ``lo`` up, otherwise ``hi`` down.  ``count(s >= mid) >= keep`` holds
exactly when ``w >= mid``, w being the keep-th largest non-NaN score (never
when fewer than keep scores are non-NaN), so the steps can be replayed from w
alone.  The device kernel does that; this test checks the claim against the
oracle's own 32-step threshold on rows with ties, signed zeros, infinities,
NaNs, huge scores and the reference's sink boost.  In float32, (hi - lo) * 0.5
is exact, so the unfused ``lo + (hi - lo) * 0.5`` below is the fused value.
"""
from __future__ import annotations

import numpy as np
import pytest

import oracle as O

F = np.float32


def replay_threshold(s: np.ndarray, retain_ratio: float, sinks: int) -> np.float32:
    s = s.astype(F).copy()
    L = s.size
    s[: min(max(sinks, 0), L)] = F(1e38)
    keep = max(1, min(L, int(np.ceil(F(retain_ratio) * F(L)))))
    cmp = s[~np.isnan(s)]
    gmin = F(min(F(1e38), cmp.min())) if cmp.size else F(1e38)
    gmax = F(max(F(-1e38), cmp.max())) if cmp.size else F(-1e38)
    if gmin >= gmax:
        return F(gmin - F(1.0))
    w = F(np.sort(cmp)[::-1][keep - 1]) if cmp.size >= keep else F(np.nan)
    lo, hi = gmin, gmax
    with np.errstate(invalid="ignore", over="ignore"):
        for _ in range(32):
            mid = F(lo + F(F(hi - lo) * F(0.5)))
            if w >= mid:
                lo = mid
            else:
                hi = mid
    return lo


def _rows(seed: int, L: int, kind: str) -> np.ndarray:
    rng = np.random.default_rng(seed)
    if kind == "lognormal":
        return rng.lognormal(0, 1, L).astype(F)
    if kind == "ties":
        return rng.integers(-3, 4, L).astype(F)
    if kind == "signed_zero":
        x = -rng.integers(0, 3, L).astype(F)
        x[rng.random(L) < 0.4] = -0.0
        return x
    if kind == "specials":
        x = rng.standard_normal(L).astype(F)
        m = rng.random(L)
        x[m < 0.05] = np.nan
        x[(m >= 0.05) & (m < 0.07)] = np.inf
        x[(m >= 0.07) & (m < 0.09)] = -np.inf
        x[(m >= 0.09) & (m < 0.1)] = 3e38
        return x
    if kind == "neg_inf_only_low":  # a -inf with a finite maximum: the first midpoint is NaN
        x = rng.standard_normal(L).astype(F)
        x[0] = -np.inf
        return x
    if kind == "mostly_nan":
        x = rng.standard_normal(L).astype(F)
        x[rng.random(L) < 0.9] = np.nan
        return x
    return rng.standard_normal(L).astype(F)


KINDS = ["lognormal", "ties", "signed_zero", "specials", "neg_inf_only_low", "mostly_nan", "normal"]


@pytest.mark.parametrize("kind", KINDS)
@pytest.mark.parametrize("sinks", [0, 4])
def test_replay_from_the_keep_th_largest_matches_the_bisection(kind, sinks):
    for trial, (L, r) in enumerate([(1, 0.5), (7, 0.3), (100, 0.75), (777, 0.01), (1024, 1.0), (3001, 0.6)]):
        s = _rows(trial * 31 + len(kind), L, kind)
        sc = s.reshape(1, 1, L)
        bt = np.zeros((1, L), np.int32)
        kp = np.zeros((1, 1, 1, 32), np.float16)
        _, _, thr = O.evict_tokens(sc, bt, np.zeros(1, np.int32), kp, kp.copy(), r, sinks)
        got = replay_threshold(s, r, sinks)
        ref = F(thr[0, 0])
        assert (np.isnan(got) and np.isnan(ref)) or got.view(np.uint32) == ref.view(np.uint32), (kind, L, r, got, ref)
