"""The exact top-k eviction restatement on small hand-checked cases (CPU)."""
from __future__ import annotations

import numpy as np

import oracle as O


def _pools(NB, BS, H, D):
    kp = np.arange(NB * BS * H * D, dtype=np.float32).reshape(NB, BS, H, D).astype(np.float16)
    return kp, -kp


def test_keep_count_sinks_ties_and_compaction():
    BS, H, D = 4, 2, 8
    kp, vp = _pools(6, BS, H, D)
    L = 10
    sc = np.zeros((1, H, L), np.float32)
    sc[0, 0] = [9, 0, 5, 5, 1, 5, 7, 0, 2, 5]
    bt = np.array([[3, 0, 5, -1]], np.int32)
    ctx = np.array([L], np.int32)
    k0, v0 = kp.copy(), vp.copy()
    kept, cnt, freed, fcnt = O.evict_topk_compact(sc, bt, ctx, kp, vp, 0.5, num_sink_tokens=2)
    # keep = ceil(0.5 * 10) = 5: sinks 0, 1; then 6 (7), then the first two 5s: 2, 3
    assert cnt[0] == 5 and kept[0, :5].tolist() == [0, 1, 2, 3, 6] and (kept[0, 5:] == -1).all()
    assert ctx[0] == 5 and bt[0].tolist() == [3, 0, -1, -1]
    assert fcnt[0] == 1 and freed[0].tolist() == [5, -1, -1, -1]
    old = [3, 0, 5]
    for i, t in enumerate([0, 1, 2, 3, 6]):
        np.testing.assert_array_equal(kp[bt[0, i // BS], i % BS], k0[old[t // BS], t % BS])
        np.testing.assert_array_equal(vp[bt[0, i // BS], i % BS], v0[old[t // BS], t % BS])


def test_holes_nan_and_empty():
    BS, H, D = 4, 1, 8
    kp, vp = _pools(8, BS, H, D)
    sc = np.array([[[1, 2, 3, 4, 9, 9, 9, 9, np.nan, 8, 0, 7]]], np.float32)
    bt = np.array([[2, -1, 4], [6, 7, 1]], np.int32)
    sc = np.concatenate([sc, np.zeros_like(sc)])
    ctx = np.array([12, 0], np.int32)
    kept, cnt, freed, fcnt = O.evict_topk_compact(sc, bt, ctx, kp, vp, 0.5, num_sink_tokens=0)
    # tokens 4..7 sit on a hole: 8 valid tokens, keep 4: 9 (8), 11 (7), 3 (4), 2 (3); NaN ranks lowest
    assert kept[0, :4].tolist() == [2, 3, 9, 11] and cnt[0] == 4
    assert bt[0].tolist() == [2, -1, -1] and freed[0, :fcnt[0]].tolist() == [4]
    assert cnt[1] == 0 and ctx[1] == 0 and bt[1].tolist() == [-1, -1, -1] and sorted(freed[1, :3]) == [1, 6, 7]
