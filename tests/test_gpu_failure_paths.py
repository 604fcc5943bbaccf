"""Failure paths of the bounded device waits, made without a GPU fault.

The in-place row movers of the exact top-k compaction wait, with a bound, for
the rows at their destinations to be read.  A test hook withholds every
"read" flag (a flag that nothing sets) and shortens the bound, so each wait
on one runs out: the call must report MEMOPT_ERR_TIMEOUT through
memopt_evict_topk_status, no kept row may have been overwritten before it
was read, and the next normal call on the same buffers must succeed.
"""
from __future__ import annotations

import numpy as np
import pytest
import torch

import capi
import oracle as O

pytestmark = pytest.mark.gpu
DEV = "cuda"
TIMEOUT = -7  # MEMOPT_ERR_TIMEOUT


def _case(S, H, L, BS, D, seed):
    rng = np.random.default_rng(seed)
    MB = (L + BS - 1) // BS
    NB = S * MB + 3
    bt = rng.permutation(NB)[: S * MB].astype(np.int32).reshape(S, MB)
    sc = rng.lognormal(0.0, 1.0, (S, H, L)).astype(np.float32)
    kp = rng.standard_normal((NB, BS, H, D)).astype(np.float16)
    vp = rng.standard_normal((NB, BS, H, D)).astype(np.float16)
    return sc, bt, kp, vp


@pytest.fixture
def hooks():
    capi.evict_topk_set_test_hooks(4096, True)
    try:
        yield
    finally:
        capi.evict_topk_set_test_hooks(0, False)


def _sources_intact(kept, cnt, bt_old, BS, before, after):
    for b in range(kept.shape[0]):
        for i in range(int(cnt[b])):
            t = int(kept[b, i])
            pg, pos = bt_old[b, t // BS], t % BS
            assert np.array_equal(before[pg, pos].view(np.uint16), after[pg, pos].view(np.uint16)), (b, i, t)


def test_fp16_mover_gives_up_reports_and_overwrites_nothing(hooks):
    S, H, L, BS, D = 2, 4, 700, 16, 64
    sc, bt, kp, vp = _case(S, H, L, BS, D, 1)
    ctx = np.full(S, L, np.int32)
    gk, gv = torch.from_numpy(kp).to(DEV), torch.from_numpy(vp).to(DEV)
    gbt, gctx = torch.from_numpy(bt).to(DEV), torch.from_numpy(ctx).to(DEV)
    status = []
    kept, cnt, _, _ = capi.evict_topk_compact(torch.from_numpy(sc).to(DEV), gbt, gctx, gk, gv, 0.5, 4, status=status)
    assert status == [TIMEOUT]
    assert b"gave up" in capi.lib().memopt_last_error()
    k_, c_ = kept.cpu().numpy(), cnt.cpu().numpy()
    _sources_intact(k_, c_, bt, BS, kp, gk.cpu().numpy())
    _sources_intact(k_, c_, bt, BS, vp, gv.cpu().numpy())


def test_int4_mover_gives_up_reports_and_overwrites_nothing(hooks):
    S, H, L, BS, D = 2, 4, 600, 16, 128
    sc, bt, kp, vp = _case(S, H, L, BS, D, 2)
    NB = kp.shape[0]
    T = NB * BS
    pages = torch.zeros(NB, H, capi.int4_page_bytes(BS, D), dtype=torch.uint8, device=DEV)
    capi.write_cache_int4(torch.from_numpy(kp.reshape(T, H, D)).to(DEV), torch.from_numpy(vp.reshape(T, H, D)).to(DEV),
                          torch.from_numpy(np.arange(T, dtype=np.int32)).to(DEV), pages, BS)
    before = [np.ascontiguousarray(a) for a in O.int4_views(pages.cpu().numpy(), BS, D)]
    gbt = torch.from_numpy(bt).to(DEV)
    gctx = torch.full((S,), L, dtype=torch.int32, device=DEV)
    status = []
    kept, cnt, _, _ = capi.evict_topk_compact_int4(torch.from_numpy(sc).to(DEV), gbt, gctx, pages, BS, D, 0.5, 4,
                                                   status=status)
    assert status == [TIMEOUT]
    after = O.int4_views(pages.cpu().numpy(), BS, D)
    k_, c_ = kept.cpu().numpy(), cnt.cpu().numpy()
    for b in range(S):
        for i in range(int(c_[b])):
            t = int(k_[b, i])
            pg, pos = bt[b, t // BS], t % BS
            for x, y in zip(before, after):
                assert np.array_equal(x[pg, :, pos].view(np.uint8), y[pg, :, pos].view(np.uint8))


def test_timeout_surfaces_as_python_error_then_recovers():
    import memopt_C

    H, D, BS, L = 2, 64, 16, 400
    memopt_C.init_pool(64, BS, H, D)
    kp, vp = memopt_C.get_pool_tensors()
    kp.normal_()
    vp.normal_()
    bt = torch.arange(25, dtype=torch.int32, device=DEV).reshape(1, 25)
    sc = torch.rand(1, H, L, device=DEV)
    capi.evict_topk_set_test_hooks(4096, True)
    try:
        with pytest.raises(RuntimeError, match="gave up"):
            memopt_C.evict_topk_compact(sc, bt.clone(), torch.full((1,), L, dtype=torch.int32, device=DEV), 0.5, 4)
    finally:
        capi.evict_topk_set_test_hooks(0, False)
    # the hooks are off again: a normal call on the same pool succeeds
    kept, cnt, _, _ = memopt_C.evict_topk_compact(sc, bt.clone(), torch.full((1,), L, dtype=torch.int32, device=DEV),
                                                  0.5, 4)
    assert int(cnt.item()) == 200
