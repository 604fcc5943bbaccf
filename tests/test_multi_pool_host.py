"""Host side of the multi-device page pool (memopt_mdpool_*), on CPU: the
per-device FIFO free-lists, home-first allocation with spill to the device
with the most free blocks, errors, and the gather plan."""
from __future__ import annotations

import ctypes as C

import pytest

from memopt import _capi
from memopt.multi_pool import mdpool_plan


def _init(blocks):
    arr = (C.c_int * len(blocks))(*blocks)
    return _capi.lib().memopt_mdpool_init(C.c_int(len(blocks)), arr)


def _alloc(pref):
    d = C.c_int(-9)
    b = _capi.lib().memopt_mdpool_allocate(C.c_int(pref), C.byref(d))
    return d.value, b


def test_allocate_home_first_then_spill_to_most_free():
    lib = _capi.lib()
    assert _init([2, 3, 1]) == 0
    assert [_alloc(0) for _ in range(2)] == [(0, 0), (0, 1)]  # FIFO on the home device
    assert _alloc(0) == (1, 0)  # device 0 full: device 1 has the most free blocks
    assert _alloc(2) == (2, 0)
    assert _alloc(2) == (1, 1)  # device 2 full, device 1 (1 left)... has most
    assert _alloc(0) == (1, 2)
    assert _alloc(1)[1] == -1  # every device exhausted
    assert [lib.memopt_mdpool_free_count(d) for d in range(3)] == [0, 0, 0]
    assert lib.memopt_mdpool_free(C.c_int(1), C.c_int(1)) == 0
    assert lib.memopt_mdpool_free(C.c_int(1), C.c_int(1)) == -1  # already free
    assert lib.memopt_mdpool_free(C.c_int(1), C.c_int(7)) == -5  # out of range
    assert lib.memopt_mdpool_free(C.c_int(3), C.c_int(0)) == -5
    assert _alloc(0) == (1, 1)  # the freed block comes back
    assert _alloc(5)[1] == -5  # preferred device out of range


def test_ties_take_the_lowest_device_and_errors_without_init():
    lib = _capi.lib()
    assert _init([0, 2, 2]) == 0
    assert _alloc(0) == (1, 0)
    lib.memopt_mdpool_reset()
    assert _alloc(0)[1] == -2  # not initialized
    assert lib.memopt_mdpool_free_count(0) == -2
    assert _init([1, -1]) == -1
    arr = (C.c_int * 1)(1)
    assert lib.memopt_mdpool_init(C.c_int(0), arr) == -1


def test_gather_plan_groups_remote_pages_by_owner_and_dedupes():
    dev = [0, 2, 1, 0, 2, 1, 0, 2]
    blk = [5, 3, 4, -1, 3, 9, 6, 8]  # (2, 3) twice; a hole
    local, copies = mdpool_plan(dev, blk, home=0, staging_base=100, staging_capacity=10)
    # owners in device order (1 then 2), first appearance within each
    assert copies == [(1, 4, 100), (1, 9, 101), (2, 3, 102), (2, 8, 103)]
    assert local == [5, 102, 100, -1, 102, 101, 6, 103]
    # a different home device reads its own pages in place
    local1, copies1 = mdpool_plan(dev, blk, home=1, staging_base=50, staging_capacity=10)
    assert local1[2] == 4 and local1[5] == 9 and [c[0] for c in copies1] == [0, 0, 2, 2]
    with pytest.raises(_capi.MemoptError, match="staging"):
        mdpool_plan(dev, blk, home=0, staging_base=100, staging_capacity=3)
    assert mdpool_plan([], [], 0, 0, 0) == ([], [])


def _cpu_pool(blocks, staging=4, H=2, D=64, BS=16):
    import torch

    from memopt.multi_pool import MultiDevicePagePool
    from memopt.sharding import RankGroup

    def write_rows(k, v, slots):
        kp, vp = pool.tensors
        kp.view(-1, H, D)[slots.long()] = k
        vp.view(-1, H, D)[slots.long()] = v

    pool = MultiDevicePagePool(RankGroup(), blocks, staging, BS, H, D, device=torch.device("cpu"),
                               pack=lambda src, ids, out: out.copy_(src.index_select(0, ids.long())),
                               write_rows=write_rows, attend_fn=lambda *a: None)
    return pool


def test_single_rank_pool_bookkeeping_and_exhaustion():
    import torch

    pool = _cpu_pool(4)
    a = pool.add_sequence(0)
    b = pool.add_sequence(0)
    k = torch.randn(40, 2, 64).half()
    pool.append(a, k, k)  # 3 pages
    assert pool.length(a) == 40 and [p[0] for p in pool.pages(a)] == [0, 0, 0] and pool.free_count(0) == 1
    kp, _ = pool.tensors
    pg = pool.pages(a)
    assert torch.equal(kp[pg[2][1], :8], k[32:40])  # token t in page t // 16, slot t % 16
    with pytest.raises(MemoryError):
        pool.append(b, torch.randn(20, 2, 64).half(), torch.randn(20, 2, 64).half())  # needs 2 pages, 1 left
    assert pool.length(b) == 0 and pool.free_count(0) == 1  # the failed append took nothing
    pool.append(b, k[:16], k[:16])
    assert pool.free_count(0) == 0
    pool.free_sequence(a)
    assert pool.free_count(0) == 3
    with pytest.raises(ValueError):
        pool.add_sequence(1)  # a world of one rank
    with pytest.raises(ValueError):
        pool.append(b)  # the home rank must pass k and v
