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
