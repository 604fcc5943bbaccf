"""Host logic of the incremental paged cache: page table bookkeeping against
a fake FIFO allocator, and the scheduler-policy decisions (CPU only)."""
from __future__ import annotations

import pytest

from memopt.kv_cache import PagedKVCache, PageTable
from memopt.scheduler import MemoryScheduler, SchedulerConfig


class FifoPool:
    def __init__(self, n):
        self.free = list(range(n))

    def alloc(self):
        return self.free.pop(0) if self.free else -1

    def release(self, p):
        self.free.append(p)


def test_page_table_slots_and_growth():
    pool = FifoPool(8)
    t = PageTable(4, pool.alloc, pool.release)
    a, b = t.add_sequence(), t.add_sequence()
    assert t.reserve(a, 6) == [0, 1, 2, 3, 4, 5]          # pages 0, 1
    assert t.reserve(b, 1) == [8]                           # page 2
    assert t.reserve(a, 3) == [6, 7, 12]                    # page 1 fills, page 3 opens
    assert t.pages(a) == [0, 1, 3] and t.length(a) == 9
    assert t.block_table([a, b]) == [[0, 1, 3], [2, -1, -1]]
    assert t.block_table([b], max_blocks=2) == [[2, -1]]
    t.free_sequence(a)
    assert pool.free[-3:] == [0, 1, 3] and a not in t


def test_page_table_exhaustion_rolls_back():
    pool = FifoPool(2)
    t = PageTable(16, pool.alloc, pool.release)
    s = t.add_sequence()
    t.reserve(s, 16)
    with pytest.raises(MemoryError):
        t.reserve(s, 40)  # needs 3 more pages, only 1 left
    assert t.length(s) == 16 and t.pages(s) == [0] and pool.free == [1]
    with pytest.raises(ValueError):
        t.reserve(s, -1)


class StubCache(PagedKVCache):
    """The policy logic of PagedKVCache with its data path recorded."""

    def __init__(self, fmt="fp16"):  # noqa: D107 - no pool
        self.fmt = fmt
        self.eviction = "reference"
        self.calls = []
        self._applied = (1.0, fmt == "int4")

    @property
    def kv_format(self):
        return self.fmt

    def token_scores(self, q, sids):
        self.calls.append("scores")
        return "S"

    def evict(self, sids, scores, retain_ratio, num_sink_tokens=4):
        self.calls.append(("evict", retain_ratio, num_sink_tokens))
        return "evicted"

    def to_int4(self):
        self.calls.append("int4")
        self.fmt = "int4"


def test_apply_policy_follows_the_scheduler_once_per_change():
    util = {"v": 0.2}
    sched = MemoryScheduler(SchedulerConfig(drop_retain_ratio=0.5), sampler=lambda: util["v"])
    cache = StubCache()
    sched.adjust_policy()
    assert cache.apply_policy(sched, q="q", sids=[0]) is None and cache.calls == []
    util["v"] = 0.99
    sched.adjust_policy()
    assert cache.apply_policy(sched, q="q", sids=[0], num_sink_tokens=2) == "evicted"
    assert cache.calls == ["scores", ("evict", 0.5, 2), "int4"]
    cache.calls.clear()
    assert cache.apply_policy(sched, q="q", sids=[0]) is None and cache.calls == []  # unchanged policy
    util["v"] = 0.1
    sched.adjust_policy()
    cache.apply_policy(sched, q="q", sids=[0])
    assert cache.calls == [] and cache.kv_format == "int4"  # quantised tokens stay INT4


def test_page_table_compact_frees_tail_pages():
    pool = FifoPool(6)
    t = PageTable(4, pool.alloc, pool.release)
    s = t.add_sequence()
    t.reserve(s, 15)  # pages 0..3
    assert t.compact(s, 6) == [2, 3]
    assert t.pages(s) == [0, 1] and t.length(s) == 6 and pool.free == [4, 5, 2, 3]
    assert t.reserve(s, 3) == [6, 7, 16]  # continues after the compacted tokens
    with pytest.raises(ValueError):
        t.compact(s, 100)
