"""Multi-rank host logic on CPU (gloo, world_size 2): sequence sharding, the
max-over-ranks timing reduction and the whole-job rate that bench.py reports,
and sharded decode reproducing the unsharded result."""
from __future__ import annotations

import os
import socket
import subprocess
import sys

import numpy as np
import pytest

import oracle as O
from memopt.sharding import job_rate, shard_range

HERE = os.path.dirname(os.path.abspath(__file__))


def test_shard_range_partitions():
    for s in range(0, 23):
        for n in range(1, 9):
            ranges = [shard_range(s, n, r) for r in range(n)]
            covered = [i for a, b in ranges for i in range(a, b)]
            assert covered == list(range(s))
            sizes = [b - a for a, b in ranges]
            assert max(sizes) - min(sizes) <= 1
    with pytest.raises(ValueError):
        shard_range(4, 2, 2)


def test_job_rate_uses_slowest_rank():
    assert job_rate(100.0, 10.0, 4) == pytest.approx(40000.0)
    with pytest.raises(ValueError):
        job_rate(1.0, 0.0, 1)


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def test_two_rank_gloo_sharded_decode(tmp_path):
    world, port = 2, _free_port()
    procs = []
    for r in range(world):
        env = dict(os.environ, MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), WORLD_SIZE=str(world),
                   RANK=str(r), LOCAL_RANK=str(r))
        procs.append(subprocess.Popen([sys.executable, os.path.join(HERE, "multirank_worker.py"), str(tmp_path)],
                                      env=env, stdout=subprocess.PIPE, stderr=subprocess.STDOUT))
    for p in procs:
        out, _ = p.communicate(timeout=240)
        assert p.returncode == 0, out.decode()[-2000:]
    sys.path.insert(0, HERE)
    import multirank_worker as W

    q, kp, vp, bt, ctx = W.global_workload()
    ref = O.paged_attention_f16(q, kp, vp, bt, ctx, 96, 96)
    got = np.zeros_like(ref)
    seen = []
    for r in range(world):
        z = np.load(tmp_path / f"rank{r}.npz")
        a, b = int(z["start"]), int(z["stop"])
        got[a:b] = z["out"]
        seen.extend(range(a, b))
        assert float(z["mx"]) == 10.0 + world - 1  # max over ranks reached every rank
    assert sorted(seen) == list(range(W.S))
    assert np.array_equal(got, ref)


def _spawn(worker: str, world: int, args, extra_env=None, timeout=240):
    port = _free_port()
    procs = []
    for r in range(world):
        env = dict(os.environ, MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), WORLD_SIZE=str(world),
                   RANK=str(r), LOCAL_RANK=str(r), **(extra_env or {}))
        procs.append(subprocess.Popen([sys.executable, os.path.join(HERE, worker), *map(str, args)],
                                      env=env, stdout=subprocess.PIPE, stderr=subprocess.STDOUT))
    try:
        for p in procs:
            out, _ = p.communicate(timeout=timeout)
            assert p.returncode == 0, out.decode()[-3000:]
    finally:
        for p in procs:  # a rank that failed or timed out must not outlive the test
            if p.poll() is None:
                p.kill()
                p.wait()


def check_head_sharded_evict(out_dir, world: int) -> None:
    """Every rank's outputs equal the oracle's decision on the rank-ordered
    partial sums, and its pool rows equal its head slice of the compacted pool."""
    sys.path.insert(0, HERE)
    import multirank_evict_worker as W

    sc, bt, ctx, kp, vp = W.global_workload()
    hs = W.H // world
    parts = np.stack([O.evict_topk_head_sum(sc[:, r * hs:(r + 1) * hs]) for r in range(world)])
    rbt, rctx, rkp, rvp = bt.copy(), ctx.copy(), kp.copy(), vp.copy()
    rk, rc, rf, rfc = O.evict_topk_compact_parts(parts, rbt, rctx, rkp, rvp, W.RETAIN, W.SINKS)
    assert 0 < rc.sum() < ctx.sum()  # the case evicts something
    for r in range(world):
        z = np.load(os.path.join(out_dir, f"rank{r}.npz"))
        assert (int(z["h0"]), int(z["h1"])) == (r * hs, (r + 1) * hs)
        for name, ref in (("kept", rk), ("cnt", rc), ("freed", rf), ("fcnt", rfc), ("bt", rbt), ("ctx", rctx)):
            assert np.array_equal(z[name], ref), (r, name)
        for b in range(W.S):
            for i in range(int(rc[b])):
                pg, pos = rbt[b, i // W.BS], i % W.BS
                assert np.array_equal(z["k"][pg, pos].view(np.uint16), rkp[pg, pos, r * hs:(r + 1) * hs].view(np.uint16))
                assert np.array_equal(z["v"][pg, pos].view(np.uint16), rvp[pg, pos, r * hs:(r + 1) * hs].view(np.uint16))


def test_two_rank_gloo_head_sharded_exact_eviction(tmp_path):
    _spawn("multirank_evict_worker.py", 2, [tmp_path, "gloo"])
    check_head_sharded_evict(tmp_path, 2)


def test_head_range_and_single_rank_gather():
    from memopt.sharding import RankGroup, head_range

    assert [head_range(32, 4, r) for r in range(4)] == [(0, 8), (8, 16), (16, 24), (24, 32)]
    with pytest.raises(ValueError):
        head_range(6, 4, 0)
    import torch

    t = torch.arange(6.0).reshape(2, 3)
    g = RankGroup()
    assert torch.equal(g.all_gather_rows(t), t[None])


def check_multi_pool(out_dir, world: int) -> None:
    """Each home rank's attention over its sequence (pages on both GPUs)
    equals the oracle over the sequence's rows; the page placement is the
    replicated allocator's (home first, spill to the GPU with most room)."""
    sys.path.insert(0, HERE)
    import multirank_pool_worker as W

    zs = [np.load(os.path.join(out_dir, f"rank{r}.npz")) for r in range(world)]
    for z in zs[1:]:  # identical replicas
        assert np.array_equal(z["pagesA"], zs[0]["pagesA"]) and np.array_equal(z["pagesB"], zs[0]["pagesB"])
        assert np.array_equal(z["free"], zs[0]["free"])
    pa, pb = zs[0]["pagesA"], zs[0]["pagesB"]
    assert [int(d) for d, _ in pa] == [0] * W.BLOCKS + [1, 1]  # A: 130 tokens, 9 pages, 2 spilled
    assert all(int(d) == 1 for d, _ in pb)
    assert list(zs[0]["free"]) == [0, W.BLOCKS - 2 - len(pb)]
    for r, name in ((0, "A"), (1, "B")):
        k, v = W.full_rows(name)
        L = k.shape[0]
        MB = (L + W.BS - 1) // W.BS
        kp = np.zeros((MB, W.BS, W.H, W.D), np.float16)
        vp = np.zeros_like(kp)
        kp.reshape(-1, W.H, W.D)[:L] = k
        vp.reshape(-1, W.H, W.D)[:L] = v
        ref = O.paged_attention_f16(W.query(name), kp, vp, np.arange(MB, dtype=np.int32)[None],
                                    np.array([L], np.int32), L, L)
        np.testing.assert_allclose(zs[r]["out"], ref, atol=2e-3, rtol=1e-2)


def test_two_rank_gloo_multi_device_pool(tmp_path):
    _spawn("multirank_pool_worker.py", 2, [tmp_path, "gloo"])
    check_multi_pool(tmp_path, 2)
