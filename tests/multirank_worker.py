"""One rank of the CPU multi-rank tests (gloo): run by tests/test_multirank.py.

Argument: a scratch directory.  The rank joins the gloo group from the
torchrun-style environment, checks the max-over-ranks reduction, decodes its
shard of a seeded paged fp16 workload with the oracle (its own pool holding
only its sequences' pages, as one GPU would) and writes its result to
<dir>/rank<r>.npz.
"""
from __future__ import annotations

import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(HERE)
for p in (os.path.join(REPO, "memopt-transformer-runtime_b200"), os.path.join(REPO, "oracle")):
    sys.path.insert(0, p)

from memopt.sharding import RankGroup, dist_env, shard_range  # noqa: E402
import oracle as O  # noqa: E402

S, H, D, BS, MB = 5, 2, 64, 16, 6


def global_workload(seed: int = 17):
    rng = np.random.default_rng(seed)
    nb = S * MB
    bt = rng.permutation(nb).astype(np.int32).reshape(S, MB)
    kp = rng.standard_normal((nb, BS, H, D)).astype(np.float16)
    vp = rng.standard_normal((nb, BS, H, D)).astype(np.float16)
    q = rng.standard_normal((S, 1, H, D)).astype(np.float16)
    ctx = np.array([96, 1, 50, 80, 17], np.int32)
    return q, kp, vp, bt, ctx


def main() -> None:
    out_dir = sys.argv[1]
    world, rank, _ = dist_env()
    group = RankGroup.init("gloo")
    assert group.world_size == world and group.rank == rank
    mx = group.max(10.0 + rank)
    q, kp, vp, bt, ctx = global_workload()
    start, stop = shard_range(S, world, rank)
    # This rank's pool holds only its sequences' pages, renumbered 0..n-1.
    pages = bt[start:stop].reshape(-1)
    local_bt = np.arange(pages.size, dtype=np.int32).reshape(stop - start, MB)
    out = O.paged_attention_f16(q[start:stop], kp[pages], vp[pages], local_bt, ctx[start:stop], 96, 96)
    group.barrier()
    group.destroy()
    np.savez(os.path.join(out_dir, f"rank{rank}.npz"), out=out, start=start, stop=stop, mx=mx)


if __name__ == "__main__":
    main()
