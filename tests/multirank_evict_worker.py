"""One rank of the head-sharded exact eviction tests.

Arguments: a scratch directory and a backend ("gloo" or "nccl").  Every rank
holds one head shard of the same seeded sequences (scores and pool rows of
its heads, identical block tables), runs
``memopt.sharding.evict_exact_head_sharded`` and writes its outputs and its
compacted pool rows to <dir>/rank<r>.npz.

* gloo (CPU, run by tests/test_multirank.py): the operators are a stand-in
  built on the oracle, so the test covers the host logic (the partial rows
  reach every rank in rank order, one decision, in-place updates).
* nccl (one GPU per rank, run by tests/test_gpu_multigpu.py): the operators
  are ``memopt_C`` on this rank's pool; the exchange is an NCCL all-gather.
"""
from __future__ import annotations

import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(HERE)
for p in (os.path.join(REPO, "memopt-transformer-runtime_b200"), os.path.join(REPO, "oracle")):
    sys.path.insert(0, p)

import torch  # noqa: E402

from memopt.sharding import RankGroup, dist_env, evict_exact_head_sharded, head_range  # noqa: E402

S, H, D, BS, L = 3, 4, 64, 16, 200
RETAIN, SINKS = 0.6, 3


def global_workload(seed: int = 23):
    rng = np.random.default_rng(seed)
    MB = (L + BS - 1) // BS
    NB = S * MB + 4
    bt = rng.permutation(NB)[: S * MB].astype(np.int32).reshape(S, MB)
    bt[1, 3] = -1  # a hole
    sc = rng.integers(0, 6, (S, H, L)).astype(np.float32) * 0.5  # many ties across the head sums
    sc[2, 1, 17] = np.nan
    kp = rng.standard_normal((NB, BS, H, D)).astype(np.float16)
    vp = rng.standard_normal((NB, BS, H, D)).astype(np.float16)
    ctx = np.array([L, 150, 97], np.int32)
    return sc, bt, ctx, kp, vp


class OracleOps:
    """CPU stand-in for the two memopt_C operators, over this rank's pool."""

    def __init__(self, kp, vp):
        self.kp, self.vp = kp, vp

    def evict_topk_head_sum(self, scores):
        import oracle as O

        return torch.from_numpy(O.evict_topk_head_sum(scores.numpy()))

    def evict_topk_compact_parts(self, parts, block_tables, context_lens, retain_ratio, num_sink_tokens):
        import oracle as O

        res = O.evict_topk_compact_parts(parts.numpy(), block_tables.numpy(), context_lens.numpy(), self.kp,
                                         self.vp, retain_ratio, num_sink_tokens)
        return tuple(torch.from_numpy(x) for x in res)


def main() -> None:
    out_dir, backend = sys.argv[1], sys.argv[2]
    world, rank, local = dist_env()
    sc, bt, ctx, kp, vp = global_workload()
    h0, h1 = head_range(H, world, rank)
    my_k = np.ascontiguousarray(kp[:, :, h0:h1])
    my_v = np.ascontiguousarray(vp[:, :, h0:h1])
    if backend == "nccl":
        import memopt_C

        dev = torch.device("cuda", local)
        torch.cuda.set_device(dev)
        group = RankGroup.init("nccl", dev)
        memopt_C.init_pool(kp.shape[0], BS, h1 - h0, D)
        kc, vc = memopt_C.get_pool_tensors()
        kc.copy_(torch.from_numpy(my_k))
        vc.copy_(torch.from_numpy(my_v))
        ops = memopt_C
    else:
        dev = torch.device("cpu")
        group = RankGroup.init("gloo")
        ops = OracleOps(my_k, my_v)
    scores = torch.from_numpy(np.ascontiguousarray(sc[:, h0:h1])).to(dev)
    tbt = torch.from_numpy(bt.copy()).to(dev)
    tctx = torch.from_numpy(ctx.copy()).to(dev)
    kept, cnt, freed, fcnt = evict_exact_head_sharded(group, scores, tbt, tctx, RETAIN, SINKS, ops)
    if backend == "nccl":
        torch.cuda.synchronize()
        kc, vc = memopt_C.get_pool_tensors()
        my_k, my_v = kc.cpu().numpy(), vc.cpu().numpy()
    group.barrier()
    group.destroy()
    np.savez(os.path.join(out_dir, f"rank{rank}.npz"), kept=kept.cpu().numpy(), cnt=cnt.cpu().numpy(),
             freed=freed.cpu().numpy(), fcnt=fcnt.cpu().numpy(), bt=tbt.cpu().numpy(), ctx=tctx.cpu().numpy(),
             k=my_k, v=my_v, h0=h0, h1=h1)


if __name__ == "__main__":
    main()
