"""One rank of the multi-device page pool tests.

Arguments: a scratch directory and a backend ("gloo" or "nccl").  Two
sequences with seeded K/V rows are appended in several chunks to a
``memopt.multi_pool.MultiDevicePagePool`` of 7 blocks per rank: sequence A
(home rank 0, 130 tokens) fills rank 0 and spills two pages onto rank 1,
sequence B (home rank 1) stays on rank 1.  Each rank then attends for its
home sequence and writes its output, its pool's page owners and the free
counts to <dir>/rank<r>.npz.

* gloo (CPU, tests/test_multirank.py): the page pack, the row writer and the
  attention are stand-ins (numpy indexing and the oracle), so the test covers
  the replicated allocator, the append routing and the staging exchange.
* nccl (one GPU per rank, tests/test_gpu_multigpu.py): the library's CUDA
  kernels (write_cache, memopt_copy_pages, paged attention) over NCCL.
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

from memopt.multi_pool import MultiDevicePagePool  # noqa: E402
from memopt.sharding import RankGroup, dist_env  # noqa: E402

H, D, BS, BLOCKS, STAGING = 2, 64, 16, 7, 8
CHUNKS = {"A": [37, 1, 60, 32], "B": [40, 1, 29]}  # appended in this interleaved order


def rows(seed: int, n: int):
    rng = np.random.default_rng(seed)
    return (rng.standard_normal((n, H, D)).astype(np.float16), rng.standard_normal((n, H, D)).astype(np.float16))


def full_rows(name: str):
    ks, vs = [], []
    for i, n in enumerate(CHUNKS[name]):
        k, v = rows(ord(name) * 100 + i, n)
        ks.append(k)
        vs.append(v)
    return np.concatenate(ks), np.concatenate(vs)


def query(name: str):
    return np.random.default_rng(len(name) * 7 + ord(name)).standard_normal((1, 1, H, D)).astype(np.float16)


def main() -> None:
    out_dir, backend = sys.argv[1], sys.argv[2]
    world, rank, local = dist_env()
    if backend == "nccl":
        torch.cuda.set_device(local)
        dev = torch.device("cuda", local)
    else:
        dev = torch.device("cpu")
    group = RankGroup.init(backend, dev)
    kw = {}
    if backend == "gloo":
        import oracle as O

        def pack(src, ids, out):
            out.copy_(src.index_select(0, ids.long()))

        def attend_fn(q, table, ctx, msl, win):
            kp, vp = pool.tensors
            r = O.paged_attention_f16(q.numpy(), kp.numpy(), vp.numpy(), table.numpy(), ctx.numpy(), msl, win)
            return torch.from_numpy(r)

        def write_rows(k, v, slots):
            kp, vp = pool.tensors
            kp.view(-1, H, D)[slots.long()] = k
            vp.view(-1, H, D)[slots.long()] = v

        kw = dict(pack=pack, attend_fn=attend_fn, write_rows=write_rows)
    pool = MultiDevicePagePool(group, BLOCKS, STAGING, BS, H, D, device=dev, **kw)
    sid = {"A": pool.add_sequence(0), "B": pool.add_sequence(1)}
    order = [("A", 0), ("B", 0), ("A", 1), ("B", 1), ("A", 2), ("B", 2), ("A", 3)]
    for name, i in order:
        n = CHUNKS[name][i]
        home = 0 if name == "A" else 1
        if rank == home:
            k, v = rows(ord(name) * 100 + i, n)
            pool.append(sid[name], torch.from_numpy(k).to(dev), torch.from_numpy(v).to(dev))
        else:
            pool.append(sid[name], n=n)
    mine = "A" if rank == 0 else "B"
    q = torch.from_numpy(query(mine)).to(dev)
    out = pool.attend([sid["A"], sid["B"]], q)
    if dev.type == "cuda":
        torch.cuda.synchronize()
    np.savez(os.path.join(out_dir, f"rank{rank}.npz"), out=out.float().cpu().numpy(),
             pagesA=np.array(pool.pages(sid["A"]), np.int32), pagesB=np.array(pool.pages(sid["B"]), np.int32),
             free=np.array([pool.free_count(r) for r in range(world)], np.int32))
    # pages return to their owners' free-lists
    pool.free_sequence(sid["A"])
    assert [pool.free_count(r) for r in range(world)] == [BLOCKS, BLOCKS - len(pool.pages(sid["B"]))]
    group.barrier()
    group.destroy()


if __name__ == "__main__":
    main()
