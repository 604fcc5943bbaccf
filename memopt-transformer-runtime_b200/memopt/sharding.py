"""Sequence sharding across GPUs: one process and one KV-cache pool per GPU.

Every (sequence, head) pair of the data plane is independent: ``write_cache``,
the INT4 quantiser, ``evict_tokens`` (per head) and decode attention read and
write only that sequence's pages.  A job of ``S`` sequences therefore runs as
``N`` independent shards, each rank owning a contiguous range of sequences,
its own pool and its own block tables; no collective is on the data path.
The only cross-rank traffic is host-side bookkeeping: a barrier around timed
regions and the max over ranks of a device time (the job finishes when its
slowest shard does).  The reference runs on one device only (its README lists
multi-GPU pools as future work), so this module has no reference counterpart.

Heads can be sharded instead (each rank's pool holds H/N heads of every
sequence, for batches smaller than the GPU count).  Everything stays local
then too, except the exact eviction whose decision is shared across heads:
:func:`evict_exact_head_sharded` exchanges one fp32 row of partial token
scores per sequence and rank (an all-gather, 1 MB per rank at 8 sequences of
32768 tokens) and every rank ranks tokens by the same rank-ordered sum.
"""
from __future__ import annotations

import os
from dataclasses import dataclass
from typing import Optional, Tuple


def dist_env() -> Tuple[int, int, int]:
    """(world_size, rank, local_rank) as set by torchrun (1, 0, 0 without it)."""
    return (int(os.environ.get("WORLD_SIZE", "1")), int(os.environ.get("RANK", "0")),
            int(os.environ.get("LOCAL_RANK", "0")))


def shard_range(num_sequences: int, world_size: int, rank: int) -> Tuple[int, int]:
    """Contiguous [start, stop) of the sequences owned by ``rank``.

    Shards differ in size by at most one sequence; the first ``S % N`` ranks
    take the extra one.  Ranks beyond the work get an empty range.
    """
    if world_size <= 0 or not 0 <= rank < world_size:
        raise ValueError(f"rank {rank} outside a world of {world_size}")
    if num_sequences < 0:
        raise ValueError("num_sequences must be >= 0")
    base, extra = divmod(num_sequences, world_size)
    start = rank * base + min(rank, extra)
    return start, start + base + (1 if rank < extra else 0)


def job_rate(units_per_rank: float, slowest_ms: float, world_size: int) -> float:
    """Whole-job throughput (units per second) of ``world_size`` equal shards
    that each process ``units_per_rank`` units, timed by the slowest rank."""
    if slowest_ms <= 0:
        raise ValueError("slowest_ms must be > 0")
    return units_per_rank * world_size / (slowest_ms * 1e-3)


@dataclass
class RankGroup:
    """The process group of a sharded job (``None`` group: a single process).

    ``device`` is where reduction tensors live: a CUDA device for NCCL, the
    CPU for gloo.
    """

    dist: Optional[object] = None
    device: Optional[object] = None

    @classmethod
    def init(cls, backend: str, device=None) -> "RankGroup":
        """Joins the torchrun rendezvous when WORLD_SIZE > 1 (else a 1-rank group)."""
        world, _, _ = dist_env()
        if world <= 1:
            return cls(None, device)
        import torch
        import torch.distributed as dist

        if not dist.is_initialized():
            if backend == "nccl":
                dist.init_process_group("nccl", device_id=device)
            else:
                dist.init_process_group(backend)
        return cls(dist, device if backend == "nccl" else torch.device("cpu"))

    @property
    def world_size(self) -> int:
        return 1 if self.dist is None else self.dist.get_world_size()

    @property
    def rank(self) -> int:
        return 0 if self.dist is None else self.dist.get_rank()

    def barrier(self) -> None:
        if self.dist is not None:
            self.dist.barrier()

    def max(self, x: float) -> float:
        """The largest ``x`` over all ranks (every rank gets it)."""
        if self.dist is None:
            return float(x)
        import torch

        t = torch.tensor([float(x)], dtype=torch.float64, device=self.device)
        self.dist.all_reduce(t, op=self.dist.ReduceOp.MAX)
        return float(t.item())

    def all_gather_rows(self, t):
        """Every rank's ``t`` (same shape on all ranks), stacked in rank order
        into ``[world_size, *t.shape]`` on every rank."""
        if self.dist is None:
            return t.unsqueeze(0)
        t = t.contiguous()
        out = t.new_empty((self.world_size,) + tuple(t.shape))
        if t.is_cuda:
            self.dist.all_gather_into_tensor(out, t)
        else:
            self.dist.all_gather(list(out.unbind(0)), t)
        return out

    def destroy(self) -> None:
        if self.dist is not None and self.dist.is_initialized():
            self.dist.destroy_process_group()


def head_range(num_heads: int, world_size: int, rank: int) -> Tuple[int, int]:
    """Contiguous [start, stop) of the heads a rank holds under head sharding."""
    if num_heads % world_size:
        raise ValueError(f"{num_heads} heads do not split evenly over {world_size} ranks")
    return shard_range(num_heads, world_size, rank)


def evict_exact_head_sharded(group: RankGroup, scores, block_tables, context_lens, retain_ratio: float,
                             num_sink_tokens: int = 4, ops=None):
    """Exact top-k eviction shared across heads when the heads are sharded.

    ``scores`` [S, H_local, L] are this rank's heads; ``block_tables`` /
    ``context_lens`` are the sequences' (the same on every rank) and are
    updated in place.  Each rank sums its own heads, the partial rows are
    all-gathered in rank order, and ``evict_topk_compact_parts`` ranks tokens
    by their fp32 sum in rank order and compacts this rank's pool, so every
    rank keeps the same tokens and frees the same pages.  With one rank this
    is ``evict_topk_compact``.  ``ops`` is the operator module (``memopt_C``).
    Returns ``(kept_idx, kept_count, freed_pages, freed_count)``.
    """
    if ops is None:
        import memopt_C as ops
    part = ops.evict_topk_head_sum(scores)
    parts = group.all_gather_rows(part)
    return ops.evict_topk_compact_parts(parts, block_tables, context_lens, float(retain_ratio),
                                        int(num_sink_tokens))
