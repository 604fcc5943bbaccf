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

    def destroy(self) -> None:
        if self.dist is not None and self.dist.is_initialized():
            self.dist.destroy_process_group()
