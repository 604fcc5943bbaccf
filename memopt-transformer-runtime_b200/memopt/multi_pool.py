"""KV-cache pages spread over the GPUs of a job (one process per GPU).

The reference's pool is one tensor pair on one device (its kv_cache.cu:97
leaves "extend to multi-GPU via device_id key if needed"; its README lists a
block allocator spanning devices as future work).  Here a sequence has a
*home* rank, where its attention runs, and its pages may live on any rank: a
page is allocated on the home GPU while it has free blocks and spills to the
GPU with the most free blocks otherwise, so one context can use the HBM of
several GPUs.

Every rank holds a replica of the host-side state (the allocator of
``memopt_mdpool_*`` in the C library, sequence tables, lengths) and makes the
same calls in the same order (SPMD), so all replicas agree without messages.
Page data moves only in two places, both point-to-point over the process
group (NCCL over NVLink on GPUs):

* ``append``: the home rank sends the new token rows that belong to pages
  owned by another rank to that rank, which writes them into its own pool
  with ``write_cache`` (fused INT4 quantisation for an INT4 pool);
* ``attend``: before attention, every rank packs the pages it owns that a
  peer's home sequences read (``memopt_copy_pages``), sends them, and the
  peer receives them straight into consecutive staging blocks of its pool
  (``memopt_mdpool_plan`` groups each owner's pages into one run); attention
  then runs on the home GPU over local blocks only.

No kernel reads another GPU's memory and no TMA multicast is involved.
``pack`` / ``write_rows`` / ``attend_fn`` can be replaced (the CPU tests run
the exchange logic on gloo with numpy-backed versions); the defaults are the
CUDA kernels of this library and refuse CPU tensors.
"""
from __future__ import annotations

import ctypes as C
from dataclasses import dataclass, field
from typing import Callable, Dict, List, Optional, Sequence

import torch

from . import _capi

__all__ = ["MultiDevicePagePool", "mdpool_plan"]


def _lib():
    return _capi.lib()


def mdpool_plan(page_dev: Sequence[int], page_blk: Sequence[int], home: int, staging_base: int,
                staging_capacity: int):
    """Python view of ``memopt_mdpool_plan``: (local_blk, [(src_dev, src_blk,
    dst_blk), ...])."""
    n = len(page_blk)
    arr = C.c_int32 * max(n, 1)
    pd, pb = arr(*page_dev), arr(*page_blk)
    local, sd, sb, db = arr(), arr(), arr(), arr()
    nc = C.c_int(0)
    _capi.check(_lib().memopt_mdpool_plan(pd, pb, C.c_int(n), C.c_int(home), C.c_int(staging_base),
                                          C.c_int(staging_capacity), local, sd, sb, db, C.byref(nc)),
                "memopt_mdpool_plan")
    return list(local)[:n], [(sd[k], sb[k], db[k]) for k in range(nc.value)]


@dataclass
class _Seq:
    home: int
    pages: List[tuple] = field(default_factory=list)  # (owner rank, block)
    length: int = 0


def _cuda_pack(src: torch.Tensor, ids: torch.Tensor, out: torch.Tensor) -> None:
    if not src.is_cuda:
        raise RuntimeError("MultiDevicePagePool: the page copy kernel needs CUDA tensors")
    page_bytes = src[0].numel() * src.element_size()
    _capi.check(_lib().memopt_copy_pages(C.c_void_p(src.data_ptr()), C.c_void_p(ids.data_ptr()),
                                         C.c_void_p(out.data_ptr()), C.c_void_p(0), C.c_int(ids.numel()),
                                         C.c_int64(page_bytes),
                                         C.c_void_p(torch.cuda.current_stream(src.device).cuda_stream)),
                "memopt_copy_pages")


class MultiDevicePagePool:
    """Paged KV storage of one layer over ``group.world_size`` GPUs.

    Each rank owns ``blocks_per_rank`` allocatable blocks plus
    ``staging_blocks`` receive blocks, in local pool tensors of
    ``blocks_per_rank + staging_blocks`` pages (fp16: K and V
    [blocks, block_size, H, D]; INT4: pages [blocks, H, page_bytes]).
    """

    def __init__(self, group, blocks_per_rank: int, staging_blocks: int, block_size: int, num_heads: int,
                 head_dim: int, kv_format: str = "fp16", device=None,
                 pack: Optional[Callable] = None, write_rows: Optional[Callable] = None,
                 attend_fn: Optional[Callable] = None) -> None:
        if kv_format not in ("fp16", "int4"):
            raise ValueError("kv_format must be 'fp16' or 'int4'")
        self.group = group
        self.world = group.world_size
        self.rank = group.rank
        self.nb, self.ns = blocks_per_rank, staging_blocks
        self.bs, self.h, self.d = block_size, num_heads, head_dim
        self.kv_format = kv_format
        self.device = device if device is not None else torch.device("cuda", torch.cuda.current_device())
        total = blocks_per_rank + staging_blocks
        if kv_format == "fp16":
            shape = (total, block_size, num_heads, head_dim)
            self.tensors = [torch.zeros(shape, dtype=torch.float16, device=self.device) for _ in range(2)]
        else:
            pb = block_size * head_dim + block_size * (head_dim // 64) * 4
            self.tensors = [torch.zeros((total, num_heads, pb), dtype=torch.uint8, device=self.device)]
        blocks = (C.c_int * self.world)(*([blocks_per_rank] * self.world))
        _capi.check(_lib().memopt_mdpool_init(C.c_int(self.world), blocks), "memopt_mdpool_init")
        self._seqs: Dict[int, _Seq] = {}
        self._next = 0
        self._pack = pack or _cuda_pack
        self._write_rows = write_rows or self._cuda_write_rows
        self._attend_fn = attend_fn or self._cuda_attend

    # ---- bookkeeping (replicated) --------------------------------------------
    def add_sequence(self, home: int) -> int:
        if not 0 <= home < self.world:
            raise ValueError(f"home rank {home} outside a world of {self.world}")
        sid = self._next
        self._next += 1
        self._seqs[sid] = _Seq(home)
        return sid

    def free_sequence(self, sid: int) -> None:
        for dev, blk in self._seqs.pop(sid).pages:
            _capi.check(_lib().memopt_mdpool_free(C.c_int(dev), C.c_int(blk)), "memopt_mdpool_free")

    def pages(self, sid: int) -> List[tuple]:
        return list(self._seqs[sid].pages)

    def length(self, sid: int) -> int:
        return self._seqs[sid].length

    def free_count(self, rank: int) -> int:
        return int(_lib().memopt_mdpool_free_count(C.c_int(rank)))

    def _reserve(self, sid: int, n: int) -> List[tuple]:
        """(owner, slot) of n new tokens; pages allocated home-first."""
        seq = self._seqs[sid]
        need = (seq.length + n + self.bs - 1) // self.bs - len(seq.pages)
        got = []
        for _ in range(max(0, need)):
            dev = C.c_int(-1)
            blk = _lib().memopt_mdpool_allocate(C.c_int(seq.home), C.byref(dev))
            if blk < 0:
                for d_, b_ in got:
                    _lib().memopt_mdpool_free(C.c_int(d_), C.c_int(b_))
                if blk == -1:
                    raise MemoryError(f"every GPU's pages are in use (appending {n} tokens to sequence {sid})")
                _capi.check(blk, "memopt_mdpool_allocate")
            got.append((dev.value, blk))
        seq.pages.extend(got)
        out = []
        for t in range(seq.length, seq.length + n):
            dev, blk = seq.pages[t // self.bs]
            out.append((dev, blk * self.bs + t % self.bs))
        seq.length += n
        return out

    # ---- data path -------------------------------------------------------------
    def _cuda_write_rows(self, k: torch.Tensor, v: torch.Tensor, slots: torch.Tensor) -> None:
        st = torch.cuda.current_stream(self.device).cuda_stream
        if self.kv_format == "fp16":
            _capi.write_cache_f16(k, v, slots, self.tensors[0], self.tensors[1], st)
        else:
            _capi.write_cache_int4(k, v, slots, self.tensors[0], self.bs, st)

    def append(self, sid: int, k: Optional[torch.Tensor] = None, v: Optional[torch.Tensor] = None,
               n: Optional[int] = None) -> None:
        """Appends n token rows ([n, H, D] fp16) to ``sid``.  Every rank calls
        it; the home rank passes ``k``/``v`` (the others may pass None and
        give ``n``).  Rows whose page another rank owns are sent there."""
        seq = self._seqs[sid]
        home = seq.home
        if self.rank == home:
            if k is None or v is None:
                raise ValueError("append: the home rank must pass k and v")
            n = k.shape[0]
        if n is None:
            raise ValueError("append: ranks other than the home rank must pass n")
        where = self._reserve(sid, n)
        dist = self.group.dist
        for owner in range(self.world):
            idx = [i for i, (dev, _) in enumerate(where) if dev == owner]
            if not idx:
                continue
            slots = torch.tensor([where[i][1] for i in idx], dtype=torch.int32, device=self.device)
            if owner == home:
                if self.rank == home:
                    sel = torch.tensor(idx, dtype=torch.long, device=k.device)
                    self._write_rows(k.index_select(0, sel).contiguous(), v.index_select(0, sel).contiguous(),
                                     slots)
            elif self.rank == home:
                sel = torch.tensor(idx, dtype=torch.long, device=k.device)
                dist.send(k.index_select(0, sel).contiguous(), dst=owner)
                dist.send(v.index_select(0, sel).contiguous(), dst=owner)
            elif self.rank == owner:
                kr = torch.empty((len(idx), self.h, self.d), dtype=torch.float16, device=self.device)
                vr = torch.empty_like(kr)
                dist.recv(kr, src=home)
                dist.recv(vr, src=home)
                self._write_rows(kr, vr, slots)

    def _plans(self, sids: Sequence[int]):
        """Per home rank: (its sequences, local tables, copies)."""
        plans = {}
        width = max((len(self._seqs[s].pages) for s in sids), default=0)
        for home in range(self.world):
            mine = [s for s in sids if self._seqs[s].home == home]
            dev, blk = [], []
            for s in mine:
                pg = self._seqs[s].pages
                dev += [p[0] for p in pg] + [home] * (width - len(pg))
                blk += [p[1] for p in pg] + [-1] * (width - len(pg))
            local, copies = mdpool_plan(dev, blk, home, self.nb, self.ns)
            plans[home] = (mine, local, copies, width)
        return plans

    def gather(self, sids: Sequence[int]):
        """Moves the remote pages this rank's home sequences read into its
        staging blocks (and serves its own pages to the peers).  Returns
        (home sequences of this rank, local block table [S, width])."""
        plans = self._plans(sids)
        dist = self.group.dist
        ops = []
        keep = []
        for home, (_, _, copies, _) in plans.items():
            for owner in range(self.world):
                run = [c for c in copies if c[0] == owner]
                if not run or owner == home:
                    continue
                if self.rank == owner:  # pack and send my pages to `home`
                    ids = torch.tensor([c[1] for c in run], dtype=torch.int32, device=self.device)
                    for t in self.tensors:
                        buf = torch.empty((len(run),) + tuple(t.shape[1:]), dtype=t.dtype, device=t.device)
                        self._pack(t, ids, buf)
                        keep.append(buf)
                        ops.append(dist.P2POp(dist.isend, buf, home))
                elif self.rank == home:  # receive straight into consecutive staging blocks
                    d0 = run[0][2]
                    for t in self.tensors:
                        ops.append(dist.P2POp(dist.irecv, t[d0:d0 + len(run)], owner))
        if ops:
            for r in dist.batch_isend_irecv(ops):
                r.wait()
        mine, local, _, width = plans[self.rank]
        table = torch.tensor(local, dtype=torch.int32, device=self.device).reshape(len(mine), width)
        return mine, table

    def _cuda_attend(self, q, table, ctx, msl, win):
        import memopt_C

        if self.kv_format == "fp16":
            return memopt_C.dynamic_sparse_attention(q, self.tensors[0], self.tensors[1], table, ctx, msl, win)
        return memopt_C.dynamic_sparse_attention_int4(q, self.tensors[0], table, ctx, msl, win)

    def attend(self, sids: Sequence[int], q: Optional[torch.Tensor], window_size: int = -1):
        """Attention of each rank's home sequences among ``sids`` (every rank
        passes the same ``sids``; ``q`` [S_home, n, H, D] holds this rank's
        home sequences in ``sids`` order).  Returns this rank's output, or
        None when it is home to none of them."""
        mine, table = self.gather(sids)
        if not mine:
            return None
        ctx = torch.tensor([self._seqs[s].length for s in mine], dtype=torch.int32, device=self.device)
        msl = max(1, int(ctx.max().item()))
        win = msl if window_size <= 0 else window_size
        return self._attend_fn(q.to(torch.float16).contiguous(), table, ctx, msl, win)
