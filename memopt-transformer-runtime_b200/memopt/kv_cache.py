"""Incremental paged KV cache over the module pool, driven by the
:class:`~memopt.scheduler.MemoryScheduler` policy.

The reference promises (README) that the scheduler's ``retain_ratio`` /
``use_int4`` drive the attention layer, but nothing in it reads them; this
module is that missing caller of the data-plane operators:

* :class:`PageTable` — pure-Python bookkeeping of sequences, pages, block
  tables, slot mappings and context lengths on top of a page allocator
  (``memopt_C.allocate_block`` / ``free_block``: FIFO, -1 when exhausted, as
  in the reference kv_cache.cu:146-201).  It has no device state and is
  tested on CPU.
* :class:`PagedKVCache` — one cache per process over the ``memopt_C`` pool:
  ``append`` writes new K/V tokens (``write_cache``), ``attend`` runs paged
  attention over each sequence's whole cached context (decode when the
  sequences get one new token per step, prefill otherwise), ``evict`` runs
  ``evict_tokens`` with per-token attention scores, ``to_int4`` re-quantises
  every cached token into an INT4 pool with the same block ids, and
  ``apply_policy`` maps a scheduler snapshot onto those actions.
"""
from __future__ import annotations

from dataclasses import dataclass, field
from typing import Callable, Dict, List, Optional, Sequence

import torch

__all__ = ["PageTable", "PagedKVCache"]


@dataclass
class _Seq:
    pages: List[int] = field(default_factory=list)
    length: int = 0


class PageTable:
    """Sequences -> pages, with slot mappings for appended tokens.

    ``alloc()`` returns a free page id or -1; ``free(page)`` returns it.
    Token ``t`` of a sequence lives in page ``pages[t // block_size]`` at slot
    ``page * block_size + t % block_size`` (the reference's slot convention).
    """

    def __init__(self, block_size: int, alloc: Callable[[], int], free: Callable[[int], None]) -> None:
        if block_size <= 0:
            raise ValueError("block_size must be > 0")
        self.block_size = block_size
        self._alloc = alloc
        self._free = free
        self._seqs: Dict[int, _Seq] = {}
        self._next_id = 0

    def add_sequence(self) -> int:
        sid = self._next_id
        self._next_id += 1
        self._seqs[sid] = _Seq()
        return sid

    def free_sequence(self, sid: int) -> None:
        seq = self._seqs.pop(sid)
        for p in seq.pages:
            self._free(p)

    def __contains__(self, sid: int) -> bool:
        return sid in self._seqs

    def length(self, sid: int) -> int:
        return self._seqs[sid].length

    def pages(self, sid: int) -> List[int]:
        return list(self._seqs[sid].pages)

    def reserve(self, sid: int, n_new: int) -> List[int]:
        """Slots for ``n_new`` tokens appended to ``sid`` (pages allocated as
        needed).  Raises ``MemoryError`` when the pool is exhausted; pages
        taken by the failed call are returned first."""
        if n_new < 0:
            raise ValueError("n_new must be >= 0")
        seq = self._seqs[sid]
        bs = self.block_size
        need = (seq.length + n_new + bs - 1) // bs - len(seq.pages)
        got: List[int] = []
        for _ in range(max(0, need)):
            p = self._alloc()
            if p < 0:
                for q in got:
                    self._free(q)
                raise MemoryError(f"KV pool exhausted while appending {n_new} tokens to sequence {sid}")
            got.append(p)
        seq.pages.extend(got)
        slots = [seq.pages[t // bs] * bs + t % bs for t in range(seq.length, seq.length + n_new)]
        seq.length += n_new
        return slots

    def compact(self, sid: int, new_length: int) -> List[int]:
        """After an in-place compaction of ``sid`` to its first ``new_length``
        tokens: keeps the first ceil(new_length / block_size) pages, returns
        the others to the allocator and lists them."""
        seq = self._seqs[sid]
        if not 0 <= new_length <= seq.length:
            raise ValueError(f"compact: new length {new_length} outside [0, {seq.length}]")
        need = (new_length + self.block_size - 1) // self.block_size
        freed = seq.pages[need:]
        seq.pages = seq.pages[:need]
        seq.length = new_length
        for p in freed:
            self._free(p)
        return freed

    def block_table(self, sids: Sequence[int], max_blocks: Optional[int] = None) -> List[List[int]]:
        """Rows of page ids, -1 padded to ``max_blocks`` (default: the longest)."""
        rows = [self._seqs[s].pages for s in sids]
        width = max((len(r) for r in rows), default=0) if max_blocks is None else max_blocks
        return [r[:width] + [-1] * (width - len(r[:width])) for r in rows]


class PagedKVCache:
    """Paged KV cache of one attention layer over the process-wide pool."""

    def __init__(self, num_blocks: int, num_heads: int, head_dim: int, block_size: int = 16,
                 kv_format: str = "fp16", device: Optional[torch.device] = None,
                 eviction: str = "exact") -> None:
        """``eviction``: "exact" (the default) runs ``evict_topk_compact``
        (one exact top-k per sequence shared by all heads, sinks always
        kept, kept rows compacted, emptied pages freed), so a scheduler
        decision of ``retain_ratio < 1`` returns pages to the pool;
        "reference" runs ``evict_tokens`` (the reference's semantics:
        per-head threshold, rows zeroed, no page released; with sink tokens
        its sink boost makes the bisection keep every token, so it frees
        nothing)."""
        if eviction not in ("reference", "exact"):
            raise ValueError("eviction must be 'reference' or 'exact'")
        self.eviction = eviction
        import memopt_C

        self._C = memopt_C
        self.num_blocks, self.num_heads, self.head_dim, self.block_size = num_blocks, num_heads, head_dim, block_size
        self.device = device or torch.device("cuda", torch.cuda.current_device())
        memopt_C.init_pool(num_blocks, block_size, num_heads, head_dim, kv_format=kv_format)
        self.table = PageTable(block_size, memopt_C.allocate_block, memopt_C.free_block)
        self._applied = (1.0, kv_format == "int4")  # policy state the cache currently reflects

    # ---- bookkeeping ---------------------------------------------------------
    @property
    def kv_format(self) -> str:
        return self._C.pool_format()

    def add_sequence(self) -> int:
        return self.table.add_sequence()

    def free_sequence(self, sid: int) -> None:
        self.table.free_sequence(sid)

    def context_lens(self, sids: Sequence[int]) -> torch.Tensor:
        return torch.tensor([self.table.length(s) for s in sids], dtype=torch.int32, device=self.device)

    def block_tables(self, sids: Sequence[int]) -> torch.Tensor:
        rows = self.table.block_table(sids)
        return torch.tensor(rows, dtype=torch.int32, device=self.device).reshape(len(sids), -1)

    # ---- data path -------------------------------------------------------------
    def append(self, sids: Sequence[int], k: torch.Tensor, v: torch.Tensor) -> None:
        """Writes ``k``/``v`` of shape [B, n, H, D] as the next n tokens of each
        sequence (``write_cache``; fused INT4 quantisation for an int4 pool)."""
        B, n, H, D = k.shape
        if B != len(sids) or (H, D) != (self.num_heads, self.head_dim):
            raise ValueError(f"append: k of shape {tuple(k.shape)} does not match {len(sids)} sequences x "
                             f"{self.num_heads} heads x {self.head_dim}")
        slots: List[int] = []
        for s in sids:
            slots.extend(self.table.reserve(s, n))
        slot_t = torch.tensor(slots, dtype=torch.int32, device=self.device)
        bt = self.block_tables(sids)
        self._C.write_cache(k.reshape(B * n, H, D).to(torch.float16).contiguous(),
                            v.reshape(B * n, H, D).to(torch.float16).contiguous(), bt, slot_t)

    def attend(self, q: torch.Tensor, sids: Sequence[int], window_size: int = -1) -> torch.Tensor:
        """Attention of ``q`` [B, n, H, D] over each sequence's cached context
        (non-causal, the reference semantics); window <= 0: whole context."""
        bt = self.block_tables(sids)
        ctx = self.context_lens(sids)
        msl = max(1, int(ctx.max().item()) if len(sids) else 1)
        win = msl if window_size <= 0 else window_size
        q16 = q.to(torch.float16).contiguous()
        if self.kv_format == "int4":
            return self._C.dynamic_sparse_attention_int4(q16, self._C.get_int4_pages(), bt, ctx, msl, win)
        kc, vc = self._C.get_pool_tensors()
        return self._C.dynamic_sparse_attention(q16, kc, vc, bt, ctx, msl, win)

    def _keys(self, pages: torch.Tensor, n: int) -> torch.Tensor:
        """fp32 keys [n, H, D] of a sequence's first n tokens: the fp16 pool's
        rows, or the INT4 pool's codes dequantised as the reference does
        (fp16((c - 8) * scale), quantization.cu:254-268)."""
        H, D = self.num_heads, self.head_dim
        if self.kv_format == "fp16":
            kc, _ = self._C.get_pool_tensors()
            return kc[pages].reshape(-1, H, D)[:n].float()
        kcodes, kscale, _, _ = self._C.get_int4_pool_tensors()
        c = kcodes[pages].transpose(1, 2).reshape(-1, H, D // 2)[:n]  # [n, H, D/2]: byte i = dims 2i, 2i+1
        codes = torch.stack([c & 15, c >> 4], dim=-1).reshape(n, H, D).float() - 8.0
        sc = kscale[pages].transpose(1, 2).reshape(-1, H, D // 64)[:n].float().repeat_interleave(64, dim=-1)
        return (codes * sc).half().float()

    def token_scores(self, q: torch.Tensor, sids: Sequence[int]) -> torch.Tensor:
        """Per-token attention weights [B, H, L] of the last query row of ``q``
        over the cached context (fp16 or INT4 pool), the eviction signal of
        Ada-KV.  Padding past a sequence's length is 0."""
        lens = [self.table.length(s) for s in sids]
        L = max(lens, default=0)
        H, D, bs = self.num_heads, self.head_dim, self.block_size
        out = torch.zeros(len(sids), H, L, dtype=torch.float32, device=self.device)
        scale = D ** -0.5
        for i, s in enumerate(sids):
            n = lens[i]
            if n == 0:
                continue
            pages = torch.tensor(self.table.pages(s), dtype=torch.long, device=self.device)
            keys = self._keys(pages, n)  # [n, H, D]
            logits = torch.einsum("hd,nhd->hn", q[i, -1].float(), keys) * scale
            out[i, :, :n] = torch.softmax(logits, dim=-1)
        return out

    def evict(self, sids: Sequence[int], scores: torch.Tensor, retain_ratio: float, num_sink_tokens: int = 4):
        """``evict_tokens`` over the sequences (reference semantics: evicted
        rows are zeroed in the pool; pages stay allocated).  Returns the
        retained-token indices and counts [B, H, L] / [B, H]."""
        if self.kv_format != "fp16":
            raise RuntimeError("evict: evict_tokens works on the fp16 pool")
        bt = self.block_tables(sids)
        ibf = torch.zeros(self.num_blocks, dtype=torch.int32, device=self.device)
        return self._C.evict_tokens(scores.float().contiguous(), bt, ibf, float(retain_ratio), int(num_sink_tokens),
                                    return_retained=True)

    def evict_exact(self, sids: Sequence[int], scores: torch.Tensor, retain_ratio: float,
                    num_sink_tokens: int = 4, group=None) -> List[List[int]]:
        """``evict_topk_compact`` over the sequences: the kept tokens (exact
        top-k of the head-summed scores, sinks always kept) move to the front
        of each sequence, lengths shrink, and the emptied pages return to the
        pool.  Returns the kept original token indices per sequence.

        ``group`` (a :class:`memopt.sharding.RankGroup`): this cache holds one
        head shard of every sequence and ``scores`` are its heads; the ranks
        exchange partial token scores and take one shared decision."""
        if group is not None and group.world_size > 1 and self.kv_format != "fp16":
            raise RuntimeError("evict_exact: the head-sharded form works on the fp16 pool")
        bt = self.block_tables(sids).contiguous()
        ctx = self.context_lens(sids).contiguous()
        sc = scores.float().contiguous()
        if group is not None and group.world_size > 1:
            from .sharding import evict_exact_head_sharded

            kept, cnt, _, _ = evict_exact_head_sharded(group, sc, bt, ctx, retain_ratio, num_sink_tokens, self._C)
        else:
            kept, cnt, _, _ = self._C.evict_topk_compact(sc, bt, ctx, float(retain_ratio), int(num_sink_tokens))
        counts = cnt.tolist()
        kept_h = kept.cpu()
        out = []
        for i, s in enumerate(sids):
            self.table.compact(s, counts[i])
            out.append(kept_h[i, :counts[i]].tolist())
        return out

    def to_int4(self) -> None:
        """Re-quantises every cached token into an INT4 pool with the same
        block ids (page tables and lengths are unchanged)."""
        if self.kv_format == "int4":
            return
        kc, vc = self._C.get_pool_tensors()
        sids = list(self.table._seqs.keys())
        entries = []
        for s in sids:
            n = self.table.length(s)
            if n == 0:
                continue
            bs = self.block_size
            slots = [self.table.pages(s)[t // bs] * bs + t % bs for t in range(n)]
            st = torch.tensor(slots, dtype=torch.long, device=self.device)
            k = kc.reshape(-1, self.num_heads, self.head_dim)[st].clone()
            v = vc.reshape(-1, self.num_heads, self.head_dim)[st].clone()
            entries.append((st.to(torch.int32), k, v))
        # The pool is a per-process singleton: re-initialise it as INT4 and
        # restore the allocator state (the same pages in use, FIFO of the rest).
        used = {p for s in sids for p in self.table.pages(s)}
        self._C.init_pool(self.num_blocks, self.block_size, self.num_heads, self.head_dim, kv_format="int4")
        taken = []
        while True:
            p = self._C.allocate_block()
            if p < 0:
                break
            taken.append(p)
        for p in taken:
            if p not in used:
                self._C.free_block(p)
        dummy_bt = torch.zeros(1, 1, dtype=torch.int32, device=self.device)
        for st, k, v in entries:
            self._C.write_cache(k, v, dummy_bt, st)

    def apply_policy(self, scheduler, q: Optional[torch.Tensor] = None, sids: Optional[Sequence[int]] = None,
                     num_sink_tokens: int = 4) -> Optional[tuple]:
        """Maps a scheduler snapshot onto the cache when it differs from the one
        last applied: ``retain_ratio < 1`` evicts (scores from
        ``q``'s last row), then ``use_int4`` converts the pool to INT4.  A
        return to (1.0, fp16) only affects new caches (quantised tokens cannot
        be restored).  Returns the eviction result or None."""
        retain, use_int4 = scheduler.snapshot()
        if (retain, use_int4) == self._applied:
            return None
        self._applied = (retain, use_int4)
        result = None
        if retain < 1.0 and q is not None and sids and (self.kv_format == "fp16" or self.eviction == "exact"):
            scores = self.token_scores(q, sids)
            if self.eviction == "exact":
                result = self.evict_exact(sids, scores, retain, num_sink_tokens)
            else:
                result = self.evict(sids, scores, retain, num_sink_tokens)
        if use_int4 and self.kv_format == "fp16":
            self.to_int4()
        return result
