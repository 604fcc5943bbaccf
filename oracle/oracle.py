"""ctypes/numpy front end of the CPU oracle (memopt_oracle.c).

TEST INFRASTRUCTURE ONLY: used by tests/, ``__graft_entry__.smoke()`` and the
CPU-baseline leg of bench.py as the checker.  Arrays are numpy; fp16 data is
passed as ``np.float16``.
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
SRC = os.path.join(HERE, "memopt_oracle.c")
LIB = os.path.join(HERE, "liboracle.so")
CFLAGS = ["-O2", "-fopenmp", "-ffp-contract=off", "-fno-fast-math", "-fPIC", "-shared"]


def build() -> str:
    if not os.path.exists(LIB) or os.path.getmtime(LIB) < os.path.getmtime(SRC):
        tmp = LIB + ".tmp"
        subprocess.run(["gcc", *CFLAGS, SRC, "-o", tmp, "-lm"], check=True)
        os.replace(tmp, LIB)
    return LIB


_lib = None


def lib() -> C.CDLL:
    global _lib
    if _lib is None:
        build()
        _lib = C.CDLL(LIB)
        _lib.oracle_f16_to_f32.restype = C.c_float
        _lib.oracle_f16_to_f32.argtypes = [C.c_uint16]
        _lib.oracle_f32_to_f16.restype = C.c_uint16
        _lib.oracle_f32_to_f16.argtypes = [C.c_float]
    return _lib


def _p(a: np.ndarray) -> C.c_void_p:
    assert a.flags["C_CONTIGUOUS"], "oracle inputs must be C-contiguous"
    return C.c_void_p(a.ctypes.data)


I64, I32, F32 = C.c_int64, C.c_int, C.c_float
_c = np.ascontiguousarray


def f32_to_f16_bits(x: float) -> int:
    return int(lib().oracle_f32_to_f16(C.c_float(x)))


def f16_bits_to_f32(b: int) -> float:
    return float(lib().oracle_f16_to_f32(C.c_uint16(b)))


def quantize_int4(x: np.ndarray) -> tuple[np.ndarray, np.ndarray]:
    """Reference quantize_kv_cache_int4: packed (shape[..., D/2]) and fp32 scales."""
    x = _c(x, dtype=np.float16)
    n = x.size
    packed = np.zeros(x.shape[:-1] + (x.shape[-1] // 2,), np.uint8)
    scales = np.zeros(n // 64, np.float32)
    lib().oracle_quantize_int4(_p(x), I64(n), _p(packed), _p(scales))
    return packed, scales


def dequantize_int4(packed: np.ndarray, scales: np.ndarray) -> np.ndarray:
    packed = _c(packed, dtype=np.uint8)
    scales = _c(scales, dtype=np.float32)
    out = np.zeros(packed.shape[:-1] + (packed.shape[-1] * 2,), np.float16)
    lib().oracle_dequantize_int4(_p(packed), _p(scales), I64(out.size), _p(out))
    return out


def write_cache_f16(keys, values, slots, kpool, vpool) -> None:
    """In place on kpool/vpool [NB, BS, H, D] fp16 (C-contiguous numpy)."""
    T, H, D = keys.shape
    NB, BS = kpool.shape[0], kpool.shape[1]
    keys, values, slots = _c(keys, np.float16), _c(values, np.float16), _c(slots, np.int32)
    lib().oracle_write_cache_f16(_p(keys), _p(values), _p(slots), I64(T), I32(H), I32(D),
                                 _p(kpool), _p(vpool), I64(NB), I32(BS))


def int4_page_bytes(block_size: int, head_dim: int) -> int:
    return block_size * head_dim + block_size * (head_dim // 64) * 4


def write_cache_int4(keys, values, slots, pages, block_size) -> None:
    """In place on INT4 pages uint8 [NB, H, page_bytes]."""
    T, H, D = keys.shape
    NB = pages.shape[0]
    keys, values, slots = _c(keys, np.float16), _c(values, np.float16), _c(slots, np.int32)
    lib().oracle_write_cache_int4(_p(keys), _p(values), _p(slots), I64(T), I32(H), I32(D), _p(pages),
                                  I64(NB), I32(block_size))


def int4_views(pages, block_size, head_dim):
    """(k_codes, k_scales, v_codes, v_scales) of the INT4 pages in logical order:
    codes [NB, H, BS, D/2] (byte i = code(2i) | code(2i+1) << 4), fp16 scales
    [NB, H, BS, D/64].  The V rows and V scales are un-permuted from the stored
    order (for D == 128 the 32-byte halves of V rows whose index has bit 1 set
    are exchanged; V scales are [BS/16][D/64][16] in a per-tile token order)."""
    NB, H, PB = pages.shape
    BS, D, G = block_size, head_dim, head_dim // 64
    cb = BS * D // 2
    kc = pages[:, :, :cb].reshape(NB, H, BS, D // 2)
    vc = pages[:, :, cb:2 * cb].reshape(NB, H, BS, D // 2).copy()
    if D == 128:
        swap = (np.arange(BS) & 2) != 0
        vc[:, :, swap] = np.concatenate([vc[:, :, swap, 32:], vc[:, :, swap, :32]], axis=-1)
    ks = np.ascontiguousarray(pages[:, :, 2 * cb:2 * cb + BS * G * 2]).view(np.float16).reshape(NB, H, BS, G)
    vraw = np.ascontiguousarray(pages[:, :, 2 * cb + BS * G * 2:]).view(np.float16).reshape(NB, H, BS // 16, G, 16)
    r = np.arange(16)
    slot = 2 * (r & 3) + ((r >> 2) & 1) + 8 * (r >> 3)
    vs = vraw[..., slot].transpose(0, 1, 2, 4, 3).reshape(NB, H, BS, G)
    return kc, ks, vc, vs


def evict_tokens(scores, block_tables, is_block_free, kpool, vpool, retain_ratio, num_sink_tokens=4):
    """In place on block_tables / is_block_free / pools.  Returns (idx, cnt, thr)."""
    scores = _c(scores, np.float32)
    S, H, L = scores.shape
    MB = block_tables.shape[1]
    NBF = is_block_free.shape[0]
    BS, D = kpool.shape[1], kpool.shape[3]
    idx = np.full((S, H, L), -1, np.int32)
    cnt = np.zeros((S, H), np.int32)
    thr = np.zeros((S, H), np.float32)
    lib().oracle_evict_tokens(_p(scores), I32(S), I32(H), I32(L), _p(block_tables), I32(MB),
                              _p(is_block_free), I32(NBF), _p(kpool), _p(vpool), I32(BS), I32(D),
                              F32(retain_ratio), I32(num_sink_tokens), _p(idx), _p(cnt), _p(thr))
    return idx, cnt, thr


def evict_cache(scores, kpool, vpool, retain_ratio) -> None:
    scores = _c(scores, np.float32)
    NB, BS, H = scores.shape
    D = kpool.shape[3]
    lib().oracle_evict_cache(_p(scores), I32(NB), I32(BS), I32(H), I32(D), _p(kpool), _p(vpool),
                             F32(retain_ratio))


def paged_attention_f16(q, kpool, vpool, block_tables, context_lens, max_seq_len, window_size, causal=False):
    """fp64 output [B, QL, H, D].  The pool's head count (kpool.shape[2]) may
    divide H (grouped-query attention: query head h reads KV head h / (H/KVH));
    causal=True: row i is the token at ctx - QL + i (an extension)."""
    q = _c(q, np.float16)
    B, QL, H, D = q.shape
    NB, BS, KVH = kpool.shape[0], kpool.shape[1], kpool.shape[2]
    bt, cl = _c(block_tables, np.int32), _c(context_lens, np.int32)
    out = np.zeros((B, QL, H, D), np.float64)
    lib().oracle_paged_attention_f16_ex(_p(q), _p(_c(kpool)), _p(_c(vpool)), _p(bt), _p(cl), I32(B),
                                        I32(QL), I32(H), I32(KVH), I32(D), I32(bt.shape[1]), I64(NB), I32(BS),
                                        I32(max_seq_len), I32(window_size), I32(int(causal)), _p(out))
    return out


def paged_attention_int4(q, pages, block_tables, context_lens, max_seq_len, window_size, block_size,
                         causal=False):
    """pages [NB, KVH, page_bytes]; KVH may divide H as in paged_attention_f16."""
    q = _c(q, np.float16)
    B, QL, H, D = q.shape
    NB, KVH = pages.shape[0], pages.shape[1]
    bt, cl = _c(block_tables, np.int32), _c(context_lens, np.int32)
    out = np.zeros((B, QL, H, D), np.float64)
    lib().oracle_paged_attention_int4_ex(_p(q), _p(_c(pages)), _p(bt), _p(cl), I32(B), I32(QL), I32(H), I32(KVH),
                                         I32(D), I32(bt.shape[1]), I64(NB), I32(block_size), I32(max_seq_len),
                                         I32(window_size), I32(int(causal)), _p(out))
    return out


def evict_topk_head_sum(scores):
    """fp32 sum over heads, in head order, of scores [S, H, L] -> [S, L]
    (starting from +0, as the device kernel does)."""
    S, H, L = scores.shape
    tot = np.zeros((S, L), np.float32)
    for h in range(H):
        tot = (tot + scores[:, h].astype(np.float32)).astype(np.float32)
    return tot


def evict_topk_compact(scores, block_tables, context_lens, kpool, vpool, retain_ratio, num_sink_tokens=4):
    """Restatement of the exact top-k eviction with compaction (this build's
    operator; no reference counterpart).  In place on block_tables,
    context_lens and the fp16 pools; returns (kept_idx, kept_count,
    freed_pages, freed_count).  Pure numpy: token score = fp32 sum over heads
    in head order, sinks always kept, invalid tokens never kept, ties by lower
    index, NaN lowest."""
    return evict_topk_compact_parts(evict_topk_head_sum(scores)[None], block_tables, context_lens, kpool, vpool,
                                    retain_ratio, num_sink_tokens)


def evict_topk_compact_parts(parts, block_tables, context_lens, kpool, vpool, retain_ratio, num_sink_tokens=4):
    """The head-sharded form: parts [G, S, L] are the ranks' partial token
    scores (evict_topk_head_sum of each rank's heads) in rank order; the token
    score is their fp32 sum in rank order.  kpool/vpool hold this rank's heads."""
    NB, BS = kpool.shape[0], kpool.shape[1]
    get = lambda pg, pos: (kpool[pg, pos].copy(), vpool[pg, pos].copy())

    def put(pg, pos, row):
        kpool[pg, pos], vpool[pg, pos] = row

    return _topk_compact_rows(parts, block_tables, context_lens, NB, BS, get, put, retain_ratio, num_sink_tokens)


def evict_topk_compact_int4(scores, block_tables, context_lens, kc, ks, vc, vs, retain_ratio, num_sink_tokens=4):
    """The same operator on an INT4 pool, in the logical views of int4_views
    (codes [NB, H, BS, D/2], fp16 scales [NB, H, BS, D/64]; modified in
    place): a kept token's codes and scales move with it, every head."""
    NB, BS = kc.shape[0], kc.shape[2]
    get = lambda pg, pos: (kc[pg, :, pos].copy(), ks[pg, :, pos].copy(), vc[pg, :, pos].copy(), vs[pg, :, pos].copy())

    def put(pg, pos, row):
        kc[pg, :, pos], ks[pg, :, pos], vc[pg, :, pos], vs[pg, :, pos] = row

    return _topk_compact_rows(evict_topk_head_sum(scores)[None], block_tables, context_lens, NB, BS, get, put,
                              retain_ratio, num_sink_tokens)


def _topk_compact_rows(parts, block_tables, context_lens, NB, BS, get, put, retain_ratio, num_sink_tokens):
    """Decision and row moves shared by both pool formats: get(page, pos) reads
    a token row of every head, put(page, pos, row) writes one."""
    G, S, L = parts.shape
    MB = block_tables.shape[1]
    kept_idx = np.full((S, L), -1, np.int32)
    kept_count = np.zeros(S, np.int32)
    freed = np.full((S, MB), -1, np.int32)
    freed_count = np.zeros(S, np.int32)
    total = np.zeros((S, L), np.float32)
    for g in range(G):
        total = (total + parts[g].astype(np.float32)).astype(np.float32)
    for b in range(S):
        n = min(max(int(context_lens[b]), 0), L)
        tot = total[b]
        row = block_tables[b].copy()
        valid_pages = [int(p) for p in row if 0 <= p < NB]
        cand = []
        for t in range(n):
            lb = t // BS
            pg = int(row[lb]) if lb < MB else -1
            if 0 <= pg < NB:
                s = tot[t]
                key = (3, 0.0) if t < num_sink_tokens else ((0, 0.0) if np.isnan(s) else (1, float(s)))
                cand.append((key, t))
        nv = len(cand)
        keep = 0 if nv == 0 else max(1, min(nv, int(np.ceil(np.float32(retain_ratio) * np.float32(nv)))))
        # largest first; ties: lower index first
        order = sorted(cand, key=lambda kt: (-kt[0][0], -kt[0][1], kt[1]))
        kept = sorted(t for _, t in order[:keep])
        kept_idx[b, :keep] = kept
        kept_count[b] = keep
        old = row.copy()
        rows = [get(old[t // BS], t % BS) for t in kept]
        need = (keep + BS - 1) // BS
        new_row = np.full(MB, -1, np.int32)
        new_row[:need] = valid_pages[:need]
        fl = valid_pages[need:]
        freed[b, :len(fl)] = fl
        freed_count[b] = len(fl)
        block_tables[b] = new_row
        for i in range(keep):
            put(new_row[i // BS], i % BS, rows[i])
        context_lens[b] = keep
    return kept_idx, kept_count, freed, freed_count
