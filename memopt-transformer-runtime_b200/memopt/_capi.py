"""ctypes binding of libmemopt_b200.so (the C-ABI in include/memopt_b200.h).

This is the binding a host without PyTorch extensions would use; tensors are
passed as raw device pointers.  bench.py times the kernels through it.
"""
from __future__ import annotations

import ctypes as C
import os

# MEMOPT_LIB names another build of the same library (a variant compiled with
# different tuning macros); by default the in-tree build is loaded.
_LIB_PATH = os.environ.get("MEMOPT_LIB") or os.path.join(
    os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "libmemopt_b200.so")
P, I, I64, F, SZ = C.c_void_p, C.c_int, C.c_int64, C.c_float, C.c_size_t
_lib = None


class MemoptError(RuntimeError):
    pass


def lib() -> C.CDLL:
    global _lib
    if _lib is None:
        if not os.path.exists(_LIB_PATH):
            raise MemoptError(f"{_LIB_PATH} is missing; run memopt-transformer-runtime_b200/build.py")
        _lib = C.CDLL(_LIB_PATH)
        _lib.memopt_last_error.restype = C.c_char_p
        _lib.memopt_paged_attention_workspace_size.restype = SZ
        _lib.memopt_paged_attention_workspace_size_ex.restype = SZ
        _lib.memopt_paged_attention_int4_workspace_size_ex.restype = SZ
        _lib.memopt_paged_attention_ticket_bytes.restype = SZ
    return _lib


def check(status: int, what: str) -> None:
    if status != 0:
        raise MemoptError(f"{what}: {lib().memopt_last_error().decode()} (status {status})")


def paged_attention_f16(q, kpool, vpool, bt, ctx, out, msl, win, ws, ws_bytes, stream):
    B, QL, H, D = q.shape
    check(lib().memopt_paged_attention_f16(
        P(q.data_ptr()), P(kpool.data_ptr()), P(vpool.data_ptr()), P(bt.data_ptr()), P(ctx.data_ptr()),
        I(B), I(QL), I(H), I(D), I(bt.shape[1]), I64(kpool.shape[0]), I(kpool.shape[1]), I(msl), I(win),
        P(out.data_ptr()), P(ws.data_ptr() if ws is not None else 0), SZ(ws_bytes), P(stream)),
        "memopt_paged_attention_f16")


def paged_attention_int4(q, pages, block_size, bt, ctx, out, msl, win, ws, ws_bytes, stream):
    B, QL, H, D = q.shape
    check(lib().memopt_paged_attention_int4(
        P(q.data_ptr()), P(pages.data_ptr()), P(bt.data_ptr()), P(ctx.data_ptr()), I(B), I(QL), I(H), I(D),
        I(bt.shape[1]), I64(pages.shape[0]), I(block_size), I(msl), I(win), P(out.data_ptr()),
        P(ws.data_ptr() if ws is not None else 0), SZ(ws_bytes), P(stream)), "memopt_paged_attention_int4")


def paged_attention_f16_ex(q, kpool, vpool, bt, ctx, out, msl, win, causal, ws, ws_bytes, stream):
    """Pools of kpool.shape[2] heads (dividing the query's H)."""
    B, QL, H, D = q.shape
    check(lib().memopt_paged_attention_f16_ex(
        P(q.data_ptr()), P(kpool.data_ptr()), P(vpool.data_ptr()), P(bt.data_ptr()), P(ctx.data_ptr()),
        I(B), I(QL), I(H), I(kpool.shape[2]), I(D), I(bt.shape[1]), I64(kpool.shape[0]), I(kpool.shape[1]),
        I(msl), I(win), I(int(causal)), P(out.data_ptr()), P(ws.data_ptr() if ws is not None else 0),
        SZ(ws_bytes), P(stream)), "memopt_paged_attention_f16_ex")


def paged_attention_int4_ex(q, pages, block_size, bt, ctx, out, msl, win, causal, ws, ws_bytes, stream):
    """INT4 pages [NB, KVH, page_bytes] with KVH dividing the query's H."""
    B, QL, H, D = q.shape
    check(lib().memopt_paged_attention_int4_ex(
        P(q.data_ptr()), P(pages.data_ptr()), P(bt.data_ptr()), P(ctx.data_ptr()), I(B), I(QL), I(H),
        I(pages.shape[1]), I(D), I(bt.shape[1]), I64(pages.shape[0]), I(block_size), I(msl), I(win),
        I(int(causal)), P(out.data_ptr()), P(ws.data_ptr() if ws is not None else 0), SZ(ws_bytes), P(stream)),
        "memopt_paged_attention_int4_ex")


def evict_topk_workspace_size(S, L, H, D) -> int:
    lib().memopt_evict_topk_workspace_size.restype = SZ
    return int(lib().memopt_evict_topk_workspace_size(I(S), I(L), I(H), I(D)))


def evict_topk_compact_int4(scores, bt, ctx, pages, block_size, head_dim, retain_ratio, sinks, kept, cnt, freed,
                            fcnt, ws, ws_bytes, stream):
    """Exact top-k eviction with compaction on INT4 pages [NB, H, page_bytes]."""
    S, H, L = scores.shape
    check(lib().memopt_evict_topk_compact_int4(
        P(scores.data_ptr()), I(S), I(H), I(L), P(bt.data_ptr()), I(bt.shape[1]), P(ctx.data_ptr()),
        P(pages.data_ptr()), I(pages.shape[0]), I(block_size), I(head_dim), C.c_float(retain_ratio), I(sinks),
        P(kept.data_ptr()), P(cnt.data_ptr()), P(freed.data_ptr()), P(fcnt.data_ptr()), P(ws.data_ptr()),
        SZ(ws_bytes), P(stream)), "memopt_evict_topk_compact_int4")


def workspace_size_ex(B, QL, H, KVH, D, MB, BS, msl, win) -> int:
    return int(lib().memopt_paged_attention_workspace_size_ex(B, QL, H, KVH, D, MB, BS, msl, win))


def int4_workspace_size_ex(B, QL, H, KVH, D, MB, BS, msl, win) -> int:
    """Workspace of an INT4-pool call: the split workspace plus, for q_len >=
    64, the fp16 page scratch of the prefill path."""
    return int(lib().memopt_paged_attention_int4_workspace_size_ex(B, QL, H, KVH, D, MB, BS, msl, win))


def workspace_size(B, QL, H, D, MB, BS, msl, win) -> int:
    return int(lib().memopt_paged_attention_workspace_size(B, QL, H, D, MB, BS, msl, win))


def evict_tokens(scores, bt, ibf, kpool, vpool, retain_ratio, num_sinks, idx, cnt, stream):
    S, Hh, L = scores.shape
    check(lib().memopt_evict_tokens(
        P(scores.data_ptr()), I(S), I(Hh), I(L), P(bt.data_ptr()), I(bt.shape[1]), P(ibf.data_ptr()),
        I(ibf.shape[0]), P(kpool.data_ptr()), P(vpool.data_ptr()), I(kpool.shape[0]), I(kpool.shape[1]),
        I(kpool.shape[3]), F(retain_ratio), I(num_sinks), P(idx.data_ptr() if idx is not None else 0),
        P(cnt.data_ptr() if cnt is not None else 0), P(stream)), "memopt_evict_tokens")


def quantize_int4(x, packed, scales, stream):
    check(lib().memopt_quantize_int4(P(x.data_ptr()), I64(x.numel()), I(64), P(packed.data_ptr()),
                                     P(scales.data_ptr()), P(stream)), "memopt_quantize_int4")


def dequantize_int4(packed, scales, out, stream):
    check(lib().memopt_dequantize_int4(P(packed.data_ptr()), P(scales.data_ptr()), I64(out.numel()), I(64),
                                       P(out.data_ptr()), P(stream)), "memopt_dequantize_int4")


def write_cache_f16(keys, values, slots, kpool, vpool, stream):
    T, H, D = keys.shape
    check(lib().memopt_write_cache_f16(P(keys.data_ptr()), P(values.data_ptr()), P(slots.data_ptr()), I64(T), I(H),
                                       I(D), P(kpool.data_ptr()), P(vpool.data_ptr()), I64(kpool.shape[0]),
                                       I(kpool.shape[1]), P(0), P(stream)), "memopt_write_cache_f16")


def write_cache_int4(keys, values, slots, pages, block_size, stream):
    T, H, D = keys.shape
    check(lib().memopt_write_cache_int4(P(keys.data_ptr()), P(values.data_ptr()), P(slots.data_ptr()), I64(T), I(H),
                                        I(D), P(pages.data_ptr()), I64(pages.shape[0]), I(block_size), P(0),
                                        P(stream)), "memopt_write_cache_int4")


def evict_cache(scores, kpool, vpool, retain_ratio, stream):
    NB, BS, H = scores.shape
    check(lib().memopt_evict_cache(P(scores.data_ptr()), I(NB), I(BS), I(H), I(kpool.shape[3]),
                                   P(kpool.data_ptr()), P(vpool.data_ptr()), F(retain_ratio), P(stream)),
          "memopt_evict_cache")
