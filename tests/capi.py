"""ctypes access to libmemopt_b200.so for the GPU parity tests.

Every call goes through the C-ABI declared in include/memopt_b200.h with raw
device pointers of torch tensors and the current torch stream.
"""
from __future__ import annotations

import ctypes as C
import os

import torch

from conftest import PKG

_lib = None
P, I, I64, F, SZ = C.c_void_p, C.c_int, C.c_int64, C.c_float, C.c_size_t


def lib() -> C.CDLL:
    global _lib
    if _lib is None:
        _lib = C.CDLL(os.environ.get("MEMOPT_LIB") or os.path.join(PKG, "libmemopt_b200.so"))
        _lib.memopt_last_error.restype = C.c_char_p
        _lib.memopt_paged_attention_workspace_size.restype = SZ
        _lib.memopt_paged_attention_ticket_bytes.restype = SZ
    return _lib


def ptr(t: torch.Tensor | None) -> P:
    return P(0 if t is None else t.data_ptr())


def stream() -> P:
    return P(torch.cuda.current_stream().cuda_stream)


def ok(st: int) -> None:
    assert st == 0, f"status {st}: {lib().memopt_last_error().decode()}"


def write_cache_f16(keys, values, slots, kpool, vpool, bad=None):
    T, H, D = keys.shape
    ok(lib().memopt_write_cache_f16(ptr(keys), ptr(values), ptr(slots), I64(T), I(H), I(D), ptr(kpool),
                                    ptr(vpool), I64(kpool.shape[0]), I(kpool.shape[1]), ptr(bad), stream()))


def write_cache_int4(keys, values, slots, pages, block_size, bad=None):
    T, H, D = keys.shape
    ok(lib().memopt_write_cache_int4(ptr(keys), ptr(values), ptr(slots), I64(T), I(H), I(D), ptr(pages),
                                     I64(pages.shape[0]), I(block_size), ptr(bad), stream()))


def quantize(x):
    n = x.numel()
    packed = torch.empty(x.shape[:-1] + (x.shape[-1] // 2,), dtype=torch.uint8, device=x.device)
    scales = torch.empty(n // 64, dtype=torch.float32, device=x.device)
    ok(lib().memopt_quantize_int4(ptr(x), I64(n), I(64), ptr(packed), ptr(scales), stream()))
    return packed, scales


def dequantize(packed, scales):
    out = torch.empty(packed.shape[:-1] + (packed.shape[-1] * 2,), dtype=torch.float16, device=packed.device)
    ok(lib().memopt_dequantize_int4(ptr(packed), ptr(scales), I64(out.numel()), I(64), ptr(out), stream()))
    return out


def evict_tokens(scores, bt, ibf, kpool, vpool, r, sinks, retained=True):
    S, H, L = scores.shape
    idx = torch.full((S, H, L), -7, dtype=torch.int32, device=scores.device) if retained else None
    cnt = torch.full((S, H), -7, dtype=torch.int32, device=scores.device) if retained else None
    ok(lib().memopt_evict_tokens(ptr(scores), I(S), I(H), I(L), ptr(bt), I(bt.shape[1]), ptr(ibf),
                                 I(ibf.shape[0]), ptr(kpool), ptr(vpool), I(kpool.shape[0]), I(kpool.shape[1]),
                                 I(kpool.shape[3]), F(r), I(sinks), ptr(idx), ptr(cnt), stream()))
    return idx, cnt


def evict_cache(scores, kpool, vpool, r):
    NB, BS, H = scores.shape
    ok(lib().memopt_evict_cache(ptr(scores), I(NB), I(BS), I(H), I(kpool.shape[3]), ptr(kpool), ptr(vpool),
                                F(r), stream()))


def workspace(B, QL, H, D, MB, BS, msl, win, device="cuda", kvh=None, int4=False):
    fn = lib().memopt_paged_attention_int4_workspace_size_ex if int4 else lib().memopt_paged_attention_workspace_size_ex
    fn.restype = SZ
    n = fn(B, QL, H, H if kvh is None else kvh, D, MB, BS, msl, win)
    if n == 0:
        return None, 0
    ws = torch.zeros(n, dtype=torch.uint8, device=device)
    return ws, n


def attention_f16(q, kpool, vpool, bt, ctx, msl, win, ws=None):
    B, QL, H, D = q.shape
    MB = bt.shape[1]
    out = torch.empty_like(q)
    if ws is None:
        ws, n = workspace(B, QL, H, D, MB, kpool.shape[1], msl, win)
    else:
        n = ws.numel()
    ok(lib().memopt_paged_attention_f16(ptr(q), ptr(kpool), ptr(vpool), ptr(bt), ptr(ctx), I(B), I(QL), I(H),
                                        I(D), I(MB), I64(kpool.shape[0]), I(kpool.shape[1]), I(msl), I(win),
                                        ptr(out), ptr(ws), SZ(n), stream()))
    return out


def attention_int4(q, pages, block_size, bt, ctx, msl, win, ws=None):
    B, QL, H, D = q.shape
    MB = bt.shape[1]
    out = torch.empty_like(q)
    if ws is None:
        ws, n = workspace(B, QL, H, D, MB, block_size, msl, win, int4=True)
    else:
        n = ws.numel()
    ok(lib().memopt_paged_attention_int4(ptr(q), ptr(pages), ptr(bt), ptr(ctx), I(B), I(QL), I(H), I(D), I(MB),
                                         I64(pages.shape[0]), I(block_size), I(msl), I(win), ptr(out), ptr(ws),
                                         SZ(n), stream()))
    return out


def int4_page_bytes(block_size, head_dim):
    lib().memopt_int4_page_bytes.restype = SZ
    return int(lib().memopt_int4_page_bytes(I(block_size), I(head_dim)))


def _topk_status(ws, S, L, status):
    """memopt_evict_topk_status after a compaction: asserted OK, or appended
    to ``status`` (a list) when the caller checks it itself."""
    st = lib().memopt_evict_topk_status(ptr(ws), I(S), I(L), stream())
    if status is None:
        ok(st)
    else:
        status.append(st)


def evict_topk_compact(scores, bt, ctx, kpool, vpool, retain_ratio, sinks, status=None):
    S, H, L = scores.shape
    MB = bt.shape[1]
    dev = scores.device
    kept = torch.empty(S, L, dtype=torch.int32, device=dev)
    cnt = torch.empty(S, dtype=torch.int32, device=dev)
    freed = torch.empty(S, MB, dtype=torch.int32, device=dev)
    fcnt = torch.empty(S, dtype=torch.int32, device=dev)
    lib().memopt_evict_topk_workspace_size.restype = SZ
    wsb = int(lib().memopt_evict_topk_workspace_size(I(S), I(L), I(H), I(kpool.shape[3])))
    ws = torch.empty(max(wsb, 16), dtype=torch.uint8, device=dev)
    ok(lib().memopt_evict_topk_compact(ptr(scores), I(S), I(H), I(L), ptr(bt), I(MB), ptr(ctx), ptr(kpool),
                                       ptr(vpool), I(kpool.shape[0]), I(kpool.shape[1]), I(kpool.shape[3]),
                                       F(retain_ratio), I(sinks), ptr(kept), ptr(cnt), ptr(freed), ptr(fcnt),
                                       ptr(ws), SZ(wsb), stream()))
    _topk_status(ws, S, L, status)
    return kept, cnt, freed, fcnt


def evict_topk_compact_int4(scores, bt, ctx, pages, block_size, head_dim, retain_ratio, sinks, status=None):
    S, H, L = scores.shape
    MB = bt.shape[1]
    dev = scores.device
    kept = torch.empty(S, L, dtype=torch.int32, device=dev)
    cnt = torch.empty(S, dtype=torch.int32, device=dev)
    freed = torch.empty(S, MB, dtype=torch.int32, device=dev)
    fcnt = torch.empty(S, dtype=torch.int32, device=dev)
    lib().memopt_evict_topk_workspace_size.restype = SZ
    wsb = int(lib().memopt_evict_topk_workspace_size(I(S), I(L), I(H), I(head_dim)))
    ws = torch.empty(max(wsb, 16), dtype=torch.uint8, device=dev)
    ok(lib().memopt_evict_topk_compact_int4(ptr(scores), I(S), I(H), I(L), ptr(bt), I(MB), ptr(ctx), ptr(pages),
                                            I(pages.shape[0]), I(block_size), I(head_dim), F(retain_ratio), I(sinks),
                                            ptr(kept), ptr(cnt), ptr(freed), ptr(fcnt), ptr(ws), SZ(wsb), stream()))
    _topk_status(ws, S, L, status)
    return kept, cnt, freed, fcnt


def evict_topk_head_sum(scores):
    S, H, L = scores.shape
    out = torch.empty(S, L, dtype=torch.float32, device=scores.device)
    ok(lib().memopt_evict_topk_head_sum(ptr(scores), I(S), I(H), I(L), ptr(out), stream()))
    return out


def evict_topk_compact_parts(parts, bt, ctx, kpool, vpool, retain_ratio, sinks, status=None):
    G, S, L = parts.shape
    MB = bt.shape[1]
    dev = parts.device
    H, D = kpool.shape[2], kpool.shape[3]
    kept = torch.empty(S, L, dtype=torch.int32, device=dev)
    cnt = torch.empty(S, dtype=torch.int32, device=dev)
    freed = torch.empty(S, MB, dtype=torch.int32, device=dev)
    fcnt = torch.empty(S, dtype=torch.int32, device=dev)
    lib().memopt_evict_topk_workspace_size.restype = SZ
    wsb = int(lib().memopt_evict_topk_workspace_size(I(S), I(L), I(H), I(D)))
    ws = torch.empty(max(wsb, 16), dtype=torch.uint8, device=dev)
    ok(lib().memopt_evict_topk_compact_parts(ptr(parts), I(G), I(S), I(L), ptr(bt), I(MB), ptr(ctx), ptr(kpool),
                                             ptr(vpool), I(kpool.shape[0]), I(kpool.shape[1]), I(H), I(D),
                                             F(retain_ratio), I(sinks), ptr(kept), ptr(cnt), ptr(freed), ptr(fcnt),
                                             ptr(ws), SZ(wsb), stream()))
    _topk_status(ws, S, L, status)
    return kept, cnt, freed, fcnt


def attention_f16_ex(q, kpool, vpool, bt, ctx, msl, win, causal=False):
    """memopt_paged_attention_f16_ex: the pool's head count may divide H."""
    B, QL, H, D = q.shape
    MB = bt.shape[1]
    out = torch.empty_like(q)
    ws, n = workspace(B, QL, H, D, MB, kpool.shape[1], msl, win, kvh=kpool.shape[2])
    ok(lib().memopt_paged_attention_f16_ex(ptr(q), ptr(kpool), ptr(vpool), ptr(bt), ptr(ctx), I(B), I(QL), I(H),
                                           I(kpool.shape[2]), I(D), I(MB), I64(kpool.shape[0]), I(kpool.shape[1]),
                                           I(msl), I(win), I(int(causal)), ptr(out), ptr(ws), SZ(n), stream()))
    return out


def attention_int4_ex(q, pages, block_size, bt, ctx, msl, win, causal=False):
    B, QL, H, D = q.shape
    MB = bt.shape[1]
    out = torch.empty_like(q)
    ws, n = workspace(B, QL, H, D, MB, block_size, msl, win, kvh=pages.shape[1], int4=True)
    ok(lib().memopt_paged_attention_int4_ex(ptr(q), ptr(pages), ptr(bt), ptr(ctx), I(B), I(QL), I(H),
                                            I(pages.shape[1]), I(D), I(MB), I64(pages.shape[0]), I(block_size),
                                            I(msl), I(win), I(int(causal)), ptr(out), ptr(ws), SZ(n), stream()))
    return out


def evict_topk_set_test_hooks(flag_poll_limit: int, withhold_read_flags: bool) -> None:
    ok(lib().memopt_evict_topk_set_test_hooks(C.c_uint32(flag_poll_limit), I(int(withhold_read_flags))))
