"""The allocation-free paged decode entry point, through the C-ABI.

memopt_paged_attention_f16_noalloc serves callers that cannot allocate device
memory when they run attention (hosts with their own allocator-free runtime,
or steps where allocator calls are forbidden): its split-K scratch is a fixed
array inside the library.  Its output must match memopt_paged_attention_f16
(caller-provided workspace) within the attention tolerance, on two calls in a
row (the second call reuses the scratch the first one left behind), and a
call whose scratch would not fit must be rejected cleanly.

This file is collected last on purpose; it must pass on its own in a fresh
process as well as after every other test.
"""
from __future__ import annotations

import ctypes as C

import numpy as np
import pytest
import torch

import capi

pytestmark = pytest.mark.gpu
ATOL, RTOL = 2e-3, 1e-2


def _noalloc(q, kp, vp, bt, cl, msl, win, out):
    B, QL, H, D = q.shape
    lib = capi.lib()
    return lib.memopt_paged_attention_f16_noalloc(
        capi.ptr(q), capi.ptr(kp), capi.ptr(vp), capi.ptr(bt), capi.ptr(cl), C.c_int(B), C.c_int(QL),
        C.c_int(H), C.c_int(D), C.c_int(bt.shape[1]), C.c_int64(kp.shape[0]), C.c_int(kp.shape[1]),
        C.c_int(msl), C.c_int(win), capi.ptr(out), capi.stream())


def _case(B, H, D, BS, ctx, seed):
    g = torch.Generator().manual_seed(seed)
    MB = max(ctx) // BS
    NB = B * MB + 3
    bt = torch.randperm(NB, generator=g)[: B * MB].reshape(B, MB).to(torch.int32).cuda()
    kp = torch.randn(NB, BS, H, D, generator=g).half().cuda()
    vp = torch.randn(NB, BS, H, D, generator=g).half().cuda()
    q = torch.randn(B, 1, H, D, generator=g).half().cuda()
    cl = torch.tensor(ctx, dtype=torch.int32).cuda()
    return q, kp, vp, bt, cl, MB * BS


@pytest.mark.parametrize("B,H,D,BS,ctx,win", [(4, 32, 128, 16, [4096, 4000, 17, 2048], 4096),
                                              (2, 8, 64, 32, [1024, 999], 300)])
def test_noalloc_matches_workspace_entry_point_twice(B, H, D, BS, ctx, win):
    q, kp, vp, bt, cl, msl = _case(B, H, D, BS, ctx, sum(ctx))
    need = capi.lib().memopt_paged_attention_workspace_size(B, 1, H, D, bt.shape[1], BS, msl, win)
    assert need > 0  # the case exercises the split-K scratch
    ref = capi.attention_f16(q, kp, vp, bt, cl, msl, win)
    for _ in range(2):
        out = torch.full_like(q, float("nan"))
        st = _noalloc(q, kp, vp, bt, cl, msl, win, out)
        assert st == 0, capi.lib().memopt_last_error().decode()
        torch.cuda.synchronize()
        np.testing.assert_allclose(out.float().cpu().numpy(), ref.float().cpu().numpy(), atol=ATOL, rtol=RTOL)


def test_noalloc_rejects_oversized_calls():
    lib = capi.lib()
    lib.memopt_paged_attention_noalloc_max_bytes.restype = C.c_size_t
    cap = lib.memopt_paged_attention_noalloc_max_bytes()
    # ~4700 (sequence, head) rows split in two chunks need ~4.9 MB of partials.
    B, H, D, BS, MB = 47, 100, 128, 16, 64
    need = lib.memopt_paged_attention_workspace_size(B, 1, H, D, MB, BS, MB * BS, MB * BS)
    assert need > cap
    q = torch.zeros(B, 1, H, D, dtype=torch.float16, device="cuda")
    kp = torch.zeros(4, BS, H, D, dtype=torch.float16, device="cuda")
    bt = torch.zeros(B, MB, dtype=torch.int32, device="cuda")
    cl = torch.zeros(B, dtype=torch.int32, device="cuda")
    out = torch.empty_like(q)
    st = _noalloc(q, kp, kp, bt, cl, MB * BS, MB * BS, out)
    assert st == -6  # MEMOPT_ERR_WORKSPACE
    assert b"static scratch" in lib.memopt_last_error()


def test_noalloc_rejects_bad_arguments_before_touching_the_scratch():
    """A call with invalid arguments fails before any work is queued (so it
    cannot clear the tickets of another call that is using the scratch)."""
    q, kp, vp, bt, cl, msl = _case(2, 8, 128, 16, [300, 200], 9)
    out = torch.empty_like(q)
    lib = capi.lib()
    bad = kp.view(-1)[1:]  # a pool pointer 2 bytes off alignment
    st = lib.memopt_paged_attention_f16_noalloc(
        capi.ptr(q), capi.ptr(bad), capi.ptr(vp), capi.ptr(bt), capi.ptr(cl), C.c_int(2), C.c_int(1), C.c_int(8),
        C.c_int(128), C.c_int(bt.shape[1]), C.c_int64(kp.shape[0]), C.c_int(16), C.c_int(msl), C.c_int(msl),
        capi.ptr(out), capi.stream())
    assert st == -1  # MEMOPT_ERR_INVALID_ARG
    assert b"16-byte aligned" in lib.memopt_last_error()
