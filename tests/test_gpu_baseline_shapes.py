"""GPU parity at the shapes the benchmark times, and on pools past 2^31.

* configs[1] decode: the benchmark's own seeded workload (batch 32, 32 heads
  x 128, 4096 tokens), a subset of its sequences checked against the oracle.
* configs[4] prefill: the benchmark's own seeded workload (4 x 8192 queries
  over 8192 tokens, 32 heads), 128 sampled query rows of every sequence and
  head against the fp64 oracle (non-causal rows are independent, so the
  oracle runs on the sampled rows alone).
* configs[4] prefill over INT4 pages (the same rows written by the fused
  writer): 64 sampled query rows of every sequence and head.
* configs[4] decode: INT4 pages written by the fused write_cache for a
  131072-token sequence, 32 heads, decode against the oracle.
* 64-bit offsets: an fp16 pool of 40000 pages x 16 x 32 x 128 (2.6e9
  elements per pool) and an INT4 pool of 32000 pages x 32 heads x 2176 B
  (2.2e9 bytes), with the sequences on the highest physical pages; write,
  decode (one-row and multi-query), prefill (fp16 and INT4), evict_tokens and both
  compactions run there and are checked on a compact copy of the touched
  pages.

Tolerances: bit-exact for pages, codes, tables and indices; attention within
2e-3 absolute + 1e-2 relative of the fp64 oracle.
"""
from __future__ import annotations

import numpy as np
import pytest
import torch

import bench
import capi
import oracle as O

pytestmark = pytest.mark.gpu
ATOL, RTOL = 2e-3, 1e-2
DEV = torch.device("cuda", 0)


def np16(t):
    return t.detach().cpu().numpy()


def _close(got, ref):
    np.testing.assert_allclose(np16(got).astype(np.float64), ref, atol=ATOL, rtol=RTOL)


def _compact(bt, *pools):
    """Pages referenced by bt gathered into a small pool: (bt remapped, pages
    used in ascending order, gathered copies of each pool)."""
    bt = np.asarray(bt)
    used = np.unique(bt[bt >= 0])
    remap = np.full(int(used.max()) + 1 if used.size else 1, -1, np.int64)
    remap[used] = np.arange(used.size)
    cbt = np.where(bt >= 0, remap[np.maximum(bt, 0)], -1).astype(np.int32)
    idx = torch.from_numpy(used).to(DEV)
    return cbt, used, [np.ascontiguousarray(np16(p.index_select(0, idx))) for p in pools]


# ------------------------------------------------------ benchmark workloads
def test_cfg1_benchmark_decode_workload():
    kp, vp, bt, q, ctx = bench.make_fp16_workload(torch, 1234, DEV)
    msl = bench.CTX
    out = capi.attention_f16(q, kp, vp, bt, ctx, msl, msl)
    seqs = [0, 13, 31]
    cbt, _, (ckp, cvp) = _compact(np16(bt)[seqs], kp, vp)
    ref = O.paged_attention_f16(np16(q)[seqs], ckp, cvp, cbt, np16(ctx)[seqs], msl, msl)
    _close(out[seqs], ref)


def test_cfg4_prefill_benchmark_workload_sampled_rows():
    kp, vp, bt, q, ctx = bench.make_prefill_workload(torch, DEV)
    QL = bench.PREFILL_QL
    out = capi.attention_f16(q, kp, vp, bt, ctx, QL, QL)
    rows = np.sort(np.random.default_rng(8192).choice(QL, size=128, replace=False))
    rows[0], rows[-1] = 0, QL - 1
    rt = torch.from_numpy(rows).to(DEV)
    bt_h, ctx_h = np16(bt), np16(ctx)
    for b in range(q.shape[0]):
        cbt, _, (ckp, cvp) = _compact(bt_h[b:b + 1], kp, vp)
        qs = np.ascontiguousarray(np16(q[b:b + 1].index_select(1, rt)))
        ref = O.paged_attention_f16(qs, ckp, cvp, cbt, ctx_h[b:b + 1], QL, QL)
        _close(out[b:b + 1].index_select(1, rt), ref)


def test_cfg4_prefill_on_int4_pages_sampled_rows():
    # the benchmark's int4_prefill leg: its K/V rows written into INT4 pages by the fused writer
    kp, vp, bt, q, ctx = bench.make_prefill_workload(torch, DEV)
    QL = bench.PREFILL_QL
    NB, BSZ, NH, HD = kp.shape
    pages = torch.zeros(NB, NH, capi.int4_page_bytes(BSZ, HD), dtype=torch.uint8, device=DEV)
    capi.write_cache_int4(kp.view(-1, NH, HD), vp.view(-1, NH, HD),
                          torch.arange(NB * BSZ, dtype=torch.int32, device=DEV), pages, BSZ)
    del kp, vp
    out = capi.attention_int4(q, pages, BSZ, bt, ctx, QL, QL)
    rows = np.sort(np.random.default_rng(4096).choice(QL, size=64, replace=False))
    rows[0], rows[-1] = 0, QL - 1
    rt = torch.from_numpy(rows).to(DEV)
    bt_h, ctx_h = np16(bt), np16(ctx)
    for b in range(q.shape[0]):
        cbt, _, (cpages,) = _compact(bt_h[b:b + 1], pages)
        qs = np.ascontiguousarray(np16(q[b:b + 1].index_select(1, rt)))
        ref = O.paged_attention_int4(qs, cpages, cbt, ctx_h[b:b + 1], QL, QL, BSZ)
        _close(out[b:b + 1].index_select(1, rt), ref)


def test_cfg4_int4_decode_131072_tokens_written_by_fused_writer():
    L, H, D, BS = 131072, 32, 128, 16
    MB = L // BS
    NB = MB + 7
    g = torch.Generator(device=DEV).manual_seed(131072)
    bt = torch.randperm(NB, generator=torch.Generator().manual_seed(3))[:MB].to(torch.int32).reshape(1, MB).to(DEV)
    pages = torch.zeros(NB, H, capi.int4_page_bytes(BS, D), dtype=torch.uint8, device=DEV)
    slots = (bt.reshape(-1).repeat_interleave(BS) * BS + torch.arange(BS, device=DEV, dtype=torch.int32).repeat(MB))
    slots = slots.to(torch.int32)
    chunk = 16384
    for c0 in range(0, L, chunk):
        k = torch.randn(chunk, H, D, device=DEV, dtype=torch.float16, generator=g)
        v = torch.randn(chunk, H, D, device=DEV, dtype=torch.float16, generator=g)
        capi.write_cache_int4(k, v, slots[c0:c0 + chunk].contiguous(), pages, BS)
    q = torch.randn(1, 1, H, D, device=DEV, dtype=torch.float16, generator=g)
    ctx = torch.full((1,), L, dtype=torch.int32, device=DEV)
    out = capi.attention_int4(q, pages, BS, bt, ctx, L, L)
    ref = O.paged_attention_int4(np16(q), np16(pages), np16(bt), np16(ctx), L, L, BS)
    _close(out, ref)
    # the same pages with a window (configs[3]-style block skipping)
    out_w = capi.attention_int4(q, pages, BS, bt, ctx, L, 4096)
    _close(out_w, O.paged_attention_int4(np16(q), np16(pages), np16(bt), np16(ctx), L, 4096, BS))


# ---------------------------------------------------------- 64-bit offsets
F16_NB, INT4_NB = 40000, 32000
H, D, BS, LSEQ = 32, 128, 16, 1024


def _top_tables(NB, S, MB, seed):
    rng = np.random.default_rng(seed)
    top = NB - S * MB - 16 + rng.permutation(S * MB + 16)[: S * MB]
    return top.astype(np.int32).reshape(S, MB)


@pytest.fixture(scope="module")
def big_f16():
    assert F16_NB * BS * H * D > 2 ** 31
    kp = torch.empty(F16_NB, BS, H, D, dtype=torch.float16, device=DEV)
    vp = torch.empty_like(kp)
    yield kp, vp
    del kp, vp
    torch.cuda.empty_cache()


def _fill(pools, bt, seed):
    g = torch.Generator(device=DEV).manual_seed(seed)
    idx = torch.from_numpy(np.unique(bt)).long().to(DEV)
    for p in pools:
        p[idx] = torch.randn((idx.numel(),) + tuple(p.shape[1:]), device=DEV, dtype=p.dtype, generator=g)


def test_f16_pool_beyond_2p31_write_and_attention(big_f16):
    kp, vp = big_f16
    S, MB = 2, LSEQ // BS
    bt = _top_tables(F16_NB, S, MB, 1)
    _fill((kp, vp), bt, 1)
    # write_cache of every token of both sequences (new values)
    T = S * LSEQ
    slots = (np.repeat(bt.reshape(-1), BS) * BS + np.tile(np.arange(BS), S * MB)).astype(np.int32)
    assert int(slots.max()) * H * D > 2 ** 31
    rng = np.random.default_rng(2)
    k = rng.standard_normal((T, H, D)).astype(np.float16)
    v = rng.standard_normal((T, H, D)).astype(np.float16)
    capi.write_cache_f16(torch.from_numpy(k).to(DEV), torch.from_numpy(v).to(DEV), torch.from_numpy(slots).to(DEV),
                         kp, vp)
    cbt, used, (ckp, cvp) = _compact(bt, kp, vp)
    remap = {int(p): i for i, p in enumerate(used)}
    rk, rv = np.zeros_like(ckp), np.zeros_like(cvp)
    cslots = np.array([remap[int(s) // BS] * BS + int(s) % BS for s in slots], np.int32)
    O.write_cache_f16(k, v, cslots, rk, rv)
    assert np.array_equal(ckp.view(np.uint16), rk.view(np.uint16))
    assert np.array_equal(cvp.view(np.uint16), rv.view(np.uint16))
    gbt = torch.from_numpy(bt).to(DEV)
    ctx = np.array([LSEQ, LSEQ - 77], np.int32)
    gctx = torch.from_numpy(ctx).to(DEV)
    for QL, nh in ((1, H), (4, H), (128, H), (1, 2 * H)):
        q = torch.from_numpy(rng.standard_normal((S, QL, nh, D)).astype(np.float16)).to(DEV)
        if nh == H:
            got = capi.attention_f16(q, kp, vp, gbt, gctx, LSEQ, LSEQ)
        else:  # grouped-query: the multi-query kernel
            got = capi.attention_f16_ex(q, kp, vp, gbt, gctx, LSEQ, LSEQ)
        _close(got, O.paged_attention_f16(np16(q), ckp, cvp, cbt, ctx, LSEQ, LSEQ))


def test_f16_pool_beyond_2p31_evict_tokens(big_f16):
    kp, vp = big_f16
    S, MB = 2, LSEQ // BS
    bt = _top_tables(F16_NB, S, MB, 3)
    _fill((kp, vp), bt, 3)
    sc = np.random.default_rng(4).lognormal(0, 1, (S, H, LSEQ)).astype(np.float32)
    cbt, used, (ckp, cvp) = _compact(bt, kp, vp)
    gbt = torch.from_numpy(bt).to(DEV)
    ibf = torch.zeros(F16_NB, dtype=torch.int32, device=DEV)
    idx, cnt = capi.evict_tokens(torch.from_numpy(sc).to(DEV), gbt, ibf, kp, vp, 0.5, 0)
    cibf = np.zeros(used.size, np.int32)
    ridx, rcnt, _ = O.evict_tokens(sc, cbt, cibf, ckp, cvp, 0.5, 0)
    assert np.array_equal(np16(cnt), rcnt) and np.array_equal(np16(idx), ridx)
    assert int(rcnt.sum()) < S * H * LSEQ  # rows were evicted (and zeroed) at high offsets
    _, _, (gk, gv) = _compact(bt, kp, vp)
    assert np.array_equal(gk.view(np.uint16), ckp.view(np.uint16))
    assert np.array_equal(gv.view(np.uint16), cvp.view(np.uint16))
    back = np.where(cbt >= 0, used[np.maximum(cbt, 0)], cbt)
    assert np.array_equal(np16(gbt), back)
    assert np.array_equal(np16(ibf)[used], cibf)


def test_f16_pool_beyond_2p31_exact_compaction(big_f16):
    kp, vp = big_f16
    S, MB = 2, LSEQ // BS
    bt = _top_tables(F16_NB, S, MB, 5)
    _fill((kp, vp), bt, 5)
    sc = np.random.default_rng(6).lognormal(0, 1, (S, H, LSEQ)).astype(np.float32)
    ctx = np.array([LSEQ, LSEQ - 5], np.int32)
    cbt, used, (ckp, cvp) = _compact(bt, kp, vp)
    gbt, gctx = torch.from_numpy(bt).to(DEV), torch.from_numpy(ctx).to(DEV)
    kept, cnt, freed, fcnt = capi.evict_topk_compact(torch.from_numpy(sc).to(DEV), gbt, gctx, kp, vp, 0.75, 4)
    rctx = ctx.copy()
    rk, rc, rf, rfc = O.evict_topk_compact(sc, cbt, rctx, ckp, cvp, 0.75, 4)
    assert np.array_equal(np16(cnt), rc) and np.array_equal(np16(kept), rk) and np.array_equal(np16(gctx), rctx)
    back = lambda a: np.where(a >= 0, used[np.maximum(a, 0)], a)  # noqa: E731
    assert np.array_equal(np16(gbt), back(cbt)) and np.array_equal(np16(freed), back(rf))
    assert np.array_equal(np16(fcnt), rfc)
    gbt_h = np16(gbt)
    for b in range(S):
        for i in range(0, int(rc[b]), 7):
            pg, pos = gbt_h[b, i // BS], i % BS
            cpg = cbt[b, i // BS]
            assert np.array_equal(np16(kp[pg, pos]).view(np.uint16), ckp[cpg, pos].view(np.uint16))
            assert np.array_equal(np16(vp[pg, pos]).view(np.uint16), cvp[cpg, pos].view(np.uint16))


@pytest.fixture(scope="module")
def big_int4():
    pb = capi.int4_page_bytes(BS, D)
    assert INT4_NB * H * pb > 2 ** 31
    pages = torch.zeros(INT4_NB, H, pb, dtype=torch.uint8, device=DEV)
    yield pages
    del pages
    torch.cuda.empty_cache()


def test_int4_pool_beyond_2p31_write_attention_compaction(big_int4):
    pages = big_int4
    S, MB = 2, LSEQ // BS
    bt = _top_tables(INT4_NB, S, MB, 7)
    T = S * LSEQ
    slots = (np.repeat(bt.reshape(-1), BS) * BS + np.tile(np.arange(BS), S * MB)).astype(np.int32)
    rng = np.random.default_rng(8)
    k = rng.standard_normal((T, H, D)).astype(np.float16)
    v = rng.standard_normal((T, H, D)).astype(np.float16)
    capi.write_cache_int4(torch.from_numpy(k).to(DEV), torch.from_numpy(v).to(DEV), torch.from_numpy(slots).to(DEV),
                          pages, BS)
    cbt, used, (cpages,) = _compact(bt, pages)
    remap = {int(p): i for i, p in enumerate(used)}
    rpages = np.zeros_like(cpages)
    cslots = np.array([remap[int(s) // BS] * BS + int(s) % BS for s in slots], np.int32)
    O.write_cache_int4(k, v, cslots, rpages, BS)
    assert np.array_equal(cpages, rpages)
    gbt = torch.from_numpy(bt).to(DEV)
    ctx = np.array([LSEQ, LSEQ - 300], np.int32)
    gctx = torch.from_numpy(ctx).to(DEV)
    for QL, nh in ((1, H), (1, 2 * H), (3, H), (96, H)):  # q_len 96: the INT4 prefill path
        q = torch.from_numpy(rng.standard_normal((S, QL, nh, D)).astype(np.float16)).to(DEV)
        got = capi.attention_int4_ex(q, pages, BS, gbt, gctx, LSEQ, LSEQ)
        _close(got, O.paged_attention_int4(np16(q), cpages, cbt, ctx, LSEQ, LSEQ, BS))
    # exact compaction on the same pages
    sc = rng.lognormal(0, 1, (S, H, LSEQ)).astype(np.float32)
    views = [np.ascontiguousarray(a) for a in O.int4_views(cpages, BS, D)]
    kept, cnt, freed, fcnt = capi.evict_topk_compact_int4(torch.from_numpy(sc).to(DEV), gbt, gctx, pages, BS, D,
                                                          0.75, 4)
    rbt, rctx = cbt.copy(), ctx.copy()
    rk, rc, rf, rfc = O.evict_topk_compact_int4(sc, rbt, rctx, *views, 0.75, 4)
    assert np.array_equal(np16(cnt), rc) and np.array_equal(np16(kept), rk)
    back = lambda a: np.where(a >= 0, used[np.maximum(a, 0)], a)  # noqa: E731
    assert np.array_equal(np16(gbt), back(rbt)) and np.array_equal(np16(freed), back(rf))
    _, _, (after,) = _compact(bt, pages)  # same page set, same order
    got = O.int4_views(after, BS, D)
    for b in range(S):
        for i in range(int(rc[b])):
            pg, pos = rbt[b, i // BS], i % BS
            for a, ref in zip(got, views):
                assert np.array_equal(a[pg, :, pos].view(np.uint8), ref[pg, :, pos].view(np.uint8))
