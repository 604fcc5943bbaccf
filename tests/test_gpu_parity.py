"""GPU parity: every kernel, called through the C-ABI, against the CPU oracle.

Bit-exact for codes, scales, written pages, block tables, vote counters and
retained-token indices; attention within 2e-3 absolute + 1e-2 relative of the
fp64 oracle (the tolerance stated for fp16 attention outputs).
"""
from __future__ import annotations

import numpy as np
import pytest
import torch

import capi
import oracle as O

pytestmark = pytest.mark.gpu
ATOL, RTOL = 2e-3, 1e-2
WORKSPACE_ERR = -6  # MEMOPT_ERR_WORKSPACE
DEV = "cuda"


def np16(t):
    return t.detach().cpu().numpy()


# ----------------------------------------------------------------- quant
@pytest.mark.parametrize("shape", [(64,), (4, 128), (2, 8, 64), (2, 4, 8, 64), (3, 1000, 64), (7, 32, 128)])
@pytest.mark.parametrize("dist", ["normal", "uniform", "small", "large", "zeros", "const"])
def test_quantize_bit_exact(shape, dist):
    g = torch.Generator(device="cpu").manual_seed(hash((shape, dist)) & 0xFFFF)
    if dist == "normal":
        x = torch.randn(shape, generator=g)
    elif dist == "uniform":
        x = torch.rand(shape, generator=g) * 2 - 1
    elif dist == "small":
        x = torch.rand(shape, generator=g) * 0.2 - 0.1
    elif dist == "large":
        x = torch.rand(shape, generator=g) * 200 - 100
    elif dist == "zeros":
        x = torch.zeros(shape)
    else:
        x = torch.full(shape, 0.5)
    x = x.half()
    p, s = capi.quantize(x.to(DEV))
    pr, sr = O.quantize_int4(x.numpy())
    assert np.array_equal(np16(p), pr)
    assert np.array_equal(np16(s).view(np.uint32), sr.view(np.uint32))
    d = capi.dequantize(p, s)
    dr = O.dequantize_int4(pr, sr)
    assert np.array_equal(np16(d).view(np.uint16), dr.view(np.uint16))


def test_quantize_special_values():
    x = torch.zeros(8, 64)
    x[0, 3] = float("inf")
    x[1, 5] = float("nan")
    x[2] = torch.linspace(-65504, 65504, 64)
    x[3, :] = 6e-8  # fp16 subnormals
    x[4, ::2] = 2.5
    x[4, 1] = 7.0
    x = x.half()
    p, s = capi.quantize(x.to(DEV))
    pr, sr = O.quantize_int4(x.numpy())
    assert np.array_equal(np16(p), pr)
    assert np.array_equal(np16(s).view(np.uint32), sr.view(np.uint32))


# ------------------------------------------------------------ write_cache
def _slots(T, NB, BS, seed, bad=0):
    rng = np.random.default_rng(seed)
    s = rng.choice(NB * BS, size=T, replace=False).astype(np.int32)
    if bad:
        s[rng.choice(T, size=bad, replace=False)] = rng.choice([-1, NB * BS, NB * BS + 7, -100], size=bad)
    return s


@pytest.mark.parametrize("T,H,D,NB,BS", [(1, 8, 64, 4, 16), (100, 8, 64, 20, 16), (333, 32, 128, 64, 16),
                                          (77, 4, 128, 10, 32), (50, 3, 10, 8, 16)])
def test_write_cache_f16_bit_exact(T, H, D, NB, BS):
    rng = np.random.default_rng(T)
    k = rng.standard_normal((T, H, D)).astype(np.float16)
    v = rng.standard_normal((T, H, D)).astype(np.float16)
    s = _slots(T, NB, BS, T, bad=min(3, T - 1))
    kp = np.zeros((NB, BS, H, D), np.float16)
    vp = np.zeros_like(kp)
    O.write_cache_f16(k, v, s, kp, vp)
    gk = torch.zeros(NB, BS, H, D, dtype=torch.float16, device=DEV)
    gv = torch.zeros_like(gk)
    bad = torch.zeros(1, dtype=torch.int32, device=DEV)
    capi.write_cache_f16(torch.from_numpy(k).to(DEV), torch.from_numpy(v).to(DEV), torch.from_numpy(s).to(DEV),
                         gk, gv, bad)
    assert np.array_equal(np16(gk), kp) and np.array_equal(np16(gv), vp)
    assert int(bad.item()) == int(((s < 0) | (s >= NB * BS)).sum())


@pytest.mark.parametrize("T,H,D,NB,BS", [(1, 8, 64, 4, 16), (129, 8, 64, 20, 16), (300, 32, 128, 64, 16),
                                          (77, 4, 128, 10, 32), (40, 2, 192, 8, 16)])
def test_write_cache_int4_bit_exact(T, H, D, NB, BS):
    rng = np.random.default_rng(T + 1)
    k = rng.standard_normal((T, H, D)).astype(np.float16)
    v = (rng.standard_normal((T, H, D)) * 3).astype(np.float16)
    k[0, 0, :64] = 0  # all-zero group -> scale 1.0
    s = _slots(T, NB, BS, T + 1, bad=min(2, T - 1))
    PB = O.int4_page_bytes(BS, D)
    assert PB == capi.int4_page_bytes(BS, D)
    pages = np.zeros((NB, H, PB), np.uint8)
    O.write_cache_int4(k, v, s, pages, BS)
    g = torch.zeros(NB, H, PB, dtype=torch.uint8, device=DEV)
    capi.write_cache_int4(torch.from_numpy(k).to(DEV), torch.from_numpy(v).to(DEV), torch.from_numpy(s).to(DEV),
                          g, BS)
    assert np.array_equal(np16(g), pages)
    # codes and scales agree with the standalone reference quantizer on each (token, head) row
    kc, ks, vc, vs = O.int4_views(pages, BS, D)
    ok_t = [i for i in range(T) if 0 <= s[i] < NB * BS]
    for t in ok_t[:3]:
        blk, pos = divmod(int(s[t]), BS)
        pr, sr = O.quantize_int4(k[t])
        assert np.array_equal(kc[blk, :, pos, :], pr.reshape(H, D // 2))
        assert np.array_equal(ks[blk, :, pos, :].reshape(-1).view(np.uint16), sr.astype(np.float16).view(np.uint16))
        pr, sr = O.quantize_int4(v[t])
        assert np.array_equal(vc[blk, :, pos, :], pr.reshape(H, D // 2))
        assert np.array_equal(vs[blk, :, pos, :].reshape(-1).view(np.uint16), sr.astype(np.float16).view(np.uint16))


# ------------------------------------------------------------ evict_tokens
def _evict_case(S, H, L, BS, D, r, sinks, seed, dist="lognormal", extra_pages=3, holes=False):
    rng = np.random.default_rng(seed)
    if dist == "lognormal":
        sc = rng.lognormal(0, 1, (S, H, L)).astype(np.float32)
    elif dist == "ties":
        sc = rng.integers(0, 4, (S, H, L)).astype(np.float32)
    elif dist == "const":
        sc = np.full((S, H, L), 2.0, np.float32)
    elif dist == "specials":  # NaN, +-inf and huge scores scattered through lognormal rows
        sc = rng.lognormal(0, 1, (S, H, L)).astype(np.float32)
        m = rng.random((S, H, L))
        sc[m < 0.02] = np.nan
        sc[(m >= 0.02) & (m < 0.025)] = np.inf
        sc[(m >= 0.025) & (m < 0.03)] = -np.inf
        sc[(m >= 0.03) & (m < 0.032)] = 3e38
        sc[0, 0, : min(L, 70)] = np.nan  # a whole thread's worth of NaN
    elif dist == "maxheavy":  # most scores equal to the row maximum
        sc = rng.lognormal(0, 1, (S, H, L)).astype(np.float32)
        sc[rng.random((S, H, L)) < 0.8] = 50.0
    elif dist == "signed_zero":  # -0, +0 and negative scores only
        sc = -rng.integers(0, 3, (S, H, L)).astype(np.float32)
        sc[rng.random((S, H, L)) < 0.3] = -0.0
    elif dist == "mostly_nan":  # fewer comparable scores than kept tokens
        sc = rng.standard_normal((S, H, L)).astype(np.float32)
        sc[rng.random((S, H, L)) < 0.9] = np.nan
    else:
        sc = rng.standard_normal((S, H, L)).astype(np.float32)
    MB = (L + BS - 1) // BS
    NB = S * MB + extra_pages
    bt = rng.permutation(NB)[: S * MB].astype(np.int32).reshape(S, MB)
    if holes:
        bt[rng.random(bt.shape) < 0.1] = -1
    kp = rng.standard_normal((NB, BS, H, D)).astype(np.float16)
    vp = rng.standard_normal((NB, BS, H, D)).astype(np.float16)
    return sc, bt, kp, vp


@pytest.mark.parametrize("S,H,L,BS,D,r,sinks,dist,holes", [
    (2, 4, 512, 16, 64, 0.75, 4, "lognormal", False),
    (2, 4, 512, 16, 64, 0.75, 0, "lognormal", False),
    (3, 2, 1000, 16, 128, 0.5, 0, "normal", True),
    (1, 8, 4096, 16, 128, 0.75, 0, "lognormal", False),
    (2, 2, 777, 32, 64, 0.3, 2, "ties", False),
    (1, 2, 100, 16, 64, 1.0, 0, "normal", False),
    (1, 2, 100, 16, 64, 0.01, 0, "normal", False),
    (1, 2, 64, 16, 64, 0.5, 0, "const", False),
    (1, 3, 1, 16, 64, 0.5, 0, "normal", False),
    (2, 2, 32768, 16, 64, 0.75, 0, "lognormal", False),
    (2, 2, 32768, 16, 64, 0.75, 4, "lognormal", False),
    (1, 2, 300, 1, 32, 0.5, 0, "normal", False),
    (2, 3, 1023, 16, 64, 0.6, 0, "specials", False),
    (2, 3, 4097, 16, 64, 0.75, 3, "specials", True),
    (1, 2, 9001, 16, 64, 0.4, 0, "specials", False),
    (1, 2, 20001, 16, 64, 0.75, 0, "specials", False),
    (1, 2, 32767, 16, 64, 0.75, 5, "specials", False),
    (1, 2, 16384, 16, 64, 0.9, 0, "ties", False),
    (1, 2, 32768, 16, 64, 0.5, 0, "maxheavy", False),   # keep-th largest among the maxima
    (1, 2, 32768, 16, 64, 0.9, 0, "maxheavy", False),   # ... and below them
    (1, 2, 5000, 16, 64, 0.6, 0, "signed_zero", False),
    (1, 2, 32768, 16, 64, 0.5, 0, "mostly_nan", False),
    (1, 2, 32768, 16, 64, 0.05, 0, "mostly_nan", False),
])
def test_evict_tokens_bit_exact(S, H, L, BS, D, r, sinks, dist, holes):
    sc, bt, kp, vp = _evict_case(S, H, L, BS, D, r, sinks, L + S, dist, holes=holes)
    NB = kp.shape[0]
    ibf = np.zeros(NB, np.int32)
    gk, gv = torch.from_numpy(kp).to(DEV), torch.from_numpy(vp).to(DEV)
    gbt, gibf = torch.from_numpy(bt).to(DEV), torch.from_numpy(ibf).to(DEV)
    idx, cnt = capi.evict_tokens(torch.from_numpy(sc).to(DEV), gbt, gibf, gk, gv, r, sinks)
    ridx, rcnt, _ = O.evict_tokens(sc, bt, ibf, kp, vp, r, sinks)
    assert np.array_equal(np16(cnt), rcnt)
    assert np.array_equal(np16(idx), ridx)
    assert np.array_equal(np16(gbt), bt)
    assert np.array_equal(np16(gibf), ibf)
    assert np.array_equal(np16(gk).view(np.uint16), kp.view(np.uint16))
    assert np.array_equal(np16(gv).view(np.uint16), vp.view(np.uint16))


@pytest.mark.parametrize("S,H,L,BS,D,r,sinks,dist,holes", [
    (2, 4, 512, 16, 64, 0.75, 4, "lognormal", False),
    (3, 2, 1000, 16, 128, 0.5, 0, "normal", True),
    (2, 2, 777, 32, 64, 0.3, 2, "ties", False),
    (1, 2, 100, 16, 64, 1.0, 0, "normal", False),
    (1, 2, 100, 16, 64, 0.01, 0, "normal", False),
    (2, 3, 4097, 16, 64, 0.75, 3, "specials", True),
    (1, 2, 32768, 16, 64, 0.75, 4, "lognormal", False),
    (2, 2, 16384, 16, 64, 0.6, 0, "ties", True),
    (2, 32, 4096, 16, 128, 0.75, 4, "lognormal", True),  # 8 KB rows, the bench's geometry
    (1, 4, 20000, 16, 64, 0.05, 0, "normal", False),     # long forward moves
    (2, 2, 70000, 16, 64, 0.75, 4, "lognormal", True),   # streaming select: > 32768 tokens, > 2048 pages
    (1, 2, 40000, 32, 64, 0.5, 3, "ties", False),        # > 32768 tokens, 1250 pages
    (1, 2, 50000, 16, 64, 0.6, 0, "specials", True),
])
def test_evict_topk_compact_bit_exact(S, H, L, BS, D, r, sinks, dist, holes):
    sc, bt, kp, vp = _evict_case(S, H, L, BS, D, r, sinks, L + 7 * S, dist, holes=holes)
    rng = np.random.default_rng(L)
    ctx = np.array([L - int(rng.integers(0, min(L, 40))) for _ in range(S)], np.int32)
    ctx[0] = L
    gk, gv = torch.from_numpy(kp).to(DEV), torch.from_numpy(vp).to(DEV)
    gbt, gctx = torch.from_numpy(bt).to(DEV), torch.from_numpy(ctx).to(DEV)
    kept, cnt, freed, fcnt = capi.evict_topk_compact(torch.from_numpy(sc).to(DEV), gbt, gctx, gk, gv, r, sinks)
    rk, rc, rf, rfc = O.evict_topk_compact(sc, bt, ctx, kp, vp, r, sinks)
    assert np.array_equal(np16(cnt), rc)
    assert np.array_equal(np16(kept), rk)
    assert np.array_equal(np16(fcnt), rfc)
    assert np.array_equal(np16(freed), rf)
    assert np.array_equal(np16(gbt), bt)
    assert np.array_equal(np16(gctx), ctx)
    # every live row of every kept page is bit-identical (rows past the kept tokens are unspecified)
    for b in range(S):
        for i in range(int(rc[b])):
            pg, pos = bt[b, i // BS], i % BS
            assert np.array_equal(np16(gk[pg, pos]).view(np.uint16), kp[pg, pos].view(np.uint16))
            assert np.array_equal(np16(gv[pg, pos]).view(np.uint16), vp[pg, pos].view(np.uint16))


@pytest.mark.parametrize("S,H,L,BS,D,r,sinks,dist,holes", [
    (2, 4, 1000, 16, 128, 0.5, 4, "lognormal", True),
    (2, 2, 777, 32, 64, 0.3, 2, "ties", False),
    (1, 32, 4096, 16, 128, 0.75, 4, "lognormal", False),   # 32 heads: one per lane
    (1, 40, 600, 16, 128, 0.6, 0, "specials", True),       # 40 heads: lanes take two
    (1, 2, 20000, 16, 64, 0.05, 0, "normal", False),       # long forward moves
    (1, 4, 66000, 16, 128, 0.75, 4, "lognormal", True),    # streaming select
])
def test_evict_topk_compact_int4_bit_exact(S, H, L, BS, D, r, sinks, dist, holes):
    """INT4 pool: every kept token's codes and scales (all heads) land at its
    new position, with the position-dependent V layout re-applied."""
    sc, bt, kp, vp = _evict_case(S, H, L, BS, D, r, sinks, L + 3 * S, dist, holes=holes)
    rng = np.random.default_rng(L + H)
    ctx = np.array([L - int(rng.integers(0, min(L, 40))) for _ in range(S)], np.int32)
    ctx[0] = L
    NB = kp.shape[0]
    T = NB * BS
    pages = torch.zeros(NB, H, capi.int4_page_bytes(BS, D), dtype=torch.uint8, device=DEV)
    capi.write_cache_int4(torch.from_numpy(kp.reshape(T, H, D)).to(DEV), torch.from_numpy(vp.reshape(T, H, D)).to(DEV),
                          torch.from_numpy(np.arange(T, dtype=np.int32)).to(DEV), pages, BS)
    views = [np.ascontiguousarray(a) for a in O.int4_views(np16(pages), BS, D)]
    gbt, gctx = torch.from_numpy(bt).to(DEV), torch.from_numpy(ctx).to(DEV)
    kept, cnt, freed, fcnt = capi.evict_topk_compact_int4(torch.from_numpy(sc).to(DEV), gbt, gctx, pages, BS, D, r, sinks)
    rbt, rctx = bt.copy(), ctx.copy()
    rk, rc, rf, rfc = O.evict_topk_compact_int4(sc, rbt, rctx, *views, r, sinks)
    assert np.array_equal(np16(cnt), rc) and np.array_equal(np16(kept), rk)
    assert np.array_equal(np16(fcnt), rfc) and np.array_equal(np16(freed), rf)
    assert np.array_equal(np16(gbt), rbt) and np.array_equal(np16(gctx), rctx)
    got = O.int4_views(np16(pages), BS, D)
    for b in range(S):
        for i in range(int(rc[b])):
            pg, pos = rbt[b, i // BS], i % BS
            for a, ref in zip(got, views):
                assert np.array_equal(a[pg, :, pos].view(np.uint8), ref[pg, :, pos].view(np.uint8))


@pytest.mark.parametrize("S,H,G,L,BS,D,r,sinks,dist,holes", [
    (2, 4, 2, 512, 16, 64, 0.75, 4, "lognormal", False),
    (3, 4, 4, 1000, 16, 128, 0.5, 0, "normal", True),
    (2, 6, 3, 777, 32, 64, 0.3, 2, "ties", False),
    (2, 4, 2, 4097, 16, 64, 0.75, 3, "specials", True),
    (1, 8, 8, 32768, 16, 64, 0.75, 4, "lognormal", False),
])
def test_evict_topk_head_sharded_bit_exact(S, H, G, L, BS, D, r, sinks, dist, holes):
    """Heads split over G shards: partial sums per shard, decision on their
    rank-ordered sum; each shard's pool (its heads) compacted identically."""
    sc, bt, kp, vp = _evict_case(S, H, L, BS, D, r, sinks, L + 7 * S, dist, holes=holes)
    rng = np.random.default_rng(L + G)
    ctx = np.array([L - int(rng.integers(0, min(L, 40))) for _ in range(S)], np.int32)
    ctx[0] = L
    hs = H // G
    gsc = torch.from_numpy(sc).to(DEV)
    parts = torch.stack([capi.evict_topk_head_sum(gsc[:, g * hs:(g + 1) * hs].contiguous()) for g in range(G)])
    rparts = np.stack([O.evict_topk_head_sum(sc[:, g * hs:(g + 1) * hs]) for g in range(G)])
    assert np.array_equal(np16(parts), rparts, equal_nan=True)  # NaN payloads may differ
    rbt, rctx = bt.copy(), ctx.copy()
    rkp, rvp = kp.copy(), vp.copy()
    rk, rc, rf, rfc = O.evict_topk_compact_parts(rparts, rbt, rctx, rkp, rvp, r, sinks)
    for g in range(G):
        gk = torch.from_numpy(np.ascontiguousarray(kp[:, :, g * hs:(g + 1) * hs])).to(DEV)
        gv = torch.from_numpy(np.ascontiguousarray(vp[:, :, g * hs:(g + 1) * hs])).to(DEV)
        gbt, gctx = torch.from_numpy(bt).to(DEV), torch.from_numpy(ctx).to(DEV)
        kept, cnt, freed, fcnt = capi.evict_topk_compact_parts(parts, gbt, gctx, gk, gv, r, sinks)
        assert np.array_equal(np16(cnt), rc) and np.array_equal(np16(kept), rk)
        assert np.array_equal(np16(fcnt), rfc) and np.array_equal(np16(freed), rf)
        assert np.array_equal(np16(gbt), rbt) and np.array_equal(np16(gctx), rctx)
        for b in range(S):
            for i in range(int(rc[b])):
                pg, pos = rbt[b, i // BS], i % BS
                assert np.array_equal(np16(gk[pg, pos]).view(np.uint16), rkp[pg, pos, g * hs:(g + 1) * hs].view(np.uint16))
                assert np.array_equal(np16(gv[pg, pos]).view(np.uint16), rvp[pg, pos, g * hs:(g + 1) * hs].view(np.uint16))


def test_evict_topk_one_part_equals_unsharded():
    sc, bt, kp, vp = _evict_case(2, 4, 3000, 16, 64, 0.6, 4, 3000 + 14, "lognormal", holes=True)
    ctx = np.array([3000, 2980], np.int32)
    gsc = torch.from_numpy(sc).to(DEV)
    a = [torch.from_numpy(x).to(DEV) for x in (kp, vp, bt, ctx)]
    b = [torch.from_numpy(x.copy()).to(DEV) for x in (kp, vp, bt, ctx)]
    r1 = capi.evict_topk_compact(gsc, a[2], a[3], a[0], a[1], 0.6, 4)
    r2 = capi.evict_topk_compact_parts(capi.evict_topk_head_sum(gsc)[None], b[2], b[3], b[0], b[1], 0.6, 4)
    for x, y in zip(list(r1) + a, list(r2) + b):
        assert torch.equal(x, y)


@pytest.mark.parametrize("NB,BS,H,D,r", [(10, 16, 4, 64, 0.75), (7, 32, 3, 128, 0.5), (5, 8, 2, 64, 0.9),
                                         (6, 5, 2, 64, 0.6), (3, 16, 2, 64, 0.01), (37, 16, 32, 128, 0.75),
                                         (9, 16, 40, 128, 0.5), (4, 32, 33, 64, 0.3), (5, 16, 3, 20, 0.5)])
def test_evict_cache_bit_exact(NB, BS, H, D, r):
    rng = np.random.default_rng(NB * BS)
    sc = rng.integers(0, 5, (NB, BS, H)).astype(np.float32)  # many ties
    sc[0, 0, 0] = np.nan
    kp = rng.standard_normal((NB, BS, H, D)).astype(np.float16)
    vp = rng.standard_normal((NB, BS, H, D)).astype(np.float16)
    gk, gv = torch.from_numpy(kp).to(DEV), torch.from_numpy(vp).to(DEV)
    capi.evict_cache(torch.from_numpy(sc).to(DEV), gk, gv, r)
    O.evict_cache(sc, kp, vp, r)
    assert np.array_equal(np16(gk).view(np.uint16), kp.view(np.uint16))
    assert np.array_equal(np16(gv).view(np.uint16), vp.view(np.uint16))


# --------------------------------------------------------------- attention
def _attn_case(B, QL, H, D, BS, ctx, MB, seed, holes=0.0, dist="normal"):
    rng = np.random.default_rng(seed)
    NB = B * MB + 5
    bt = rng.permutation(NB)[: B * MB].astype(np.int32).reshape(B, MB)
    if holes:
        bt[rng.random(bt.shape) < holes] = -1
        bt[0, 0] = NB + 3  # beyond the pool: skipped like -1
    f = (lambda s: rng.standard_normal(s)) if dist == "normal" else (lambda s: rng.random(s))
    kp = f((NB, BS, H, D)).astype(np.float16)
    vp = f((NB, BS, H, D)).astype(np.float16)
    q = f((B, QL, H, D)).astype(np.float16)
    return q, kp, vp, bt, np.asarray(ctx, np.int32)


ATTN_CASES = [
    # B, QL, H, D, BS, ctx, MB, max_seq_len, window, holes
    (2, 1, 8, 64, 16, [512, 512], 32, 512, 512, 0.0),
    (3, 1, 4, 128, 16, [1, 17, 300], 20, 320, 320, 0.0),
    (2, 1, 4, 128, 32, [1000, 64], 40, 1280, 100, 0.0),
    (2, 3, 4, 64, 32, [300, 301], 10, 320, -1, 0.2),
    (4, 1, 2, 128, 16, [0, 5, 4096, 4095], 256, 4096, 4096, 0.0),
    (1, 2, 2, 64, 16, [4096], 256, 4096, 77, 0.1),
    (2, 1, 4, 128, 16, [700, 900], 64, 1024, 0, 0.0),
    (2, 1, 32, 128, 16, [4096, 4000], 256, 4096, 4096, 0.0),
    (1, 1, 2, 128, 16, [40000], 2500, 40000, 40000, 0.0),
    (2, 1, 2, 64, 16, [100, 100], 8, 128, 128, 0.0),  # ctx beyond the table
]


@pytest.mark.parametrize("case", ATTN_CASES)
def test_attention_f16_vs_oracle(case):
    B, QL, H, D, BS, ctx, MB, msl, win, holes = case
    q, kp, vp, bt, cl = _attn_case(B, QL, H, D, BS, ctx, MB, sum(ctx) + H, holes)
    got = capi.attention_f16(torch.from_numpy(q).to(DEV), torch.from_numpy(kp).to(DEV),
                             torch.from_numpy(vp).to(DEV), torch.from_numpy(bt).to(DEV),
                             torch.from_numpy(cl).to(DEV), msl, win)
    ref = O.paged_attention_f16(q, kp, vp, bt, cl, msl, win)
    np.testing.assert_allclose(np16(got).astype(np.float64), ref, atol=ATOL, rtol=RTOL)


@pytest.mark.parametrize("case", ATTN_CASES)
def test_attention_int4_vs_oracle(case):
    B, QL, H, D, BS, ctx, MB, msl, win, holes = case
    q, kp, vp, bt, cl = _attn_case(B, QL, H, D, BS, ctx, MB, sum(ctx) + H + 1, holes)
    NB = kp.shape[0]
    # Fill the INT4 pages from the fp16 pool rows with the fused writer.
    T = NB * BS
    keys = kp.reshape(T, H, D)
    vals = vp.reshape(T, H, D)
    slots = np.arange(T, dtype=np.int32)
    pages = torch.zeros(NB, H, capi.int4_page_bytes(BS, D), dtype=torch.uint8, device=DEV)
    capi.write_cache_int4(torch.from_numpy(keys).to(DEV), torch.from_numpy(vals).to(DEV),
                          torch.from_numpy(slots).to(DEV), pages, BS)
    got = capi.attention_int4(torch.from_numpy(q).to(DEV), pages, BS, torch.from_numpy(bt).to(DEV),
                              torch.from_numpy(cl).to(DEV), msl, win)
    ref = O.paged_attention_int4(q, np16(pages), bt, cl, msl, win, BS)
    np.testing.assert_allclose(np16(got).astype(np.float64), ref, atol=ATOL, rtol=RTOL)


@pytest.mark.parametrize("qmul,vmean,win", [(8.0, 0.0, 32768), (0.05, 0.0, 32768), (1.0, 2.5, 32768),
                                             (4.0, -1.5, 5000)])
def test_attention_int4_long_context_stress(qmul, vmean, win):
    """Long rows with peaked / flat attention and V with a large common mean:
    the INT4 P.V path folds a per-code offset out of its fp32 accumulators
    every few steps, which these cases would expose."""
    B, H, D, BS, L = 1, 2, 128, 16, 32768
    MB = L // BS
    rng = np.random.default_rng(int(qmul * 100 + vmean * 10))
    NB = MB + 3
    bt = rng.permutation(NB)[:MB].astype(np.int32).reshape(1, MB)
    k = rng.standard_normal((NB * BS, H, D)).astype(np.float16)
    v = (rng.standard_normal((NB * BS, H, D)) + vmean).astype(np.float16)
    q = (rng.standard_normal((B, 1, H, D)) * qmul).astype(np.float16)
    pages = torch.zeros(NB, H, capi.int4_page_bytes(BS, D), dtype=torch.uint8, device=DEV)
    capi.write_cache_int4(torch.from_numpy(k).to(DEV), torch.from_numpy(v).to(DEV),
                          torch.from_numpy(np.arange(NB * BS, dtype=np.int32)).to(DEV), pages, BS)
    cl = np.array([L], np.int32)
    got = capi.attention_int4(torch.from_numpy(q).to(DEV), pages, BS, torch.from_numpy(bt).to(DEV),
                              torch.from_numpy(cl).to(DEV), L, win)
    ref = O.paged_attention_int4(q, np16(pages), bt, cl, L, win, BS)
    np.testing.assert_allclose(np16(got).astype(np.float64), ref, atol=ATOL, rtol=RTOL)


GQA_CASES = [
    # B, QL, H, KVH, D, BS, ctx, MB, max_seq_len, window, causal, holes
    (2, 1, 8, 2, 128, 16, [700, 1000], 64, 1024, 1024, False, 0.0),     # decode, GQA 4
    (2, 3, 8, 8, 64, 16, [300, 301], 20, 320, 320, True, 0.1),          # multi-row decode, causal
    (2, 5, 8, 1, 128, 32, [400, 90], 16, 512, 100, True, 0.0),          # MQA, causal, window
    (1, 1, 4, 2, 128, 16, [40000], 2500, 40000, 40000, False, 0.0),     # split-K, GQA
    (1, 200, 4, 2, 128, 16, [777], 64, 1024, 1024, True, 0.0),          # prefill, causal, GQA
    (2, 130, 8, 2, 64, 16, [300, 1000], 64, 1024, 256, True, 0.1),      # prefill, causal window, holes
    (1, 512, 2, 1, 128, 32, [4096], 128, 4096, 4096, False, 0.0),       # prefill, MQA, non-causal
    (1, 300, 2, 2, 128, 16, [300], 32, 512, 512, True, 0.0),            # prefill: rows == context
]


def _gqa_case(B, QL, H, KVH, D, BS, ctx, MB, holes, seed):
    rng = np.random.default_rng(seed)
    NB = B * MB + 5
    bt = rng.permutation(NB)[: B * MB].astype(np.int32).reshape(B, MB)
    if holes:
        bt[rng.random(bt.shape) < holes] = -1
    kp = rng.standard_normal((NB, BS, KVH, D)).astype(np.float16)
    vp = rng.standard_normal((NB, BS, KVH, D)).astype(np.float16)
    q = rng.standard_normal((B, QL, H, D)).astype(np.float16)
    return q, kp, vp, bt, np.asarray(ctx, np.int32)


@pytest.mark.parametrize("case", GQA_CASES)
def test_attention_gqa_causal_f16_vs_oracle(case):
    B, QL, H, KVH, D, BS, ctx, MB, msl, win, causal, holes = case
    q, kp, vp, bt, cl = _gqa_case(B, QL, H, KVH, D, BS, ctx, MB, holes, QL * 7 + H)
    got = capi.attention_f16_ex(torch.from_numpy(q).to(DEV), torch.from_numpy(kp).to(DEV),
                                torch.from_numpy(vp).to(DEV), torch.from_numpy(bt).to(DEV),
                                torch.from_numpy(cl).to(DEV), msl, win, causal)
    ref = O.paged_attention_f16(q, kp, vp, bt, cl, msl, win, causal=causal)
    np.testing.assert_allclose(np16(got).astype(np.float64), ref, atol=ATOL, rtol=RTOL)


@pytest.mark.parametrize("case", [c for c in GQA_CASES if c[1] < 64])
def test_attention_gqa_causal_int4_vs_oracle(case):
    B, QL, H, KVH, D, BS, ctx, MB, msl, win, causal, holes = case
    q, kp, vp, bt, cl = _gqa_case(B, QL, H, KVH, D, BS, ctx, MB, holes, QL * 11 + H)
    NB = kp.shape[0]
    T = NB * BS
    pages = torch.zeros(NB, KVH, capi.int4_page_bytes(BS, D), dtype=torch.uint8, device=DEV)
    capi.write_cache_int4(torch.from_numpy(kp.reshape(T, KVH, D)).to(DEV),
                          torch.from_numpy(vp.reshape(T, KVH, D)).to(DEV),
                          torch.from_numpy(np.arange(T, dtype=np.int32)).to(DEV), pages, BS)
    got = capi.attention_int4_ex(torch.from_numpy(q).to(DEV), pages, BS, torch.from_numpy(bt).to(DEV),
                                 torch.from_numpy(cl).to(DEV), msl, win, causal)
    ref = O.paged_attention_int4(q, np16(pages), bt, cl, msl, win, BS, causal=causal)
    np.testing.assert_allclose(np16(got).astype(np.float64), ref, atol=ATOL, rtol=RTOL)


# Multi-query decode (fp16, >= 2 query rows per KV head, q_len < 64): one page
# load serves the group's query heads x the q_len rows (tiles of 16 rows).
MQ_CASES = [
    # B, QL, H, KVH, D, BS, ctx, MB, max_seq_len, window, causal, holes
    (3, 1, 32, 8, 128, 16, [4096, 1000, 17], 256, 4096, 4096, False, 0.0),   # GQA 4, ragged
    (2, 1, 16, 2, 128, 16, [3000, 2999], 200, 3200, 3200, False, 0.05),     # GQA 8, holes
    (2, 1, 4, 2, 64, 32, [511, 64], 16, 512, 512, False, 0.0),              # GQA 2, D 64, 32-token pages
    (2, 4, 8, 8, 128, 16, [900, 4], 64, 1024, 1024, True, 0.0),             # MHA q_len 4, causal (4 <= q_len ctx)
    (2, 4, 32, 4, 128, 16, [1200, 700], 80, 1280, 1280, True, 0.1),         # 32 rows per KV head: 2 tiles
    (1, 3, 6, 2, 64, 16, [333], 24, 384, 100, True, 0.0),                   # 9 rows (partial tile), window
    (2, 2, 16, 1, 128, 32, [2048, 1500], 64, 2048, 300, False, 0.0),        # MQA 32 rows, window
    (1, 1, 8, 2, 128, 16, [40000], 2500, 40000, 40000, False, 0.0),         # split-K, GQA 4
    (2, 8, 8, 2, 128, 16, [20000, 5], 1250, 20000, 1024, True, 0.0),        # split-K, causal window, q_len > ctx
    (1, 1, 8, 2, 128, 16, [0], 4, 64, 64, False, 0.0),                      # empty context
]


@pytest.mark.parametrize("case", MQ_CASES)
def test_attention_multi_query_f16_vs_oracle(case):
    B, QL, H, KVH, D, BS, ctx, MB, msl, win, causal, holes = case
    q, kp, vp, bt, cl = _gqa_case(B, QL, H, KVH, D, BS, ctx, MB, holes, QL * 13 + H + KVH)
    got = capi.attention_f16_ex(torch.from_numpy(q).to(DEV), torch.from_numpy(kp).to(DEV),
                                torch.from_numpy(vp).to(DEV), torch.from_numpy(bt).to(DEV),
                                torch.from_numpy(cl).to(DEV), msl, win, causal)
    ref = O.paged_attention_f16(q, kp, vp, bt, cl, msl, win, causal=causal)
    np.testing.assert_allclose(np16(got).astype(np.float64), ref, atol=ATOL, rtol=RTOL)


@pytest.mark.parametrize("case", MQ_CASES + [
    (2, 70, 4, 2, 128, 16, [200, 90], 16, 256, 256, True, 0.0),    # q_len 70: the INT4 prefill path
    (1, 2, 2, 2, 64, 16, [50], 4, 64, 64, False, 0.0),             # MHA q_len 2, D 64
])
def test_attention_multi_query_int4_vs_oracle(case):
    B, QL, H, KVH, D, BS, ctx, MB, msl, win, causal, holes = case
    q, kp, vp, bt, cl = _gqa_case(B, QL, H, KVH, D, BS, ctx, MB, holes, QL * 17 + H + KVH)
    NB = kp.shape[0]
    T = NB * BS
    pages = torch.zeros(NB, KVH, capi.int4_page_bytes(BS, D), dtype=torch.uint8, device=DEV)
    capi.write_cache_int4(torch.from_numpy(kp.reshape(T, KVH, D)).to(DEV),
                          torch.from_numpy(vp.reshape(T, KVH, D)).to(DEV),
                          torch.from_numpy(np.arange(T, dtype=np.int32)).to(DEV), pages, BS)
    got = capi.attention_int4_ex(torch.from_numpy(q).to(DEV), pages, BS, torch.from_numpy(bt).to(DEV),
                                 torch.from_numpy(cl).to(DEV), msl, win, causal)
    ref = O.paged_attention_int4(q, np16(pages), bt, cl, msl, win, BS, causal=causal)
    np.testing.assert_allclose(np16(got).astype(np.float64), ref, atol=ATOL, rtol=RTOL)


# --------------------- INT4 prefill (q_len >= 64: pages -> fp16 scratch -> tcgen05)
INT4_PREFILL_CASES = [
    # B, QL, H, KVH, D, BS, ctx, MB, max_seq_len, window, causal, holes
    (1, 64, 2, 2, 128, 16, [128], 8, 128, 128, False, 0.0),
    (2, 130, 4, 2, 128, 16, [300, 77], 20, 320, 320, False, 0.0),
    (2, 256, 4, 4, 64, 16, [1000, 1024], 64, 1024, 1024, False, 0.1),
    (1, 200, 4, 2, 128, 32, [777], 30, 960, 300, False, 0.1),
    (1, 200, 4, 2, 128, 16, [777], 64, 1024, 1024, True, 0.0),   # causal GQA
    (2, 130, 8, 2, 64, 16, [300, 1000], 64, 1024, 256, True, 0.1),  # causal window, holes
    (2, 64, 2, 1, 64, 32, [64, 0], 4, 128, -1, False, 0.0),        # MQA, an empty context
    (1, 512, 8, 8, 128, 16, [4096], 256, 4096, 1000, False, 0.0),
]


def _int4_pages(kp, vp, BS):
    NB, _, KVH, D = kp.shape
    T = NB * BS
    pages = torch.zeros(NB, KVH, capi.int4_page_bytes(BS, D), dtype=torch.uint8, device=DEV)
    capi.write_cache_int4(torch.from_numpy(kp.reshape(T, KVH, D)).to(DEV), torch.from_numpy(vp.reshape(T, KVH, D)).to(DEV),
                          torch.from_numpy(np.arange(T, dtype=np.int32)).to(DEV), pages, BS)
    return pages


@pytest.mark.parametrize("case", INT4_PREFILL_CASES)
def test_prefill_int4_vs_oracle(case):
    B, QL, H, KVH, D, BS, ctx, MB, msl, win, causal, holes = case
    q, kp, vp, bt, cl = _gqa_case(B, QL, H, KVH, D, BS, ctx, MB, holes, QL * 19 + H + KVH)
    pages = _int4_pages(kp, vp, BS)
    got = capi.attention_int4_ex(torch.from_numpy(q).to(DEV), pages, BS, torch.from_numpy(bt).to(DEV),
                                 torch.from_numpy(cl).to(DEV), msl, win, causal)
    # the oracle dequantises exactly (fp64); the device rounds K and V to fp16 as the reference does
    ref = O.paged_attention_int4(q, np16(pages), bt, cl, msl, win, BS, causal=causal)
    np.testing.assert_allclose(np16(got).astype(np.float64), ref, atol=ATOL, rtol=RTOL)


def test_prefill_int4_workspace_size_scratch_and_reuse():
    B, QL, H, KVH, D, BS, ctx, MB, msl, win, causal, holes = INT4_PREFILL_CASES[1]
    q, kp, vp, bt, cl = _gqa_case(B, QL, H, KVH, D, BS, ctx, MB, holes, 3)
    pages = _int4_pages(kp, vp, BS)
    gq, gbt, gcl = (torch.from_numpy(a).to(DEV) for a in (q, bt, cl))
    small, n_small = capi.workspace(B, QL, H, D, MB, BS, msl, win, kvh=KVH)
    ws, n = capi.workspace(B, QL, H, D, MB, BS, msl, win, kvh=KVH, int4=True)
    assert n >= n_small + B * MB * BS * KVH * D * 4  # fp16 K and V scratch past the split workspace
    lib = capi.lib()

    def call(qt, out, ws_t, n_ws, causal_flag):
        return lib.memopt_paged_attention_int4_ex(
            capi.ptr(qt), capi.ptr(pages), capi.ptr(gbt), capi.ptr(gcl), capi.I(B), capi.I(qt.shape[1]), capi.I(H),
            capi.I(KVH), capi.I(D), capi.I(MB), capi.I64(pages.shape[0]), capi.I(BS), capi.I(msl), capi.I(win),
            capi.I(int(causal_flag)), capi.ptr(out), capi.ptr(ws_t), capi.SZ(n_ws), capi.stream())

    out = torch.empty_like(gq)
    if small is not None:
        assert call(gq, out, small, n_small, causal) == WORKSPACE_ERR  # no room for the scratch
        assert b"workspace" in lib.memopt_last_error()
    assert call(gq, out, ws, n, causal) == 0
    ref = O.paged_attention_int4(q, np16(pages), bt, cl, msl, win, BS, causal=causal)
    np.testing.assert_allclose(np16(out).astype(np.float64), ref, atol=ATOL, rtol=RTOL)
    tickets = lib.memopt_paged_attention_ticket_bytes(B, QL, H)
    assert int(ws[:tickets].count_nonzero().item()) == 0
    # a decode call (one query row) on the same workspace after the prefill
    q1 = np.ascontiguousarray(q[:, -1:])
    g1 = torch.from_numpy(q1).to(DEV)
    o1 = torch.empty_like(g1)
    assert call(g1, o1, ws, n, False) == 0
    ref1 = O.paged_attention_int4(q1, np16(pages), bt, cl, msl, win, BS, causal=False)
    np.testing.assert_allclose(np16(o1).astype(np.float64), ref1, atol=ATOL, rtol=RTOL)


def test_attention_multi_query_deterministic_and_tickets_reset():
    B, QL, H, KVH, D, BS, ctx, MB, msl, win, causal, holes = MQ_CASES[7]
    q, kp, vp, bt, cl = _gqa_case(B, QL, H, KVH, D, BS, ctx, MB, holes, 5)
    args = [torch.from_numpy(a).to(DEV) for a in (q, kp, vp, bt, cl)]
    o1 = capi.attention_f16_ex(*args, msl, win, causal)
    o2 = capi.attention_f16_ex(*args, msl, win, causal)
    assert torch.equal(o1, o2)


def test_attention_deterministic_and_workspace_reuse():
    B, QL, H, D, BS, ctx, MB, msl, win, holes = ATTN_CASES[7]
    q, kp, vp, bt, cl = _attn_case(B, QL, H, D, BS, ctx, MB, 11, holes)
    args = [torch.from_numpy(a).to(DEV) for a in (q, kp, vp, bt, cl)]
    ws, n = capi.workspace(B, QL, H, D, MB, BS, msl, win)
    assert n > 0  # this case uses split-K
    o1 = capi.attention_f16(*args, msl, win, ws=ws)
    o2 = capi.attention_f16(*args, msl, win, ws=ws)
    assert torch.equal(o1, o2)
    tickets = capi.lib().memopt_paged_attention_ticket_bytes(B, QL, H)
    assert int(ws[:tickets].count_nonzero().item()) == 0  # tickets left zero


# --------------------------------------------- prefill (q_len >= 64: tcgen05)
PREFILL_CASES = [
    # B, QL, H, D, BS, ctx, MB, max_seq_len, window, holes
    (1, 64, 1, 128, 16, [128], 8, 128, 128, 0.0),
    (1, 128, 2, 128, 16, [256], 16, 256, 256, 0.0),
    (2, 130, 2, 128, 16, [300, 77], 20, 320, 320, 0.0),
    (2, 256, 4, 64, 16, [1000, 1024], 64, 1024, 1024, 0.1),
    (1, 200, 2, 128, 32, [777], 30, 960, 300, 0.1),
    (2, 64, 2, 64, 32, [64, 0], 4, 128, -1, 0.0),
    (1, 512, 8, 128, 16, [4096], 256, 4096, 1000, 0.0),
]


@pytest.mark.parametrize("case", PREFILL_CASES)
def test_prefill_f16_vs_oracle(case):
    B, QL, H, D, BS, ctx, MB, msl, win, holes = case
    q, kp, vp, bt, cl = _attn_case(B, QL, H, D, BS, ctx, MB, sum(ctx) + QL, holes)
    got = capi.attention_f16(torch.from_numpy(q).to(DEV), torch.from_numpy(kp).to(DEV),
                             torch.from_numpy(vp).to(DEV), torch.from_numpy(bt).to(DEV),
                             torch.from_numpy(cl).to(DEV), msl, win)
    ref = O.paged_attention_f16(q, kp, vp, bt, cl, msl, win)
    np.testing.assert_allclose(np16(got).astype(np.float64), ref, atol=ATOL, rtol=RTOL)
