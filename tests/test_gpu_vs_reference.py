"""GPU parity against the reference's OWN kernels, built from its sources
into oracle/_ref/ by oracle/build_ref.py (skipped when that build is absent).

This pins both the oracle and this project's kernels to the reference
implementation run on the same device and inputs:
  * quantize / dequantize: bit-exact (codes, fp32 scales, fp16 outputs);
  * write_cache into the fp16 pool: bit-exact pool contents;
  * evict_tokens (seq_len <= 4096, the reference's limit) and evict_cache:
    bit-exact pool contents, block tables and vote counters;
  * dynamic_sparse_attention: within 2e-3 abs + 1e-2 rel of the reference.
"""
from __future__ import annotations

import numpy as np
import pytest
import torch

import capi
import oracle as O
from build_ref import load as load_ref

pytestmark = pytest.mark.gpu
DEV = "cuda"


@pytest.fixture(scope="module")
def ref():
    m = load_ref()
    if m is None:
        pytest.skip("reference extension not built (oracle/build_ref.py)")
    return m


def np16(t):
    return t.detach().cpu().numpy()


@pytest.mark.parametrize("shape,dist", [((4, 128), "u"), ((2, 8, 64), "n"), ((64, 4096), "n"),
                                        ((8, 64), "z"), ((5, 192), "big")])
def test_quant_matches_reference_kernel(ref, shape, dist):
    g = torch.Generator().manual_seed(7)
    x = {"u": torch.rand(shape, generator=g) * 2 - 1, "n": torch.randn(shape, generator=g),
         "z": torch.zeros(shape), "big": torch.randn(shape, generator=g) * 3000}[dist].half().to(DEV)
    pr, sr = ref.quantize_kv_cache_int4(x, 64)
    p, s = capi.quantize(x)
    assert torch.equal(p, pr)
    assert torch.equal(s.view(torch.int32), sr.view(torch.int32))
    po, so = O.quantize_int4(np16(x))  # the oracle agrees with the reference too
    assert np.array_equal(po, np16(pr)) and np.array_equal(so, np16(sr))
    dr = ref.dequantize_kv_cache_int4(pr, sr, 64)
    d = capi.dequantize(p, s)
    assert torch.equal(d.view(torch.int16), dr.view(torch.int16))


def test_write_cache_matches_reference_kernel(ref):
    NB, BS, H, D, T = 40, 16, 8, 64, 500
    ref.init_pool(NB, BS, H, D)
    rng = np.random.default_rng(1)
    slots = torch.from_numpy(rng.choice(NB * BS, T, replace=False).astype(np.int32)).to(DEV)
    k = torch.randn(T, H, D, device=DEV).half()
    v = torch.randn(T, H, D, device=DEV).half()
    rk, rv = ref.get_pool_tensors()
    rk.zero_()
    rv.zero_()
    ref.write_cache(k, v, torch.zeros(1, 1, dtype=torch.int32, device=DEV), slots)
    gk = torch.zeros(NB, BS, H, D, dtype=torch.float16, device=DEV)
    gv = torch.zeros_like(gk)
    capi.write_cache_f16(k, v, slots, gk, gv)
    assert torch.equal(gk, rk) and torch.equal(gv, rv)


@pytest.mark.parametrize("S,H,L,r,sinks,dist", [(2, 4, 512, 0.75, 4, "ln"), (2, 4, 1000, 0.75, 0, "ln"),
                                                (1, 8, 4096, 0.5, 0, "n"), (3, 2, 333, 0.3, 2, "ties"),
                                                (1, 4, 4096, 0.75, 4, "ln")])
def test_evict_tokens_matches_reference_kernel(ref, S, H, L, r, sinks, dist):
    BS, D = 16, 64
    MB = (L + BS - 1) // BS
    NB = S * MB + 2
    rng = np.random.default_rng(L + S)
    sc = {"ln": rng.lognormal(0, 1, (S, H, L)), "n": rng.standard_normal((S, H, L)),
          "ties": rng.integers(0, 3, (S, H, L))}[dist].astype(np.float32)
    bt = rng.permutation(NB)[: S * MB].astype(np.int32).reshape(S, MB)
    kp = torch.randn(NB, BS, H, D, device=DEV).half()
    vp = torch.randn(NB, BS, H, D, device=DEV).half()
    ref.init_pool(NB, BS, H, D)
    rk, rv = ref.get_pool_tensors()
    rk.copy_(kp)
    rv.copy_(vp)
    rbt = torch.from_numpy(bt).to(DEV)
    ribf = torch.zeros(NB, dtype=torch.int32, device=DEV)
    gsc = torch.from_numpy(sc).to(DEV)
    ref.evict_tokens(gsc, rbt, ribf, r, sinks)
    gbt = torch.from_numpy(bt).to(DEV)
    gibf = torch.zeros(NB, dtype=torch.int32, device=DEV)
    gk, gv = kp.clone(), vp.clone()
    capi.evict_tokens(gsc, gbt, gibf, gk, gv, r, sinks)
    assert torch.equal(gbt, rbt) and torch.equal(gibf, ribf)
    assert torch.equal(gk.view(torch.int16), rk.view(torch.int16))
    assert torch.equal(gv.view(torch.int16), rv.view(torch.int16))
    # and the oracle replays the same state
    ok_, ov = np16(kp).copy(), np16(vp).copy()
    obt, oibf = bt.copy(), np.zeros(NB, np.int32)
    O.evict_tokens(sc, obt, oibf, ok_, ov, r, sinks)
    assert np.array_equal(ok_.view(np.uint16), np16(rk).view(np.uint16))


def test_evict_cache_matches_reference_kernel(ref):
    NB, BS, H, D = 30, 16, 4, 64
    rng = np.random.default_rng(9)
    sc = torch.from_numpy(rng.integers(0, 6, (NB, BS, H)).astype(np.float32)).to(DEV)
    kp = torch.randn(NB, BS, H, D, device=DEV).half()
    vp = torch.randn(NB, BS, H, D, device=DEV).half()
    ref.init_pool(NB, BS, H, D)
    rk, rv = ref.get_pool_tensors()
    rk.copy_(kp)
    rv.copy_(vp)
    ref.evict_cache(torch.zeros(1, 1, dtype=torch.int32, device=DEV), sc, 0.75, 4)
    gk, gv = kp.clone(), vp.clone()
    capi.evict_cache(sc, gk, gv, 0.75)
    assert torch.equal(gk, rk) and torch.equal(gv, rv)


@pytest.mark.parametrize("B,QL,H,D,BS,ctx,MB,win", [(2, 1, 8, 64, 16, [512, 300], 32, 512),
                                                   (2, 4, 4, 128, 32, [777, 64], 25, 100),
                                                   (3, 1, 32, 128, 16, [4096, 1, 2000], 256, 4096)])
def test_attention_matches_reference_kernel(ref, B, QL, H, D, BS, ctx, MB, win):
    NB = B * MB + 3
    rng = np.random.default_rng(sum(ctx))
    bt = rng.permutation(NB)[: B * MB].astype(np.int32).reshape(B, MB)
    bt[rng.random(bt.shape) < 0.05] = -1
    bt_t = torch.from_numpy(bt).to(DEV)
    kp = torch.randn(NB, BS, H, D, device=DEV).half()
    vp = torch.randn(NB, BS, H, D, device=DEV).half()
    q = torch.randn(B, QL, H, D, device=DEV).half()
    cl = torch.tensor(ctx, dtype=torch.int32, device=DEV)
    msl = MB * BS
    r = ref.dynamic_sparse_attention(q, kp, vp, bt_t, cl, msl, win)
    g = capi.attention_f16(q, kp, vp, bt_t, cl, msl, win)
    torch.testing.assert_close(g.float(), r.float(), atol=2e-3, rtol=1e-2)
