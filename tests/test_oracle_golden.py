"""Pins the CPU oracle (oracle/memopt_oracle.c) against the reference.

* INT4 known answers from the reference test-suite (tests/test_quant.py:439-566):
  all-zero groups, constant 0.5, alternating +/-7, single group.
* fp16 conversions against numpy (IEEE round-to-nearest-even).
* paged attention against golden outputs of the reference's own CPU path
  (``_sdpa_fallback``, src/memopt/triton_attention.py:473-550), recorded by
  tests/golden/make_golden.py.
* evict_tokens against the behaviour the reference kernel's arithmetic
  implies (kv_cache.cu:714-870): with sinks nothing is evicted, without sinks
  exactly ``keep`` distinct scores survive.
"""
from __future__ import annotations

import os

import numpy as np
import pytest

import oracle as O

GOLDEN = os.path.join(os.path.dirname(__file__), "golden", "attention_sdpa.npz")


def test_f16_to_f32_all_halves():
    bits = np.arange(65536, dtype=np.uint16)
    ref = bits.view(np.float16).astype(np.float32)
    got = np.array([O.f16_bits_to_f32(int(b)) for b in bits[::7]], np.float32)
    r = ref[::7]
    nan = np.isnan(r)
    assert np.array_equal(np.isnan(got), nan)
    assert np.array_equal(got[~nan], r[~nan])


def test_f32_to_f16_random_and_edges():
    rng = np.random.default_rng(0)
    vals = np.concatenate([
        rng.standard_normal(4000).astype(np.float32) * 10,
        rng.standard_normal(2000).astype(np.float32) * 1e-6,
        np.array([0.0, -0.0, 65504, 65519.99, 65520, 1e9, -1e9, 5.96e-8, 2.98e-8, 2.99e-8,
                  6.1035e-5, np.inf, -np.inf], np.float32),
    ])
    ref = vals.astype(np.float16).view(np.uint16)
    got = np.array([O.f32_to_f16_bits(float(v)) for v in vals], np.uint16)
    assert np.array_equal(got, ref)


def test_quant_all_zeros():
    packed, scales = O.quantize_int4(np.zeros((4, 128), np.float16))
    assert np.all(packed == 0x88) and np.all(scales == 1.0)
    assert np.all(O.dequantize_int4(packed, scales) == 0)


def test_quant_constant_half():
    x = np.full((4, 128), 0.5, np.float16)
    packed, scales = O.quantize_int4(x)
    assert np.all(packed == 0xFF)
    assert np.all(scales == np.float32(0.5) / np.float32(7.0))
    mse = np.mean((O.dequantize_int4(packed, scales).astype(np.float32) - 0.5) ** 2)
    assert mse < 1e-6


def test_quant_plus_minus_seven_exact():
    x = np.empty(64, np.float16)
    x[::2], x[1::2] = 7.0, -7.0
    packed, scales = O.quantize_int4(x)
    assert scales.tolist() == [1.0]
    assert np.all(packed == (15 | (1 << 4)))
    assert np.array_equal(O.dequantize_int4(packed, scales), x)


def test_quant_single_group_shapes():
    x = np.random.default_rng(1).uniform(-1, 1, 64).astype(np.float16)
    packed, scales = O.quantize_int4(x)
    assert packed.shape == (32,) and scales.shape == (1,)


def test_quant_ties_round_away_from_zero():
    # 2.5 * scale must give code round(2.5)+8 = 11 (ties away), not 10.
    x = np.zeros(64, np.float16)
    x[0], x[1], x[2] = 7.0, 2.5, -2.5
    packed, scales = O.quantize_int4(x)
    assert scales[0] == 1.0
    assert packed[0] & 0xF == 15 and packed[0] >> 4 == 11 and packed[1] & 0xF == 5


def test_quant_matches_torch_reference_within_one_code():
    # tests/test_quant.py:650-694 of the reference: codes within +/-1 of the
    # ties-to-even torch reference, scales within 1e-4.
    rng = np.random.default_rng(42)
    x = rng.uniform(-1, 1, (4, 128)).astype(np.float16)
    packed, scales = O.quantize_int4(x)
    g = x.astype(np.float32).reshape(-1, 64)
    s_ref = np.abs(g).max(1) / 7.0
    assert np.allclose(scales, s_ref, atol=1e-4, rtol=1e-4)
    q_ref = np.clip(np.round(g / s_ref[:, None]) + 8, 0, 15).reshape(-1)
    flat = packed.reshape(-1)
    q = np.empty(flat.size * 2, np.int32)
    q[0::2], q[1::2] = flat & 0xF, flat >> 4
    assert np.abs(q - q_ref).max() <= 1


@pytest.mark.parametrize("ci", range(4))
def test_attention_oracle_matches_reference_cpu_path(ci):
    z = np.load(GOLDEN)
    q, k, v = z[f"c{ci}_q"], z[f"c{ci}_k"], z[f"c{ci}_v"]
    bt, ctx, msl = z[f"c{ci}_bt"], z[f"c{ci}_ctx"], int(z[f"c{ci}_max_seq_len"])
    ref = z[f"c{ci}_out"].astype(np.float64)
    got = O.paged_attention_f16(q, k, v, bt, ctx, msl, msl)
    # The reference rounds its fp32 SDPA to fp16: one fp16 ulp plus fp32 noise.
    np.testing.assert_allclose(got, ref, atol=2e-3, rtol=1e-2)


def _pool(NB, BS, H, D, seed=0):
    rng = np.random.default_rng(seed)
    return (rng.standard_normal((NB, BS, H, D)).astype(np.float16),
            rng.standard_normal((NB, BS, H, D)).astype(np.float16))


def test_evict_tokens_with_sinks_evicts_nothing():
    S, H, L, BS, D = 2, 2, 512, 16, 64
    rng = np.random.default_rng(3)
    scores = rng.lognormal(0, 1, (S, H, L)).astype(np.float32)
    k, v = _pool(S * L // BS, BS, H, D)
    k0, v0 = k.copy(), v.copy()
    bt = np.arange(S * L // BS, dtype=np.int32).reshape(S, -1)
    ibf = np.zeros(S * L // BS, np.int32)
    idx, cnt, _ = O.evict_tokens(scores, bt, ibf, k, v, 0.75, 4)
    assert np.all(cnt == L)
    assert np.array_equal(k, k0) and np.array_equal(v, v0)


def test_evict_tokens_without_sinks_keeps_exactly_keep():
    S, H, L, BS, D = 2, 3, 1000, 16, 64
    rng = np.random.default_rng(4)
    scores = rng.lognormal(0, 1, (S, H, L)).astype(np.float32)
    NB = S * ((L + BS - 1) // BS)
    k, v = _pool(NB, BS, H, D)
    k0 = k.copy()
    bt = np.arange(NB, dtype=np.int32).reshape(S, -1)
    ibf = np.zeros(NB, np.int32)
    idx, cnt, thr = O.evict_tokens(scores, bt, ibf, k, v, 0.75, 0)
    keep = int(np.ceil(np.float32(0.75) * np.float32(L)))
    assert np.all(cnt == keep)
    for s in range(S):
        for h in range(H):
            kept = idx[s, h, :cnt[s, h]]
            assert np.array_equal(kept, np.nonzero(scores[s, h] >= thr[s, h])[0])
            ev = np.nonzero(scores[s, h] < thr[s, h])[0]
            t = ev[0]
            row = k[bt[s, t // BS], t % BS, h]
            zero_d = np.arange(t % 32, D, 32)
            assert np.all(row[zero_d] == 0)
            other = np.setdiff1d(np.arange(D), zero_d)
            assert np.array_equal(row[other], k0[bt[s, t // BS], t % BS, h][other])
    assert np.all(ibf == 0)


def test_evict_tokens_block_size_one_unlinks():
    S, H, L, BS, D = 1, 2, 64, 1, 32
    scores = np.ones((S, H, L), np.float32)
    scores[:, :, 0] = 0.0   # token 0 (t % 32 == 0) is the lowest in both heads
    scores[:, :, 32] = 0.5  # token 32 too
    k, v = _pool(L, BS, H, D)
    bt = np.arange(L, dtype=np.int32).reshape(S, L)
    ibf = np.zeros(L, np.int32)
    O.evict_tokens(scores, bt, ibf, k, v, 0.96875, 0)  # keep 62 of 64
    assert ibf[0] == 2 and ibf[32] == 2
    assert bt[0, 0] == -1 and bt[0, 32] == -1
    assert np.count_nonzero(bt == -1) == 2


def test_evict_cache_keeps_top_keep():
    NB, BS, H, D = 5, 16, 3, 64
    rng = np.random.default_rng(5)
    scores = rng.standard_normal((NB, BS, H)).astype(np.float32)
    k, v = _pool(NB, BS, H, D)
    O.evict_cache(scores, k, v, 0.75)
    keep = int(0.75 * 16)
    for b in range(NB):
        for h in range(H):
            order = np.argsort(-scores[b, :, h], kind="stable")
            zeroed = np.all(k[b, :, h] == 0, axis=-1)
            assert not zeroed[order[:keep]].any()
            assert zeroed[order[keep:]].all()
