"""Incremental decode through PagedKVCache / DynamicAttention on the GPU, and
the MemoryScheduler policy applied to a live cache."""
from __future__ import annotations

import numpy as np
import pytest
import torch

import oracle as O

import memopt
from memopt import DynamicAttention, MemoryScheduler, PagedKVCache, SchedulerConfig

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda", 0)


def _ref_attention(q, k, v):
    # q [n, H, D], k/v [L, H, D] -> [n, H, D], non-causal, fp32
    s = torch.einsum("nhd,lhd->hnl", q.float(), k.float()) / q.shape[-1] ** 0.5
    return torch.einsum("hnl,lhd->nhd", torch.softmax(s, dim=-1), v.float())


def test_incremental_decode_matches_full_attention():
    torch.manual_seed(0)
    H, D = 4, 64
    cache = PagedKVCache(64, H, D, 16)
    sids = [cache.add_sequence(), cache.add_sequence()]
    ks, vs = [[], []], [[], []]
    for step, n in enumerate([37, 1, 1, 1, 20, 1]):  # prefill-sized chunks and single tokens
        k = torch.randn(2, n, H, D, device=DEV, dtype=torch.float16)
        v = torch.randn(2, n, H, D, device=DEV, dtype=torch.float16)
        q = torch.randn(2, n, H, D, device=DEV, dtype=torch.float16)
        cache.append(sids, k, v)
        for i in range(2):
            ks[i].append(k[i])
            vs[i].append(v[i])
        out = cache.attend(q, sids)
        for i in range(2):
            ref = _ref_attention(q[i], torch.cat(ks[i]), torch.cat(vs[i]))
            torch.testing.assert_close(out[i].float(), ref, atol=2e-3, rtol=1e-2)
    assert cache.context_lens(sids).tolist() == [61, 61]
    cache.free_sequence(sids[0])
    assert memopt.memopt_C.free_blocks_count() == 64 - 4


def _oracle_int4_attend(q, k_rows, v_rows, BS):
    """fp64 oracle attention of q [1, n, H, D] over the tokens k/v [L, H, D]
    (fp16) written in order into a fresh INT4 pool by the oracle's writer;
    returns (out, pages)."""
    L, H, D = k_rows.shape
    MB = (L + BS - 1) // BS
    pages = np.zeros((MB, H, O.int4_page_bytes(BS, D)), np.uint8)
    O.write_cache_int4(k_rows, v_rows, np.arange(L, dtype=np.int32), pages, BS)
    bt = np.arange(MB, dtype=np.int32)[None]
    out = O.paged_attention_int4(q, pages, bt, np.array([L], np.int32), L, L, BS)
    return out, pages


def test_scheduler_pressure_evict_int4_decode_matches_oracle():
    """Scheduler decision (retain 0.75 + INT4) applied to a live cache: exact
    eviction keeps the top tokens, the pool is re-quantised, and decode on the
    INT4 pool matches the oracle over the kept tokens, step after step; the
    pages themselves are bit-identical to the oracle's writer's."""
    torch.manual_seed(11)
    H, D, BS = 4, 128, 16
    util = {"v": 0.1}
    sched = MemoryScheduler(SchedulerConfig(drop_retain_ratio=0.75), sampler=lambda: util["v"])
    cache = PagedKVCache(32, H, D, BS)
    assert cache.eviction == "exact"
    sid = cache.add_sequence()
    k = torch.randn(1, 41, H, D, device=DEV, dtype=torch.float16)
    v = torch.randn(1, 41, H, D, device=DEV, dtype=torch.float16)
    cache.append([sid], k[:, :40], v[:, :40])
    assert cache.apply_policy(sched, None, [sid]) is None and cache.kv_format == "fp16"
    util["v"] = 0.99
    sched.adjust_policy()
    assert sched.snapshot() == (0.75, True)
    free0 = memopt.memopt_C.free_blocks_count()
    cache.append([sid], k[:, 40:], v[:, 40:])  # 41 tokens: 3 pages
    q = torch.randn(1, 1, H, D, device=DEV, dtype=torch.float16)
    kept = cache.apply_policy(sched, q, [sid], num_sink_tokens=4)[0]
    assert cache.kv_format == "int4" and len(kept) == 31 and kept[:4] == [0, 1, 2, 3]
    assert memopt.memopt_C.free_blocks_count() == free0 + 1  # 41 -> 31 tokens: 3 -> 2 pages
    # the kept set is the exact top-31 of the head-summed scores (sinks first)
    s_ = torch.einsum("hd,lhd->hl", q[0, 0].float(), k[0].float()) * D ** -0.5
    tot = torch.softmax(s_, -1).sum(0)
    assert set(kept[4:]) == set((torch.argsort(tot[4:], descending=True)[:27] + 4).tolist())
    kr = k[0, kept].cpu().numpy()
    vr = v[0, kept].cpu().numpy()
    for step in range(4):
        qn = torch.randn(1, 1, H, D, device=DEV, dtype=torch.float16)
        got = cache.attend(qn, [sid])
        ref, pages = _oracle_int4_attend(qn.cpu().numpy(), kr, vr, BS)
        np.testing.assert_allclose(got.float().cpu().numpy(), ref, atol=2e-3, rtol=1e-2)
        live = memopt.memopt_C.get_int4_pages()[torch.tensor(cache.table.pages(sid), device=DEV)].cpu().numpy()
        L = kr.shape[0]
        for a, b in zip(O.int4_views(live, BS, D), O.int4_views(pages, BS, D)):
            for t in range(L):  # every live token row, codes and scales
                assert np.array_equal(a[t // BS, :, t % BS].view(np.uint8), b[t // BS, :, t % BS].view(np.uint8))
        nk = torch.randn(1, 1, H, D, device=DEV, dtype=torch.float16)
        nv = torch.randn(1, 1, H, D, device=DEV, dtype=torch.float16)
        cache.append([sid], nk, nv)  # decode continues on the INT4 pool (fused quantising writer)
        kr = np.concatenate([kr, nk[0].cpu().numpy()])
        vr = np.concatenate([vr, nv[0].cpu().numpy()])
    assert cache.context_lens([sid]).tolist() == [35]


def test_reference_eviction_with_sinks_frees_nothing():
    """The reference-semantics mode (evict_tokens) under the same decision:
    with sink tokens, the sink boost makes the 32-step bisection keep every
    token, so no row is evicted and no page is released; exact eviction (the
    default) is the mode that frees memory."""
    torch.manual_seed(12)
    H, D, BS = 2, 64, 16
    cache = PagedKVCache(16, H, D, BS, eviction="reference")
    sid = cache.add_sequence()
    cache.append([sid], torch.randn(1, 64, H, D, device=DEV, dtype=torch.float16),
                 torch.randn(1, 64, H, D, device=DEV, dtype=torch.float16))
    before = memopt.memopt_C.get_pool_tensors()[0].clone()
    free0 = memopt.memopt_C.free_blocks_count()
    scores = torch.rand(1, H, 64, device=DEV)
    idx, cnt = cache.evict([sid], scores, 0.5, num_sink_tokens=4)
    assert cnt.tolist() == [[64, 64]]
    assert torch.equal(memopt.memopt_C.get_pool_tensors()[0], before)
    assert memopt.memopt_C.free_blocks_count() == free0 and cache.table.length(sid) == 64


def test_dynamic_attention_with_cache_and_scheduler():
    torch.manual_seed(1)
    E, H = 256, 4
    D = E // H
    util = {"v": 0.1}
    sched = MemoryScheduler(SchedulerConfig(drop_retain_ratio=0.75), sampler=lambda: util["v"])
    layer = DynamicAttention(E, H, scheduler=sched, num_sink_tokens=0).to(DEV)
    cache = PagedKVCache(32, H, D, 16)
    sids = [cache.add_sequence()]
    x = torch.randn(1, 40, E, device=DEV)
    y0 = layer(x, kv_cache=cache, seq_ids=sids)
    assert y0.shape == (1, 40, E) and torch.isfinite(y0).all() and cache.kv_format == "fp16"
    # pressure: exact eviction on the fp16 pool (41 -> 31 tokens), then INT4
    util["v"] = 0.99
    sched.adjust_policy()
    y1 = layer(torch.randn(1, 1, E, device=DEV), kv_cache=cache, seq_ids=sids)
    assert cache.kv_format == "int4" and torch.isfinite(y1).all()
    assert cache.context_lens(sids).tolist() == [31]
    # decode continues on the INT4 pool; the layer's output is out_proj of the
    # oracle's attention over the live INT4 pages
    for _ in range(3):
        xs = torch.randn(1, 1, E, device=DEV)
        y = layer(xs, kv_cache=cache, seq_ids=sids)
        q = layer.q_proj(xs).detach().reshape(1, 1, H, D).half().cpu().numpy()
        pages = memopt.memopt_C.get_int4_pages().cpu().numpy()
        bt = cache.block_tables(sids).cpu().numpy()
        cl = cache.context_lens(sids).cpu().numpy()
        att = O.paged_attention_int4(q, pages, bt, cl, int(cl[0]), int(cl[0]), 16)
        ref = layer.out_proj(torch.from_numpy(att).float().reshape(1, 1, E).to(DEV))
        torch.testing.assert_close(y.detach(), ref.detach(), atol=5e-3, rtol=1e-2)
    assert cache.context_lens(sids).tolist() == [34]


def test_to_int4_keeps_tokens_and_pages():
    torch.manual_seed(2)
    H, D = 2, 128
    cache = PagedKVCache(16, H, D, 16)
    s = cache.add_sequence()
    k = torch.randn(1, 50, H, D, device=DEV, dtype=torch.float16)
    v = torch.randn(1, 50, H, D, device=DEV, dtype=torch.float16)
    cache.append([s], k, v)
    q = torch.randn(1, 1, H, D, device=DEV, dtype=torch.float16)
    before = cache.attend(q, [s]).float()
    pages = cache.table.pages(s)
    free_before = memopt.memopt_C.free_blocks_count()
    cache.to_int4()
    assert cache.kv_format == "int4" and cache.table.pages(s) == pages
    assert memopt.memopt_C.free_blocks_count() == free_before
    after = cache.attend(q, [s]).float()
    assert (after - before).abs().max().item() < 0.1  # INT4 g64 quantisation error only


def test_exact_eviction_frees_pages_and_keeps_top_tokens():
    torch.manual_seed(3)
    H, D, BS = 2, 64, 16
    cache = PagedKVCache(40, H, D, BS, eviction="exact")
    sids = [cache.add_sequence(), cache.add_sequence()]
    k = torch.randn(2, 200, H, D, device=DEV, dtype=torch.float16)
    v = torch.randn(2, 200, H, D, device=DEV, dtype=torch.float16)
    cache.append(sids, k, v)
    free0 = memopt.memopt_C.free_blocks_count()
    scores = torch.rand(2, H, 200, device=DEV)
    kept = cache.evict_exact(sids, scores, 0.5, num_sink_tokens=4)
    tot = scores.sum(1)
    for i, s in enumerate(sids):
        assert len(kept[i]) == 100 and cache.table.length(s) == 100
        assert kept[i][:4] == [0, 1, 2, 3]  # sinks
        rest = set(torch.argsort(tot[i, 4:], descending=True)[:96].add(4).tolist())
        assert set(kept[i][4:]) == rest
        # the compacted rows are the kept tokens, in order
        q = torch.randn(1, 1, H, D, device=DEV, dtype=torch.float16)
        out = cache.attend(q, [s])
        ki = torch.tensor(kept[i], device=DEV)
        s_ = torch.einsum("hd,lhd->hl", q[0, 0].float(), k[i, ki].float()) / D ** 0.5
        ref = torch.einsum("hl,lhd->hd", torch.softmax(s_, -1), v[i, ki].float())
        torch.testing.assert_close(out[0, 0].float(), ref, atol=2e-3, rtol=1e-2)
    # 200 tokens = 13 pages each -> 100 tokens = 7 pages: 12 pages back in the pool
    assert memopt.memopt_C.free_blocks_count() == free0 + 12


def test_exact_eviction_on_the_int4_pool():
    torch.manual_seed(5)
    H, D, BS = 2, 128, 16
    cache = PagedKVCache(40, H, D, BS, kv_format="int4", eviction="exact")
    sids = [cache.add_sequence(), cache.add_sequence()]
    k = torch.randn(2, 200, H, D, device=DEV, dtype=torch.float16)
    v = torch.randn(2, 200, H, D, device=DEV, dtype=torch.float16)
    cache.append(sids, k, v)
    q = torch.randn(2, 1, H, D, device=DEV, dtype=torch.float16)
    before = cache.attend(q, sids)
    free0 = memopt.memopt_C.free_blocks_count()
    scores = cache.token_scores(q, sids)  # from the dequantised INT4 keys
    assert scores.shape == (2, H, 200)
    torch.testing.assert_close(scores.sum(-1), torch.ones(2, H, device=DEV), atol=1e-4, rtol=0)
    kept = cache.evict_exact(sids, scores, 0.5, num_sink_tokens=4)
    assert memopt.memopt_C.free_blocks_count() == free0 + 12
    after = cache.attend(q, sids)
    # The compacted cache must attend exactly like a cache that was only ever
    # given the kept tokens (INT4 codes and scales depend on the token alone).
    ref_cache_kept = [torch.tensor(kk, device=DEV) for kk in kept]
    for i, s in enumerate(sids):
        assert cache.table.length(s) == 100 and kept[i][:4] == [0, 1, 2, 3]
    fresh = PagedKVCache(40, H, D, BS, kv_format="int4")  # the same process-wide pool: new pages
    fs = [fresh.add_sequence(), fresh.add_sequence()]
    fresh.append(fs, torch.stack([k[i, ref_cache_kept[i]] for i in range(2)]),
                 torch.stack([v[i, ref_cache_kept[i]] for i in range(2)]))
    torch.testing.assert_close(after, fresh.attend(q, fs), atol=0, rtol=0)
    assert not torch.equal(before, after)



def test_int4_cache_prefill_chunk_matches_oracle():
    """A 96-row chunk on the INT4 cache takes the prefill path (pages
    dequantised into the workspace's fp16 scratch, then the tcgen05 kernel)
    through memopt_C, which sizes that workspace itself."""
    torch.manual_seed(4)
    H, D, BS = 4, 128, 16
    cache = PagedKVCache(64, H, D, BS)
    sids = [cache.add_sequence(), cache.add_sequence()]
    cache.append(sids, torch.randn(2, 300, H, D, device=DEV, dtype=torch.float16),
                 torch.randn(2, 300, H, D, device=DEV, dtype=torch.float16))
    cache.to_int4()
    cache.append(sids, torch.randn(2, 96, H, D, device=DEV, dtype=torch.float16),
                 torch.randn(2, 96, H, D, device=DEV, dtype=torch.float16))
    q = torch.randn(2, 96, H, D, device=DEV, dtype=torch.float16)
    out = cache.attend(q, sids)
    pages = memopt.memopt_C.get_int4_pages().cpu().numpy()
    bt = cache.block_tables(sids).cpu().numpy()
    cl = cache.context_lens(sids).cpu().numpy()
    assert cl.tolist() == [396, 396]
    ref = O.paged_attention_int4(q.cpu().numpy(), pages, bt, cl, int(cl.max()), int(cl.max()), BS)
    np.testing.assert_allclose(out.float().cpu().numpy(), ref, atol=2e-3, rtol=1e-2)
    # a decode step afterwards reuses the same cached workspace
    q1 = torch.randn(2, 1, H, D, device=DEV, dtype=torch.float16)
    ref1 = O.paged_attention_int4(q1.cpu().numpy(), pages, bt, cl, int(cl.max()), int(cl.max()), BS)
    np.testing.assert_allclose(cache.attend(q1, sids).float().cpu().numpy(), ref1, atol=2e-3, rtol=1e-2)
