"""Head-sharded exact eviction on two GPUs: one process per GPU, memopt_C on
each rank's pool, the partial token scores all-gathered over NCCL."""
from __future__ import annotations

import pytest
import torch

from test_multirank import _spawn, check_head_sharded_evict


@pytest.mark.gpu
@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_two_gpu_nccl_head_sharded_exact_eviction(tmp_path):
    _spawn("multirank_evict_worker.py", 2, [tmp_path, "nccl"], extra_env={"NCCL_NVLS_ENABLE": "0"}, timeout=300)
    check_head_sharded_evict(tmp_path, 2)


@pytest.mark.gpu
@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_two_gpu_multi_device_pool_attention(tmp_path):
    """A sequence whose pages spill onto the second GPU: pages packed with
    memopt_copy_pages, sent over NCCL into the home GPU's staging blocks,
    attention on the home GPU, checked against the oracle."""
    from test_multirank import check_multi_pool

    _spawn("multirank_pool_worker.py", 2, [tmp_path, "nccl"], extra_env={"NCCL_NVLS_ENABLE": "0"}, timeout=300)
    check_multi_pool(tmp_path, 2)


@pytest.mark.gpu
def test_copy_pages_pack_and_unpack_bit_exact():
    import ctypes as C

    import capi

    g = torch.Generator(device="cuda").manual_seed(5)
    pool = torch.randn(50, 16, 4, 64, device="cuda", generator=g).half()
    ids = torch.tensor([7, 3, 49, 0, 3], dtype=torch.int32, device="cuda")
    buf = torch.empty(5, 16, 4, 64, dtype=torch.float16, device="cuda")
    pb = C.c_int64(16 * 4 * 64 * 2)
    capi.ok(capi.lib().memopt_copy_pages(capi.ptr(pool), capi.ptr(ids), capi.ptr(buf), capi.P(0), C.c_int(5), pb,
                                         capi.stream()))
    assert torch.equal(buf, pool[ids.long()])
    dst = torch.zeros_like(pool)
    slots = torch.tensor([40, 41, 42, 43, -1], dtype=torch.int32, device="cuda")  # -1: skipped
    capi.ok(capi.lib().memopt_copy_pages(capi.ptr(buf), capi.P(0), capi.ptr(dst), capi.ptr(slots), C.c_int(5), pb,
                                         capi.stream()))
    assert torch.equal(dst[40:44], buf[:4]) and int(dst[:40].count_nonzero()) == 0 and int(dst[44:].count_nonzero()) == 0
    assert capi.lib().memopt_copy_pages(capi.ptr(pool), capi.P(0), capi.ptr(dst), capi.P(0), C.c_int(1),
                                        C.c_int64(24), capi.stream()) == -3  # not a multiple of 16


@pytest.mark.gpu
@pytest.mark.parametrize("kv_format", ["fp16", "int4"])
def test_single_gpu_multi_device_pool_matches_oracle(kv_format):
    """World of one: the pool's CUDA defaults (write_cache into its own
    tensors, gather with no remote pages, paged attention) against the oracle."""
    import numpy as np

    import oracle as O
    from memopt.multi_pool import MultiDevicePagePool
    from memopt.sharding import RankGroup

    H, D, BS = 4, 128, 16
    pool = MultiDevicePagePool(RankGroup(), 20, 4, BS, H, D, kv_format=kv_format, device=torch.device("cuda", 0))
    s = pool.add_sequence(0)
    rng = np.random.default_rng(3)
    k = rng.standard_normal((150, H, D)).astype(np.float16)
    v = rng.standard_normal((150, H, D)).astype(np.float16)
    pool.append(s, torch.from_numpy(k[:100]).cuda(), torch.from_numpy(v[:100]).cuda())
    pool.append(s, torch.from_numpy(k[100:]).cuda(), torch.from_numpy(v[100:]).cuda())
    q = rng.standard_normal((1, 1, H, D)).astype(np.float16)
    out = pool.attend([s], torch.from_numpy(q).cuda())
    MB = 10
    bt = np.arange(MB, dtype=np.int32)[None]
    if kv_format == "fp16":
        kp = np.zeros((MB, BS, H, D), np.float16)
        vp = np.zeros_like(kp)
        kp.reshape(-1, H, D)[:150], vp.reshape(-1, H, D)[:150] = k, v
        ref = O.paged_attention_f16(q, kp, vp, bt, np.array([150], np.int32), 150, 150)
    else:
        pages = np.zeros((MB, H, O.int4_page_bytes(BS, D)), np.uint8)
        O.write_cache_int4(k, v, np.arange(150, dtype=np.int32), pages, BS)
        ref = O.paged_attention_int4(q, pages, bt, np.array([150], np.int32), 150, 150, BS)
    np.testing.assert_allclose(out.float().cpu().numpy(), ref, atol=2e-3, rtol=1e-2)
    assert [p[0] for p in pool.pages(s)] == [0] * MB
