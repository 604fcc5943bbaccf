"""Host-side tests that need no GPU: the C-ABI library, the pool free-list,
the memopt_C module surface, the scheduler policy and the Python API."""
from __future__ import annotations

import ctypes as C
import os
import re
import threading
import time

import pytest
import torch

from conftest import PKG, REPO

HEADER = os.path.join(REPO, "include", "memopt_b200.h")
LIB = os.path.join(PKG, "libmemopt_b200.so")


def declared_symbols() -> list[str]:
    text = open(HEADER).read()
    return sorted(set(re.findall(r"\b(memopt_[a-z0-9_]+)\s*\(", text)))


@pytest.fixture(scope="module")
def lib():
    if not os.path.exists(LIB):
        pytest.fail("libmemopt_b200.so is not built (run memopt-transformer-runtime_b200/build.py)")
    return C.CDLL(LIB)


def test_library_exports_every_declared_symbol(lib):
    syms = declared_symbols()
    assert len(syms) >= 20
    for s in syms:
        assert hasattr(lib, s), f"{s} declared in memopt_b200.h but not exported"


def test_status_strings(lib):
    lib.memopt_status_string.restype = C.c_char_p
    assert lib.memopt_status_string(0) == b"ok"
    assert b"pool" in lib.memopt_status_string(-2)
    assert lib.memopt_abi_version() == 1


def test_pool_free_list_fifo(lib):
    lib.memopt_pool_reset()
    assert lib.memopt_pool_allocate_block() == -2  # not initialized
    assert lib.memopt_pool_init(4, 16, 2, 64) == 0
    assert lib.memopt_pool_free_blocks_count() == 4
    got = [lib.memopt_pool_allocate_block() for _ in range(5)]
    assert got == [0, 1, 2, 3, -1]
    assert lib.memopt_pool_free_block(2) == 0
    assert lib.memopt_pool_free_block(0) == 0
    assert lib.memopt_pool_free_block(4) == -5  # out of range
    assert [lib.memopt_pool_allocate_block() for _ in range(2)] == [2, 0]
    # same geometry: idempotent (free-list unchanged)
    assert lib.memopt_pool_init(4, 16, 2, 64) == 0
    assert lib.memopt_pool_free_blocks_count() == 0
    # bad geometry: error and uninitialised afterwards
    assert lib.memopt_pool_init(0, 16, 2, 64) == -1
    assert lib.memopt_pool_is_initialized() == 0
    assert lib.memopt_pool_init(3, 16, 2, 63) == -1  # odd head_dim
    lib.memopt_pool_reset()


def test_pool_thread_safety(lib):
    lib.memopt_pool_reset()
    assert lib.memopt_pool_init(20000, 16, 2, 64) == 0
    out: list[list[int]] = [[] for _ in range(4)]

    def worker(i):
        for _ in range(5000):
            out[i].append(lib.memopt_pool_allocate_block())

    ts = [threading.Thread(target=worker, args=(i,)) for i in range(4)]
    for t in ts:
        t.start()
    for t in ts:
        t.join()
    allb = sorted(x for o in out for x in o)
    assert allb == list(range(20000))
    lib.memopt_pool_reset()


def test_kernel_entry_points_validate_without_gpu(lib):
    # Argument errors are reported before any device work.
    assert lib.memopt_quantize_int4(None, C.c_int64(64), 32, None, None, None) == -1
    assert lib.memopt_evict_tokens(None, 1, 1, 1, None, 1, None, 1, None, None, 1, 16, 64,
                                   C.c_float(1.5), 4, None, None, None) == -1
    sz = lib.memopt_paged_attention_workspace_size
    sz.restype = C.c_size_t
    assert sz(0, 1, 1, 64, 1, 16, 16, 16) == 0


def test_int4_workspace_adds_the_prefill_scratch_only_for_prefill_calls(lib):
    gen = lib.memopt_paged_attention_workspace_size_ex
    i4 = lib.memopt_paged_attention_int4_workspace_size_ex
    gen.restype = i4.restype = C.c_size_t
    # decode (q_len 1): the same size for both pool formats
    assert i4(4, 1, 32, 8, 128, 512, 16, 8192, 8192) == gen(4, 1, 32, 8, 128, 512, 16, 8192, 8192)
    # prefill (q_len >= 64): the split workspace (256-aligned) + fp16 K and V pages + a table
    B, QL, H, KVH, D, MB, BS = 4, 8192, 32, 32, 128, 512, 16
    split = gen(B, QL, H, KVH, D, MB, BS, 8192, 8192)
    kv = B * MB * BS * KVH * D * 2
    table = -(-(B * MB * 4) // 256) * 256
    assert i4(B, QL, H, KVH, D, MB, BS, 8192, 8192) == -(-split // 256) * 256 + 2 * kv + table
    # head_dim / block_size pairs without a prefill kernel keep the multi-query path's size
    assert i4(1, 128, 4, 2, 192, 8, 16, 128, 128) == gen(1, 128, 4, 2, 192, 8, 16, 128, 128)
    assert i4(0, 128, 4, 2, 128, 8, 16, 128, 128) == 0


def test_memopt_c_module_surface():
    import memopt_C

    for name in ["get_hello", "init_pool", "allocate_block", "free_block", "get_pool_tensors",
                 "free_blocks_count", "write_cache", "evict_cache", "evict_tokens",
                 "dynamic_sparse_attention", "quantize_kv_cache_int4", "dequantize_kv_cache_int4",
                 "get_key_pool", "get_value_pool", "dynamic_sparse_attention_int4",
                 "get_int4_pool_tensors", "get_int4_pages"]:
        assert hasattr(memopt_C, name), name
    assert "MemOpt C++ Backend Initialized" in memopt_C.get_hello()


def test_memopt_c_errors_on_cpu_tensors():
    import memopt_C

    with pytest.raises(RuntimeError):
        memopt_C.quantize_kv_cache_int4(torch.zeros(4, 128, dtype=torch.float16), 64)
    # init_pool(0, ...) raises and leaves no pool behind (the reference kept the
    # previous pool, which made tests/test_attention.py:252-290 order-dependent).
    with pytest.raises(RuntimeError):
        memopt_C.init_pool(0, 16, 8, 64)
    with pytest.raises(RuntimeError, match="pool not initialized"):
        memopt_C.write_cache(torch.zeros(1, 8, 64, dtype=torch.float16),
                             torch.zeros(1, 8, 64, dtype=torch.float16),
                             torch.zeros(1, 1, dtype=torch.int32), torch.zeros(1, dtype=torch.int32))


def test_reference_import_contract():
    import memopt

    assert memopt.__version__ == "0.1.0"
    assert "MemOpt C++ Backend Initialized" in memopt.get_hello()


def test_dynamic_attention_sdpa_path_matches_torch():
    import memopt

    torch.manual_seed(0)
    m = memopt.DynamicAttention(512, 8)
    x = torch.randn(2, 64, 512)
    out = m(x)
    q = m.q_proj(x).reshape(2, 64, 8, 64).transpose(1, 2)
    k = m.k_proj(x).reshape(2, 64, 8, 64).transpose(1, 2)
    v = m.v_proj(x).reshape(2, 64, 8, 64).transpose(1, 2)
    ref = torch.softmax(q @ k.transpose(-1, -2) / 8.0, -1) @ v
    ref = m.out_proj(ref.transpose(1, 2).reshape(2, 64, 512))
    torch.testing.assert_close(out, ref, atol=1e-5, rtol=1e-4)


def test_dynamic_attention_window_truncates_keys():
    import memopt

    torch.manual_seed(0)
    m = memopt.DynamicAttention(64, 2, window_size=8)
    x = torch.randn(1, 32, 64)
    out = m(x)
    m2 = memopt.DynamicAttention(64, 2)
    m2.load_state_dict(m.state_dict())
    assert not torch.allclose(out, m2(x))


def test_dynamic_attention_paged_cpu_falls_back_with_warning():
    import memopt

    m = memopt.DynamicAttention(64, 2)
    x = torch.randn(1, 4, 64)
    bt = torch.zeros(1, 1, dtype=torch.int32)
    sm = torch.arange(4, dtype=torch.int32)
    cl = torch.full((1,), 4, dtype=torch.int32)
    with pytest.warns(RuntimeWarning):
        m(x, bt, sm, cl)
    assert m._fallback_count == 1 and not m._use_custom_kernel
    strict = memopt.DynamicAttention(64, 2, strict=True)
    with pytest.raises(RuntimeError):
        strict(x, bt, sm, cl)


def test_scheduler_config_validation():
    from memopt import SchedulerConfig

    SchedulerConfig()
    for kw in [dict(vram_high_threshold=0.0), dict(vram_low_threshold=0.9),
               dict(drop_retain_ratio=1.0), dict(poll_interval_sec=0.0)]:
        with pytest.raises(ValueError):
            SchedulerConfig(**kw)


def test_scheduler_hysteresis_with_fake_sampler():
    from memopt import MemoryScheduler

    util = [0.2]
    s = MemoryScheduler(sampler=lambda: util[0])
    s.adjust_policy()
    assert s.snapshot() == (1.0, False)
    util[0] = 0.9
    s.adjust_policy()
    assert s.snapshot() == (0.75, True)
    util[0] = 0.7  # dead band: unchanged
    s.adjust_policy()
    assert s.snapshot() == (0.75, True)
    util[0] = 0.5
    s.adjust_policy()
    assert s.snapshot() == (1.0, False)


def test_scheduler_thread_and_hook():
    from memopt import MemoryScheduler, SchedulerConfig

    util = [0.95]
    s = MemoryScheduler(SchedulerConfig(poll_interval_sec=0.01), sampler=lambda: util[0])
    s.start()
    deadline = time.time() + 5
    while s.retain_ratio != 0.75 and time.time() < deadline:
        time.sleep(0.01)
    assert s.use_int4
    s.stop()
    s.start()  # restartable
    s.stop()
    util[0] = 0.1
    lin = torch.nn.Linear(2, 2)
    s.attach_hook(lin)
    lin(torch.zeros(1, 2))
    assert s.snapshot() == (1.0, False)
    s.detach_hook()
    with pytest.raises(TypeError):
        s.attach_hook("not a module")


def test_scheduler_survives_sampler_exceptions():
    from memopt import MemoryScheduler

    def bad():
        raise RuntimeError("boom")

    s = MemoryScheduler(sampler=bad)
    s.adjust_policy()
    assert s.snapshot() == (1.0, False)
    assert "MemoryScheduler(" in repr(s)
