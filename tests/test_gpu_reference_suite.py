"""The reference's own GPU test contracts, run against this build's memopt_C.

Restates the checks of the reference test-suite (tests/test_attention.py and
tests/test_quant.py of the reference project): non-causal SDPA equivalence of
dynamic_sparse_attention at 1e-3 for S in {512, 1024, 2048}, output shape,
bit-determinism, the uninitialised-pool error, and the INT4 shape / dtype /
MSE / edge-case / error-guard contracts.  Also exercises DynamicAttention's
paged path end to end (no fallback allowed).
"""
from __future__ import annotations

import math

import pytest
import torch
import torch.nn.functional as F

import memopt_C

pytestmark = pytest.mark.gpu
BS, H, D, B = 16, 8, 64, 2


def setup_pool(seq_len):
    nbps = math.ceil(seq_len / BS)
    memopt_C.init_pool(B * nbps + 2, BS, H, D)
    rows = [[memopt_C.allocate_block() for _ in range(nbps)] for _ in range(B)]
    assert min(min(r) for r in rows) >= 0, "pool exhausted (idempotent init_pool kept a used free-list)"
    slots = [rows[b][t // BS] * BS + t % BS for b in range(B) for t in range(seq_len)]
    return (torch.tensor(slots, dtype=torch.int32, device="cuda"),
            torch.tensor(rows, dtype=torch.int32, device="cuda"))


def _run(seq_len):
    torch.manual_seed(42)
    q, k, v = (torch.rand(B, H, seq_len, D, dtype=torch.float16, device="cuda") for _ in range(3))
    base = F.scaled_dot_product_attention(q, k, v)
    slots, bt = setup_pool(seq_len)
    memopt_C.write_cache(k.permute(0, 2, 1, 3).reshape(B * seq_len, H, D).contiguous(),
                         v.permute(0, 2, 1, 3).reshape(B * seq_len, H, D).contiguous(), bt, slots)
    kc, vc = memopt_C.get_pool_tensors()
    cl = torch.full((B,), seq_len, dtype=torch.int32, device="cuda")
    out = memopt_C.dynamic_sparse_attention(q.permute(0, 2, 1, 3).contiguous(), kc, vc, bt, cl, seq_len, seq_len)
    return base, out, (q, kc, vc, bt, cl)


@pytest.mark.parametrize("seq_len", [512, 1024, 2048])
def test_math_equivalence(seq_len):
    base, out, _ = _run(seq_len)
    assert out.shape == (B, seq_len, H, D)
    assert torch.allclose(base, out.permute(0, 2, 1, 3), atol=1e-3, rtol=1e-3)


def test_determinism():
    _, out, (q, kc, vc, bt, cl) = _run(512)
    again = memopt_C.dynamic_sparse_attention(q.permute(0, 2, 1, 3).contiguous(), kc, vc, bt, cl, 512, 512)
    assert torch.equal(out, again)


def test_pool_not_initialized_raises():
    with pytest.raises(RuntimeError):
        memopt_C.init_pool(0, BS, H, D)
    z = torch.zeros(1, H, D, dtype=torch.float16, device="cuda")
    with pytest.raises(RuntimeError, match="pool not initialized|out of bounds|exhausted"):
        memopt_C.write_cache(z, z, torch.zeros(1, 1, dtype=torch.int32, device="cuda"),
                             torch.zeros(1, dtype=torch.int32, device="cuda"))


def test_get_key_value_pool_alias_pool_tensors():
    setup_pool(64)
    k, v = memopt_C.get_pool_tensors()
    assert memopt_C.get_key_pool().data_ptr() == k.data_ptr()
    assert memopt_C.get_value_pool().data_ptr() == v.data_ptr()


@pytest.mark.parametrize("shape", [(128,), (4, 128), (2, 8, 64), (2, 4, 8, 64)])
def test_quant_shapes_dtypes(shape):
    x = (torch.rand(shape, device="cuda") * 2 - 1).half()
    p, s = memopt_C.quantize_kv_cache_int4(x, 64)
    assert p.shape == shape[:-1] + (shape[-1] // 2,) and p.dtype == torch.uint8
    assert s.shape == (math.prod(shape) // 64,) and s.dtype == torch.float32
    d = memopt_C.dequantize_kv_cache_int4(p, s, 64)
    assert d.shape == shape and d.dtype == torch.float16


@pytest.mark.parametrize("dist,thr", [("u", 5e-3), ("n", 5e-2), ("s", 5e-5)])
def test_quant_mse(dist, thr):
    torch.manual_seed(42)
    x = {"u": torch.rand(8192, device="cuda") * 2 - 1, "n": torch.randn(8192, device="cuda"),
         "s": torch.rand(8192, device="cuda") * 0.2 - 0.1}[dist].half()
    p, s = memopt_C.quantize_kv_cache_int4(x, 64)
    d = memopt_C.dequantize_kv_cache_int4(p, s, 64)
    assert ((x.float() - d.float()) ** 2).mean().item() < thr


def test_quant_error_guards():
    x = torch.rand(4, 128, device="cuda").half()
    with pytest.raises(RuntimeError):
        memopt_C.quantize_kv_cache_int4(x, 32)
    with pytest.raises(RuntimeError):
        memopt_C.quantize_kv_cache_int4(x.float(), 64)
    with pytest.raises(RuntimeError):
        memopt_C.quantize_kv_cache_int4(x.cpu(), 64)
    with pytest.raises(RuntimeError):
        memopt_C.quantize_kv_cache_int4(torch.rand(128, 4, device="cuda").half().t(), 64)
    with pytest.raises(RuntimeError):
        memopt_C.quantize_kv_cache_int4(torch.rand(4, 3, device="cuda").half(), 64)
    with pytest.raises(RuntimeError):
        memopt_C.quantize_kv_cache_int4(torch.rand(50, 2, device="cuda").half(), 64)


def test_attention_unsupported_geometry_raises():
    q = torch.zeros(1, 1, 2, 96, dtype=torch.float16, device="cuda")
    kc = torch.zeros(4, 16, 2, 96, dtype=torch.float16, device="cuda")
    with pytest.raises(RuntimeError, match="unsupported"):
        memopt_C.dynamic_sparse_attention(q, kc, kc, torch.zeros(1, 1, dtype=torch.int32, device="cuda"),
                                          torch.ones(1, dtype=torch.int32, device="cuda"), 16, 16)


@pytest.mark.parametrize("fmt", ["fp16", "int4"])
def test_dynamic_attention_paged_path_runs(fmt):
    import memopt

    torch.manual_seed(0)
    S = 64
    mod = memopt.DynamicAttention(512, 8, strict=True).cuda()
    memopt_C.init_pool(B * S // BS + 7, BS, 8, 64, kv_format=fmt)  # fresh geometry: fresh free-list
    rows = [[memopt_C.allocate_block() for _ in range(S // BS)] for _ in range(B)]
    assert min(min(r) for r in rows) >= 0
    slots = torch.tensor([rows[b][t // BS] * BS + t % BS for b in range(B) for t in range(S)],
                         dtype=torch.int32, device="cuda")
    bt = torch.tensor(rows, dtype=torch.int32, device="cuda")
    cl = torch.full((B,), S, dtype=torch.int32, device="cuda")
    x = torch.randn(B, S, 512, device="cuda")
    out = mod(x, bt, slots, cl)
    dense = mod(x)  # SDPA path, same math (non-causal, full window)
    assert mod._fallback_count == 0
    tol = 5e-3 if fmt == "fp16" else 0.15
    torch.testing.assert_close(out, dense, atol=tol, rtol=tol)
