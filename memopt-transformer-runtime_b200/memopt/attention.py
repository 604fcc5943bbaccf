"""``DynamicAttention``: multi-head attention over the paged KV pool.

Same constructor, forward signature and routing as the reference module
(src/memopt/attention.py:79-547):

* q/k/v/out projections are ``nn.Linear(E, E, bias=False)``;
* ``forward(x, block_tables=None, slot_mapping=None, context_lens=None)``
  takes the paged path when ``memopt_C`` is loaded and all three paged
  arguments are given: K/V are cast to fp16 and written with
  ``memopt_C.write_cache``, then ``memopt_C.dynamic_sparse_attention`` runs
  over the pool with ``max_seq_len = S`` and the effective window
  (``window_size <= 0`` -> S); an int4 pool is read with
  ``dynamic_sparse_attention_int4``;
* without paged arguments it computes dense SDPA, keeping only the last
  ``window_size`` keys when ``S > window_size`` (reference :475-530);
* ``forward(x, kv_cache=cache, seq_ids=ids)`` (addition) appends this
  call's K/V to a :class:`memopt.kv_cache.PagedKVCache` and attends over each
  sequence's whole cached context (incremental decode); with
  ``scheduler=MemoryScheduler(...)`` the scheduler's ``retain_ratio`` /
  ``use_int4`` are applied to the cache first (eviction, INT4 conversion);
* an exception on the paged path is reported as a RuntimeWarning, counted
  in ``_fallback_count``, disables the paged path for the instance and the
  call is answered by SDPA — unless ``strict=True``, which re-raises.

The reference's paged path always failed (it called ``get_key_pool`` /
``get_value_pool``, which its extension never exported); here both exist, so
the paged path runs.  There is no Triton backend: ``use_triton=True`` only
emits a warning.
"""
from __future__ import annotations

import warnings
from typing import Optional

import torch
import torch.nn as nn
import torch.nn.functional as F

try:
    import memopt_C as _memopt_C  # type: ignore[import]

    _C_EXT_AVAILABLE: bool = True
except ImportError:  # pragma: no cover
    _memopt_C = None  # type: ignore[assignment]
    _C_EXT_AVAILABLE = False

__all__ = ["DynamicAttention"]


class DynamicAttention(nn.Module):
    """Multi-head attention backed by the B200 paged KV-cache kernels."""

    def __init__(
        self,
        embed_dim: int,
        num_heads: int,
        dropout: float = 0.0,
        window_size: int = -1,
        num_sink_tokens: int = 4,
        use_triton: bool = False,
        strict: bool = False,
        scheduler=None,
    ) -> None:
        super().__init__()
        assert embed_dim % num_heads == 0, (
            f"embed_dim ({embed_dim}) must be divisible by num_heads ({num_heads})"
        )
        self.embed_dim = embed_dim
        self.num_heads = num_heads
        self.head_dim = embed_dim // num_heads
        self.dropout = dropout
        self.window_size = window_size
        self.num_sink_tokens = num_sink_tokens
        self.scale = self.head_dim ** -0.5
        self.strict = strict
        self.scheduler = scheduler

        self.q_proj = nn.Linear(embed_dim, embed_dim, bias=False)
        self.k_proj = nn.Linear(embed_dim, embed_dim, bias=False)
        self.v_proj = nn.Linear(embed_dim, embed_dim, bias=False)
        self.out_proj = nn.Linear(embed_dim, embed_dim, bias=False)

        self._use_custom_kernel: bool = _C_EXT_AVAILABLE
        self._fallback_count: int = 0
        if use_triton:
            warnings.warn(
                "DynamicAttention: this build has no Triton backend; use_triton is ignored "
                "and the paged CUDA kernels are used.",
                RuntimeWarning,
                stacklevel=2,
            )
        self._use_triton = False

    def _effective_window(self, seq_len: int) -> int:
        return seq_len if self.window_size <= 0 else self.window_size

    def forward(
        self,
        x: torch.Tensor,
        block_tables: Optional[torch.Tensor] = None,
        slot_mapping: Optional[torch.Tensor] = None,
        context_lens: Optional[torch.Tensor] = None,
        kv_cache=None,
        seq_ids=None,
    ) -> torch.Tensor:
        orig_dtype = x.dtype
        B, seq_len, _ = x.shape
        q = self.q_proj(x)
        k = self.k_proj(x)
        v = self.v_proj(x)
        if kv_cache is not None:
            # Incremental path: this call's tokens are appended to each
            # sequence's cache and attend over its whole cached context.
            H, D = self.num_heads, self.head_dim
            q4 = q.reshape(B, seq_len, H, D)
            kv_cache.append(seq_ids, k.reshape(B, seq_len, H, D), v.reshape(B, seq_len, H, D))
            if self.scheduler is not None:
                kv_cache.apply_policy(self.scheduler, q4, seq_ids, self.num_sink_tokens)
            out = kv_cache.attend(q4, seq_ids, self.window_size)
            return self.out_proj(out.reshape(B, seq_len, self.embed_dim).to(orig_dtype))
        paged = block_tables is not None and slot_mapping is not None and context_lens is not None
        if self._use_custom_kernel and paged:
            try:
                attn = self._custom_kernel_forward(
                    q, k, v, block_tables, slot_mapping, context_lens, seq_len, orig_dtype
                )
            except Exception as exc:  # noqa: BLE001
                if self.strict:
                    raise
                warnings.warn(
                    f"DynamicAttention: custom kernel raised {type(exc).__name__}: {exc}. "
                    "Disabling custom kernel for this instance and falling back to SDPA.",
                    RuntimeWarning,
                    stacklevel=2,
                )
                self._fallback_count += 1
                self._use_custom_kernel = False
                attn = self._sdpa_forward(q, k, v, seq_len)
        else:
            attn = self._sdpa_forward(q, k, v, seq_len)
        return self.out_proj(attn)

    def _custom_kernel_forward(
        self,
        q: torch.Tensor,
        k: torch.Tensor,
        v: torch.Tensor,
        block_tables: torch.Tensor,
        slot_mapping: torch.Tensor,
        context_lens: torch.Tensor,
        seq_len: int,
        orig_dtype: torch.dtype,
    ) -> torch.Tensor:
        B = q.shape[0]
        H, D = self.num_heads, self.head_dim
        k16 = k.to(torch.float16).reshape(B * seq_len, H, D)
        v16 = v.to(torch.float16).reshape(B * seq_len, H, D)
        _memopt_C.write_cache(k16, v16, block_tables, slot_mapping)
        q16 = q.to(torch.float16).reshape(B, seq_len, H, D).contiguous()
        window = self._effective_window(seq_len)
        if _memopt_C.pool_format() == "int4":
            pages = _memopt_C.get_int4_pages()
            out = _memopt_C.dynamic_sparse_attention_int4(
                q16, pages, block_tables, context_lens, seq_len, window
            )
        else:
            key_cache = _memopt_C.get_key_pool()
            value_cache = _memopt_C.get_value_pool()
            out = _memopt_C.dynamic_sparse_attention(
                q16, key_cache, value_cache, block_tables, context_lens, seq_len, window
            )
        return out.reshape(B, seq_len, self.embed_dim).to(orig_dtype)

    def _sdpa_forward(self, q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, seq_len: int) -> torch.Tensor:
        B = q.shape[0]
        H, D = self.num_heads, self.head_dim
        qs = q.reshape(B, seq_len, H, D).transpose(1, 2)
        ks = k.reshape(B, seq_len, H, D).transpose(1, 2)
        vs = v.reshape(B, seq_len, H, D).transpose(1, 2)
        if self.window_size > 0 and seq_len > self.window_size:
            ks = ks[:, :, -self.window_size:, :]
            vs = vs[:, :, -self.window_size:, :]
        out = F.scaled_dot_product_attention(qs, ks, vs, scale=self.scale, dropout_p=0.0)
        return out.transpose(1, 2).reshape(B, seq_len, self.embed_dim)

    def __repr__(self) -> str:  # noqa: D105
        return (
            f"DynamicAttention(embed_dim={self.embed_dim}, num_heads={self.num_heads}, "
            f"head_dim={self.head_dim}, window_size={self.window_size}, "
            f"custom_kernel={'on' if self._use_custom_kernel else 'off (fallback)'}, "
            f"triton=off, fallback_count={self._fallback_count})"
        )
