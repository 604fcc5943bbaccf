"""Restatement of the reference's CPU paged attention, for the CPU baseline.

TEST INFRASTRUCTURE ONLY: used by tests/ (pinned against the reference's own
outputs in tests/golden/attention_sdpa.npz) and by bench.py's CPU baseline and
reference arm as the stand-in for the reference's CPU path, which is Python
that this build cannot carry to the GPU box.

Algorithm of the reference's ``_sdpa_fallback``
(src/memopt/triton_attention.py:473-550), for the setting the benchmark uses
(window_size == max_seq_len, so no Ada-KV windowing): per sequence, the pages
covering its context are gathered in table order into dense K and V
[ctx, H, D], truncated to ctx rows, and PyTorch's scaled_dot_product_attention
runs on them in fp32 with scale 1/sqrt(D); the result is rounded to fp16.
With a window smaller than max_seq_len the reference keeps the sink tokens
plus the last `window` tokens; that branch is restated too.
"""
from __future__ import annotations

import math

import torch
import torch.nn.functional as F


def paged_sdpa(query: torch.Tensor, key_cache: torch.Tensor, value_cache: torch.Tensor,
               block_tables: torch.Tensor, context_lens: torch.Tensor, max_seq_len: int, window_size: int,
               num_sink_tokens: int = 4) -> torch.Tensor:
    """query [B, QL, H, D] fp16, caches [NB, BS, H, D] fp16 (CPU tensors) ->
    [B, QL, H, D] fp16."""
    B, QL, H, D = query.shape
    BS = key_cache.shape[1]
    outs = []
    for b in range(B):
        n = int(context_lens[b])
        pages = block_tables[b, : math.ceil(n / BS)].long()
        k = key_cache.index_select(0, pages).reshape(-1, H, D)[:n]
        v = value_cache.index_select(0, pages).reshape(-1, H, D)[:n]
        if window_size < max_seq_len and n > window_size:
            sink = min(num_sink_tokens, n)
            keep = torch.cat([torch.arange(sink), torch.arange(max(n - window_size, sink), n)])
            k, v = k[keep], v[keep]
        o = F.scaled_dot_product_attention(query[b].transpose(0, 1).float()[None], k.transpose(0, 1).float()[None],
                                           v.transpose(0, 1).float()[None], scale=D ** -0.5, dropout_p=0.0)
        outs.append(o[0].transpose(0, 1).half())
    return torch.stack(outs)
