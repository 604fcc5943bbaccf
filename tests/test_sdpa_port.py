"""The CPU baseline's restatement of the reference's CPU paged attention
(oracle/sdpa_port.py) against the reference's own outputs, recorded from its
``_sdpa_fallback`` by tests/golden/make_golden.py."""
from __future__ import annotations

import os

import numpy as np
import torch

from sdpa_port import paged_sdpa

GOLDEN = os.path.join(os.path.dirname(__file__), "golden", "attention_sdpa.npz")


def test_sdpa_port_reproduces_reference_outputs():
    z = np.load(GOLDEN)
    for i in range(int(z["n_cases"])):
        g = {k: torch.from_numpy(z[f"c{i}_{k}"]) for k in ("q", "k", "v", "bt", "ctx")}
        msl = int(z[f"c{i}_max_seq_len"])
        out = paged_sdpa(g["q"], g["k"], g["v"], g["bt"], g["ctx"], msl, msl)
        ref = z[f"c{i}_out"]
        # same algorithm and the same torch arithmetic: identical fp16 results
        assert np.array_equal(out.numpy().view(np.uint16), ref.view(np.uint16)), i


def test_sdpa_port_window_keeps_sinks_and_recent_tokens():
    g = torch.Generator().manual_seed(0)
    H, D, BS = 2, 64, 16
    k = torch.randn(8, BS, H, D, generator=g).half()
    v = torch.randn(8, BS, H, D, generator=g).half()
    q = torch.randn(1, 1, H, D, generator=g).half()
    bt = torch.arange(8, dtype=torch.int32)[None]
    out = paged_sdpa(q, k, v, bt, torch.tensor([100]), 128, 40, num_sink_tokens=4)
    keep = list(range(4)) + list(range(60, 100))
    kd, vd = k.reshape(-1, H, D)[keep], v.reshape(-1, H, D)[keep]
    ref = torch.nn.functional.scaled_dot_product_attention(q[0].transpose(0, 1).float()[None],
                                                           kd.transpose(0, 1).float()[None],
                                                           vd.transpose(0, 1).float()[None], scale=D ** -0.5)
    assert torch.equal(out[0], ref[0].transpose(0, 1).half())
