"""Generate golden attention fixtures from the reference's own CPU code path.

Run in a checkout that has the reference project available (its ``src``
directory given by MEMOPT_REFERENCE_ROOT, default /root/reference):

    python tests/golden/make_golden.py

It imports the reference's pure-PyTorch paged attention
(``memopt.triton_attention._sdpa_fallback``, reference
src/memopt/triton_attention.py:473-550) and evaluates it on small seeded
paged caches with ``window_size == max_seq_len`` — the setting in which its
semantics coincide with the CUDA kernel's (attention.cu:153-186: no window,
no sinks, non-causal).  The results are written to attention_sdpa.npz and
pin the CPU oracle in tests/test_oracle_golden.py.  The reference is needed
only to regenerate the file, never to run the tests.
"""
from __future__ import annotations

import os
import sys

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
REF = os.environ.get("MEMOPT_REFERENCE_ROOT", os.path.join(os.sep, "root", "reference"))


def case(seed: int, B: int, QL: int, H: int, D: int, BS: int, ctx: list[int], mb: int, dist: str):
    g = torch.Generator().manual_seed(seed)
    nb = B * mb + 3
    perm = torch.randperm(nb, generator=g)[: B * mb].reshape(B, mb).to(torch.int32)
    if dist == "normal":
        kp = torch.randn(nb, BS, H, D, generator=g).half()
        vp = torch.randn(nb, BS, H, D, generator=g).half()
        q = torch.randn(B, QL, H, D, generator=g).half()
    else:  # U[0,1) as in tests/test_attention.py of the reference
        kp = torch.rand(nb, BS, H, D, generator=g).half()
        vp = torch.rand(nb, BS, H, D, generator=g).half()
        q = torch.rand(B, QL, H, D, generator=g).half()
    cl = torch.tensor(ctx, dtype=torch.int32)
    max_seq_len = mb * BS
    return q, kp, vp, perm, cl, max_seq_len


def main() -> None:
    sys.path.insert(0, os.path.join(REF, "src"))
    from memopt.triton_attention import _sdpa_fallback  # reference code

    cases = [
        (1, 2, 1, 4, 64, 16, [37, 64], 4, "normal"),
        (2, 2, 3, 4, 128, 16, [100, 5], 7, "normal"),
        (3, 3, 1, 2, 64, 32, [64, 33, 96], 3, "uniform"),
        (4, 1, 2, 2, 128, 32, [200], 7, "uniform"),
    ]
    out = {}
    for i, c in enumerate(cases):
        q, kp, vp, bt, cl, msl = case(*c)
        with torch.no_grad():
            o = _sdpa_fallback(q, kp, vp, bt, cl, msl, msl, 4, c[5])
        for name, t in (("q", q), ("k", kp), ("v", vp), ("bt", bt), ("ctx", cl), ("out", o)):
            out[f"c{i}_{name}"] = t.numpy()
        out[f"c{i}_max_seq_len"] = np.array(msl)
    out["n_cases"] = np.array(len(cases))
    np.savez_compressed(os.path.join(HERE, "attention_sdpa.npz"), **out)
    print("wrote", len(cases), "cases")


if __name__ == "__main__":
    main()
