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
