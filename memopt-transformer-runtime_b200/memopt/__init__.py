"""MemOpt KV-cache data plane, B200 (sm_100a) build.

Drop-in for the reference package ``memopt`` (src/memopt/__init__.py:1-20):
same ``__version__``, ``get_hello``, ``DynamicAttention``, ``MemoryScheduler``
and ``SchedulerConfig``.  The compiled module ``memopt_C`` lives next to this
package directory.  The reference's ``BaselineLlama`` HF wrapper is not part
of the data plane and is not provided.

On a machine with a CUDA device the extension is mandatory: a missing or
unloadable ``memopt_C`` raises instead of silently degrading.
"""
from __future__ import annotations

import os as _os
import sys as _sys

__version__ = "0.1.0"

_here = _os.path.dirname(_os.path.dirname(_os.path.abspath(__file__)))
if _here not in _sys.path:
    _sys.path.insert(0, _here)

import torch as _torch  # noqa: E402  (loads libc10/libtorch for memopt_C)

try:
    import memopt_C  # noqa: F401

    _C_AVAILABLE = True
except ImportError as _e:  # pragma: no cover - exercised only on broken installs
    _C_AVAILABLE = False
    if _torch.cuda.is_available():
        raise ImportError(
            "memopt: the CUDA extension memopt_C could not be loaded on a CUDA machine "
            f"({_e}); build it with memopt-transformer-runtime_b200/build.py"
        ) from _e

from memopt.attention import DynamicAttention  # noqa: E402
from memopt.scheduler import MemoryScheduler, SchedulerConfig  # noqa: E402
from memopt.kv_cache import PagedKVCache, PageTable  # noqa: E402

__all__ = ["DynamicAttention", "MemoryScheduler", "SchedulerConfig", "PagedKVCache", "PageTable", "get_hello"]


def get_hello() -> str:
    """Returns a greeting from the C++ backend if available."""
    if _C_AVAILABLE:
        return memopt_C.get_hello()
    return "C++ backend not loaded."
