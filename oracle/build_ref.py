"""Compile the reference's own CUDA extension into oracle/_ref/ (checker only).

TEST INFRASTRUCTURE ONLY.  Builds the unmodified sources of the reference
project (src/csrc/kv_cache.cu, attention.cu, quantization.cu, extension.cpp
of a read-only reference checkout, located by MEMOPT_REFERENCE_ROOT) as a
torch extension named ``memopt_ref_C`` with the compiler flags of the
reference's setup.py:83-111, targeting sm_100.  Nothing is copied into this
repository; the build output lives in oracle/_ref/ (git-ignored) and is used
by the GPU parity tests to compare this project's kernels with the reference
kernels on the same inputs, and by tests/golden/make_golden_ref.py.
"""
from __future__ import annotations

import os
import shutil
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
OUT = os.path.join(HERE, "_ref")
SO = os.path.join(OUT, "memopt_ref_C.so")


def _default_root() -> str:
    return os.environ.get("MEMOPT_REFERENCE_ROOT", os.path.join(os.sep, "root", "reference"))


def build(ref_root: str | None = None, verbose: bool = False) -> str | None:
    csrc = os.path.join(ref_root or _default_root(), "src", "csrc")
    if not os.path.isdir(csrc):
        return SO if os.path.exists(SO) else None
    srcs = [os.path.join(csrc, f) for f in ("extension.cpp", "kv_cache.cu", "attention.cu", "quantization.cu")]
    if os.path.exists(SO) and all(os.path.getmtime(SO) >= os.path.getmtime(s) for s in srcs):
        return SO
    os.environ.setdefault("TORCH_CUDA_ARCH_LIST", "10.0")
    # The image's /opt/gcc wrapper (picked up by torch's default CXX) produces
    # extensions that crash when a TORCH_CHECK message carries a number;
    # the system compiler does not.
    if os.path.exists("/usr/bin/g++"):
        os.environ["CXX"] = "/usr/bin/g++"
    from torch.utils import cpp_extension

    bdir = os.path.join(OUT, "build")
    os.makedirs(bdir, exist_ok=True)
    cpp_extension.load(
        name="memopt_ref_C",
        sources=srcs,
        extra_include_paths=[csrc],
        extra_cflags=["-O3", "-std=c++17"],
        extra_cuda_cflags=["-O3", "-std=c++17", "--expt-relaxed-constexpr",
                           "-D__CUDA_NO_HALF_OPERATORS__", "-D__CUDA_NO_HALF_CONVERSIONS__"],
        build_directory=bdir,
        with_cuda=True,
        is_python_module=False,
        verbose=verbose,
    )
    shutil.copy2(os.path.join(bdir, "memopt_ref_C.so"), SO)
    return SO


def load():
    """Import the built reference module, or return None when absent."""
    if not os.path.exists(SO):
        return None
    import torch  # noqa: F401  (loads libtorch for the extension)

    if OUT not in sys.path:
        sys.path.insert(0, OUT)
    import memopt_ref_C  # type: ignore[import]

    return memopt_ref_C


if __name__ == "__main__":
    print(build(verbose="-v" in sys.argv))
