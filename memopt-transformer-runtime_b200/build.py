"""Build recipe for the B200 data plane (run from any directory).

Produces, next to this file:
  * libmemopt_b200.so — the C-ABI library (include/memopt_b200.h): every
    CUDA kernel, compiled for sm_100a only, with a static CUDA runtime;
  * memopt_C.so       — the PyTorch-facing module (a thin C++ wrapper that
    links libmemopt_b200.so through an $ORIGIN rpath).
Both are rebuilt only when a source is newer than the output.
"""
from __future__ import annotations

import os
import shutil
import subprocess
import sys

PKG = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(PKG)
CSRC = os.path.join(PKG, "csrc")
INCLUDE = os.path.join(REPO, "include")
LIB = os.path.join(PKG, "libmemopt_b200.so")
EXT = os.path.join(PKG, "memopt_C.so")
CU_SOURCES = ["host.cu", "quant.cu", "write_cache.cu", "evict.cu", "decode.cu", "decode_static.cu", "prefill.cu", "compact.cu", "mdpool.cu"]
NVCC_FLAGS = [
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-O3", "-std=c++17", "-lineinfo", "--expt-relaxed-constexpr",
    "-Xcompiler", "-fPIC", "-Xcompiler", "-fvisibility=hidden",
]


def _nvcc() -> str:
    cuda_home = os.environ.get("CUDA_HOME", "/usr/local/cuda")
    path = os.path.join(cuda_home, "bin", "nvcc")
    return path if os.path.exists(path) else "nvcc"


def _newer(out: str, deps: list[str]) -> bool:
    if not os.path.exists(out):
        return True
    t = os.path.getmtime(out)
    return any(os.path.getmtime(d) > t for d in deps if os.path.exists(d))


def _sources() -> list[str]:
    return [os.path.join(CSRC, s) for s in CU_SOURCES if os.path.exists(os.path.join(CSRC, s))]


def _compile_one(src: str, obj: str, verbose: bool) -> None:
    cmd = [_nvcc(), *NVCC_FLAGS, "-I", INCLUDE, "-I", CSRC, "-c", src, "-o", obj]
    if verbose:
        print(" ".join(cmd), flush=True)
    subprocess.run(cmd, check=True)


def build_lib(verbose: bool = False) -> str:
    srcs = _sources()
    headers = [os.path.join(CSRC, f) for f in os.listdir(CSRC) if f.endswith((".cuh", ".h"))]
    headers.append(os.path.join(INCLUDE, "memopt_b200.h"))
    if not _newer(LIB, srcs + headers + [__file__]):
        return LIB
    objdir = os.path.join(PKG, "_build", "obj")
    os.makedirs(objdir, exist_ok=True)
    objs = [os.path.join(objdir, os.path.basename(s) + ".o") for s in srcs]
    from concurrent.futures import ThreadPoolExecutor

    with ThreadPoolExecutor(max_workers=min(8, len(srcs))) as ex:
        list(ex.map(lambda so: _compile_one(so[0], so[1], verbose), zip(srcs, objs)))
    tmp = LIB + ".tmp"
    cmd = [_nvcc(), "-shared", "-gencode", "arch=compute_100a,code=sm_100a", "-cudart", "static", *objs, "-o", tmp,
           "-Xlinker", "-soname=libmemopt_b200.so"]
    subprocess.run(cmd, check=True)
    os.replace(tmp, LIB)
    return LIB


def build_ext(verbose: bool = False) -> str:
    src = os.path.join(CSRC, "memopt_C.cpp")
    if not _newer(EXT, [src, LIB, os.path.join(INCLUDE, "memopt_b200.h"), __file__]):
        return EXT
    # The image's /opt/gcc wrapper (picked up by torch's default CXX) produces
    # extensions that crash when a TORCH_CHECK message carries a number;
    # the system compiler does not.
    if os.path.exists("/usr/bin/g++"):
        os.environ["CXX"] = "/usr/bin/g++"
    from torch.utils import cpp_extension

    bdir = os.path.join(PKG, "_build", "memopt_C")
    os.makedirs(bdir, exist_ok=True)
    cpp_extension.load(
        name="memopt_C",
        sources=[src],
        extra_include_paths=[INCLUDE],
        extra_cflags=["-O2", "-std=c++17"],
        extra_ldflags=[f"-L{PKG}", "-lmemopt_b200", "-Wl,-rpath,$ORIGIN", f"-Wl,-rpath,{PKG}"],
        build_directory=bdir,
        with_cuda=True,
        is_python_module=False,
        verbose=verbose,
    )
    built = os.path.join(bdir, "memopt_C.so")
    shutil.copy2(built, EXT + ".tmp")
    os.replace(EXT + ".tmp", EXT)
    return EXT


def build(verbose: bool = False) -> None:
    build_lib(verbose)
    build_ext(verbose)


if __name__ == "__main__":
    build(verbose="-v" in sys.argv)
