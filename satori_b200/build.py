"""Build recipe for the in-tree CUDA library ``satori_b200/_build/libsatori_cuda.so`` (sm_100a).

One nvcc invocation compiles every ``csrc/*.cu`` for ``-gencode arch=compute_100a,code=sm_100a``
and links them, with the CUDA runtime linked statically, into a shared library exposing the C ABI
declared in ``include/satori_cuda.h``.  The library is built in-tree so that it travels with the
repository snapshot to the GPU machine.
"""
from __future__ import annotations

import glob
import os
import shutil
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
CSRC = os.path.join(HERE, "csrc")
BUILD_DIR = os.path.join(HERE, "_build")
LIB_PATH = os.path.join(BUILD_DIR, "libsatori_cuda.so")
HEADER = os.path.join(ROOT, "include", "satori_cuda.h")

NVCC_FLAGS = [
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-O3", "-lineinfo", "-std=c++17",
    "-Xcompiler", "-fPIC,-O2,-fvisibility=hidden",
    "-Xptxas", "-O3",
    "--expt-relaxed-constexpr",
]


def _nvcc() -> str:
    for cand in (shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError("nvcc not found")


def sources():
    return sorted(glob.glob(os.path.join(CSRC, "*.cu")) + glob.glob(os.path.join(CSRC, "*.cpp")))


def _inputs():
    return sources() + sorted(glob.glob(os.path.join(CSRC, "*.cuh"))) + \
        sorted(glob.glob(os.path.join(CSRC, "*.h"))) + [HEADER, __file__]


def stale() -> bool:
    if not os.path.exists(LIB_PATH):
        return True
    built = os.path.getmtime(LIB_PATH)
    return any(os.path.getmtime(p) > built for p in _inputs())


def _compile(src: str, extra, verbose: bool) -> str:
    obj = os.path.join(BUILD_DIR, os.path.splitext(os.path.basename(src))[0] + ".o")
    cmd = [_nvcc(), *NVCC_FLAGS, *extra, "-c", "-o", obj, src]
    if verbose:
        print(" ".join(cmd), flush=True)
    subprocess.run(cmd, check=True)
    return obj


def build(force: bool = False, verbose: bool = False, extra=()) -> str:
    """Compile the library when it is missing or older than its sources; return its path.

    Every ``.cu`` is compiled to its own object in parallel (each is a whole-program device unit: no
    device code crosses files), then nvcc links them into the shared library."""
    if not (force or stale()):
        return LIB_PATH
    from concurrent.futures import ThreadPoolExecutor
    os.makedirs(BUILD_DIR, exist_ok=True)
    srcs = sources()
    with ThreadPoolExecutor(max_workers=max(1, min(len(srcs), os.cpu_count() or 1))) as pool:
        objs = list(pool.map(lambda s: _compile(s, extra, verbose), srcs))
    tmp = LIB_PATH + ".tmp"
    cmd = [_nvcc(), "-gencode", "arch=compute_100a,code=sm_100a", "-shared", "-o", tmp, *objs, "-lcuda", "-ldl"]
    if verbose:
        print(" ".join(cmd), flush=True)
    subprocess.run(cmd, check=True)
    os.replace(tmp, LIB_PATH)
    return LIB_PATH


if __name__ == "__main__":
    print(build(force="--force" in sys.argv, verbose=True,
                extra=(["-Xptxas", "-v"] if "--ptxas-v" in sys.argv else [])))
