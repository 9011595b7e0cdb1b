"""Build recipe for the CPU oracle (test infrastructure, never the product path).

``build_oracle()`` compiles ``satori_oracle.c`` into ``oracle/_build/libsatori_oracle.so``
with gcc.  The flags matter for parity: ``-ffp-contract=off`` keeps every FP32 multiply and
add separately rounded exactly as the C# reference computes them, and the explicit FMA calls
in the source stand for the reference's ``Fma.MultiplyAdd``.  ``-mavx2 -mfma`` lets the
intrinsic restatements of the reference's AVX2 kernels compile; ``-fopenmp`` provides the
all-cores row split used for the timed CPU baseline.

The reference itself (C#/.NET) cannot be compiled in this image, so there is no
``oracle/_ref`` build; the restatement is pinned against the reference's golden vectors
instead (tests/test_oracle_golden.py).
"""
from __future__ import annotations

import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
BUILD_DIR = os.path.join(HERE, "_build")
LIB_PATH = os.path.join(BUILD_DIR, "libsatori_oracle.so")
SOURCES = [os.path.join(HERE, "satori_oracle.c")]
HEADERS = [os.path.join(HERE, "satori_oracle.h")]

CFLAGS = ["-O2", "-std=gnu11", "-fPIC", "-shared", "-ffp-contract=off", "-fno-fast-math",
          "-mavx2", "-mfma", "-fopenmp", "-Wall", "-Wextra", "-Wno-unused-parameter"]


def _stale() -> bool:
    if not os.path.exists(LIB_PATH):
        return True
    built = os.path.getmtime(LIB_PATH)
    return any(os.path.getmtime(p) > built for p in SOURCES + HEADERS + [__file__])


def build_oracle(force: bool = False) -> str:
    """Compile the oracle if it is missing or older than its sources; return the .so path."""
    if force or _stale():
        os.makedirs(BUILD_DIR, exist_ok=True)
        tmp = LIB_PATH + ".tmp"
        cmd = ["gcc", *CFLAGS, "-o", tmp, *SOURCES, "-lm"]
        subprocess.run(cmd, check=True)
        os.replace(tmp, LIB_PATH)
    return LIB_PATH


if __name__ == "__main__":
    print(build_oracle(force="--force" in sys.argv))
