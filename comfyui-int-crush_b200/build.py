"""Build libintcrush_b200.so in place (nvcc, sm_100a only).

Usage: ``python build.py`` from anywhere.  The library is written next to this
file so that it travels with the source tree; it links the CUDA runtime
statically and does not link libcuda (driver entry points are resolved at run
time), so it loads on hosts without a GPU driver.
"""
from __future__ import annotations

import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(HERE, "csrc")
LIB = os.path.join(HERE, "libintcrush_b200.so")
SOURCES = ["intcrush_b200.cu", "ic_common.cuh", "prep_common.cuh", "prep.cu", "prep_tile.cu", "gemm_tc.cu", "skinny.cu", "weights.cu", "abi.cu"]


def _nvcc() -> str:
    cand = os.path.join(os.environ.get("CUDA_HOME", "/usr/local/cuda"), "bin", "nvcc")
    return cand if os.path.exists(cand) else "nvcc"


def needs_build() -> bool:
    if not os.path.exists(LIB):
        return True
    t = os.path.getmtime(LIB)
    deps = [os.path.join(CSRC, s) for s in SOURCES]
    deps.append(os.path.join(HERE, "..", "include", "intcrush_b200.h"))
    return any(os.path.getmtime(d) > t for d in deps if os.path.exists(d))


def build(force: bool = False, verbose: bool = False) -> str:
    if not force and not needs_build():
        return LIB
    cmd = [
        _nvcc(), "-gencode", "arch=compute_100a,code=sm_100a", "-lineinfo", "-O3", "-std=c++17",
        "--shared", "-Xcompiler", "-fPIC", "-cudart", "static", "-diag-suppress", "20044",
        "-o", LIB + ".tmp", os.path.join(CSRC, "intcrush_b200.cu"),
    ]
    if verbose:
        cmd.insert(1, "-Xptxas=-v")
    subprocess.run(cmd, check=True)
    os.replace(LIB + ".tmp", LIB)
    return LIB


if __name__ == "__main__":
    build(force="--force" in sys.argv, verbose="-v" in sys.argv)
    print(LIB)
