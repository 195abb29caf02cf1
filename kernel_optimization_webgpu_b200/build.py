"""Build recipe for the in-tree CUDA library (libqdecode.so, sm_100a).

The library is compiled with nvcc directly (no torch extension machinery): it is
a plain C-ABI shared object that JavaScript, C or Python can load.
"""
from __future__ import annotations

import os
import shutil
import subprocess
import sys

PKG = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(PKG)
CSRC = os.path.join(PKG, "csrc")
LIB = os.path.join(PKG, "libqdecode.so")
SOURCES = ["engine.cu", "noalloc.cu"]
DEPS = ["engine.cu", "noalloc.cu", "kernels.cuh", "persist.cuh", "gemm_tc.cuh", "common.cuh", "json.hpp"]
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]


def nvcc() -> str:
    for cand in (shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError("nvcc not found")


def _stale() -> bool:
    if not os.path.exists(LIB):
        return True
    t = os.path.getmtime(LIB)
    paths = [os.path.join(CSRC, d) for d in DEPS] + [os.path.join(ROOT, "include", "qdecode.h")]
    return any(os.path.getmtime(p) > t for p in paths)


def build(force: bool = False, verbose: bool = False) -> str:
    if not force and not _stale():
        return LIB
    cmd = [nvcc(), "-O3", "-std=c++17", *ARCH, "-lineinfo", "-Xcompiler", "-fPIC,-O3", "-shared",
           "-I", os.path.join(ROOT, "include"), "-o", LIB + ".tmp"]
    if verbose:
        cmd += ["-Xptxas", "-v"]
    cmd += [os.path.join(CSRC, s) for s in SOURCES]
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        sys.stderr.write(res.stdout + res.stderr)
        raise RuntimeError("nvcc failed building libqdecode.so")
    if verbose:
        sys.stderr.write(res.stderr)
    os.replace(LIB + ".tmp", LIB)
    return LIB


if __name__ == "__main__":
    build(force="--force" in sys.argv, verbose="-v" in sys.argv)
    print(LIB)
