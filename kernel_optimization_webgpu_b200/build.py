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
SOURCES = ["engine.cu", "batch.cu", "noalloc.cu", "bench_api.cu", "sample.cu"]
DEPS = SOURCES + ["kernels.cuh", "persist.cuh", "gemm_tc.cuh", "batch.cuh", "internal.cuh", "tma.cuh", "common.cuh", "json.hpp"]
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
    obj_dir = os.path.join(PKG, "_build")
    os.makedirs(obj_dir, exist_ok=True)
    common = [nvcc(), "-O3", "-std=c++17", *ARCH, "-lineinfo", "-Xcompiler", "-fPIC,-O3",
              "-I", os.path.join(ROOT, "include")]
    if verbose:
        common += ["-Xptxas", "-v"]
    # one nvcc per translation unit, in parallel, then one link
    procs, objs = [], []
    for src in SOURCES:
        obj = os.path.join(obj_dir, src.replace(".cu", ".o"))
        objs.append(obj)
        procs.append((src, subprocess.Popen(common + ["-c", os.path.join(CSRC, src), "-o", obj],
                                            stdout=subprocess.PIPE, stderr=subprocess.PIPE, text=True)))
    failed = False
    for src, p in procs:
        out, err = p.communicate()
        if p.returncode != 0:
            sys.stderr.write(f"--- {src}\n" + out + err)
            failed = True
        elif verbose:
            sys.stderr.write(err)
    if failed:
        raise RuntimeError("nvcc failed building libqdecode.so")
    res = subprocess.run([nvcc(), *ARCH, "-shared", "-o", LIB + ".tmp", *objs], capture_output=True, text=True)
    if res.returncode != 0:
        sys.stderr.write(res.stdout + res.stderr)
        raise RuntimeError("nvcc failed linking libqdecode.so")
    os.replace(LIB + ".tmp", LIB)
    return LIB


if __name__ == "__main__":
    build(force="--force" in sys.argv, verbose="-v" in sys.argv)
    print(LIB)
