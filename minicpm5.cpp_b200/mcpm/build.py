"""Builds the engine's shared library (libmcpm.so) in-tree with nvcc for sm_100a.

The library holds the CUDA kernels, the host engine and the C ABI of include/mcpm.h.
It is rebuilt when any source under csrc/ or include/ is newer than the library.
"""
from __future__ import annotations

import glob
import os
import subprocess
import sys

PKG = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))      # minicpm5.cpp_b200/
REPO = os.path.dirname(PKG)
CSRC = os.path.join(PKG, "csrc")
BUILD = os.path.join(PKG, "_build")
LIB = os.path.join(BUILD, "libmcpm.so")
NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
# No --use_fast_math: the kernels rely on IEEE division, square root and denormals.
NVCC_FLAGS = ["-O3", "-std=c++17", "-lineinfo", "--expt-relaxed-constexpr", "-Xcompiler", "-fPIC,-O2",
              "-Xptxas", "-warn-spills"]


def sources():
    return sorted(glob.glob(os.path.join(CSRC, "*.cu")) + glob.glob(os.path.join(CSRC, "*.cpp")))


def _stale() -> bool:
    if not os.path.exists(LIB):
        return True
    t = os.path.getmtime(LIB)
    deps = sources() + glob.glob(os.path.join(CSRC, "*.h")) + glob.glob(os.path.join(CSRC, "*.cuh")) \
        + glob.glob(os.path.join(REPO, "include", "*.h"))
    return any(os.path.getmtime(d) > t for d in deps)


def build(force: bool = False, verbose: bool = False) -> str:
    if not force and not _stale():
        return LIB
    os.makedirs(BUILD, exist_ok=True)
    objs = []
    for src in sources():
        obj = os.path.join(BUILD, os.path.basename(src) + ".o")
        cmd = [NVCC] + ARCH + NVCC_FLAGS + ["-I" + CSRC, "-I" + os.path.join(REPO, "include"), "-c", src, "-o", obj]
        if verbose:
            print(" ".join(cmd), file=sys.stderr)
        subprocess.run(cmd, check=True)
        objs.append(obj)
    tmp = LIB + ".tmp"
    subprocess.run([NVCC] + ARCH + ["-shared", "-o", tmp] + objs + ["-lcudart", "-ldl"], check=True)
    os.replace(tmp, LIB)
    return LIB


if __name__ == "__main__":
    print(build(force="--force" in sys.argv, verbose=True))
