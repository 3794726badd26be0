"""Builds the sm_100a artefacts in-tree (no JIT cache):

  cudair/libcudair_b200.so    the C-ABI library (include/cudair_b200.h)
  cudair/cudair_kernels.cubin the loadable module with the reference's
                              kernel names (MatMul16, VecAdd, ReduceF32)

Run `python cuda-ir.go_b200/build.py` (or __graft_entry__.build()).  nvcc
cross-compiles for sm_100a, so no GPU is needed to build.
"""
from __future__ import annotations

import glob
import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(HERE, "csrc")
OUT = os.path.join(HERE, "cudair")
REPO = os.path.dirname(HERE)
NVCC = os.environ.get("NVCC", "nvcc")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
COMMON = ARCH + ["-O3", "-std=c++17", "-lineinfo", "-I" + os.path.join(REPO, "include"),
                 "-Xcompiler", "-fPIC,-fvisibility=hidden,-Wall"]

LIB = os.path.join(OUT, "libcudair_b200.so")
CUBIN = os.path.join(OUT, "cudair_kernels.cubin")


def _sources():
    return sorted(glob.glob(os.path.join(CSRC, "*.cu")) + glob.glob(os.path.join(CSRC, "*.cpp")))


def _lib_sources():
    return [s for s in _sources() if os.path.basename(s) != "module.cu"]


def _stale(target, deps):
    if not os.path.exists(target):
        return True
    t = os.path.getmtime(target)
    return any(os.path.getmtime(d) > t for d in deps)


def _deps():
    return (_sources() + glob.glob(os.path.join(CSRC, "*.cuh")) + glob.glob(os.path.join(CSRC, "*.h"))
            + glob.glob(os.path.join(REPO, "include", "*.h")))


def _run(cmd, verbose):
    if verbose:
        print(" ".join(cmd), flush=True)
    subprocess.run(cmd, check=True)


def build(force: bool = False, verbose: bool = True, ptxas_info: bool = False) -> dict:
    os.makedirs(OUT, exist_ok=True)
    deps = _deps()
    extra = ["-Xptxas", "-v"] if ptxas_info else []
    if force or _stale(LIB, deps):
        objs = []
        objdir = os.path.join(HERE, "_build")
        os.makedirs(objdir, exist_ok=True)
        for src in _lib_sources():
            obj = os.path.join(objdir, os.path.basename(src) + ".o")
            _run([NVCC] + COMMON + extra + ["-c", src, "-o", obj], verbose)
            objs.append(obj)
        _run([NVCC] + ARCH + ["-shared", "-o", LIB] + objs + ["-ldl", "-lpthread"], verbose)
    if force or _stale(CUBIN, deps):
        _run([NVCC] + COMMON + extra + ["-cubin", os.path.join(CSRC, "module.cu"), "-o", CUBIN], verbose)
    return {"lib": LIB, "cubin": CUBIN}


if __name__ == "__main__":
    print(build(force="--force" in sys.argv, ptxas_info="--ptxas-info" in sys.argv))
