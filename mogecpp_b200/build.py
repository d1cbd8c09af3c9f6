"""Builds the sm_100a shared library of the sparse-voxel path in-tree.

Output: ``mogecpp_b200/libmoge_sparse_cuda.so`` (C ABI declared in
``include/moge_sparse_cuda.h``).  nvcc cross-compiles for sm_100a without a
GPU, so this runs on any machine with CUDA 12.9.

    python -m mogecpp_b200.build [--force] [--verbose]
"""

from __future__ import annotations

import argparse
import os
import subprocess
import sys

PKG = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(PKG)
CSRC = os.path.join(PKG, "csrc")
LIB = os.path.join(PKG, "libmoge_sparse_cuda.so")
SOURCES = ["topology.cu", "prep.cu", "gn.cu", "conv_tc.cu", "plan.cu", "ops.cu", "capi.cu",
           "noalloc.cu", "image_topo.cu", "refiner.cu", "slab.cu"]
HEADERS = ["common.cuh", "conv.h", "conv_common.cuh", "gn.h", "ops.h", "plan.h", "topology.h", "image_topo.h"]
NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")
FLAGS = ["-O3", "-std=c++17", "-gencode", "arch=compute_100a,code=sm_100a", "-lineinfo",
         "-Xcompiler", "-fPIC,-O3", "--expt-relaxed-constexpr", "-I", os.path.join(ROOT, "include")]


def _stale(out: str, deps: list[str]) -> bool:
    if not os.path.exists(out):
        return True
    t = os.path.getmtime(out)
    return any(os.path.getmtime(d) > t for d in deps)


def build(force: bool = False, verbose: bool = False, extra: list[str] | None = None) -> str:
    objdir = os.path.join(PKG, "_build")
    os.makedirs(objdir, exist_ok=True)
    hdrs = [os.path.join(CSRC, h) for h in HEADERS] + [os.path.join(ROOT, "include", "moge_sparse_cuda.h")]
    objs = []
    for src in SOURCES:
        s = os.path.join(CSRC, src)
        o = os.path.join(objdir, src + ".o")
        objs.append(o)
        if force or _stale(o, [s] + hdrs):
            cmd = [NVCC, *FLAGS, *(extra or []), "-c", s, "-o", o]
            if verbose:
                print(" ".join(cmd), flush=True)
            subprocess.run(cmd, check=True)
    if force or _stale(LIB, objs):
        cmd = [NVCC, "-shared", "-gencode", "arch=compute_100a,code=sm_100a", *objs, "-o", LIB]
        if verbose:
            print(" ".join(cmd), flush=True)
        subprocess.run(cmd, check=True)
    return LIB


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--verbose", action="store_true")
    ap.add_argument("--ptxas-v", action="store_true", help="print register / smem usage")
    a = ap.parse_args()
    path = build(a.force, a.verbose, ["-Xptxas", "-v"] if a.ptxas_v else None)
    print(path)
    sys.exit(0)
