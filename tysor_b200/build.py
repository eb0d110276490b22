"""Builds libtysor_cuda.so in-tree for sm_100a.

    python -m tysor_b200.build        (or __graft_entry__.build())

Each csrc/*.cu is compiled with nvcc for `-gencode arch=compute_100a,
code=sm_100a` and linked into tysor_b200/libtysor_cuda.so (static CUDA
runtime; the driver API is reached through cudaGetDriverEntryPoint and NCCL
through dlopen, so the library has no link-time dependency on either).
ops.cu is compiled with --fmad=false so its f32 arithmetic rounds every
product and sum separately, like the reference.
"""
from __future__ import annotations

import os
import shutil
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(HERE, "csrc")
BUILD = os.path.join(HERE, "_build")
LIB = os.path.join(HERE, "libtysor_cuda.so")

SOURCES = ["gemm.cu", "ops.cu", "bridge.cu", "executor.cu", "comm.cu", "noalloc.cu"]
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
COMMON = ["-O3", "-std=c++20", "-lineinfo", "-Xcompiler", "-fPIC", "-Xcompiler", "-ffp-contract=off",
          "--expt-relaxed-constexpr", "-I" + os.path.join(os.path.dirname(HERE), "include")]
PER_FILE = {"ops.cu": ["--fmad=false"]}


def nvcc() -> str:
    for cand in (os.environ.get("NVCC"), "/usr/local/cuda/bin/nvcc", shutil.which("nvcc")):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError("nvcc not found")


def _stale(target: str, deps) -> bool:
    if not os.path.exists(target):
        return True
    t = os.path.getmtime(target)
    return any(os.path.getmtime(d) > t for d in deps)


def build(verbose: bool = False, force: bool = False) -> str:
    os.makedirs(BUILD, exist_ok=True)
    headers = [os.path.join(CSRC, f) for f in os.listdir(CSRC) if f.endswith(".cuh")]
    headers.append(os.path.join(os.path.dirname(HERE), "include", "tysor_cuda.h"))
    objs = []
    for src in SOURCES:
        path = os.path.join(CSRC, src)
        obj = os.path.join(BUILD, src.replace(".cu", ".o"))
        objs.append(obj)
        if force or _stale(obj, [path] + headers):
            cmd = [nvcc()] + ARCH + COMMON + PER_FILE.get(src, []) + ["-c", path, "-o", obj]
            if verbose:
                print(" ".join(cmd), flush=True)
            subprocess.run(cmd, check=True)
    if force or _stale(LIB, objs):
        cmd = [nvcc()] + ARCH + ["-shared", "-o", LIB] + objs + ["-ldl", "-lpthread"]
        if verbose:
            print(" ".join(cmd), flush=True)
        subprocess.run(cmd, check=True)
    return LIB


if __name__ == "__main__":
    build(verbose=True, force="--force" in sys.argv)
    print(LIB)
