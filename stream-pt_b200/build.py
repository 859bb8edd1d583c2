"""Build the sm_100a shared library ``libspt_moe.so`` in-tree with nvcc.

Usage: ``python stream-pt_b200/build.py`` (no GPU needed; nvcc cross-compiles).
"""
from __future__ import annotations

import os
import shutil
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(HERE, "csrc")
OUT = os.path.join(HERE, "libspt_moe.so")
BUILD = os.path.join(HERE, "_build")

SOURCES = ["spt_kernels.cu", "spt_mma.cu", "spt_gemv16.cu", "spt_q80.cu", "spt_q40.cu", "spt_gguf.cpp", "spt_api.cu"]

NVCC_FLAGS = [
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-lineinfo", "-O3", "-std=c++17",
    # every fused multiply-add in the kernels is written explicitly; nothing
    # else may be contracted, so results round like the reference
    "-fmad=false",
    "-Xcompiler", "-fPIC", "-Xcompiler", "-Wall",
]


def nvcc() -> str:
    for cand in (os.environ.get("NVCC"), "/usr/local/cuda/bin/nvcc", shutil.which("nvcc")):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError("nvcc not found")


def _stale(target: str, deps: list[str]) -> bool:
    if not os.path.exists(target):
        return True
    t = os.path.getmtime(target)
    return any(os.path.getmtime(d) > t for d in deps)


def build(verbose: bool = False, force: bool = False) -> str:
    os.makedirs(BUILD, exist_ok=True)
    headers = [os.path.join(CSRC, f) for f in os.listdir(CSRC) if f.endswith((".h", ".cuh"))]
    headers.append(os.path.join(HERE, "..", "include", "spt_moe.h"))
    objs = []
    for src in SOURCES:
        s = os.path.join(CSRC, src)
        o = os.path.join(BUILD, os.path.splitext(src)[0] + ".o")
        objs.append(o)
        if force or _stale(o, [s] + headers):
            cmd = [nvcc(), *NVCC_FLAGS, "-c", s, "-o", o]
            if verbose:
                cmd.insert(1, "-Xptxas=-v")
                print(" ".join(cmd), flush=True)
            subprocess.run(cmd, check=True)
    if force or _stale(OUT, objs):
        cmd = [nvcc(), "-gencode", "arch=compute_100a,code=sm_100a", "-shared",
               "-Xcompiler", "-fPIC", "-o", OUT, *objs, "-lcudart_static", "-lrt", "-ldl", "-lpthread"]
        subprocess.run(cmd, check=True)
    return OUT


if __name__ == "__main__":
    build(verbose="-v" in sys.argv, force="-f" in sys.argv)
    print(OUT)
