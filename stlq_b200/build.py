"""Builds libstlq_b200.so in-tree for sm_100a (nvcc; no JIT cache, so the library travels with the repo).

    python -m stlq_b200.build            # incremental
    python -m stlq_b200.build --force    # rebuild everything
"""
from __future__ import annotations

import os
import shutil
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(HERE, "csrc")
OUT = os.path.join(HERE, "libstlq_b200.so")
OBJDIR = os.path.join(HERE, "_build")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC = os.environ.get("NVCC", shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc")
HOST_CXX = "/usr/bin/g++" if os.path.exists("/usr/bin/g++") else "g++"
# No --use_fast_math: the kernels rely on IEEE division / square root and on denormals, like
# the reference's host build.
NVFLAGS = ["-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC", "-ccbin", HOST_CXX, "--expt-relaxed-constexpr"]


def sources():
    return sorted(f for f in os.listdir(CSRC) if f.endswith((".cu", ".cpp")))


def _stale(obj, deps):
    if not os.path.exists(obj):
        return True
    t = os.path.getmtime(obj)
    return any(os.path.getmtime(d) > t for d in deps)


def build(force: bool = False, verbose: bool = False) -> str:
    os.makedirs(OBJDIR, exist_ok=True)
    headers = [os.path.join(CSRC, f) for f in os.listdir(CSRC) if f.endswith((".h", ".cuh"))]
    headers.append(os.path.join(HERE, "..", "include", "stlq_b200.h"))
    objs = []
    for src in sources():
        path = os.path.join(CSRC, src)
        obj = os.path.join(OBJDIR, src + ".o")
        objs.append(obj)
        if force or _stale(obj, [path] + headers):
            cmd = [NVCC, *ARCH, *NVFLAGS, "-c", path, "-o", obj]
            if verbose:
                print(" ".join(cmd), flush=True)
            subprocess.run(cmd, check=True)
    if force or _stale(OUT, objs):
        cmd = [NVCC, *ARCH, "-shared", "-o", OUT, *objs, "-ccbin", HOST_CXX]
        if verbose:
            print(" ".join(cmd), flush=True)
        subprocess.run(cmd, check=True)
    return OUT


if __name__ == "__main__":
    build(force="--force" in sys.argv, verbose=True)
