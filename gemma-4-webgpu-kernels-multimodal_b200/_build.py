"""Build the g4m CUDA library (libg4m.so) in-tree for sm_100a.

Usage: python _build.py [--jobs N]
Compiles every csrc/*.cu and csrc/*.cpp with nvcc (-gencode
arch=compute_100a,code=sm_100a) and links a shared library next to this
file.  Object files go to csrc/_build/.
"""
from __future__ import annotations

import argparse
import concurrent.futures as cf
import os
import shutil
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(HERE, "csrc")
OUT = os.path.join(HERE, "libg4m.so")
BUILD = os.path.join(CSRC, "_build")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
FLAGS = ["-O3", "-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC", "-Xcompiler", "-fvisibility=hidden",
         "--expt-relaxed-constexpr", "-DG4M_BUILD"]


def nvcc() -> str:
    for c in (os.environ.get("NVCC"), "/usr/local/cuda/bin/nvcc", shutil.which("nvcc")):
        if c and os.path.exists(c):
            return c
    raise RuntimeError("nvcc not found")


def sources():
    return sorted(os.path.join(CSRC, f) for f in os.listdir(CSRC) if f.endswith((".cu", ".cpp")))


def _stale(src: str, obj: str) -> bool:
    if not os.path.exists(obj):
        return True
    t = os.path.getmtime(obj)
    deps = [src] + [os.path.join(CSRC, h) for h in os.listdir(CSRC) if h.endswith((".h", ".cuh"))]
    deps.append(os.path.join(HERE, "..", "include", "g4m.h"))
    return any(os.path.getmtime(d) > t for d in deps if os.path.exists(d))


def compile_one(src: str, verbose: bool = False) -> str:
    obj = os.path.join(BUILD, os.path.basename(src) + ".o")
    if _stale(src, obj):
        cmd = [nvcc(), *ARCH, *FLAGS, "-c", src, "-o", obj]
        if verbose:
            print(" ".join(cmd), flush=True)
        subprocess.run(cmd, check=True)
    return obj


def build(jobs: int = 8, verbose: bool = False) -> str:
    os.makedirs(BUILD, exist_ok=True)
    with cf.ThreadPoolExecutor(max_workers=jobs) as ex:
        objs = list(ex.map(lambda s: compile_one(s, verbose), sources()))
    if not os.path.exists(OUT) or any(os.path.getmtime(o) > os.path.getmtime(OUT) for o in objs):
        cmd = [nvcc(), *ARCH, "-shared", "-o", OUT, *objs, "-lcudart_static", "-lrt", "-lpthread", "-ldl"]
        if verbose:
            print(" ".join(cmd), flush=True)
        subprocess.run(cmd, check=True)
    return OUT


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--jobs", type=int, default=8)
    ap.add_argument("-v", action="store_true")
    a = ap.parse_args()
    print(build(a.jobs, a.v))
