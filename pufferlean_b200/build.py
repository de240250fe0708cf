"""Builds the CUDA library in-tree: pufferlean_b200/_build/libpufferlean_b200.so (and the Lean
adapter libpufferlean_lean.so). sm_100a only; nvcc links the CUDA runtime statically, so the
library does not depend on which libcudart another package in the process loaded.

    python -m pufferlean_b200.build [--clean] [-j N]
"""
from __future__ import annotations

import argparse
import concurrent.futures as cf
import glob
import os
import shutil
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
CSRC = os.path.join(HERE, "csrc")
BUILD = os.path.join(HERE, "_build")
NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
CUFLAGS = ["-std=c++17", "-O3", "-lineinfo", "-Xcompiler", "-fPIC,-ffp-contract=off", "-I" + os.path.join(ROOT, "include")]
CXXFLAGS = ["-std=c++17", "-O2", "-fPIC", "-ffp-contract=off", "-I" + os.path.join(ROOT, "include"),
            "-I/usr/local/cuda/include"]
LIB = os.path.join(BUILD, "libpufferlean_b200.so")
LEAN_LIB = os.path.join(BUILD, "libpufferlean_lean.so")


def _compile(src: str, verbose: bool) -> str:
    obj = os.path.join(BUILD, os.path.basename(src) + ".o")
    if os.path.exists(obj) and os.path.getmtime(obj) >= max(
            [os.path.getmtime(src)] + [os.path.getmtime(h) for h in glob.glob(os.path.join(CSRC, "*.cuh"))
                                       + glob.glob(os.path.join(CSRC, "*.h"))
                                       + glob.glob(os.path.join(ROOT, "include", "*.h"))]):
        return obj
    if src.endswith(".cu"):
        cmd = [NVCC] + ARCH + CUFLAGS + ["-c", src, "-o", obj]
    else:
        cmd = ["g++"] + CXXFLAGS + ["-c", src, "-o", obj]
    if verbose:
        print(" ".join(cmd), flush=True)
    subprocess.check_call(cmd)
    return obj


def build(jobs: int | None = None, verbose: bool = False) -> str:
    os.makedirs(BUILD, exist_ok=True)
    srcs = sorted(glob.glob(os.path.join(CSRC, "*.cu")) + glob.glob(os.path.join(CSRC, "*.cpp")))
    srcs = [s for s in srcs if not os.path.basename(s).startswith("pl_lean")]
    with cf.ThreadPoolExecutor(max_workers=jobs or os.cpu_count() or 4) as ex:
        objs = list(ex.map(lambda s: _compile(s, verbose), srcs))
    newest = max(os.path.getmtime(o) for o in objs)
    if not os.path.exists(LIB) or os.path.getmtime(LIB) < newest:
        cmd = [NVCC] + ARCH + ["-shared", "-o", LIB] + objs + ["-lpthread", "-ldl"]
        if verbose:
            print(" ".join(cmd), flush=True)
        subprocess.check_call(cmd)
    lean_src = os.path.join(CSRC, "pl_lean_abi.c")
    if os.path.exists(lean_src):
        if not os.path.exists(LEAN_LIB) or os.path.getmtime(LEAN_LIB) < max(os.path.getmtime(lean_src),
                                                                             os.path.getmtime(LIB)):
            cmd = ["gcc", "-std=gnu11", "-O2", "-fPIC", "-shared", "-o", LEAN_LIB, lean_src,
                   "-I" + os.path.join(ROOT, "include"), "-I" + os.path.join(ROOT, "include", "lean_compat"),
                   "-L" + BUILD, "-lpufferlean_b200", "-Wl,-rpath,$ORIGIN"]
            if verbose:
                print(" ".join(cmd), flush=True)
            subprocess.check_call(cmd)
    return LIB


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--clean", action="store_true")
    ap.add_argument("-j", type=int, default=None)
    ap.add_argument("-v", action="store_true")
    a = ap.parse_args()
    if a.clean and os.path.isdir(BUILD):
        shutil.rmtree(BUILD)
    print(build(a.j, a.v))


if __name__ == "__main__":
    sys.exit(main())
