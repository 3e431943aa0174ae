"""Builds librt_b200.so (the C ABI of include/rt_b200.h) from csrc/*.cu for sm_100a, in tree.

    python intel-phi-apl_b200/build.py [--force] [--verbose]

One nvcc invocation per source (objects under _build/, skipped when newer than their inputs),
then one shared-library link. The library goes next to this file so it travels with the
repository snapshot to a GPU host. Then libengine_rounds.so: engine_rounds.c, a caller of that
C ABI (rounds run as the reference engine runs them; bench.py's end-to-end timing), built with
the host C compiler and linked against librt_b200.so.
"""
from __future__ import annotations

import argparse
import glob
import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
CSRC = os.path.join(HERE, "csrc")
BUILD = os.path.join(HERE, "_build")
LIB = os.path.join(HERE, "librt_b200.so")
NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
FLAGS = ["-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC", "-Xcompiler", "-fvisibility=hidden",
         "--expt-relaxed-constexpr", "-I", os.path.join(ROOT, "include"), "-I", CSRC]
# The exact products depend on IEEE fp32 fma and division: no fast-math, no flush-to-zero.
FLAGS += ["-fmad=true", "-ftz=false", "-prec-div=true", "-prec-sqrt=true"]
LIBS = ["-lcudart", "-ldl"]  # NCCL is opened at run time, on first use
ENGINE_SRC = os.path.join(HERE, "engine_rounds.c")
ENGINE_LIB = os.path.join(HERE, "libengine_rounds.so")
CC = os.environ.get("CC", "gcc")


def _newer(target: str, deps: list[str]) -> bool:
    if not os.path.exists(target):
        return False
    t = os.path.getmtime(target)
    return all(os.path.getmtime(d) <= t for d in deps)


def build(force: bool = False, verbose: bool = False) -> str:
    os.makedirs(BUILD, exist_ok=True)
    sources = sorted(glob.glob(os.path.join(CSRC, "*.cu")))
    headers = sorted(glob.glob(os.path.join(CSRC, "*.h")) + glob.glob(os.path.join(CSRC, "*.cuh"))
                     + glob.glob(os.path.join(ROOT, "include", "*.h")))
    objects = []
    for src in sources:
        obj = os.path.join(BUILD, os.path.basename(src)[:-3] + ".o")
        objects.append(obj)
        if not force and _newer(obj, [src, *headers, __file__]):
            continue
        cmd = [NVCC, *ARCH, *FLAGS, "-c", src, "-o", obj]
        if verbose:
            cmd.insert(1, "-Xptxas=-v")
            print(" ".join(cmd), flush=True)
        subprocess.run(cmd, check=True)
    if force or not _newer(LIB, objects):
        cmd = [NVCC, *ARCH, "-shared", "-o", LIB, *objects, *LIBS]
        if verbose:
            print(" ".join(cmd), flush=True)
        subprocess.run(cmd, check=True)
    if force or not _newer(ENGINE_LIB, [ENGINE_SRC, LIB, os.path.join(ROOT, "include", "rt_b200.h"), __file__]):
        cmd = [CC, "-std=gnu11", "-O2", "-Wall", "-Wextra", "-Werror", "-fPIC", "-shared", "-I", os.path.join(ROOT, "include"),
               "-o", ENGINE_LIB, ENGINE_SRC, "-L", HERE, "-lrt_b200", "-Wl,-rpath,$ORIGIN"]
        if verbose:
            print(" ".join(cmd), flush=True)
        subprocess.run(cmd, check=True)
    return LIB


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--verbose", action="store_true")
    a = ap.parse_args()
    print(build(force=a.force, verbose=a.verbose))
    sys.exit(0)
