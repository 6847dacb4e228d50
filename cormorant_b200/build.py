"""Build libcorm_b200.so in-tree: nvcc for sm_100a (cross-compiles without a
GPU) plus g++ for the host table builders.

    python -m cormorant_b200.build [--force] [--verbose]
"""
from __future__ import annotations

import argparse
import os
import shutil
import subprocess
import sys
from concurrent.futures import ThreadPoolExecutor

PKG = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(PKG)
CSRC = os.path.join(PKG, "csrc")
INCLUDE = os.path.join(ROOT, "include")
BUILD = os.path.join(PKG, "_build")
LIB = os.path.join(PKG, "libcorm_b200.so")

CU_SOURCES = ["capi.cu", "vectorop.cu", "pool.cu", "rowops.cu", "gemm_i8x4.cu", "matmul.cu", "conv.cu", "strided.cu", "llm.cu", "llm_host.cu"]
CPP_SOURCES = ["tables.cpp"]
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]


def nvcc() -> str:
    for cand in (shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError("nvcc not found")


def _newest_input() -> float:
    t = os.path.getmtime(os.path.join(INCLUDE, "cormorant_b200.h"))
    for f in os.listdir(CSRC):
        t = max(t, os.path.getmtime(os.path.join(CSRC, f)))
    return max(t, os.path.getmtime(__file__))


def _run(cmd, verbose):
    if verbose:
        print(" ".join(cmd), flush=True)
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"build failed: {' '.join(cmd)}\n{r.stdout}\n{r.stderr}")
    return r.stdout + r.stderr


def build(force: bool = False, verbose: bool = False, ptxas_verbose: bool = False) -> str:
    """Compile every source and link the shared library; returns its path.
    Skips the work when the library is newer than every input."""
    if not force and os.path.exists(LIB) and os.path.getmtime(LIB) >= _newest_input():
        return LIB
    os.makedirs(BUILD, exist_ok=True)
    nv = nvcc()
    common = ["-O3", "-std=c++17", "-I", INCLUDE, "-I", CSRC]
    jobs = []
    for s in CU_SOURCES:
        obj = os.path.join(BUILD, s + ".o")
        cmd = [nv, *ARCH, *common, "-lineinfo", "-Xcompiler", "-fPIC", "-Xcompiler", "-ffp-contract=off",
               "--expt-relaxed-constexpr", "-c", os.path.join(CSRC, s), "-o", obj]
        if ptxas_verbose:
            cmd += ["-Xptxas", "-v"]
        jobs.append((cmd, obj))
    for s in CPP_SOURCES:
        obj = os.path.join(BUILD, s + ".o")
        cmd = ["g++", "-O2", "-std=c++17", "-fPIC", "-ffp-contract=off", "-fno-fast-math", "-I", INCLUDE, "-I", CSRC,
               "-c", os.path.join(CSRC, s), "-o", obj]
        jobs.append((cmd, obj))
    with ThreadPoolExecutor(max_workers=min(8, os.cpu_count() or 4)) as ex:
        outs = list(ex.map(lambda j: _run(j[0], verbose), jobs))
    if ptxas_verbose:
        for o in outs:
            if o.strip():
                print(o)
    tmp = LIB + ".tmp"
    _run([nv, *ARCH, "-shared", "-o", tmp, *[o for _, o in jobs], "-Xcompiler", "-fPIC"], verbose)
    os.replace(tmp, LIB)
    return LIB


def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--verbose", action="store_true")
    ap.add_argument("--ptxas", action="store_true", help="print -Xptxas -v register / smem usage")
    a = ap.parse_args(argv)
    print(build(force=a.force, verbose=a.verbose, ptxas_verbose=a.ptxas))


if __name__ == "__main__":
    sys.exit(main())
