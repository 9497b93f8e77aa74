"""Build libozaki_b200.so in-tree: every .cu of this directory compiled for sm_100a with nvcc, linked into one
shared library with a C ABI (include/ozaki_b200.h).  No torch extension: Python binds it with ctypes.

    python matrix-numbers_b200/csrc/build.py            # incremental
    python matrix-numbers_b200/csrc/build.py --force    # rebuild everything
"""
from __future__ import annotations

import os
import shutil
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
PKG = os.path.dirname(HERE)
ROOT = os.path.dirname(PKG)
OUT_DIR = os.path.join(PKG, "lib")
OBJ_DIR = os.path.join(ROOT, "_build", "ozaki_b200")
LIB = os.path.join(OUT_DIR, "libozaki_b200.so")

SOURCES = ["capi.cu", "stats.cu", "rule.cu", "split.cu", "split_tc.cu", "gemm_tc.cu", "recon.cu", "certificate.cu", "chain.cu"]
HEADERS = ["ozk_common.cuh", "tc_ptx.cuh"]


def nvcc() -> str:
    for cand in (os.environ.get("NVCC"), "/usr/local/cuda/bin/nvcc", shutil.which("nvcc")):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError("nvcc not found")


FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a", "-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC",
         "-Xcompiler", "-ffp-contract=off", "--expt-relaxed-constexpr", "-I", os.path.join(ROOT, "include")]


def _stale(target: str, deps) -> bool:
    if not os.path.exists(target):
        return True
    t = os.path.getmtime(target)
    return any(os.path.getmtime(d) > t for d in deps)


def build(force: bool = False, verbose: bool = False) -> str:
    os.makedirs(OUT_DIR, exist_ok=True)
    os.makedirs(OBJ_DIR, exist_ok=True)
    hdrs = [os.path.join(HERE, h) for h in HEADERS] + [os.path.join(ROOT, "include", "ozaki_b200.h")]
    objs = []
    for src in SOURCES:
        s = os.path.join(HERE, src)
        o = os.path.join(OBJ_DIR, src.replace(".cu", ".o"))
        objs.append(o)
        if force or _stale(o, [s] + hdrs):
            cmd = [nvcc()] + FLAGS + ["-c", s, "-o", o]
            if verbose:
                print(" ".join(cmd), flush=True)
            subprocess.run(cmd, check=True)
    if force or _stale(LIB, objs):
        cmd = [nvcc(), "-shared", "-gencode", "arch=compute_100a,code=sm_100a", "-o", LIB] + objs
        if verbose:
            print(" ".join(cmd), flush=True)
        subprocess.run(cmd, check=True)
    return LIB


if __name__ == "__main__":
    print(build(force="--force" in sys.argv, verbose=True))
