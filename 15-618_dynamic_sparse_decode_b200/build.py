"""Build recipe for the sm_100a library (run from any directory).

    python 15-618_dynamic_sparse_decode_b200/build.py

produces, in this package directory:
    libdsd_b200.so        the C ABI (include/dsd_b200.h) + CUDA kernels
"""
from __future__ import annotations

import os
import subprocess
import sys

PKG = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(PKG)
CSRC = os.path.join(PKG, "csrc")
INCLUDE = os.path.join(ROOT, "include")
NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
LIB = os.path.join(PKG, "libdsd_b200.so")

SOURCES = ["dsd_capi.cu"]
HEADERS = ["dsd_kernels.cuh"]


def _newer(target: str, deps: list[str]) -> bool:
    if not os.path.exists(target):
        return False
    t = os.path.getmtime(target)
    return all(os.path.getmtime(d) <= t for d in deps)


def build_library(force: bool = False, verbose: bool = False) -> str:
    deps = [os.path.join(CSRC, s) for s in SOURCES + HEADERS] + [os.path.join(INCLUDE, "dsd_b200.h")]
    if not force and _newer(LIB, deps):
        return LIB
    cmd = [NVCC, *ARCH, "-lineinfo", "-O3", "-std=c++17", "-Xcompiler", "-fPIC", "-shared",
           f"-I{INCLUDE}", f"-I{CSRC}", "-o", LIB, *[os.path.join(CSRC, s) for s in SOURCES]]
    if verbose:
        cmd.insert(1, "-Xptxas=-v")
        print(" ".join(cmd))
    subprocess.run(cmd, check=True)
    return LIB


def build(force: bool = False, verbose: bool = False) -> None:
    build_library(force=force, verbose=verbose)


if __name__ == "__main__":
    build(force="--force" in sys.argv, verbose="-v" in sys.argv)
