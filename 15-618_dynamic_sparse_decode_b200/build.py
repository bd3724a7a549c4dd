"""Build recipe for the sm_100a library (run from any directory).

    python 15-618_dynamic_sparse_decode_b200/build.py

produces, in this package directory:
    libdsd_b200.so        the C ABI (include/dsd_b200.h) + CUDA kernels
    libdsd_host.so        the drop-in C++ API (include/dsd/*.h) over the C ABI
    bin/dsd_bench, bin/dsd_continuous_bench   the drop-in CLIs
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


def build_library(force: bool = False, verbose: bool = False, out: str = LIB,
                  defines: tuple = ()) -> str:
    """nvcc the C ABI + kernels into `out` (extra -D `defines` for experiments)."""
    deps = [os.path.join(CSRC, s) for s in SOURCES + HEADERS] + [os.path.join(INCLUDE, "dsd_b200.h")]
    if not force and _newer(out, deps):
        return out
    cmd = [NVCC, *ARCH, "-lineinfo", "-O3", "-std=c++17", "-Xcompiler", "-fPIC", "-shared",
           *[f"-D{d}" for d in defines],
           f"-I{INCLUDE}", f"-I{CSRC}", "-o", out, *[os.path.join(CSRC, s) for s in SOURCES]]
    if verbose:
        cmd.insert(1, "-Xptxas=-v")
        print(" ".join(cmd))
    subprocess.run(cmd, check=True)
    return out


HOST_DIR = os.path.join(CSRC, "host")
HOST_SOURCES = ["page_pool.cpp", "paged_kv_cache.cpp", "reference_kernels.cpp",
                "synthetic_data.cpp", "device_page_pool.cpp", "sparse_cuda_context.cpp",
                "decode_pipeline.cpp", "continuous_batching.cpp", "dense_stub.cpp"]
HOST_LIB = os.path.join(PKG, "libdsd_host.so")
BIN = os.path.join(PKG, "bin")
CLIS = {"dsd_bench": "bench_decode_main.cpp", "dsd_continuous_bench": "bench_continuous_main.cpp"}
CXX = os.environ.get("CXX", "g++")
# -ffp-contract=off: the CPU backends keep the reference's unfused arithmetic
CXXFLAGS = ["-O3", "-std=c++17", "-fPIC", "-ffp-contract=off", "-Wall", "-Wextra",
            f"-I{INCLUDE}", f"-I{HOST_DIR}"]


def build_host(force: bool = False) -> None:
    headers = [os.path.join(INCLUDE, "dsd", h) for h in os.listdir(os.path.join(INCLUDE, "dsd"))]
    headers += [os.path.join(HOST_DIR, h) for h in os.listdir(HOST_DIR) if h.endswith(".h")]
    headers += [os.path.join(INCLUDE, "dsd_b200.h")]
    srcs = [os.path.join(HOST_DIR, s) for s in HOST_SOURCES]
    if force or not _newer(HOST_LIB, srcs + headers + [LIB]):
        subprocess.run([CXX, *CXXFLAGS, "-shared", "-o", HOST_LIB, *srcs, f"-L{PKG}",
                        "-ldsd_b200", "-Wl,-rpath,$ORIGIN"], check=True)
    os.makedirs(BIN, exist_ok=True)
    for exe, src in CLIS.items():
        out = os.path.join(BIN, exe)
        s = os.path.join(HOST_DIR, src)
        if force or not _newer(out, [s, HOST_LIB] + headers):
            subprocess.run([CXX, *CXXFLAGS, "-o", out, s, f"-L{PKG}", "-ldsd_host", "-ldsd_b200",
                            "-Wl,-rpath,$ORIGIN/.."], check=True)


def build(force: bool = False, verbose: bool = False) -> None:
    build_library(force=force, verbose=verbose)
    build_host(force=force)


if __name__ == "__main__":
    build(force="--force" in sys.argv, verbose="-v" in sys.argv)
