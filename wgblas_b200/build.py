"""Builds libwgblas_b200.so (the C ABI of include/wgblas.h) in-tree with nvcc for sm_100a.

Usage: python wgblas_b200/build.py [--force] [-v]   (runs without importing the package)
"""
from __future__ import annotations

import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(HERE, "csrc")
ROOT = os.path.dirname(HERE)
LIB = os.path.join(HERE, "libwgblas_b200.so")
BUILD_DIR = os.path.join(HERE, "_build")

SOURCES = ["runtime.cu", "gemm.cu", "gemm_simt.cu", "sgemm_tf32x3.cu", "sgemm_fused.cu", "probe.cu", "sgemm_noalloc.cu", "dgemm_dmma.cu", "shard.cu", "level3_aux.cu", "trsm.cu", "gemv.cu"]
HEADERS = ["internal.h", "tcgen05.cuh", "tf32x3_common.cuh", "simt_tile.cuh"]

NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
FLAGS = ["-O3", "-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC,-ffp-contract=off",
         "--expt-relaxed-constexpr", "-I" + os.path.join(ROOT, "include")]


def _stale(target: str, deps) -> bool:
    if not os.path.exists(target):
        return True
    t = os.path.getmtime(target)
    return any(os.path.exists(d) and os.path.getmtime(d) > t for d in deps)


def build(force: bool = False, verbose: bool = False) -> str:
    os.makedirs(BUILD_DIR, exist_ok=True)
    headers = [os.path.join(CSRC, h) for h in HEADERS] + [os.path.join(ROOT, "include", "wgblas.h")]
    objs, jobs = [], []
    for src in SOURCES:
        path = os.path.join(CSRC, src)
        obj = os.path.join(BUILD_DIR, src.replace(".cu", ".o"))
        objs.append(obj)
        if force or _stale(obj, [path] + headers):
            cmd = [NVCC, *ARCH, *FLAGS, "-c", path, "-o", obj]
            if verbose:
                cmd.insert(1, "-Xptxas=-v")
            jobs.append(cmd)
    # The translation units compile independently: run them side by side.
    procs = [subprocess.Popen(cmd) for cmd in jobs]
    failed = [cmd for cmd, proc in zip(jobs, procs) if proc.wait() != 0]
    if failed:
        raise subprocess.CalledProcessError(1, failed[0])
    if force or _stale(LIB, objs):
        subprocess.run([NVCC, *ARCH, "-shared", "-o", LIB, *objs, "-ldl"], check=True)
    build_napi(force)
    return LIB


NAPI_SRC = os.path.join(HERE, "napi", "wgblas_napi.c")
NAPI_ADDON = os.path.join(HERE, "napi", "wgblas_napi.node")
CUDA_HOME = os.path.dirname(os.path.dirname(NVCC))


def napi_command(out: str) -> list[str]:
    """gcc command line of the Node-API addon (Node resolves its napi_* symbols at load)."""
    return ["gcc", "-std=c11", "-O2", "-Wall", "-Wextra", "-Werror", "-shared", "-fPIC", "-fvisibility=hidden",
            "-I" + os.path.join(ROOT, "include"), "-I" + os.path.join(CUDA_HOME, "include"), NAPI_SRC,
            "-L" + HERE, "-lwgblas_b200", "-L" + os.path.join(CUDA_HOME, "lib64"), "-lcudart",
            "-Wl,-rpath,$ORIGIN/..", "-o", out]


def build_napi(force: bool = False) -> str:
    """Builds wgblas_napi.node next to its source (the JavaScript shim in napi/js loads it)."""
    if force or _stale(NAPI_ADDON, [NAPI_SRC, LIB, os.path.join(ROOT, "include", "wgblas.h")]):
        subprocess.run(napi_command(NAPI_ADDON), check=True)
    return NAPI_ADDON


if __name__ == "__main__":
    build(force="--force" in sys.argv, verbose="-v" in sys.argv)
    print(LIB)
