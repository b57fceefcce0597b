"""Builds the in-tree CUDA library libmomiru_gemm.so for sm_100a with nvcc.

Each translation unit compiles to an object in parallel (the tcgen05 kernel
families are split over four units), then nvcc links the shared library.
"""
from __future__ import annotations

import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(HERE, "csrc")
LIB_DIR = os.path.join(HERE, "lib")
LIB_PATH = os.path.join(LIB_DIR, "libmomiru_gemm.so")
SOURCES = ["momiru_gemm.cu", "tc_strict_pair.cu", "tc_tf32_pair.cu", "tc_strict_1cta.cu", "tc_tf32_1cta.cu"]
HEADERS = ["ptx.cuh", "epilogue.cuh", "tc_gemm.cuh", "tc_gemm_2sm.cuh", "simt_gemm.cuh", "gemv.cuh", "gemv_tc.cuh", "fixup.cuh",
           "tc_launch.h", "tc_launch.cuh", "launch.cuh"]
OBJ_DIR = os.path.join(LIB_DIR, "obj")
NVCC_FLAGS = [
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-O3", "-lineinfo", "-std=c++17",
    "-ftz=false", "-prec-div=true", "-prec-sqrt=true", "-fmad=true",
    "-Xcompiler", "-fPIC", "-Xcompiler", "-fvisibility=hidden",
    "-Xcompiler", "-Wall",
    "--expt-relaxed-constexpr",
]


def _nvcc() -> str:
    cand = os.path.join(os.environ.get("CUDA_HOME", "/usr/local/cuda"), "bin", "nvcc")
    return cand if os.path.exists(cand) else "nvcc"


def _stale() -> bool:
    if not os.path.exists(LIB_PATH):
        return True
    t = os.path.getmtime(LIB_PATH)
    deps = [os.path.join(CSRC, f) for f in SOURCES + HEADERS]
    deps.append(os.path.join(HERE, "..", "include", "momiru_gemm.h"))
    return any(os.path.getmtime(d) > t for d in deps if os.path.exists(d))


def build(force: bool = False, verbose: bool = False, extra: list[str] | None = None) -> str:
    if not force and not _stale():
        return LIB_PATH
    os.makedirs(OBJ_DIR, exist_ok=True)
    headers = [os.path.join(CSRC, f) for f in HEADERS] + [os.path.join(HERE, "..", "include", "momiru_gemm.h")]
    newest_header = max(os.path.getmtime(h) for h in headers if os.path.exists(h))
    objs, jobs = [], []
    for src in SOURCES:
        obj = os.path.join(OBJ_DIR, os.path.splitext(src)[0] + ".o")
        objs.append(obj)
        path = os.path.join(CSRC, src)
        # an object is rebuilt when forced, missing, or older than its unit or any header
        if not force and os.path.exists(obj) and os.path.getmtime(obj) >= max(os.path.getmtime(path), newest_header):
            continue
        cmd = [_nvcc(), *NVCC_FLAGS, *(extra or []), "-c", "-o", obj, path]
        if verbose:
            print(" ".join(cmd), file=sys.stderr)
        jobs.append((obj, subprocess.Popen(cmd)))
    failed = [obj for obj, proc in jobs if proc.wait() != 0]
    if failed:
        raise subprocess.CalledProcessError(1, f"nvcc ({', '.join(os.path.basename(f) for f in failed)})")
    link = [_nvcc(), "-gencode", "arch=compute_100a,code=sm_100a", "-shared", "-o", LIB_PATH, *objs]
    if verbose:
        print(" ".join(link), file=sys.stderr)
    subprocess.run(link, check=True)
    return LIB_PATH


if __name__ == "__main__":
    build(force="--force" in sys.argv, verbose=True,
          extra=["-Xptxas", "-v"] if "--ptxas-v" in sys.argv else None)
    print(LIB_PATH)
