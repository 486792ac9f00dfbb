"""Build the sm_100a C-ABI library `libslokv.so` in-tree with nvcc.

The library is a plain shared object (static CUDA runtime, no torch symbols):
the Python host code binds it with ctypes, and any other host language can bind
the same `extern "C"` entry points declared in include/slokv.h.

    python slo-aware-llm-serving-engine_b200/build.py [--force] [--verbose]
"""
from __future__ import annotations

import argparse
import os
import shutil
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
CSRC = os.path.join(HERE, "csrc")
LIB_NAME = "libslokv.so"
LIB_PATH = os.path.join(HERE, LIB_NAME)

SOURCES = [
    "kv_append.cu",
    "paged_decode.cu",
    "kv_block_copy.cu",
    "kv_append_fp8.cu",
    "paged_prefill.cu",
    "qk_norm_rope.cu",
    "fp8_pages_dequant.cu",
    "row_parallel.cu",
]
HEADERS = ["common.cuh", "fp8_e4m3.cuh", "tcgen05.cuh"]

ARCH_FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = [
    "-O3", "-std=c++17", "-lineinfo", "--expt-relaxed-constexpr",
    "-Xcompiler", "-fPIC", "-Xcompiler", "-Wall",
    "-cudart", "static",
]


def nvcc_path() -> str:
    cand = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not os.path.exists(cand):
        raise RuntimeError("nvcc not found; the CUDA toolkit is required to build libslokv.so")
    return cand


def _stale() -> bool:
    if not os.path.exists(LIB_PATH):
        return True
    built = os.path.getmtime(LIB_PATH)
    deps = [os.path.join(CSRC, s) for s in SOURCES + HEADERS]
    deps.append(os.path.join(ROOT, "include", "slokv.h"))
    deps.append(os.path.abspath(__file__))
    return any(os.path.getmtime(d) > built for d in deps if os.path.exists(d))


def build(force: bool = False, verbose: bool = False, ptxas_info: bool = False) -> str:
    """Compile every kernel for sm_100a into LIB_PATH; returns the path."""
    if not force and not ptxas_info and not _stale():
        return LIB_PATH
    tmp = LIB_PATH + ".tmp"
    cmd = [nvcc_path(), *ARCH_FLAGS, *NVCC_FLAGS, "-shared", "-o", tmp]
    if ptxas_info:
        cmd += ["-Xptxas", "-v"]
    cmd += [os.path.join(CSRC, s) for s in SOURCES]
    if verbose:
        print(" ".join(cmd), file=sys.stderr)
    res = subprocess.run(cmd, cwd=CSRC, capture_output=True, text=True)
    if verbose or ptxas_info or res.returncode != 0:
        sys.stderr.write(res.stdout)
        sys.stderr.write(res.stderr)
    if res.returncode != 0:
        raise RuntimeError(f"nvcc failed with exit code {res.returncode}")
    os.replace(tmp, LIB_PATH)
    return LIB_PATH


if __name__ == "__main__":
    ap = argparse.ArgumentParser(description=__doc__)
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--verbose", action="store_true")
    ap.add_argument("--ptxas-info", action="store_true", help="print registers/spills per kernel")
    args = ap.parse_args()
    print(build(force=args.force, verbose=args.verbose, ptxas_info=args.ptxas_info))
