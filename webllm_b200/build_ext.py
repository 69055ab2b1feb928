"""Build libwllm_mulmat.so in-tree with nvcc for sm_100a.

    python -m webllm_b200.build_ext            # build if sources changed
    python -m webllm_b200.build_ext --force    # rebuild

The library is a plain C-ABI shared object (no torch types), linked
against the static CUDA runtime, so any host (ctypes, bun:ffi, cgo, C++)
can dlopen it.
"""
from __future__ import annotations

import argparse
import os
import shutil
import subprocess
import sys

PKG_DIR = os.path.dirname(os.path.abspath(__file__))
REPO_DIR = os.path.dirname(PKG_DIR)
CSRC = os.path.join(PKG_DIR, "csrc")
LIB_PATH = os.path.join(PKG_DIR, "libwllm_mulmat.so")

SOURCES = ["runtime.cpp", "mulmat_gemv.cu", "mulmat_stream.cu", "mulmat_prefill.cu", "mulmat_batched.cu",
           "mulmat_batched_tc.cu"]
HEADERS = ["wllm_internal.h", "quant_blocks.cuh"]
ARCH_FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a"]


def nvcc_path() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError("nvcc not found")


def _inputs() -> list[str]:
    files = [os.path.join(CSRC, f) for f in SOURCES + HEADERS]
    files.append(os.path.join(REPO_DIR, "include", "wllm_mulmat.h"))
    files.append(os.path.abspath(__file__))
    return files


def up_to_date() -> bool:
    if not os.path.exists(LIB_PATH):
        return False
    t = os.path.getmtime(LIB_PATH)
    return all(os.path.getmtime(f) <= t for f in _inputs())


def build(force: bool = False, verbose: bool = False) -> str:
    if not force and up_to_date():
        return LIB_PATH
    tmp = LIB_PATH + ".tmp"
    cmd = [
        nvcc_path(),
        *ARCH_FLAGS,
        "-lineinfo",
        "-O3",
        "-std=c++17",
        "-ccbin",
        "/usr/bin/g++" if os.path.exists("/usr/bin/g++") else "g++",
        "-Xcompiler",
        "-fPIC,-fvisibility=hidden",
        "-shared",
        "-cudart",
        "static",
        "-I",
        os.path.join(REPO_DIR, "include"),
        "-o",
        tmp,
        *[os.path.join(CSRC, f) for f in SOURCES],
    ]
    if verbose:
        cmd.insert(1, "-Xptxas=-v")
        print(" ".join(cmd), file=sys.stderr)
    subprocess.run(cmd, check=True, cwd=CSRC)
    os.replace(tmp, LIB_PATH)
    return LIB_PATH


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--verbose", action="store_true")
    a = ap.parse_args()
    print(build(force=a.force, verbose=a.verbose))


if __name__ == "__main__":
    main()
