"""Build libqwenb200.so (sm_100a) in-tree with nvcc.

    python -m qwen_fpga_b200.build

The library lands next to this file so it travels with the repository
snapshot; nothing is installed into site-packages.
"""

from __future__ import annotations

import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(HERE)
LIB = os.path.join(HERE, "libqwenb200.so")
SOURCES = ["csrc/runtime.cu", "csrc/batch.cu", "csrc/delta.cu", "csrc/gemv.cu", "csrc/persist.cu", "csrc/persist_tp.cu",
           "csrc/noalloc.cu", "csrc/pack.cpp"]
HEADERS = ["csrc/common.cuh", "csrc/batch.cuh", "csrc/tc.cuh", "csrc/delta.cuh", "csrc/gemv.cuh", "csrc/persist.cuh", "csrc/noalloc.cuh",
           "../include/qwen_b200.h"]
NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")
FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a", "-O3", "-lineinfo", "-std=c++17",
         "-Xcompiler", "-fPIC", "-shared", "-Xptxas", "-warn-spills"]


def stale() -> bool:
    if not os.path.exists(LIB):
        return True
    t = os.path.getmtime(LIB)
    return any(os.path.getmtime(os.path.join(HERE, s)) > t for s in SOURCES + HEADERS)


def build(force: bool = False, verbose: bool = False) -> str:
    if force or stale():
        cmd = [NVCC, *FLAGS, *[os.path.join(HERE, s) for s in SOURCES], "-o", LIB + ".tmp"]
        if verbose:
            print(" ".join(cmd), flush=True)
        subprocess.run(cmd, check=True, cwd=HERE)
        os.replace(LIB + ".tmp", LIB)
    return LIB


if __name__ == "__main__":
    print(build(force="--force" in sys.argv, verbose=True))
