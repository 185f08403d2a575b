"""Builds libqgemv_b200.so in-tree with nvcc for sm_100a.

    python -m qgemv_roofline_b200.build        (or: make -C qgemv_roofline_b200/csrc)

The library is plain CUDA C++ behind a C ABI (include/qgemv_b200.h); no
torch headers are involved, so it builds on a machine without a GPU.
"""

from __future__ import annotations

import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(HERE)
CSRC = os.path.join(HERE, "csrc")
LIB = os.path.join(HERE, "libqgemv_b200.so")
SOURCES = ["capi.cu", "gemv_soa.cu", "gemv_aos.cu", "quant.cu", "roof.cu", "harness.cu", "gemv_tma.cu", "gemv_mma.cu",
           "gemv_tc.cu", "static_ws.cu", "multi_gpu.cu"]
HEADERS = ["qgemv_common.cuh", "qgemv_internal.h", "gemv_core.cuh"]
NVCC = os.environ.get("NVCC", "nvcc")
FLAGS = [
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-O3", "-lineinfo", "-std=c++17",
    "-Xcompiler", "-fPIC,-fvisibility=hidden",
    "-shared",
]


def _stale() -> bool:
    if not os.path.exists(LIB):
        return True
    t = os.path.getmtime(LIB)
    deps = [os.path.join(CSRC, f) for f in SOURCES + HEADERS]
    deps.append(os.path.join(REPO, "include", "qgemv_b200.h"))
    return any(os.path.getmtime(p) > t for p in deps)


def build(force: bool = False, verbose: bool = False) -> str:
    if not force and not _stale():
        return LIB
    cmd = [NVCC, *FLAGS, "-I", os.path.join(REPO, "include"), "-I", CSRC,
           *[os.path.join(CSRC, f) for f in SOURCES], "-o", LIB + ".tmp"]
    if verbose:
        cmd.insert(1, "-Xptxas=-v")
        print(" ".join(cmd))
    subprocess.run(cmd, check=True)
    os.replace(LIB + ".tmp", LIB)
    return LIB


if __name__ == "__main__":
    build(force="--force" in sys.argv, verbose="-v" in sys.argv)
    print(LIB)
