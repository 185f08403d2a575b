"""ctypes binding of oracle/_ref/libqgemv_ref.so (test infrastructure only).

The library is the reference's own src/bench.cu host code (quantizers
bench.cu:32-69, float64 matvec bench.cu:75-111) compiled where it lies by
oracle/Makefile, behind the C ABI of oracle/ref_shim.cu.  It is optional:
``load()`` returns None when it has not been built.
"""

from __future__ import annotations

import ctypes
import os

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "_ref", "libqgemv_ref.so")
_lib = None


def load():
    global _lib
    if _lib is not None:
        return _lib
    if not os.path.exists(LIB_PATH):
        return None
    lib = ctypes.CDLL(LIB_PATH)
    vp, i32 = ctypes.c_void_p, ctypes.c_int
    lib.ref_block_bytes.argtypes = [i32]
    lib.ref_block_bytes.restype = i32
    for name in ("ref_quantize_q8_0", "ref_quantize_q4_0"):
        f = getattr(lib, name)
        f.argtypes = [vp, i32, i32, vp]
        f.restype = i32
    lib.ref_matvec.argtypes = [i32, vp, vp, i32, i32, vp]
    lib.ref_matvec.restype = i32
    lib.ref_plan_create.argtypes = [i32, vp, i32, i32, i32]
    lib.ref_plan_create.restype = vp
    lib.ref_plan_run.argtypes = [vp, vp, vp]
    lib.ref_plan_run.restype = i32
    lib.ref_plan_destroy.argtypes = [vp]
    lib.ref_plan_destroy.restype = None
    _lib = lib
    return lib


def _fmt_code(fmt: str) -> int:
    return 8 if fmt == "q8_0" else 4


def quantize_aos(fmt: str, W: np.ndarray) -> np.ndarray:
    """Reference C++ quantizer -> ggml blocks uint8 [M, K/32, 34|18]."""
    lib = load()
    W = np.ascontiguousarray(W, dtype=np.float32)
    M, K = W.shape
    bs = lib.ref_block_bytes(_fmt_code(fmt))
    out = np.zeros((M, K // 32, bs), dtype=np.uint8)
    fn = lib.ref_quantize_q8_0 if fmt == "q8_0" else lib.ref_quantize_q4_0
    rc = fn(W.ctypes.data, M, K, out.ctypes.data)
    assert rc == 0
    return out


def matvec(fmt: str, blocks: np.ndarray, x: np.ndarray) -> np.ndarray:
    """Reference float64 matvec over ggml blocks [M, K/32, bs] -> float64 [M]."""
    lib = load()
    blocks = np.ascontiguousarray(blocks, dtype=np.uint8)
    x = np.ascontiguousarray(x, dtype=np.float32)
    M, nb, _ = blocks.shape
    y = np.zeros(M, dtype=np.float64)
    rc = lib.ref_matvec(_fmt_code(fmt), blocks.ctypes.data, x.ctypes.data, M, nb * 32,
                        y.ctypes.data)
    assert rc == 0
    return y


class Plan:
    """The reference matvec over all rows, split across ``nthreads`` threads."""

    def __init__(self, fmt: str, blocks: np.ndarray, nthreads: int):
        self.lib = load()
        blocks = np.ascontiguousarray(blocks, dtype=np.uint8)
        self.M, nb, _ = blocks.shape
        self.K = nb * 32
        self.nthreads = nthreads
        self.h = self.lib.ref_plan_create(_fmt_code(fmt), blocks.ctypes.data, self.M,
                                          self.K, nthreads)
        if not self.h:
            raise RuntimeError("ref_plan_create failed")
        self.y = np.zeros(self.M, dtype=np.float64)

    def run(self, x: np.ndarray) -> np.ndarray:
        x = np.ascontiguousarray(x, dtype=np.float32)
        rc = self.lib.ref_plan_run(self.h, x.ctypes.data, self.y.ctypes.data)
        assert rc == 0
        return self.y

    def close(self):
        if self.h:
            self.lib.ref_plan_destroy(self.h)
            self.h = None

    def __del__(self):
        self.close()
