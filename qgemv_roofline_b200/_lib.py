"""ctypes binding of libqgemv_b200.so (the C ABI in include/qgemv_b200.h).

Loading is strict: if the shared library is missing or does not export a
declared symbol, ``lib()`` raises.  There is no CPU fallback anywhere in
this package; every compute call goes to the sm_100a kernels.
"""

from __future__ import annotations

import ctypes
import os
import threading

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libqgemv_b200.so")
HEADER = os.path.join(os.path.dirname(HERE), "include", "qgemv_b200.h")

OK = 0
STATUS_NAMES = {
    0: "QGEMV_OK", 1: "QGEMV_ERR_NULL", 2: "QGEMV_ERR_SHAPE", 3: "QGEMV_ERR_ALIGN",
    4: "QGEMV_ERR_CUDA", 5: "QGEMV_ERR_UNSUPPORTED", 6: "QGEMV_ERR_TIMEOUT", 7: "QGEMV_ERR_ARG",
}
FORMAT_CODE = {"q8_0": 8, "q4_0": 4}


MAX_RANKS = 8


class FuseDesc(ctypes.Structure):
    """qgemv_fuse of include/qgemv_b200.h."""
    _fields_ = [("peer_y", ctypes.c_void_p * MAX_RANKS), ("sig_out", ctypes.c_void_p * MAX_RANKS),
                ("cta_count", ctypes.c_void_p), ("sig_in", ctypes.c_void_p),
                ("tok", ctypes.c_void_p), ("npeer", ctypes.c_int32), ("nranks", ctypes.c_int32)]


class StackGemvDesc(ctypes.Structure):
    """qgemv_stack_gemv of include/qgemv_b200.h."""
    _fields_ = [("q", ctypes.c_void_p), ("d", ctypes.c_void_p), ("x", ctypes.c_void_p),
                ("y", ctypes.c_void_p), ("r0", ctypes.c_int64), ("M", ctypes.c_int64),
                ("M_total", ctypes.c_int64), ("K", ctypes.c_int64)]


class StackRanksDesc(ctypes.Structure):
    """qgemv_stack_ranks of include/qgemv_b200.h."""
    _fields_ = [("nranks", ctypes.c_int32), ("rank", ctypes.c_int32), ("peer_y", ctypes.c_void_p)]


class QGemvError(RuntimeError):
    """A C-ABI call returned a non-zero qgemv_status."""

    def __init__(self, func: str, status: int, message: str):
        self.func, self.status, self.message = func, status, message
        super().__init__(f"{func} failed: {STATUS_NAMES.get(status, status)}: {message}")


class CallDesc(ctypes.Structure):
    """qgemv_call_desc of include/qgemv_b200.h."""

    _fields_ = [
        ("format", ctypes.c_int32),
        ("layout", ctypes.c_int32),
        ("ncopies", ctypes.c_int32),
        ("ncols", ctypes.c_int32),
        ("M", ctypes.c_int64),
        ("K", ctypes.c_int64),
        ("ldx", ctypes.c_int64),
        ("ldy", ctypes.c_int64),
        ("q", ctypes.POINTER(ctypes.c_void_p)),
        ("d", ctypes.POINTER(ctypes.c_void_p)),
        ("x", ctypes.c_void_p),
        ("y", ctypes.c_void_p),
    ]


class DeviceInfo(ctypes.Structure):
    _fields_ = [
        ("name", ctypes.c_char * 256),
        ("device", ctypes.c_int),
        ("cc_major", ctypes.c_int),
        ("cc_minor", ctypes.c_int),
        ("sms", ctypes.c_int),
        ("l2_bytes", ctypes.c_int),
        ("mem_clock_khz", ctypes.c_int),
        ("bus_width_bits", ctypes.c_int),
        ("sm_clock_khz", ctypes.c_int),
        ("smem_per_block_optin", ctypes.c_int),
        ("datasheet_gbps", ctypes.c_double),
    ]


_vp, _i32, _i64, _sz = ctypes.c_void_p, ctypes.c_int32, ctypes.c_int64, ctypes.c_size_t
# name -> (argtypes, restype); every function of include/qgemv_b200.h.
SIGNATURES = {
    "qgemv_version": ([], ctypes.c_int),
    "qgemv_last_error": ([], ctypes.c_char_p),
    "qgemv_status_string": ([ctypes.c_int], ctypes.c_char_p),
    "qgemv_device_info_get": ([ctypes.c_int, ctypes.POINTER(DeviceInfo)], ctypes.c_int),
    "qgemv_q8_0_soa": ([_vp, _vp, _vp, _vp, _i64, _i64, _i32, _i64, _i64, _vp], ctypes.c_int),
    "qgemv_q4_0_soa": ([_vp, _vp, _vp, _vp, _i64, _i64, _i32, _i64, _i64, _vp], ctypes.c_int),
    "qgemv_q8_0_aos": ([_vp, _vp, _vp, _i64, _i64, _i32, _i64, _i64, _vp], ctypes.c_int),
    "qgemv_q4_0_aos": ([_vp, _vp, _vp, _i64, _i64, _i32, _i64, _i64, _vp], ctypes.c_int),
    "qgemv_soa_variant_count": ([], ctypes.c_int),
    "qgemv_soa_variant_name": ([ctypes.c_int], ctypes.c_char_p),
    "qgemv_soa_variant": ([ctypes.c_int, ctypes.c_int, _i32, _vp, _vp, _vp, _vp, _i64, _i64, _vp],
                          ctypes.c_int),
    "qgemv_check_device_error": ([ctypes.c_int, _vp], ctypes.c_int),
    "qgemv_set_wait_limit": ([_i64], ctypes.c_int),
    "qgemv_tile_counters_used": ([ctypes.c_int], _i32),
    "qgemv_tile_counters_capacity": ([], _i32),
    "qgemv_soa_workspace_bytes": ([ctypes.c_int, _i64, _i64, _i32], ctypes.c_size_t),
    "qgemv_soa_ws": ([ctypes.c_int, _vp, _vp, _vp, _vp, _i64, _i64, _i32, _i64, _i64, _vp,
                      ctypes.c_size_t, _vp], ctypes.c_int),
    "qgemv_release_workspaces": ([], ctypes.c_int),
    "qgemv_soa_q8_1": ([ctypes.c_int, _vp, _vp, _vp, _vp, _i64, _i64, _vp], ctypes.c_int),
    "qgemv_aos_q8_1": ([ctypes.c_int, _vp, _vp, _vp, _i64, _i64, _vp], ctypes.c_int),
    "qgemv_soa_fused": ([ctypes.c_int, _vp, _vp, _vp, _vp, _i64, _i64, _vp, _vp], ctypes.c_int),
    "qgemv_token_fence": ([_vp, _i32, _vp, _vp, _vp], ctypes.c_int),
    "qgemv_stack_create": ([ctypes.c_int, _vp, _i32, ctypes.POINTER(ctypes.c_void_p)],
                           ctypes.c_int),
    "qgemv_stack_create_ranks": ([ctypes.c_int, _vp, _i32, _vp, ctypes.POINTER(ctypes.c_void_p)],
                                 ctypes.c_int),
    "qgemv_stack_run": ([_vp, _vp], ctypes.c_int),
    "qgemv_stack_reset": ([_vp, _vp], ctypes.c_int),
    "qgemv_stack_destroy": ([_vp], ctypes.c_int),
    "qgemv_mg_init": ([_i32, ctypes.POINTER(_i32), ctypes.POINTER(_vp)], ctypes.c_int),
    "qgemv_mg_shard": ([_vp, ctypes.c_int, ctypes.c_int, _vp, _vp, _i64, _i64], ctypes.c_int),
    "qgemv_mg_rows": ([_vp, _i32, ctypes.POINTER(_i64), ctypes.POINTER(_i64)], ctypes.c_int),
    "qgemv_mg_gemv": ([_vp, ctypes.POINTER(_vp), ctypes.POINTER(_vp), _i32, _i32,
                       ctypes.POINTER(_vp)], ctypes.c_int),
    "qgemv_mg_synchronize": ([_vp], ctypes.c_int),
    "qgemv_mg_destroy": ([_vp], ctypes.c_int),
    "qgemv_soa_static_ws": ([ctypes.c_int, _vp, _vp, _vp, _vp, _i64, _i64, _i32, _i64, _i64, _vp],
                            ctypes.c_int),
    "qgemv_tiled_bytes": ([ctypes.c_int, _i64, _i64], ctypes.c_size_t),
    "qgemv_tile_weights": ([ctypes.c_int, ctypes.c_int, _vp, _vp, _i64, _i64, _vp, _vp],
                           ctypes.c_int),
    "qgemv_tiled_workspace_bytes": ([_i64, _i32], ctypes.c_size_t),
    "qgemv_tiled_gemv": ([ctypes.c_int, _vp, _i64, _i64, _vp, _vp, _i32, _i64, _i64, _vp,
                          ctypes.c_size_t, _vp], ctypes.c_int),
    "qgemv_tc_bytes": ([ctypes.c_int, _i64, _i64], ctypes.c_size_t),
    "qgemv_tc_tile": ([ctypes.c_int, ctypes.c_int, _vp, _vp, _i64, _i64, _vp, _vp], ctypes.c_int),
    "qgemv_tc_workspace_bytes": ([_i64, _i64], ctypes.c_size_t),
    "qgemv_tc_gemv": ([ctypes.c_int, _vp, _i64, _i64, _vp, _vp, _i32, _i64, _i64, _vp,
                       ctypes.c_size_t, _vp], ctypes.c_int),
    "qgemv_q8_0_tc_bytes": ([_i64, _i64], ctypes.c_size_t),
    "qgemv_q8_0_tc_tile": ([ctypes.c_int, _vp, _vp, _i64, _i64, _vp, _vp], ctypes.c_int),
    "qgemv_q8_0_tc_workspace_bytes": ([_i64, _i64], ctypes.c_size_t),
    "qgemv_q8_0_tc": ([_vp, _i64, _i64, _vp, _vp, _i32, _i64, _i64, _vp, ctypes.c_size_t, _vp],
                      ctypes.c_int),
    "qgemv_quantize_soa": ([ctypes.c_int, _vp, _i64, _i64, _i64, _vp, _vp, _vp], ctypes.c_int),
    "qgemv_quantize_aos": ([ctypes.c_int, _vp, _i64, _i64, _i64, _vp, _vp], ctypes.c_int),
    "qgemv_dequant_soa": ([ctypes.c_int, _vp, _vp, _vp, _i64, _i64, _vp], ctypes.c_int),
    "qgemv_repack": ([ctypes.c_int, ctypes.c_int, _vp, _vp, _vp, _i64, _i64, _vp], ctypes.c_int),
    "qgemv_roof_stream_read": ([_vp, _sz, _vp, _i32, _vp], ctypes.c_int),
    "qgemv_roof_bulk_read": ([_vp, _sz, _vp, _vp, _vp], ctypes.c_int),
    "qgemv_roof_d2d": ([_vp, _vp, _sz, _vp], ctypes.c_int),
    "qgemv_time_steps": ([ctypes.POINTER(CallDesc), _i32, _i32, _i32, _i32, _vp,
                          ctypes.POINTER(ctypes.c_float)], ctypes.c_int),
}

_lock = threading.Lock()
_lib = None


def lib() -> ctypes.CDLL:
    """The loaded library (built by qgemv_roofline_b200.build); raises if absent."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is None:
            if not os.path.exists(LIB_PATH):
                raise RuntimeError(
                    f"{LIB_PATH} is missing: build it with `python -m qgemv_roofline_b200.build` "
                    "(there is no CPU fallback)")
            h = ctypes.CDLL(LIB_PATH)
            for name, (argt, rest) in SIGNATURES.items():
                f = getattr(h, name)
                f.argtypes = argt
                f.restype = rest
            _lib = h
    return _lib


def last_error() -> str:
    return lib().qgemv_last_error().decode(errors="replace")


def call(name: str, *args) -> None:
    """Calls a status-returning entry point; raises QGemvError on failure."""
    rc = getattr(lib(), name)(*args)
    if rc != OK:
        raise QGemvError(name, rc, last_error())


def device_info(device: int = 0) -> dict:
    info = DeviceInfo()
    call("qgemv_device_info_get", device, ctypes.byref(info))
    out = {f: getattr(info, f) for f, _ in DeviceInfo._fields_}
    out["name"] = info.name.decode()
    return out
