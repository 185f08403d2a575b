"""The C ABI library without a GPU: it loads, exports every symbol the header
declares, and rejects bad arguments before touching the device."""

import ctypes
import re

import pytest

from qgemv_roofline_b200 import _lib


def declared_symbols():
    text = open(_lib.HEADER).read()
    return re.findall(r"QGEMV_API\s+[\w\s\*]+?\b(qgemv_\w+)\s*\(", text)


def test_library_loads_and_exports_every_declared_symbol():
    lib = _lib.lib()
    names = declared_symbols()
    assert len(names) >= 15
    for n in names:
        assert hasattr(lib, n), n
    # the ctypes signature table covers the whole header
    assert set(names) == set(_lib.SIGNATURES)


def test_version_and_status_strings():
    lib = _lib.lib()
    assert lib.qgemv_version() == 100
    for code, name in _lib.STATUS_NAMES.items():
        assert lib.qgemv_status_string(code).decode() == name


FAKE = 0x100000  # 16-byte aligned, never dereferenced: validation fails first


def rc(name, *args):
    return getattr(_lib.lib(), name)(*args)


@pytest.mark.parametrize("fn", ["qgemv_q8_0_soa", "qgemv_q4_0_soa"])
def test_soa_validation(fn):
    E = _lib
    assert rc(fn, FAKE, FAKE, FAKE, FAKE, 64, 100, 1, 100, 64, None) == 2  # K % 32
    assert "multiple of 32" in E.last_error()
    assert rc(fn, FAKE, FAKE, FAKE, FAKE, -1, 64, 1, 64, 1, None) == 2
    assert rc(fn, FAKE, FAKE, FAKE, FAKE, 64, 64, -1, 64, 64, None) == 2
    assert rc(fn, None, FAKE, FAKE, FAKE, 64, 64, 1, 64, 64, None) == 1
    assert rc(fn, FAKE, FAKE, None, FAKE, 64, 64, 1, 64, 64, None) == 1
    assert rc(fn, FAKE + 8, FAKE, FAKE, FAKE, 64, 64, 1, 64, 64, None) == 3  # q not 16-B
    assert rc(fn, FAKE, FAKE + 1, FAKE, FAKE, 64, 64, 1, 64, 64, None) == 3  # d not 2-B
    assert rc(fn, FAKE, FAKE, FAKE + 2, FAKE, 64, 64, 1, 64, 64, None) == 3  # x not 4-B
    assert rc(fn, FAKE, FAKE, FAKE, FAKE, 64, 64, 2, 32, 64, None) == 2  # ldx < K
    assert rc(fn, FAKE, FAKE, FAKE, FAKE, 64, 64, 2, 64, 32, None) == 2  # ldy < M
    assert rc(fn, FAKE, FAKE, FAKE, FAKE, 1 << 31, 64, 1, 64, 1, None) == 5
    # empty work is a no-op that needs no device
    assert rc(fn, None, None, None, None, 0, 64, 1, 64, 0, None) == 0
    assert rc(fn, None, None, None, None, 64, 64, 0, 64, 64, None) == 0


@pytest.mark.parametrize("fn", ["qgemv_q8_0_aos", "qgemv_q4_0_aos"])
def test_aos_validation(fn):
    assert rc(fn, FAKE, FAKE, FAKE, 64, 48, 1, 48, 64, None) == 2
    assert rc(fn, None, FAKE, FAKE, 64, 64, 1, 64, 64, None) == 1
    assert rc(fn, FAKE + 2, FAKE, FAKE, 64, 64, 1, 64, 64, None) == 3


def test_quantize_repack_roof_validation():
    assert rc("qgemv_quantize_soa", 5, FAKE, 4, 64, 64, FAKE, FAKE, None) == 7  # format
    assert rc("qgemv_quantize_soa", 8, FAKE, 4, 40, 40, FAKE, FAKE, None) == 2
    assert rc("qgemv_quantize_soa", 4, FAKE, 4, 64, 32, FAKE, FAKE, None) == 2  # ldw < K
    assert rc("qgemv_quantize_soa", 4, None, 4, 64, 64, FAKE, FAKE, None) == 1
    assert rc("qgemv_quantize_aos", 8, FAKE + 1, 4, 64, 64, FAKE, None) == 3
    assert rc("qgemv_dequant_soa", 4, FAKE, FAKE + 1, FAKE, 4, 64, None) == 3
    assert rc("qgemv_repack", 8, 2, FAKE, FAKE, FAKE, 4, 64, None) == 7
    assert rc("qgemv_repack", 8, 1, None, FAKE, FAKE, 4, 64, None) == 1
    assert rc("qgemv_roof_stream_read", FAKE, 100, FAKE, 4, None) == 2
    assert rc("qgemv_roof_stream_read", FAKE + 4, 128, FAKE, 4, None) == 3
    assert rc("qgemv_roof_stream_read", FAKE, 128, FAKE, 0, None) == 7
    assert rc("qgemv_roof_bulk_read", FAKE, 128, FAKE, None, None) == 1
    assert rc("qgemv_roof_d2d", None, FAKE, 16, None) == 1
    assert rc("qgemv_device_info_get", 0, None) == 1


def test_errors_are_per_thread_messages():
    import threading
    rc("qgemv_q8_0_soa", FAKE, FAKE, FAKE, FAKE, 64, 100, 1, 100, 64, None)
    seen = {}

    def other():
        seen["msg"] = _lib.last_error()

    t = threading.Thread(target=other)
    t.start()
    t.join()
    assert seen["msg"] == ""
    assert "multiple of 32" in _lib.last_error()


def test_python_raises_typed_error():
    with pytest.raises(_lib.QGemvError) as ei:
        _lib.call("qgemv_q8_0_soa", FAKE, FAKE, FAKE, FAKE, 64, 100, 1, 100, 64, None)
    assert ei.value.status == 2 and "QGEMV_ERR_SHAPE" in str(ei.value)


def test_workspace_and_tile_sizes_are_host_computations():
    lib = _lib.lib()
    # batched SoA calls with no device: the mma.sync kernel's 128 + 2064 * ceil(K / 512) *
    # min(N, 16) bytes, 0 when no workspace (on a B200 the tcgen05 kernel's need, larger)
    assert lib.qgemv_soa_workspace_bytes(8, 1000, 4096, 4) == 128 + 2064 * 8 * 4
    assert lib.qgemv_soa_workspace_bytes(4, 1000, 4096, 40) == 128 + 2064 * 8 * 16
    assert lib.qgemv_soa_workspace_bytes(8, 1000, 4096, 1) == 0
    assert lib.qgemv_soa_workspace_bytes(8, 1000, 4000, 4) == 0     # K % 256 != 0
    assert lib.qgemv_soa_workspace_bytes(3, 1000, 4096, 4) == 0     # bad format
    assert lib.qgemv_tiled_workspace_bytes(800, 3) == 128 + 2064 * 2 * 3
    assert lib.qgemv_tiled_workspace_bytes(800, 0) == 0
    # batch tiles: ceil(M/16) * ceil(K/512) blocks of 16 x 512 quants + 512 scale bytes
    assert lib.qgemv_tiled_bytes(8, 17, 800) == 2 * 2 * (16 * 512 + 512)
    assert lib.qgemv_tiled_bytes(4, 16, 512) == 1 * 1 * (16 * 256 + 512)
    assert lib.qgemv_tiled_bytes(8, 16, 33) == 0                    # K % 32 != 0


def test_fused_and_tiled_validation():
    from qgemv_roofline_b200._lib import FuseDesc
    f = FuseDesc()
    f.nranks = 0
    assert rc("qgemv_soa_fused", 8, FAKE, FAKE, FAKE, FAKE, 64, 4096, ctypes.byref(f), None) == 7
    f.nranks, f.npeer = 2, 1
    assert rc("qgemv_soa_fused", 8, FAKE, FAKE, FAKE, FAKE, 64, 4096, ctypes.byref(f), None) == 1
    assert rc("qgemv_soa_fused", 8, FAKE, FAKE, FAKE, FAKE, 64, 4096, None, None) == 1
    assert rc("qgemv_token_fence", None, 0, FAKE, FAKE, None) == 7
    assert rc("qgemv_token_fence", None, 2, FAKE, FAKE, None) == 1
    assert rc("qgemv_tile_weights", 8, 2, FAKE, FAKE, 16, 512, FAKE, None) == 7   # bad layout
    assert rc("qgemv_tile_weights", 8, 0, FAKE, FAKE, 16, 512, FAKE + 8, None) == 3
    assert rc("qgemv_tiled_gemv", 8, FAKE, 16, 100, FAKE, FAKE, 1, 100, 16, None, 0, None) == 2
    assert rc("qgemv_tiled_gemv", 8, FAKE, 16, 1 << 21, FAKE, FAKE, 1, 1 << 21, 16, None, 0,
              None) == 5
    assert rc("qgemv_tiled_gemv", 8, FAKE + 4, 16, 512, FAKE, FAKE, 1, 512, 16, None, 0,
              None) == 3


def test_multi_gpu_handle_validation():
    lib = _lib.lib()
    h = ctypes.c_void_p()
    devs = (ctypes.c_int32 * 2)(0, 1)
    assert lib.qgemv_mg_init(2, None, ctypes.byref(h)) == 1
    assert lib.qgemv_mg_init(2, devs, None) == 1
    assert lib.qgemv_mg_init(0, devs, ctypes.byref(h)) == 7
    assert lib.qgemv_mg_init(9, devs, ctypes.byref(h)) == 7
    assert not h.value
    # a NULL handle is refused by every entry point; destroying it is a no-op
    r0, rows = ctypes.c_int64(), ctypes.c_int64()
    assert lib.qgemv_mg_shard(None, 8, 0, FAKE, FAKE, 64, 64) == 1
    assert lib.qgemv_mg_rows(None, 0, ctypes.byref(r0), ctypes.byref(rows)) == 1
    assert lib.qgemv_mg_gemv(None, None, None, 1, 1, None) == 1
    assert lib.qgemv_mg_synchronize(None) == 1
    assert lib.qgemv_mg_destroy(None) == 0
