"""Bounded device-side waits run out and report, without a fault or a hang.

The reference's harness exits on any CUDA error (src/bench.cu:19-27); here
every device-side wait of the library gives up after a limit and records
QGEMV_ERR_TIMEOUT in the device error word instead.  These tests make a wait
run out on purpose by waiting on a counter that nothing increments (the
allowed form: a flag nobody sets, with a short limit), check that the call
returns, that the error word says QGEMV_ERR_TIMEOUT, that a timed-out fused
call sends no signal, and that after clearing the word the next plain call
gives the exact result again.  No fault, no trap, one GPU.
"""

import ctypes
import time

import numpy as np
import pytest
import torch

import qgemv_roofline_b200 as qg
from qgemv_roofline_b200 import _lib
from oracle import qformats_oracle as o

pytestmark = pytest.mark.gpu
DEV = "cuda"
OK, ERR_TIMEOUT = 0, 6
LIMIT_US = 2000  # 2 ms


def make(fmt, M, K, seed):
    rng = np.random.default_rng(seed)
    W = (rng.standard_normal((M, K)) * 0.02).astype(np.float32)
    x = rng.standard_normal(K).astype(np.float32)
    q, d = o.quantize(fmt, W)
    return q, d.view(np.float16), x


def planes(q, d):
    return (torch.from_numpy(np.ascontiguousarray(q)).to(DEV),
            torch.from_numpy(np.ascontiguousarray(d)).to(DEV))


@pytest.fixture
def short_wait_limit():
    lib = _lib.lib()
    assert lib.qgemv_check_device_error(1, None) == OK  # start clear
    assert lib.qgemv_set_wait_limit(LIMIT_US) == OK
    yield lib
    assert lib.qgemv_set_wait_limit(0) == OK  # back to the default (~1 s)
    lib.qgemv_check_device_error(1, None)


@pytest.mark.parametrize("fmt", ["q8_0", "q4_0"])
def test_fused_wait_on_unset_counter_times_out(short_wait_limit, fmt):
    lib = short_wait_limit
    M, K = 2048, 4096
    q, d, x = make(fmt, M, K, seed=41)
    qt, dt = planes(q, d)
    xt = torch.from_numpy(x).to(DEV)
    y_good = qg.qgemv(fmt, qt, dt, xt).clone()
    torch.cuda.synchronize()

    # counters: [0] this call's signal out, [1] the input's counter (never
    # incremented: the wait for (tok + 1) * 1 = 1 cannot complete), [2] the
    # CTA count, [3] the token count
    ctr = torch.zeros(4, dtype=torch.int32, device=DEV)
    base = ctr.data_ptr()
    fz = _lib.FuseDesc()
    fz.sig_out[0] = base
    fz.sig_in = base + 4
    fz.cta_count = base + 8
    fz.tok = base + 12
    fz.npeer, fz.nranks = 0, 1
    y = torch.zeros(M, device=DEV)
    t0 = time.perf_counter()
    _lib.call("qgemv_soa_fused", _lib.FORMAT_CODE[fmt], qt.data_ptr(), dt.data_ptr(),
              xt.data_ptr(), y.data_ptr(), M, K, ctypes.byref(fz),
              torch.cuda.current_stream().cuda_stream)
    torch.cuda.synchronize()
    assert time.perf_counter() - t0 < 20.0  # returned: the wait gave up
    c = ctr.cpu().numpy()
    assert c[0] == 0, "a timed-out call must not signal"
    assert c[1] == 0
    assert lib.qgemv_check_device_error(0, None) == ERR_TIMEOUT
    assert lib.qgemv_check_device_error(1, None) == ERR_TIMEOUT  # reports, then clears
    assert lib.qgemv_check_device_error(0, None) == OK

    # the next plain call (default limit, cleared word, reset tile counters) is exact
    assert lib.qgemv_set_wait_limit(0) == OK
    for _ in range(2):
        y2 = qg.qgemv(fmt, qt, dt, xt)
        torch.cuda.synchronize()
        assert torch.equal(y2, y_good)
    y_ref = o.matvec_ref(fmt, q, d, x[None, :])
    ok, worst = o.check_rowwise(y2.cpu().numpy()[None, :].astype(np.float64), y_ref,
                                o.row_norms(fmt, q, d), x[None, :])
    assert ok, worst
    assert lib.qgemv_check_device_error(0, None) == OK


def test_token_fence_waiting_for_a_missing_rank_times_out(short_wait_limit):
    """A token fence of two ranks where the second never arrives."""
    lib = short_wait_limit
    ctr = torch.zeros(3, dtype=torch.int32, device=DEV)  # done (local), other rank's done, tok
    base = ctr.data_ptr()
    done = (ctypes.c_void_p * 2)(base, base + 4)
    t0 = time.perf_counter()
    _lib.call("qgemv_token_fence", done, 2, base, base + 8,
              torch.cuda.current_stream().cuda_stream)
    torch.cuda.synchronize()
    assert time.perf_counter() - t0 < 20.0
    assert lib.qgemv_check_device_error(1, None) == ERR_TIMEOUT
    assert lib.qgemv_check_device_error(0, None) == OK


def test_wait_limit_argument_and_default():
    lib = _lib.lib()
    assert lib.qgemv_set_wait_limit(1 << 50) == 7  # QGEMV_ERR_ARG: absurd limit
    assert lib.qgemv_set_wait_limit(-1) == OK      # default
    assert lib.qgemv_set_wait_limit(0) == OK


def test_tc_kernel_waits_time_out_and_recover(short_wait_limit):
    """The tcgen05 batch kernel under a 1 us wait limit: its ring waits run out
    (the producer waiting for a free stage, the MMA thread for data, the
    epilogue for accumulators), the CTAs stop, wait for their copies and MMAs
    in flight, free their tensor memory and return; the error word reads
    QGEMV_ERR_TIMEOUT, and the next call at the default limit is exact."""
    lib = short_wait_limit
    assert lib.qgemv_set_wait_limit(0) == OK
    M, K, N = 28672, 8192, 4
    q, d, _ = make("q8_0", M, K, seed=43)
    qt, dt = planes(q, d)
    tiles = qg.tile_weights_tc(q=qt, d=dt)
    X = torch.randn(N, K, device=DEV, generator=torch.Generator(device=DEV).manual_seed(5))
    y_good = qg.qgemv_tc(tiles, M, K, X).clone()
    torch.cuda.synchronize()
    assert lib.qgemv_check_device_error(0, None) == OK

    assert lib.qgemv_set_wait_limit(1) == OK  # 1 us: shorter than a DRAM round trip under load
    seen = False
    for _ in range(3):
        t0 = time.perf_counter()
        y = qg.qgemv_tc(tiles, M, K, X)
        torch.cuda.synchronize()
        assert time.perf_counter() - t0 < 20.0  # returned
        if lib.qgemv_check_device_error(1, None) == ERR_TIMEOUT:
            seen = True
            break
    assert seen, "no wait of the tc kernel ran out under a 1 us limit"
    assert lib.qgemv_check_device_error(0, None) == OK

    assert lib.qgemv_set_wait_limit(0) == OK
    for _ in range(2):
        y2 = qg.qgemv_tc(tiles, M, K, X)
        torch.cuda.synchronize()
        assert torch.equal(y2, y_good)
    assert lib.qgemv_check_device_error(0, None) == OK
