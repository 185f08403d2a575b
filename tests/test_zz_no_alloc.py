"""qgemv_soa_static_ws: the batched SoA GEMV with its workspace in a static
device array (no allocation), through the C ABI, against the entry point that
takes a caller-provided workspace (qgemv_soa_ws) and against the float64
oracle.  Collected last so that it also runs after every other GPU test;
it needs nothing from them and passes alone in a fresh process too."""

import numpy as np
import pytest
import torch

from qgemv_roofline_b200 import _lib
from oracle import qformats_oracle as o

pytestmark = pytest.mark.gpu
DEV = "cuda"
FID = {"q8_0": 8, "q4_0": 4}
ERR_UNSUPPORTED = 5


def make(fmt, M, K, N, seed):
    rng = np.random.default_rng(seed)
    W = (rng.standard_normal((M, K)) * 0.02).astype(np.float32)
    X = rng.standard_normal((N, K)).astype(np.float32)
    q, d = o.quantize(fmt, W)
    return q, d.view(np.float16), X


@pytest.mark.parametrize("fmt", ["q8_0", "q4_0"])
@pytest.mark.parametrize("M,K,N", [(1000, 4096, 16), (257, 11008, 5), (64, 2048, 1),
                                   (4096, 4096, 8), (11008, 4096, 2)])
def test_static_workspace_matches_caller_workspace(fmt, M, K, N):
    lib = _lib.lib()
    q, d, X = make(fmt, M, K, N, seed=M + K + N)
    qt = torch.from_numpy(np.ascontiguousarray(q)).to(DEV)
    dt = torch.from_numpy(np.ascontiguousarray(d)).to(DEV)
    Xt = torch.from_numpy(X).to(DEV)
    st = torch.cuda.current_stream().cuda_stream
    nb = lib.qgemv_soa_workspace_bytes(FID[fmt], M, K, N)
    ws = torch.empty(max(nb, 16), dtype=torch.uint8, device=DEV)
    y_ref = torch.empty((N, M), device=DEV)
    assert lib.qgemv_soa_ws(FID[fmt], qt.data_ptr(), dt.data_ptr(), Xt.data_ptr(),
                            y_ref.data_ptr(), M, K, N, K, M, ws.data_ptr(), nb, st) == 0
    torch.cuda.synchronize()
    y64 = o.matvec_ref(fmt, q, d, X)
    wn = o.row_norms(fmt, q, d)
    for _ in range(2):  # two calls in a row
        y = torch.full((N, M), float("nan"), device=DEV)
        rc = lib.qgemv_soa_static_ws(FID[fmt], qt.data_ptr(), dt.data_ptr(), Xt.data_ptr(),
                                     y.data_ptr(), M, K, N, K, M, st)
        assert rc == 0, lib.qgemv_last_error()
        torch.cuda.synchronize()
        yh = y.cpu().numpy().astype(np.float64)
        bound = 1e-5 * wn[None, :] * np.linalg.norm(X.astype(np.float64), axis=1)[:, None]
        assert (np.abs(yh - y_ref.cpu().numpy()) <= bound).all()
        assert (np.abs(yh - y64) <= bound).all()
        if nb <= 2 << 20:
            # the whole workspace fits the array: the same (tcgen05) kernel as
            # with the caller's workspace, so the same bits
            assert torch.equal(y, y_ref)
    assert lib.qgemv_check_device_error(0, None) == 0


def test_static_workspace_rejects_oversized_calls():
    lib = _lib.lib()
    M, K, N = 16, 65536, 16   # needs 4.2 MB of workspace
    qt = torch.zeros((M, K), dtype=torch.int8, device=DEV)
    dt = torch.zeros((M, K // 32), dtype=torch.float16, device=DEV)
    Xt = torch.zeros((N, K), device=DEV)
    y = torch.full((N, M), 7.0, device=DEV)
    rc = lib.qgemv_soa_static_ws(8, qt.data_ptr(), dt.data_ptr(), Xt.data_ptr(), y.data_ptr(),
                                 M, K, N, K, M, torch.cuda.current_stream().cuda_stream)
    assert rc == ERR_UNSUPPORTED
    assert b"static workspace" in lib.qgemv_last_error()
    torch.cuda.synchronize()
    assert (y == 7.0).all()   # nothing was launched
