"""Small-batch SoA GEMV (2..16 columns per launch) on the GPU: the tensor-core
kernel through the C ABI against the float64 oracle, within the row-wise
bound |y - y_ref| <= 1e-5 ||w_row|| ||x|| and the reference gate
max|err| / max|y_ref| <= 1e-5 (tests/test_correctness.py:21 of the
reference), plus the workspace contract of qgemv_soa_ws."""

import numpy as np
import pytest
import torch

import qgemv_roofline_b200 as qg
from qgemv_roofline_b200 import _lib
from oracle import qformats_oracle as o

pytestmark = pytest.mark.gpu
TOL = 1e-5
DEV = "cuda"
ERR_ALIGN, ERR_ARG = 3, 7
FMT_ID = {"q8_0": 8, "q4_0": 4}


def make(fmt, M, K, N, seed, scale=0.02):
    rng = np.random.default_rng(seed)
    W = (rng.standard_normal((M, K)) * scale).astype(np.float32)
    X = rng.standard_normal((N, K)).astype(np.float32)
    q, d = o.quantize(fmt, W)
    return q, d, X


def planes(q, d):
    return (torch.from_numpy(np.ascontiguousarray(q)).to(DEV),
            torch.from_numpy(np.ascontiguousarray(d.view(np.float16))).to(DEV))


def check(fmt, q, d, X, Y, tol=TOL, rows=None):
    Y = np.asarray(Y, np.float64).reshape(X.shape[0], -1)
    if rows is not None:
        q, d, Y = q[rows], d[rows], Y[:, rows]
    y_ref = o.matvec_ref(fmt, q, d, X)
    wn = o.row_norms(fmt, q, d)
    ok, worst = o.check_rowwise(Y, y_ref, wn, X, tol)
    assert ok, f"row-wise bound exceeded: worst ratio {worst:.3g}"
    ok, _, rel = o.check_gate(Y, y_ref, tol)
    assert ok, f"reference gate exceeded: {rel:.3g}"
    return worst


def plain_call(fmt, qt, dt, Xt, Yt, N, ldx, ldy):
    M = qt.shape[0]
    K = Xt.shape[-1] if ldx is None else ldx
    fn = "qgemv_q8_0_soa" if fmt == "q8_0" else "qgemv_q4_0_soa"
    _lib.call(fn, qt.data_ptr(), dt.data_ptr(), Xt.data_ptr(), Yt.data_ptr(), M,
              dt.shape[1] * 32, N, ldx, ldy, torch.cuda.current_stream().cuda_stream)


BATCH_SHAPES = [
    (16, 256, 2), (1, 256, 3), (17, 768, 8), (15, 512, 9), (255, 4096, 16),
    (4099, 4096, 4), (1000, 11008, 16), (2048, 8192, 7), (333, 2304, 12),
    (4096, 4096, 15), (64, 16384, 16), (3000, 1280, 5),
]


@pytest.mark.parametrize("fmt", ["q8_0", "q4_0"])
@pytest.mark.parametrize("M,K,N", BATCH_SHAPES)
def test_batch_shapes(fmt, M, K, N):
    q, d, X = make(fmt, M, K, N, seed=M * 31 + K + N)
    qt, dt = planes(q, d)
    Xt = torch.from_numpy(X).to(DEV)
    Y = qg.qgemv(fmt, qt, dt, Xt)          # workspace from torch (qgemv_soa_ws)
    worst = check(fmt, q, d, X, Y.cpu().numpy())
    assert worst < 0.1                      # a few 1e-7 ||w|| ||x|| in practice
    Y2 = torch.empty_like(Y)                # workspace cached per stream
    plain_call(fmt, qt, dt, Xt, Y2, N, K, M)
    torch.cuda.synchronize()
    assert torch.equal(Y, Y2)


@pytest.mark.parametrize("fmt", ["q8_0", "q4_0"])
@pytest.mark.parametrize("N", [17, 33, 40])
def test_more_than_16_columns(fmt, N):
    M, K = 700, 4096
    q, d, X = make(fmt, M, K, N, seed=N)
    qt, dt = planes(q, d)
    Y = qg.qgemv(fmt, qt, dt, torch.from_numpy(X).to(DEV)).cpu().numpy()
    check(fmt, q, d, X, Y)


@pytest.mark.parametrize("fmt", ["q8_0", "q4_0"])
def test_columns_match_single_column_calls(fmt):
    M, K, N = 1536, 4096, 6
    q, d, X = make(fmt, M, K, N, seed=5)
    qt, dt = planes(q, d)
    Xt = torch.from_numpy(X).to(DEV)
    Y = qg.qgemv(fmt, qt, dt, Xt).cpu().numpy().astype(np.float64)
    wn = o.row_norms(fmt, q, d)
    for n in range(N):
        y1 = qg.qgemv(fmt, qt, dt, Xt[n]).cpu().numpy()
        # both kernels stay within ~1e-6 ||w|| ||x|| of the exact result
        bound = 3e-6 * wn * np.linalg.norm(X[n].astype(np.float64))
        assert (np.abs(Y[n] - y1) <= bound).all()


@pytest.mark.parametrize("fmt", ["q8_0", "q4_0"])
def test_per_column_extreme_scales_zero_and_non_finite(fmt):
    M, K, N = 640, 2048, 8
    q, d, X = make(fmt, M, K, N, seed=9)
    X[1] *= np.float32(1e-35)
    X[2] *= np.float32(3e30)
    X[3] = 0.0
    X[4, ::7] = 0.0
    X[5] *= np.float32(2.0 ** -140)   # subnormal column
    X[6, 100] = np.inf
    qt, dt = planes(q, d)
    Y = qg.qgemv(fmt, qt, dt, torch.from_numpy(X).to(DEV)).cpu().numpy()
    assert np.isnan(Y[6]).all()
    assert (Y[3] == 0).all()
    good = [0, 1, 2, 3, 4, 7]
    check(fmt, q, d, X[good], Y[good])
    # the subnormal column: compare against the scaled-up column
    Xs = X[5:6].astype(np.float64) * 2.0 ** 140
    y_ref = o.matvec_ref(fmt, q, d, Xs.astype(np.float32))[0] * 2.0 ** -140
    wn = o.row_norms(fmt, q, d)
    bound = 1e-5 * wn * np.linalg.norm(X[5].astype(np.float64)) + 2.0 ** -149 * 4
    assert (np.abs(Y[5] - y_ref) <= bound).all()


@pytest.mark.parametrize("fmt", ["q8_0", "q4_0"])
def test_strided_x_y_guard_bands(fmt):
    M, K, N = 517, 4096, 5
    q, d, X = make(fmt, M, K, N, seed=17)
    qt, dt = planes(q, d)
    ldx, ldy = K + 64, M + 11
    xb = torch.full((N + 1, ldx), 7.0, device=DEV)
    xb[:N, :K] = torch.from_numpy(X).to(DEV)
    yb = torch.full((N + 1, ldy), 123.0, device=DEV)
    plain_call(fmt, qt, dt, xb, yb, N, ldx, ldy)
    yh = yb.cpu().numpy()
    check(fmt, q, d, X, yh[:N, :M])
    assert (yh[:N, M:] == 123.0).all() and (yh[N] == 123.0).all()


@pytest.mark.parametrize("fmt", ["q8_0", "q4_0"])
def test_chained_calls_and_workspace_reuse(fmt):
    """y of one batched call is x of the next (same stream, programmatic
    dependent launches), interleaved with single-column calls and shapes that
    grow the per-stream workspace."""
    M = K = 2048
    q, d, X = make(fmt, M, K, 4, seed=21)
    qt, dt = planes(q, d)
    X1 = torch.from_numpy(X).to(DEV)
    Y1 = torch.empty((4, M), device=DEV)
    Y2 = torch.empty((4, M), device=DEV)
    y3 = torch.empty(M, device=DEV)
    for _ in range(3):
        plain_call(fmt, qt, dt, X1, Y1, 4, K, M)
        plain_call(fmt, qt, dt, Y1, Y2, 4, K, M)
        plain_call(fmt, qt, dt, Y2[1], y3, 1, K, M)
    torch.cuda.synchronize()
    y1 = Y1.cpu().numpy()
    check(fmt, q, d, X, y1)
    check(fmt, q, d, y1.astype(np.float32), Y2.cpu().numpy())
    # a wider K needs a larger workspace on the same stream
    q2, d2, X2 = make(fmt, 300, 16384, 16, seed=22)
    q2t, d2t = planes(q2, d2)
    Yw = torch.empty((16, 300), device=DEV)
    plain_call(fmt, q2t, d2t, torch.from_numpy(X2).to(DEV), Yw, 16, 16384, 300)
    torch.cuda.synchronize()
    check(fmt, q2, d2, X2, Yw.cpu().numpy())


@pytest.mark.parametrize("fmt", ["q8_0", "q4_0"])
def test_deterministic(fmt):
    M, K, N = 3000, 4096, 16
    q, d, X = make(fmt, M, K, N, seed=3)
    qt, dt = planes(q, d)
    Xt = torch.from_numpy(X).to(DEV)
    Y0 = qg.qgemv(fmt, qt, dt, Xt)
    for _ in range(3):
        assert torch.equal(qg.qgemv(fmt, qt, dt, Xt), Y0)


def test_workspace_contract():
    lib = _lib.lib()
    assert lib.qgemv_soa_workspace_bytes(8, 1000, 4096, 1) == 0
    assert lib.qgemv_soa_workspace_bytes(8, 1000, 4000, 4) == 0   # K % 256 != 0: no tensor cores
    n4 = lib.qgemv_soa_workspace_bytes(8, 1000, 4096, 4)
    n16 = lib.qgemv_soa_workspace_bytes(4, 1000, 4096, 16)
    assert 0 < n4 < n16 == lib.qgemv_soa_workspace_bytes(4, 1000, 4096, 40)
    # the need grows with M (the tcgen05 kernel keeps per-row-tile counters)
    assert lib.qgemv_soa_workspace_bytes(8, 64, 4096, 4) <= n4
    assert n4 <= lib.qgemv_soa_workspace_bytes(8, 100000, 4096, 4)
    n4 = lib.qgemv_soa_workspace_bytes(8, 64, 4096, 4)
    q, d, X = make("q8_0", 64, 4096, 4, seed=1)
    qt, dt = planes(q, d)
    Xt = torch.from_numpy(X).to(DEV)
    Y = torch.empty((4, 64), device=DEV)
    ws = torch.empty(n4, dtype=torch.uint8, device=DEV)
    st = torch.cuda.current_stream().cuda_stream
    args = (8, qt.data_ptr(), dt.data_ptr(), Xt.data_ptr(), Y.data_ptr(), 64, 4096, 4, 4096, 64)
    assert lib.qgemv_soa_ws(*args, ws.data_ptr(), n4 - 16, st) == ERR_ARG
    assert lib.qgemv_soa_ws(*args, None, 0, st) == ERR_ARG
    assert lib.qgemv_soa_ws(*args, ws.data_ptr() + 8, n4, st) == ERR_ALIGN
    assert lib.qgemv_soa_ws(*args, ws.data_ptr(), n4, st) == 0
    torch.cuda.synchronize()
    check("q8_0", q, d, X, Y.cpu().numpy())
    assert lib.qgemv_check_device_error(0, None) == 0


@pytest.mark.parametrize("fmt", ["q8_0", "q4_0"])
def test_graph_capture_python_api(fmt):
    """The Python API takes its workspace from torch's allocator, so batched
    calls can be captured in a CUDA graph and replayed."""
    M, K, N = 1024, 4096, 8
    q, d, X = make(fmt, M, K, N, seed=13)
    qt, dt = planes(q, d)
    Xt = torch.from_numpy(X).to(DEV)
    Y = torch.empty((N, M), device=DEV)
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        qg.qgemv(fmt, qt, dt, Xt, Y)   # warm-up outside capture
    torch.cuda.current_stream().wait_stream(s)
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        qg.qgemv(fmt, qt, dt, Xt, Y)
    Y.zero_()
    g.replay()
    torch.cuda.synchronize()
    check(fmt, q, d, X, Y.cpu().numpy())


# ------------------------------------------------------------ batch tiles
def tiles_np(fmt, q, d, M, K):
    """numpy restatement of the batch-tile layout (qgemv_tile_weights)."""
    KC, T = 512, -(-M // 16)
    nkt = -(-K // KC)
    qrow = K if fmt == "q8_0" else K // 2
    QROW = KC if fmt == "q8_0" else KC // 2
    nbox = QROW // 128
    # q8_0 quants are stored as w + 128 (sign bit flipped), padding as w = 0
    flip = 0x80 if fmt == "q8_0" else 0
    qp = np.full((T * 16, nkt * QROW), flip, np.uint8)
    qp[:M, :qrow] = q.view(np.uint8).reshape(M, qrow) ^ flip
    dp = np.zeros((T * 16, nkt * 16), np.uint16)
    dp[:M, :K // 32] = d.view(np.uint16).reshape(M, K // 32)
    out = []
    for kt in range(nkt):
        for t in range(T):
            rows = qp[16 * t:16 * t + 16, kt * QROW:(kt + 1) * QROW]
            qb = np.zeros((nbox, 16, 8, 16), np.uint8)
            for bx in range(nbox):
                for r in range(16):
                    for j in range(8):
                        qb[bx, r, j ^ (r & 7)] = rows[r, bx * 128 + 16 * j: bx * 128 + 16 * j + 16]
            out.append(qb.reshape(-1))
            out.append(dp[16 * t:16 * t + 16, kt * 16:kt * 16 + 16].reshape(-1).view(np.uint8))
    return np.concatenate(out)


@pytest.mark.parametrize("fmt", ["q8_0", "q4_0"])
@pytest.mark.parametrize("M,K", [(1, 32), (17, 800), (40, 1024)])
def test_tile_layout_bytes(fmt, M, K):
    q, d, _ = make(fmt, M, K, 1, seed=M + K)
    qt, dt = planes(q, d)
    t_soa = qg.tile_weights(fmt, q=qt, d=dt).cpu().numpy()
    assert (t_soa == tiles_np(fmt, q, d.view(np.float16), M, K)).all()
    blocks = torch.from_numpy(o.to_aos(fmt, q, d.view(np.float16))).to(DEV)
    t_aos = qg.tile_weights(fmt, blocks=blocks).cpu().numpy()
    assert (t_aos == t_soa).all()


TILED_SHAPES = [
    (1, 32, 1), (5, 96, 2), (17, 800, 3), (33, 1024, 16), (1000, 11008, 8), (300, 4000, 9),
    (2048, 4096, 1), (4099, 8192, 16), (64, 16384, 4), (700, 4096, 40),
]


@pytest.mark.parametrize("fmt", ["q8_0", "q4_0"])
@pytest.mark.parametrize("M,K,N", TILED_SHAPES)
def test_tiled_gemv(fmt, M, K, N):
    q, d, X = make(fmt, M, K, N, seed=M * 3 + K + N)
    qt, dt = planes(q, d)
    Wm = qg.QuantizedMatrix(fmt, M, K, "soa", q=qt, d=dt).to_tiled()
    Xt = torch.from_numpy(X).to(DEV)
    Y = Wm.matvec(Xt if N > 1 else Xt[0])
    check(fmt, q, d, X, Y.cpu().numpy())
    # per-stream workspace (NULL) gives the same bits
    Y2 = torch.empty((N, M), device=DEV)
    _lib.call("qgemv_tiled_gemv", FMT_ID[fmt], Wm.tiled.data_ptr(), M, K, Xt.data_ptr(),
              Y2.data_ptr(), N, K, M, None, 0, torch.cuda.current_stream().cuda_stream)
    torch.cuda.synchronize()
    assert torch.equal(Y.reshape(N, M), Y2)


@pytest.mark.parametrize("fmt", ["q8_0", "q4_0"])
@pytest.mark.parametrize("M,N", [(2000, 12), (4099, 3), (300, 16), (129, 5)])
def test_soa_batch_matches_tc_tiles(fmt, M, N):
    """Batched SoA calls of 3..16 columns run the tcgen05 kernel straight from
    the planes (2-D tensor copies, 128-byte swizzle): the same smem image as
    the tc tiles and the same arithmetic in the same order, so identical bits.
    (Two columns run the TMA pair kernel: tests/test_pair_gpu.py.)"""
    K = 8192
    q, d, X = make(fmt, M, K, N, seed=77 + M)
    qt, dt = planes(q, d)
    Xt = torch.from_numpy(X).to(DEV)
    Ys = qg.qgemv(fmt, qt, dt, Xt)
    Yc = qg.qgemv_tc(qg.tile_weights_tc(q=qt, d=dt, fmt=fmt), M, K, Xt, fmt=fmt)
    assert torch.equal(Ys, Yc)
    check(fmt, q, d, X, Ys.cpu().numpy())


@pytest.mark.parametrize("fmt", ["q8_0", "q4_0"])
def test_tiled_matches_static_ws_batch(fmt):
    """Where the tcgen05 workspace does not fit its 2 MiB array (here 12
    columns: 2.4 MB of partial sums on 148 SMs), the static-workspace entry
    runs the mma.sync kernel: on SoA planes it gives the same bits as the
    same kernel on batch tiles."""
    M, K, N = 2000, 8192, 12
    q, d, X = make(fmt, M, K, N, seed=77)
    qt, dt = planes(q, d)
    Xt = torch.from_numpy(X).to(DEV)
    Ys = torch.empty((N, M), device=DEV)
    _lib.call("qgemv_soa_static_ws", FMT_ID[fmt], qt.data_ptr(), dt.data_ptr(), Xt.data_ptr(),
              Ys.data_ptr(), M, K, N, K, M, torch.cuda.current_stream().cuda_stream)
    Yt = qg.qgemv_tiled(fmt, qg.tile_weights(fmt, q=qt, d=dt), M, K, Xt)
    assert torch.equal(Ys, Yt)
