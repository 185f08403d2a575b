"""q8_0 / q4_0 batch GEMV on the tcgen05 tensor cores (tc tiles) on the GPU, through
the C ABI: the tile layout byte for byte against a numpy restatement, every
row of Y against the float64 oracle within |y - y_ref| <= 1e-5 ||w_row|| ||x||
and the reference gate max|err| / max|y_ref| <= 1e-5 (tests/test_correctness.py:21
of the reference), at shapes where one CTA owns whole row tiles, where many
CTAs share one row tile (the partial sums added by the last CTA), ragged M and
K, 1..40 columns, extreme and non-finite column scales, strided x / y, graph
capture and run-to-run determinism."""

import numpy as np
import pytest
import torch

import qgemv_roofline_b200 as qg
from qgemv_roofline_b200 import _lib
from oracle import qformats_oracle as o

pytestmark = pytest.mark.gpu
TOL = 1e-5
DEV = "cuda"
ERR_ARG = 7
FMT_ID = {"q8_0": 8, "q4_0": 4}


def make(M, K, N, seed, scale=0.02, fmt="q8_0"):
    rng = np.random.default_rng(seed)
    W = (rng.standard_normal((M, K)) * scale).astype(np.float32)
    X = rng.standard_normal((N, K)).astype(np.float32)
    q, d = o.quantize(fmt, W)
    return q, d, X


def planes(q, d):
    return (torch.from_numpy(np.ascontiguousarray(q)).to(DEV),
            torch.from_numpy(np.ascontiguousarray(d.view(np.float16))).to(DEV))


def check(q, d, X, Y, tol=TOL, fmt="q8_0"):
    Y = np.asarray(Y, np.float64).reshape(X.shape[0], -1)
    y_ref = o.matvec_ref(fmt, q, d, X)
    wn = o.row_norms(fmt, q, d)
    ok, worst = o.check_rowwise(Y, y_ref, wn, X, tol)
    assert ok, f"row-wise bound exceeded: worst ratio {worst:.3g}"
    ok, _, rel = o.check_gate(Y, y_ref, tol)
    assert ok, f"reference gate exceeded: {rel:.3g}"
    return worst


def tc_tiles_np(q, d, M, K, fmt="q8_0"):
    """numpy restatement of the tc tile layout (qgemv_tc_tile)."""
    KT, RT = 256, 128
    nkt, nrt = -(-K // KT), -(-M // RT)
    dp = np.zeros((nrt * RT, nkt * 8), np.uint16)
    dp[:M, :K // 32] = d.view(np.uint16).reshape(M, K // 32)
    if fmt == "q8_0":
        qp = np.zeros((nrt * RT, nkt * KT), np.uint8)
        qp[:M, :K] = q.view(np.uint8).reshape(M, K)
    else:  # q4_0: 16 nibble bytes per block
        qp = np.zeros((nrt * RT, nkt * KT // 2), np.uint8)
        qp[:M, :K // 2] = q.view(np.uint8).reshape(M, K // 2)
    out = []
    for t in range(nrt):
        for kt in range(nkt):
            if fmt == "q8_0":
                rows = qp[RT * t:RT * (t + 1), kt * KT:(kt + 1) * KT]
                box = np.zeros((2, RT, 8, 16), np.uint8)
                for bx in range(2):
                    for r in range(RT):
                        for c in range(8):
                            box[bx, r, c ^ (r & 7)] = rows[r, bx * 128 + 16 * c:bx * 128 + 16 * c + 16]
                out.append(box.reshape(-1))
            else:
                rows = qp[RT * t:RT * (t + 1), kt * KT // 2:(kt + 1) * KT // 2]
                out.append(rows.reshape(RT, 8, 16).transpose(1, 0, 2).reshape(-1))  # [block][row]
            out.append(dp[RT * t:RT * (t + 1), kt * 8:(kt + 1) * 8].reshape(-1).view(np.uint8))
    return np.concatenate(out)


@pytest.mark.parametrize("fmt", ["q8_0", "q4_0"])
@pytest.mark.parametrize("M,K", [(1, 32), (130, 288), (256, 512)])
def test_tc_tile_layout_bytes(fmt, M, K):
    q, d, _ = make(M, K, 1, seed=M + K, fmt=fmt)
    qt, dt = planes(q, d)
    t_soa = qg.tile_weights_tc(q=qt, d=dt, fmt=fmt).cpu().numpy()
    assert t_soa.size == _lib.lib().qgemv_tc_bytes(FMT_ID[fmt], M, K)
    assert (t_soa == tc_tiles_np(q, d.view(np.float16), M, K, fmt)).all()
    blocks = torch.from_numpy(o.to_aos(fmt, q, d.view(np.float16))).to(DEV)
    assert (qg.tile_weights_tc(blocks=blocks, fmt=fmt).cpu().numpy() == t_soa).all()


TC_SHAPES = [
    (1, 32, 1), (5, 96, 2), (17, 800, 3), (128, 256, 4), (129, 512, 16), (300, 4000, 9),
    (1000, 11008, 8), (2048, 4096, 1), (4099, 8192, 16), (64, 16384, 5), (700, 4096, 40),
    (28672, 8192, 8), (11008, 4096, 16), (4096, 11008, 2), (333, 2304, 12), (8192, 1024, 7),
]


@pytest.mark.parametrize("fmt", ["q8_0", "q4_0"])
@pytest.mark.parametrize("M,K,N", TC_SHAPES)
def test_tc_gemv(fmt, M, K, N):
    q, d, X = make(M, K, N, seed=M * 7 + K + N, fmt=fmt)
    qt, dt = planes(q, d)
    Wm = qg.QuantizedMatrix(fmt, M, K, "soa", q=qt, d=dt).to_tc()
    Xt = torch.from_numpy(X).to(DEV)
    Y = Wm.matvec(Xt if N > 1 else Xt[0])
    torch.cuda.synchronize()
    _lib.call("qgemv_check_device_error", 0, None)
    check(q, d, X, Y.cpu().numpy(), fmt=fmt)
    # the per-stream workspace (NULL) gives the same bits, and so does a rerun
    Y2 = torch.empty((N, M), device=DEV)
    _lib.call("qgemv_tc_gemv", FMT_ID[fmt], Wm.tiled.data_ptr(), M, K, Xt.data_ptr(),
              Y2.data_ptr(), N, K, M, None, 0, torch.cuda.current_stream().cuda_stream)
    torch.cuda.synchronize()
    assert torch.equal(Y.reshape(N, M), Y2)


@pytest.mark.parametrize("fmt", ["q8_0", "q4_0"])
def test_tc_from_ggml_blocks_and_graph_capture(fmt):
    M, K, N = 3000, 4096, 6
    q, d, X = make(M, K, N, seed=5, fmt=fmt)
    blocks = torch.from_numpy(o.to_aos(fmt, q, d.view(np.float16))).to(DEV)
    Wm = qg.QuantizedMatrix(fmt, M, K, "aos", blocks=blocks).to_tc()
    Xt = torch.from_numpy(X).to(DEV)
    Y0 = Wm.matvec(Xt).clone()
    check(q, d, X, Y0.cpu().numpy(), fmt=fmt)
    # captured in a CUDA graph (workspace from the caching allocator) and replayed
    Y = torch.empty((N, M), device=DEV)
    Wm.matvec(Xt, Y)
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        Wm.matvec(Xt, Y)
    Y.zero_()
    for _ in range(3):
        g.replay()
    torch.cuda.synchronize()
    assert torch.equal(Y, Y0)


@pytest.mark.parametrize("fmt", ["q8_0", "q4_0"])
def test_tc_extreme_scales_zero_and_non_finite(fmt):
    M, K, N = 640, 2048, 8
    q, d, X = make(M, K, N, seed=9, fmt=fmt)
    X[1] *= np.float32(1e-35)
    X[2] *= np.float32(3e30)
    X[3] = 0.0
    X[4, ::7] = 0.0
    X[5] *= np.float32(2.0 ** -140)   # subnormal column
    X[6, 100] = np.inf
    X[7, 5] = np.nan
    qt, dt = planes(q, d)
    tiles = qg.tile_weights_tc(q=qt, d=dt, fmt=fmt)
    Y = qg.qgemv_tc(tiles, M, K, torch.from_numpy(X).to(DEV), fmt=fmt).cpu().numpy()
    assert np.isnan(Y[6]).all() and np.isnan(Y[7]).all()
    assert (Y[3] == 0).all()
    good = [0, 1, 2, 3, 4]
    check(q, d, X[good], Y[good], fmt=fmt)
    Xs = X[5:6].astype(np.float64) * 2.0 ** 140
    y_ref = o.matvec_ref(fmt, q, d, Xs.astype(np.float32))[0] * 2.0 ** -140
    wn = o.row_norms(fmt, q, d)
    bound = 1e-5 * wn * np.linalg.norm(X[5].astype(np.float64)) + 2.0 ** -149 * 4
    assert (np.abs(Y[5] - y_ref) <= bound).all()


def test_tc_strided_x_y_guard_bands():
    M, K, N = 517, 4096, 5
    q, d, X = make(M, K, N, seed=17)
    qt, dt = planes(q, d)
    tiles = qg.tile_weights_tc(q=qt, d=dt)
    ldx, ldy = K + 96, M + 40
    Xb = torch.full((N, ldx), float("nan"), device=DEV)
    Xb[:, :K] = torch.from_numpy(X).to(DEV)
    Yb = torch.full((N, ldy), -7.0, device=DEV)
    _lib.call("qgemv_q8_0_tc", tiles.data_ptr(), M, K, Xb.data_ptr(), Yb.data_ptr(), N, ldx, ldy,
              None, 0, torch.cuda.current_stream().cuda_stream)
    torch.cuda.synchronize()
    Yh = Yb.cpu().numpy()
    assert (Yh[:, M:] == -7.0).all()  # the guard band between rows of Y is untouched
    check(q, d, X, Yh[:, :M])


@pytest.mark.parametrize("fmt", ["q8_0", "q4_0"])
def test_tc_linearity_and_determinism(fmt):
    # x -> 2x doubles y exactly (power-of-two scaling commutes with every
    # rounding step); repeated calls give identical bits
    M, K, N = 28672, 8192, 16
    rng = np.random.default_rng(3)
    if fmt == "q8_0":
        q = rng.integers(-127, 128, size=(M, K), dtype=np.int8)
    else:  # every nibble value, -8 included
        q = rng.integers(0, 256, size=(M, K // 2), dtype=np.uint8)
    d = (rng.random((M, K // 32)) * 1e-3 + 1e-4).astype(np.float16)
    qt = torch.from_numpy(q).to(DEV)
    dt = torch.from_numpy(d).to(DEV)
    tiles = qg.tile_weights_tc(q=qt, d=dt, fmt=fmt)
    Xt = torch.randn(N, K, device=DEV, generator=torch.Generator(device=DEV).manual_seed(2))
    Y1 = qg.qgemv_tc(tiles, M, K, Xt, fmt=fmt).clone()
    Y2 = qg.qgemv_tc(tiles, M, K, 2 * Xt, fmt=fmt)
    assert torch.equal(Y2, 2 * Y1)
    for _ in range(3):
        assert torch.equal(qg.qgemv_tc(tiles, M, K, Xt, fmt=fmt), Y1)
    # every row against the oracle
    check(q, d, Xt.cpu().numpy(), Y1.cpu().numpy(), fmt=fmt)


def test_tc_workspace_contract():
    M, K = 1000, 4096
    q, d, X = make(M, K, 4, seed=1)
    qt, dt = planes(q, d)
    tiles = qg.tile_weights_tc(q=qt, d=dt)
    need = _lib.lib().qgemv_q8_0_tc_workspace_bytes(M, K)
    assert need > 0
    Xt = torch.from_numpy(X).to(DEV)
    Y = torch.empty((4, M), device=DEV)
    small = torch.empty(need - 16, dtype=torch.uint8, device=DEV)
    rc = _lib.lib().qgemv_q8_0_tc(tiles.data_ptr(), M, K, Xt.data_ptr(), Y.data_ptr(), 4, K, M,
                                  small.data_ptr(), small.numel(), None)
    assert rc == ERR_ARG
    ws = torch.empty(need, dtype=torch.uint8, device=DEV)
    _lib.call("qgemv_q8_0_tc", tiles.data_ptr(), M, K, Xt.data_ptr(), Y.data_ptr(), 4, K, M,
              ws.data_ptr(), ws.numel(), torch.cuda.current_stream().cuda_stream)
    torch.cuda.synchronize()
    check(q, d, X, Y.cpu().numpy())
