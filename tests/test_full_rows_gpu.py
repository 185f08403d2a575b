"""Every row of the timed configurations against the float64 reference.

The benchmark times the single-column kernels at W [98304, 4096] (SoA planes
and GGUF blocks), the batch-tile and SoA-plane tensor-core kernels at
W [28672, 8192] with 16 columns, two columns there (SoA planes and GGUF
blocks), and the 7B decode layer.  Here every output
row of those calls is compared with the reference's float64 dequant-matvec
(src/bench.cu:75-111: the reference's own C++ built into oracle/_ref, run on
all host threads; the numpy restatement in chunks when it was not built),
under both tolerances: the per-row bound |y - y_ref| <= 1e-5 ||w_row|| ||x||
and the reference gate max|y - y_ref| / max|y_ref| <= 1e-5
(tests/test_correctness.py:21 of the reference).  The GPU-quantized bytes of
every row are compared with the reference quantizers too.
"""

import os

import numpy as np
import pytest
import torch

import qgemv_roofline_b200 as qg
from oracle import qformats_oracle as o
from oracle import ref_lib

pytestmark = pytest.mark.gpu
DEV = "cuda"
TOL = 1e-5
CHUNK = 4096  # rows per numpy chunk (bounded host memory)


def _threads():
    return len(os.sched_getaffinity(0)) if hasattr(os, "sched_getaffinity") else os.cpu_count()


def ref_all_rows(fmt, q, d, X):
    """float64 y_ref [N, M] and ||w_row|| [M] over every row of SoA planes q, d
    (numpy) for activations X [N, K]."""
    M = q.shape[0]
    X = np.atleast_2d(np.asarray(X, np.float32))
    wn = np.empty(M)
    for r0 in range(0, M, CHUNK):
        wn[r0:r0 + CHUNK] = o.row_norms(fmt, q[r0:r0 + CHUNK], d[r0:r0 + CHUNK])
    if ref_lib.load() is not None:
        plan = ref_lib.Plan(fmt, o.to_aos(fmt, q, d), _threads())
        Y = np.stack([plan.run(x).copy() for x in X])
        plan.close()
    else:
        Y = np.empty((X.shape[0], M))
        for r0 in range(0, M, CHUNK):
            Y[:, r0:r0 + CHUNK] = o.matvec_ref(fmt, q[r0:r0 + CHUNK], d[r0:r0 + CHUNK], X)
    return Y, wn


def assert_all_rows(Y, y_ref, wn, X, what):
    Y = np.asarray(Y, np.float64).reshape(y_ref.shape)
    ok, worst = o.check_rowwise(Y, y_ref, wn, np.atleast_2d(X), TOL)
    assert ok, f"{what}: row-wise bound exceeded, worst ratio {worst:.3g}"
    ok, _, rel = o.check_gate(Y, y_ref, TOL)
    assert ok, f"{what}: reference gate exceeded, max_rel {rel:.3g}"
    return worst


def gpu_weights(fmt, M, K, seed):
    g = torch.Generator(device=DEV).manual_seed(seed)
    W = torch.randn(M, K, generator=g, device=DEV) * 0.02
    x = torch.randn(2, K, generator=g, device=DEV)
    return W, x


def check_bytes_every_row(fmt, W, q, d):
    """GPU-quantized planes equal the reference quantizer's bytes on every row."""
    Wh = W.cpu().numpy()
    qh, dh = q.cpu().numpy(), d.cpu().numpy()
    for r0 in range(0, Wh.shape[0], 16384):
        sl = slice(r0, r0 + 16384)
        if ref_lib.load() is not None:
            qo, do = o.from_aos(fmt, ref_lib.quantize_aos(fmt, Wh[sl]))
        else:
            qo, do = o.quantize(fmt, Wh[sl])
        assert np.array_equal(qh[sl].view(np.uint8), qo.view(np.uint8)), f"quants differ near row {r0}"
        assert np.array_equal(dh[sl].view(np.uint16), do.view(np.uint16)), f"scales differ near row {r0}"
    return qh, dh.view(np.float16)


@pytest.mark.parametrize("fmt", ["q8_0", "q4_0"])
def test_xl_98304x4096_every_row(fmt):
    """The headline shape: the dispatched single-column kernels on SoA planes
    and on GGUF blocks, every row, and linearity y(a x1 + b x2) = a y(x1) +
    b y(x2) per row within the same bound (no slack)."""
    M, K = 98304, 4096
    W, xs = gpu_weights(fmt, M, K, seed=2024 + (fmt == "q4_0"))
    q, d = (qg.quantize_q8_0 if fmt == "q8_0" else qg.quantize_q4_0)(W)
    qh, dh = check_bytes_every_row(fmt, W, q, d)
    del W
    x1, x2 = xs[0], xs[1]
    x12 = 0.5 * x1 + 2.0 * x2
    X = torch.stack([x1, x2, x12]).cpu().numpy()
    y_ref, wn = ref_all_rows(fmt, qh, dh, X)

    ys = [qg.qgemv(fmt, q, d, x) for x in (x1, x2, x12)]
    for i, y in enumerate(ys):
        assert_all_rows(y.cpu().numpy()[None, :], y_ref[i:i + 1], wn, X[i], f"SoA x{i}")
    blocks = qg.to_aos(fmt, q, d)
    for i, x in enumerate((x1, x2, x12)):
        ya = qg.qgemv_aos(fmt, blocks, x)
        assert_all_rows(ya.cpu().numpy()[None, :], y_ref[i:i + 1], wn, X[i], f"GGUF blocks x{i}")
    # linearity per row: each of the three outputs is within the bound of its
    # own input, so their combination is within the sum of the three bounds
    y1, y2, y12 = (y.double().cpu().numpy() for y in ys)
    lin = np.abs(y12 - (0.5 * y1 + 2.0 * y2))
    xn = np.sqrt((X.astype(np.float64) ** 2).sum(axis=1))
    bound = TOL * wn * (xn[2] + 0.5 * xn[0] + 2.0 * xn[1])
    assert (lin <= bound).all(), f"linearity: worst ratio {(lin / bound).max():.3g}"
    qg._lib.call("qgemv_check_device_error", 0, None)


@pytest.mark.parametrize("fmt", ["q8_0", "q4_0"])
def test_small_batch_28672x8192_every_row(fmt):
    """W [28672, 8192] with 16 columns: the batch-tile kernel and the SoA-plane
    kernel, every row and column; then 5 columns (a partial column group) on
    the batch tiles; and the tcgen05 kernel on tc tiles at 16, 8, 4, 2 and 1
    columns (the paths the small-batch benchmark reports)."""
    M, K, N = 28672, 8192, 16
    g = torch.Generator(device=DEV).manual_seed(4 + (fmt == "q4_0"))
    W = torch.randn(M, K, generator=g, device=DEV) * 0.02
    X = torch.randn(N, K, generator=g, device=DEV)
    q, d = (qg.quantize_q8_0 if fmt == "q8_0" else qg.quantize_q4_0)(W)
    qh, dh = check_bytes_every_row(fmt, W, q, d)
    del W
    Xh = X.cpu().numpy()
    y_ref, wn = ref_all_rows(fmt, qh, dh, Xh)
    tiles = qg.tile_weights(fmt, q=q, d=d)
    Yt = qg.qgemv_tiled(fmt, tiles, M, K, X)
    assert_all_rows(Yt.cpu().numpy(), y_ref, wn, Xh, "batch tiles, 16 columns")
    Ys = qg.qgemv(fmt, q, d, X)
    assert_all_rows(Ys.cpu().numpy(), y_ref, wn, Xh, "SoA planes, 16 columns")
    # two columns: SoA planes (q4_0: the TMA pair kernel; q8_0: tcgen05) and
    # GGUF blocks (the TMA pair kernel)
    Yp = qg.qgemv(fmt, q, d, X[6:8])
    assert_all_rows(Yp.cpu().numpy(), y_ref[6:8], wn, Xh[6:8], "SoA planes, 2 columns")
    Ya = qg.qgemv_aos(fmt, qg.to_aos(fmt, q, d), X[6:8])
    assert_all_rows(Ya.cpu().numpy(), y_ref[6:8], wn, Xh[6:8], "GGUF blocks, 2 columns")
    if fmt == "q4_0":
        assert torch.equal(Ya, Yp)  # the same kernel arithmetic on the same rows
    del Ya
    Y2 = qg.qgemv_tiled(fmt, tiles, M, K, 2.0 * X)
    assert torch.equal(Y2, 2.0 * Yt)  # power-of-two scaling is exact end to end
    Y5 = qg.qgemv_tiled(fmt, tiles, M, K, X[3:8])
    assert_all_rows(Y5.cpu().numpy(), y_ref[3:8], wn, Xh[3:8], "batch tiles, 5 columns")
    # the tcgen05 kernel on tc tiles: 16, 8, 4, 2 and 1 columns (every
    # configuration of its TMEM rings), every row
    del tiles
    tc = qg.tile_weights_tc(q=q, d=d, fmt=fmt)
    for n0, n1 in ((0, 16), (3, 11), (5, 9), (8, 10), (15, 16)):
        Yc = qg.qgemv_tc(tc, M, K, X[n0:n1] if n1 - n0 > 1 else X[n0], fmt=fmt)
        assert_all_rows(Yc.cpu().numpy(), y_ref[n0:n1], wn, Xh[n0:n1],
                        f"tc tiles, {n1 - n0} columns")
    qg._lib.call("qgemv_check_device_error", 0, None)


@pytest.mark.parametrize("fmt", ["q8_0", "q4_0"])
def test_7b_layer_every_row(fmt):
    """One full decode layer of the stack configuration (QKV 12288x4096,
    O 4096x4096, gate+up 22016x4096, down 4096x11008): every row of every
    GEMV, each checked on the input that GEMV actually received."""
    from qgemv_roofline_b200 import stack
    st = stack.DecodeStack.from_random(fmt, n_layers=1, seed=5, device=DEV, keep_full=True)
    x = torch.randn(4096, device=DEV, generator=torch.Generator(device=DEV).manual_seed(8))
    trace = []
    st(x, trace=trace)
    assert len(trace) == 4
    for (m, xin, yout), (q, d) in zip(trace, st.full):
        Xh = xin.cpu().numpy()[None, :].astype(np.float32)
        y_ref, wn = ref_all_rows(fmt, q.cpu().numpy(), d.cpu().numpy(), Xh)
        assert_all_rows(yout.cpu().numpy()[None, :], y_ref, wn, Xh, f"{m.name} [{m.M}, {m.K}]")
