"""GEMV parity on the GPU: the sm_100a kernels through the C ABI against the
float64 oracle, within the north-star bound |y - y_ref| <= 1e-5 ||w_row|| ||x||
per row and the reference gate max|err| / max|y_ref| <= 1e-5
(tests/test_correctness.py:21 of the reference)."""

import numpy as np
import pytest
import torch

import qgemv_roofline_b200 as qg
from oracle import qformats_oracle as o

pytestmark = pytest.mark.gpu
TOL = 1e-5
DEV = "cuda"


def assert_parity(fmt, q, d, X, Y, tol=TOL):
    """q, d: numpy planes; X: [N, K] numpy; Y: result, [N, M] (or [M])."""
    Y = np.asarray(Y, dtype=np.float64).reshape(X.shape[0], -1)
    y_ref = o.matvec_ref(fmt, q, d, X)
    wn = o.row_norms(fmt, q, d)
    ok, worst = o.check_rowwise(Y, y_ref, wn, X, tol)
    assert ok, f"row-wise bound exceeded: worst ratio {worst:.3g}"
    ok, max_abs, max_rel = o.check_gate(Y, y_ref, tol)
    assert ok, f"reference gate exceeded: max_rel {max_rel:.3g}"
    return max_rel


def to_gpu_planes(fmt, q, d):
    return (torch.from_numpy(np.ascontiguousarray(q)).to(DEV),
            torch.from_numpy(np.ascontiguousarray(d.view(np.float16))).to(DEV))


def make(fmt, M, K, N, seed, scale=0.02):
    rng = np.random.default_rng(seed)
    W = (rng.standard_normal((M, K)) * scale).astype(np.float32)
    X = rng.standard_normal((N, K)).astype(np.float32)
    q, d = o.quantize(fmt, W)
    return q, d, X


@pytest.mark.parametrize("fmt", ["q8_0", "q4_0"])
def test_golden_soa(golden, fmt):
    k = "8" if fmt == "q8_0" else "4"
    for name, g in golden.items():
        q, d = to_gpu_planes(fmt, g["q" + k], g["d" + k])
        X = torch.from_numpy(g["X"]).to(DEV)
        Y = qg.qgemv(fmt, q, d, X).cpu().numpy()
        assert_parity(fmt, g["q" + k], g["d" + k].view(np.float16), g["X"], Y)
        ok, _, rel = o.check_gate(Y, g["y%s_f64" % k])
        assert ok, (name, rel)


@pytest.mark.parametrize("fmt", ["q8_0", "q4_0"])
def test_golden_aos(golden, fmt):
    k = "8" if fmt == "q8_0" else "4"
    for name, g in golden.items():
        blocks = torch.from_numpy(o.to_aos(fmt, g["q" + k], g["d" + k].view(np.float16))).to(DEV)
        X = torch.from_numpy(g["X"]).to(DEV)
        Y = qg.qgemv_aos(fmt, blocks, X).cpu().numpy()
        ok, _, rel = o.check_gate(Y, g["y%s_f64" % k])
        assert ok, (name, rel)


SHAPES = [
    (4096, 4096, 1), (11008, 4096, 1), (2048, 1024, 1),   # reference test shapes
    (1, 32, 1), (3, 96, 2), (7, 96, 3), (257, 1024, 1),   # ragged / tiny
    (1000, 11008, 1), (100, 8192, 1),                      # K not a multiple of 512
    (512, 8192, 2), (384, 8192, 4), (320, 8192, 8), (300, 8192, 16),  # batch, K tiles
    (200, 4096, 5), (130, 2048, 20),                        # N rounded up / > 16
]


@pytest.mark.parametrize("fmt", ["q8_0", "q4_0"])
@pytest.mark.parametrize("M,K,N", SHAPES)
def test_soa_shapes(fmt, M, K, N):
    q, d, X = make(fmt, M, K, N, seed=M * 7 + K + N)
    qt, dt = to_gpu_planes(fmt, q, d)
    Y = qg.qgemv(fmt, qt, dt, torch.from_numpy(X).to(DEV)).cpu().numpy()
    assert_parity(fmt, q, d, X, Y)


@pytest.mark.parametrize("fmt", ["q8_0", "q4_0"])
@pytest.mark.parametrize("M,K,N", [(4096, 4096, 1), (1000, 11008, 1), (5, 96, 3),
                                   (300, 8192, 16), (257, 1024, 2), (130, 2048, 20)])
def test_aos_shapes(fmt, M, K, N):
    q, d, X = make(fmt, M, K, N, seed=M + 3 * K + N)
    blocks = torch.from_numpy(o.to_aos(fmt, q, d)).to(DEV)
    Y = qg.qgemv_aos(fmt, blocks, torch.from_numpy(X).to(DEV)).cpu().numpy()
    assert_parity(fmt, q, d, X, Y)


@pytest.mark.parametrize("fmt", ["q8_0", "q4_0"])
def test_reference_distribution_error(fmt):
    """U(-1, 1) weights and x, the reference's own inputs: the error is of the
    order the reference reports (worst 5.6e-7 relative)."""
    rng = np.random.default_rng(1234)
    W = (rng.random((4096, 4096)) * 2 - 1).astype(np.float32)
    X = (rng.random((1, 4096)) * 2 - 1).astype(np.float32)
    q, d = o.quantize(fmt, W)
    qt, dt = to_gpu_planes(fmt, q, d)
    Y = qg.qgemv(fmt, qt, dt, torch.from_numpy(X).to(DEV)).cpu().numpy()
    rel = assert_parity(fmt, q, d, X, Y)
    assert rel < 2e-6


@pytest.mark.parametrize("fmt", ["q8_0", "q4_0"])
def test_strided_x_y_and_guard_bands(fmt):
    M, K, N = 333, 2048, 3
    q, d, X = make(fmt, M, K, N, seed=9)
    qt, dt = to_gpu_planes(fmt, q, d)
    Xbig = torch.full((N, K + 64), float("nan"), device=DEV)
    Xbig[:, :K] = torch.from_numpy(X).to(DEV)
    canary = -12345.0
    Ybuf = torch.full((N + 2, M + 40), canary, device=DEV)
    Yv = Ybuf[1:N + 1, 8:8 + M]
    qg.qgemv(fmt, qt, dt, Xbig[:, :K], y=Yv)
    torch.cuda.synchronize()
    Yh = Ybuf.cpu().numpy()
    assert_parity(fmt, q, d, X, Yh[1:N + 1, 8:8 + M])
    mask = np.ones_like(Yh, dtype=bool)
    mask[1:N + 1, 8:8 + M] = False
    assert (Yh[mask] == canary).all(), "a write landed outside y"


@pytest.mark.parametrize("fmt", ["q8_0", "q4_0"])
def test_deterministic_and_stream(fmt):
    q, d, X = make(fmt, 5000, 4096, 1, seed=5)
    qt, dt = to_gpu_planes(fmt, q, d)
    x = torch.from_numpy(X[0]).to(DEV)
    s = torch.cuda.Stream()
    with torch.cuda.stream(s):
        y1 = qg.qgemv(fmt, qt, dt, x)
        y2 = qg.qgemv(fmt, qt, dt, x)
    s.synchronize()
    assert torch.equal(y1, y2)
    assert_parity(fmt, q, d, X, y1.cpu().numpy())


def test_k_zero_gives_zeros():
    q = torch.empty((10, 0), dtype=torch.int8, device=DEV)
    d = torch.empty((10, 0), dtype=torch.float16, device=DEV)
    y = torch.full((10,), 7.0, device=DEV)
    qg.qgemv("q8_0", q, d, torch.empty(0, device=DEV), y=y)
    assert torch.count_nonzero(y).item() == 0


@pytest.mark.parametrize("fmt", ["q8_0", "q4_0"])
@pytest.mark.parametrize("M,K", [(1, 256), (5, 4096), (149, 512), (300, 16384), (7, 16384),
                                 (2000, 11008), (1500, 8192), (3001, 4096)])
def test_single_column_tma_shapes(fmt, M, K):
    """Shapes of the TMA-fed kernel (K % 256 == 0): tiny, ragged tiles, the
    largest K, K = 11008 (idle slices), fewer tiles than SMs."""
    q, d, X = make(fmt, M, K, 1, seed=M + K)
    qt, dt = to_gpu_planes(fmt, q, d)
    y = qg.qgemv(fmt, qt, dt, torch.from_numpy(X[0]).to(DEV)).cpu().numpy()
    assert_parity(fmt, q, d, X, y[None, :])
    qg._lib.call("qgemv_check_device_error", 1, None)


@pytest.mark.parametrize("fmt", ["q8_0", "q4_0"])
def test_kernel_ladder_variants(fmt):
    """Every selectable single-column configuration (the --only ladder)."""
    lib = qg._lib.lib()
    M, K = 777, 4096
    q, d, X = make(fmt, M, K, 1, seed=31)
    qt, dt = to_gpu_planes(fmt, q, d)
    x = torch.from_numpy(X[0]).to(DEV)
    ran = 0
    for v in range(lib.qgemv_soa_variant_count()):
        for grid in (0, 3, 400):  # 400 CTAs: more than the matrix has tiles
            y = torch.full((M,), float("nan"), device=DEV)
            rc = lib.qgemv_soa_variant(qg._lib.FORMAT_CODE[fmt], v, grid, qt.data_ptr(),
                                       dt.data_ptr(), x.data_ptr(), y.data_ptr(), M, K, None)
            if rc == 5:  # QGEMV_ERR_UNSUPPORTED: this configuration cannot hold the shape
                continue
            assert rc == 0, qg._lib.last_error()
            assert_parity(fmt, q, d, X, y.cpu().numpy()[None, :])
            ran += 1
    assert ran >= 3 * (lib.qgemv_soa_variant_count() - 1)
    qg._lib.call("qgemv_check_device_error", 1, None)


def test_device_error_word_is_clear():
    qg._lib.call("qgemv_check_device_error", 0, None)


@pytest.mark.parametrize("fmt", ["q8_0", "q4_0"])
def test_back_to_back_dependent_calls(fmt):
    """Six GEMVs in a row on one stream, each reading the previous output and
    overwriting the buffer the previous one read (ping-pong), with no other
    kernel in between: checks the ordering of overlapped launches."""
    K = 2048
    q, d, X = make(fmt, K, K, 1, seed=7, scale=0.02)
    qt, dt = to_gpu_planes(fmt, q, d)
    a = torch.from_numpy(X[0]).to(DEV)
    b = torch.empty_like(a)
    snaps = [a.cpu().numpy()]
    for i in range(6):
        src, dst = (a, b) if i % 2 == 0 else (b, a)
        qg.qgemv(fmt, qt, dt, src, y=dst)
    torch.cuda.synchronize()
    # replay the chain step by step against the oracle
    cur = snaps[0]
    a2 = torch.from_numpy(X[0]).to(DEV)
    b2 = torch.empty_like(a2)
    for i in range(6):
        src, dst = (a2, b2) if i % 2 == 0 else (b2, a2)
        qg.qgemv(fmt, qt, dt, src, y=dst)
        torch.cuda.synchronize()
        out = dst.cpu().numpy()
        assert_parity(fmt, q, d, cur[None, :], out[None, :])
        cur = out
    final = (b if 6 % 2 == 1 else a).cpu().numpy()
    assert np.array_equal(final, cur), "overlapped chain differs from the synchronised one"


@pytest.mark.parametrize("fmt", ["q8_0", "q4_0"])
def test_unaligned_x_and_extreme_scales(fmt):
    M, K = 300, 4096
    q, d, X = make(fmt, M, K, 1, seed=13)
    qt, dt = to_gpu_planes(fmt, q, d)
    buf = torch.zeros(K + 8, device=DEV)
    # (a smaller scale would make y subnormal: no fp32 result could then meet
    # the bound, whose scale is far below the subnormal spacing)
    for scale in (1.0, 1e-35, 3e30):
        xs = (X[0].astype(np.float64) * scale).astype(np.float32)
        buf[1:K + 1] = torch.from_numpy(xs).to(DEV)      # 4-byte aligned only
        y1 = qg.qgemv(fmt, qt, dt, buf[1:K + 1]).cpu().numpy()
        y2 = qg.qgemv(fmt, qt, dt, torch.from_numpy(xs).to(DEV)).cpu().numpy()  # aligned
        for y in (y1, y2):
            assert np.isfinite(y).all()
            assert_parity(fmt, q, d, xs[None, :], y[None, :])


@pytest.mark.parametrize("fmt", ["q8_0", "q4_0"])
def test_non_finite_x_gives_non_finite_y(fmt):
    M, K = 64, 4096
    q, d, X = make(fmt, M, K, 1, seed=17)
    qt, dt = to_gpu_planes(fmt, q, d)
    for bad in (float("inf"), float("nan")):
        xs = X[0].copy()
        xs[100] = bad
        y = qg.qgemv(fmt, qt, dt, torch.from_numpy(xs).to(DEV)).cpu().numpy()
        assert not np.isfinite(y).any()


def test_sharded_wrapper_single_process():
    """ShardedQGemv without a process group: one shard holding every row."""
    from qgemv_roofline_b200.shard import ShardedQGemv
    M, K = 513, 2048
    q, d, X = make("q8_0", M, K, 2, seed=23)
    qt, dt = to_gpu_planes("q8_0", q, d)
    full = qg.QuantizedMatrix("q8_0", M, K, "soa", q=qt, d=dt)
    sh = ShardedQGemv.from_full(full, device=DEV)
    Y = sh(torch.from_numpy(X).to(DEV), gather=True).cpu().numpy()
    assert_parity("q8_0", q, d, X, Y)


@pytest.mark.parametrize("fmt", ["q8_0", "q4_0"])
@pytest.mark.parametrize("N", [1, 3])
def test_scale_plane_2_byte_aligned(fmt, N):
    """A scale plane that starts 2 bytes past a 16-byte boundary: bulk copies
    need 16-byte aligned sources, so these calls run on the register-streaming
    kernels, with the same parity."""
    M, K = 300, 4096
    q, d, X = make(fmt, M, K, N, seed=19 + N)
    qt = torch.from_numpy(q).to(DEV)
    nb = M * K // 32
    dbuf = torch.zeros(nb + 8, dtype=torch.float16, device=DEV)
    dv = dbuf[1:1 + nb].view(M, K // 32)
    dv.copy_(torch.from_numpy(d.view(np.float16)))
    assert dv.data_ptr() % 16 == 2
    Y = qg.qgemv(fmt, qt, dv, torch.from_numpy(X if N > 1 else X[0]).to(DEV)).cpu().numpy()
    assert_parity(fmt, q, d, X, Y)
    qg._lib.call("qgemv_check_device_error", 0, None)
