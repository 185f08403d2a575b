"""Two columns per launch on the TMA path (N == 2: one weight stream for both
columns, dp4a on each column's x planes), through the C ABI: q4_0 on SoA
planes and both formats on GGUF blocks (q8_0 planes stay on the tcgen05
kernel, which is faster there).  Every column equals a one-column call on the
same input bit for bit (the same per-block integer dots, the same scale form,
the same reduction tree), and every checked row is within the float64
oracle's bounds (|y - y_ref| <= 1e-5 ||w_row|| ||x|| and the reference gate
max|err| / max|y_ref| <= 1e-5, tests/test_correctness.py:21 of the
reference).  Calls that the pair kernel does not take (x columns not 16 bytes
apart) still run, on the other batch kernels."""

import numpy as np
import pytest
import torch

from qgemv_roofline_b200 import _lib
from oracle import qformats_oracle as o

pytestmark = pytest.mark.gpu
DEV = "cuda"
TOL = 1e-5
# (format, layout) of the calls the pair kernel takes
TAKEN = [("q4_0", "soa"), ("q8_0", "aos"), ("q4_0", "aos")]


def make(fmt, M, K, seed):
    rng = np.random.default_rng(seed)
    W = (rng.standard_normal((M, K)) * 0.02).astype(np.float32)
    X = rng.standard_normal((2, K)).astype(np.float32)
    q, d = o.quantize(fmt, W)
    return q, d, X


class Weights:
    """One matrix on the device as SoA planes or GGUF blocks, called through
    the C ABI's plain entry points (no workspace passed)."""

    def __init__(self, fmt, layout, q, d):
        self.fmt, self.layout = fmt, layout
        self.M, self.K = q.shape[0], d.shape[1] * 32
        if layout == "soa":
            self.q = torch.from_numpy(np.ascontiguousarray(q)).to(DEV)
            self.d = torch.from_numpy(np.ascontiguousarray(d.view(np.float16))).to(DEV)
        else:
            self.blocks = torch.from_numpy(o.to_aos(fmt, q, d.view(np.float16))).to(DEV)

    def call(self, x_ptr, Y, ncols, ldx, ldy, stream=None):
        st = torch.cuda.current_stream().cuda_stream if stream is None else stream
        if self.layout == "soa":
            fn = "qgemv_q8_0_soa" if self.fmt == "q8_0" else "qgemv_q4_0_soa"
            _lib.call(fn, self.q.data_ptr(), self.d.data_ptr(), x_ptr, Y.data_ptr(), self.M,
                      self.K, ncols, ldx, ldy, st)
        else:
            fn = "qgemv_q8_0_aos" if self.fmt == "q8_0" else "qgemv_q4_0_aos"
            _lib.call(fn, self.blocks.data_ptr(), x_ptr, Y.data_ptr(), self.M, self.K, ncols,
                      ldx, ldy, st)

    def pair(self, Xt, ldx=None, ldy=None, Y=None):
        ldx = self.K if ldx is None else ldx
        ldy = self.M if ldy is None else ldy
        if Y is None:
            Y = torch.full((2, ldy), float("nan"), device=DEV)
        self.call(Xt.data_ptr(), Y, 2, ldx, ldy)
        return Y

    def single(self, x):
        y = torch.empty(self.M, device=DEV)
        self.call(x.data_ptr(), y, 1, self.K, self.M)
        return y


def check(fmt, q, d, X, Y, rows=None):
    Y = np.asarray(Y, np.float64).reshape(X.shape[0], -1)
    if rows is not None:
        q, d, Y = q[rows], d[rows], Y[:, rows]
    y_ref = o.matvec_ref(fmt, q, d, X)
    wn = o.row_norms(fmt, q, d)
    ok, worst = o.check_rowwise(Y, y_ref, wn, X, TOL)
    assert ok, f"row-wise bound exceeded: worst ratio {worst:.3g}"
    ok, _, rel = o.check_gate(Y, y_ref, TOL)
    assert ok, f"reference gate exceeded: {rel:.3g}"


def sample_rows(M):
    if M <= 6000:
        return None
    rng = np.random.default_rng(M)
    return np.unique(np.concatenate([np.arange(64), np.arange(M - 64, M),
                                     rng.integers(0, M, 512)]))


# (M, K): tiny and ragged row counts, the smallest and largest K of the TMA
# path, the 7B down-projection K, and matrices on both sides of the
# one-CTA-per-SM switch (150 MB of q4_0, 256 MB of q8_0)
SHAPES = [(16, 256), (1, 256), (37, 768), (4099, 4096), (3001, 8192), (257, 11008),
          (700, 16384), (28672, 4096), (70000, 4096)]


@pytest.mark.parametrize("fmt,layout", TAKEN)
@pytest.mark.parametrize("M,K", SHAPES)
def test_pair_equals_single_columns(fmt, layout, M, K):
    q, d, X = make(fmt, M, K, seed=M + 3 * K)
    W = Weights(fmt, layout, q, d)
    Xt = torch.from_numpy(X).to(DEV)
    Y = W.pair(Xt)
    y0, y1 = W.single(Xt[0]), W.single(Xt[1])
    torch.cuda.synchronize()
    assert torch.equal(Y[0], y0) and torch.equal(Y[1], y1)
    check(fmt, q, d, X, Y.cpu().numpy(), rows=sample_rows(M))
    assert _lib.lib().qgemv_check_device_error(0, None) == 0


@pytest.mark.parametrize("M,K", [(4099, 4096), (28672, 8192)])
def test_q8_0_planes_two_columns(M, K):
    """q8_0 planes at two columns run the tcgen05 kernel: within the bounds."""
    q, d, X = make("q8_0", M, K, seed=5 * M + K)
    W = Weights("q8_0", "soa", q, d)
    Y = W.pair(torch.from_numpy(X).to(DEV))
    torch.cuda.synchronize()
    check("q8_0", q, d, X, Y.cpu().numpy(), rows=sample_rows(M))


@pytest.mark.parametrize("fmt,layout", TAKEN)
def test_pair_strided_columns(fmt, layout):
    """x columns ldx apart: 16-byte multiples take the pair kernel (same bits
    as one-column calls), others the other batch kernels (within the bounds);
    y columns ldy apart, the rows between them untouched."""
    M, K = 3000, 4096
    q, d, X = make(fmt, M, K, seed=11)
    W = Weights(fmt, layout, q, d)
    Xt = torch.from_numpy(X).to(DEV)
    ref = torch.stack([W.single(Xt[0]), W.single(Xt[1])])
    for ldx, ldy in ((K + 64, M + 5), (K + 1, M), (K + 6, M + 1)):
        buf = torch.zeros((2, ldx), device=DEV)
        buf[:, :K] = Xt
        Y = torch.full((2, ldy), 7.0, device=DEV)
        W.pair(buf, ldx, ldy, Y)
        torch.cuda.synchronize()
        assert (Y[:, M:] == 7.0).all()
        if ldx % 4 == 0:
            assert torch.equal(Y[:, :M], ref)
        check(fmt, q, d, X, Y[:, :M].cpu().numpy())


@pytest.mark.parametrize("fmt,layout", TAKEN)
def test_pair_dependent_chain_and_graph(fmt, layout):
    """Each call's x is the previous call's y (a square matrix): launched back
    to back (programmatic dependent launch) the chain matches the one with a
    sync after every call; then one call captured in a CUDA graph on a stream
    that never ran a batched call (the pair kernel needs no workspace) and
    replayed."""
    M = K = 4096
    q, d, X = make(fmt, M, K, seed=21)
    W = Weights(fmt, layout, q, d)
    x0 = torch.from_numpy(X).to(DEV)
    sync_chain = [x0] + [torch.empty((2, M), device=DEV) for _ in range(4)]
    for i in range(4):
        W.pair(sync_chain[i], Y=sync_chain[i + 1])
        torch.cuda.synchronize()
    chain = [x0] + [torch.empty((2, M), device=DEV) for _ in range(4)]
    for i in range(4):
        W.pair(chain[i], Y=chain[i + 1])
    torch.cuda.synchronize()
    for i in range(1, 5):
        assert torch.equal(chain[i], sync_chain[i])
    s = torch.cuda.Stream()
    Yg = torch.empty((2, M), device=DEV)
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=s):
        W.call(x0.data_ptr(), Yg, 2, K, M, stream=s.cuda_stream)
    for _ in range(3):
        Yg.zero_()
        g.replay()
        torch.cuda.synchronize()
        assert torch.equal(Yg, sync_chain[1])
    del g
    assert _lib.lib().qgemv_check_device_error(0, None) == 0


@pytest.mark.parametrize("fmt,layout", TAKEN)
def test_pair_non_finite_column(fmt, layout):
    """A non-finite value in one column makes that column's y NaN and leaves
    the other column within the bounds (the pair then takes the general scale
    form for both)."""
    M, K = 1000, 2048
    q, d, X = make(fmt, M, K, seed=31)
    X[1, 77] = np.inf
    W = Weights(fmt, layout, q, d)
    Y = W.pair(torch.from_numpy(X).to(DEV))
    torch.cuda.synchronize()
    Yh = Y.cpu().numpy()
    assert np.isnan(Yh[1]).all()
    check(fmt, q, d, X[:1], Yh[:1])


@pytest.mark.parametrize("fmt,layout", TAKEN)
@pytest.mark.parametrize("s0,s1", [(1e-35, 1.0), (1.0, 3e30), (0.0, 1.0), (2.0 ** -100, 2.0 ** 60)])
def test_pair_extreme_column_scales(fmt, layout, s0, s1):
    """Columns of very different magnitude (tiny, huge, all zero) in one pair
    call: each within the bounds of its own column."""
    M, K = 640, 2048
    q, d, X = make(fmt, M, K, seed=41)
    X[0] *= np.float32(s0)
    X[1] *= np.float32(s1)
    W = Weights(fmt, layout, q, d)
    Y = W.pair(torch.from_numpy(X).to(DEV))
    torch.cuda.synchronize()
    Yh = Y.cpu().numpy()
    if s0 == 0.0:
        assert (Yh[0] == 0).all()
    check(fmt, q, d, X, Yh)
