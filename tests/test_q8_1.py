"""The opt-in q8_1 activation path (x rounded to int8 per 32-element block,
one dp4a set per block).

CPU: the oracle's restatement against a per-element loop, its exact integer
dots, and the bound its rounding of x puts on the distance to the exact
float64 matvec; C-ABI validation.  GPU (marked): the kernels through the C ABI
against the restatement (the same quantized x, so only fp32 rounding of the
block products and of the sums separates them), SoA and GGUF blocks, edge
cases, determinism and graph capture.
"""

import struct

import numpy as np
import pytest

from oracle import qformats_oracle as o
from qgemv_roofline_b200 import _lib

FAKE = 0x100000  # 16-byte aligned, never dereferenced: validation fails first
# fp32 rounding of dw * dx, of its product with the exact block sum, and of the
# sums over blocks (a butterfly across lanes, then KS partials in order)
TOL_Q81 = 2e-6


def _f32(v):
    return struct.unpack("<f", struct.pack("<f", v))[0]


def quantize_x_loop(x):
    """Per-element restatement of quantize_x_q8_1 with Python floats rounded
    to fp32 after every operation."""
    K = len(x)
    q = np.zeros(K, dtype=np.int64)
    dx = np.zeros(K // 32, dtype=np.float64)
    for b in range(K // 32):
        blk = [float(v) for v in x[32 * b:32 * b + 32]]
        amax = max(abs(v) for v in blk)
        idv = _f32(127.0 / amax) if amax > 0 else 0.0
        dx[b] = _f32(amax / 127.0)
        for j, v in enumerate(blk):
            q[32 * b + j] = int(np.rint(_f32(v * idv)))
    return q, dx


@pytest.mark.parametrize("seed", [0, 1, 2])
def test_quantize_x_matches_per_element_loop(seed):
    rng = np.random.default_rng(seed)
    x = (rng.standard_normal(256) * rng.choice([1e-3, 1.0, 50.0])).astype(np.float32)
    x[32:64] = 0.0                                  # an all-zero block
    x[64:96] = np.float32(0.5) * np.sign(x[64:96])  # ties of x * id
    q, dx = o.quantize_x_q8_1(x)
    ql, dxl = quantize_x_loop(x)
    assert np.array_equal(q, ql)
    assert np.array_equal(dx.astype(np.float64), dxl)
    assert np.abs(q).max() <= 127
    blocks = np.abs(q.reshape(-1, 32)).max(axis=1)
    assert blocks[1] == 0 and dx[1] == 0
    assert np.all(blocks[np.arange(8) != 1] == 127)  # the block maximum maps to +-127


@pytest.mark.parametrize("fmt", ["q8_0", "q4_0"])
def test_matvec_q8_1_ref_is_the_integer_dot(fmt):
    rng = np.random.default_rng(7)
    M, K = 5, 128
    W = (rng.standard_normal((M, K)) * 0.02).astype(np.float32)
    x = rng.standard_normal(K).astype(np.float32)
    q, d = o.quantize(fmt, W)
    y = o.matvec_q8_1_ref(fmt, q, d, x)
    xq, dx = quantize_x_loop(x)
    wv = q.astype(np.int64) if fmt == "q8_0" else o.q4_nibbles(q).astype(np.int64) - 8
    for r in range(M):
        acc = 0.0
        for b in range(K // 32):
            s = int(np.dot(wv[r, 32 * b:32 * b + 32], xq[32 * b:32 * b + 32]))
            acc += s * float(d.view(np.float16)[r, b]) * dx[b]
        assert y[r] == pytest.approx(acc, rel=1e-12, abs=1e-300)


@pytest.mark.parametrize("fmt", ["q8_0", "q4_0"])
def test_q8_1_distance_to_exact_is_the_rounding_of_x(fmt):
    """|y_q81 - y_exact| <= sum_b ||w_b||_1 * 0.51 * dx_b (each x_j moves by at
    most half a step of its block, plus fp32 slack), and it is not small."""
    rng = np.random.default_rng(3)
    M, K = 64, 1024
    W = (rng.standard_normal((M, K)) * 0.02).astype(np.float32)
    x = rng.standard_normal(K).astype(np.float32)
    q, d = o.quantize(fmt, W)
    y81 = o.matvec_q8_1_ref(fmt, q, d, x)
    y = o.matvec_ref(fmt, q, d, x)
    _, dx = o.quantize_x_q8_1(x)
    Wd = o.dequant_f64(fmt, q, d)
    bound = (np.abs(Wd).reshape(M, K // 32, 32).sum(axis=2) * 0.51 * dx[None, :]).sum(axis=1)
    assert np.all(np.abs(y81 - y) <= bound)
    wn = o.row_norms(fmt, q, d)
    ok, worst = o.check_rowwise(y81, y, wn, x, 1e-5)
    assert not ok and worst > 10  # far outside the exact path's bound: why it is opt-in


def test_q8_1_entry_validation():
    lib = _lib.lib()
    assert lib.qgemv_soa_q8_1(5, FAKE, FAKE, FAKE, FAKE, 64, 4096, None) == 7   # format
    assert lib.qgemv_soa_q8_1(8, FAKE, FAKE, FAKE, FAKE, 64, 100, None) == 2    # K % 32
    assert lib.qgemv_soa_q8_1(8, None, FAKE, FAKE, FAKE, 64, 4096, None) == 1
    assert lib.qgemv_soa_q8_1(4, FAKE, None, FAKE, FAKE, 64, 4096, None) == 1
    assert lib.qgemv_soa_q8_1(8, FAKE + 8, FAKE, FAKE, FAKE, 64, 4096, None) == 3
    assert lib.qgemv_soa_q8_1(8, FAKE, FAKE, FAKE, FAKE, 64, 4064, None) == 5   # K % 256
    assert lib.qgemv_soa_q8_1(8, FAKE, FAKE, FAKE, FAKE, 64, 32768, None) == 5  # K > 16384
    assert lib.qgemv_soa_q8_1(8, FAKE, FAKE, FAKE + 4, FAKE, 64, 4096, None) == 5  # x not 16-B
    assert lib.qgemv_soa_q8_1(8, None, None, None, None, 0, 4096, None) == 0    # no rows
    assert lib.qgemv_aos_q8_1(4, None, FAKE, FAKE, 64, 4096, None) == 1
    assert lib.qgemv_aos_q8_1(4, FAKE + 2, FAKE, FAKE, 64, 4096, None) == 3
    assert lib.qgemv_aos_q8_1(8, FAKE, FAKE, FAKE, 64, 1000, None) == 2


# ------------------------------------------------------------------------ GPU

def _gpu():
    import torch

    import qgemv_roofline_b200 as qg
    return torch, qg


def _check(fmt, q, d, x, y):
    y_ref = o.matvec_q8_1_ref(fmt, q, d, x)
    wn = o.row_norms(fmt, q, d)
    ok, worst = o.check_rowwise(np.asarray(y, dtype=np.float64), y_ref, wn, x, TOL_Q81)
    assert ok, f"q8_1 kernel vs its restatement: worst ratio {worst:.3g}"
    return y_ref


@pytest.mark.gpu
@pytest.mark.parametrize("fmt", ["q8_0", "q4_0"])
@pytest.mark.parametrize("M,K", [(1, 256), (37, 4096), (4096, 4096), (3001, 11008), (300, 16384)])
def test_q8_1_kernel_matches_restatement(fmt, M, K):
    torch, qg = _gpu()
    rng = np.random.default_rng(M * 7 + K)
    W = (rng.standard_normal((M, K)) * 0.02).astype(np.float32)
    x = rng.standard_normal(K).astype(np.float32)
    q, d = o.quantize(fmt, W)
    qt = torch.from_numpy(np.ascontiguousarray(q)).cuda()
    dt = torch.from_numpy(np.ascontiguousarray(d.view(np.float16))).cuda()
    xt = torch.from_numpy(x).cuda()
    y = qg.qgemv(fmt, qt, dt, xt, activations="q8_1").cpu().numpy()
    _check(fmt, q, d.view(np.float16), x, y)
    blocks = torch.from_numpy(o.to_aos(fmt, q, d.view(np.float16))).cuda()
    ya = qg.qgemv_aos(fmt, blocks, xt, activations="q8_1").cpu().numpy()
    _check(fmt, q, d.view(np.float16), x, ya)
    assert _lib.lib().qgemv_check_device_error(0, None) == 0


@pytest.mark.gpu
@pytest.mark.parametrize("fmt", ["q8_0", "q4_0"])
def test_q8_1_edge_cases(fmt):
    torch, qg = _gpu()
    rng = np.random.default_rng(11)
    M, K = 513, 2048
    W = (rng.standard_normal((M, K)) * 0.02).astype(np.float32)
    q, d = o.quantize(fmt, W)
    m = qg.QuantizedMatrix(fmt, M, K, "soa",
                           q=torch.from_numpy(np.ascontiguousarray(q)).cuda(),
                           d=torch.from_numpy(np.ascontiguousarray(d.view(np.float16))).cuda())
    zero = torch.zeros(K, device="cuda")
    assert torch.count_nonzero(m.matvec(zero, activations="q8_1")).item() == 0
    x = rng.standard_normal(K).astype(np.float32)
    x[:64] = 0.0                                                  # zero blocks
    x[992:1024] = rng.standard_normal(32).astype(np.float32) * 1e-30  # a tiny block
    y = m.matvec(torch.from_numpy(x).cuda(), activations="q8_1").cpu().numpy()
    _check(fmt, q, d.view(np.float16), x, y)
    xh = x.copy()
    xh[100] = 1e30  # a huge element: the rest of its block rounds to 0
    yh = m.matvec(torch.from_numpy(xh).cuda(), activations="q8_1").cpu().numpy()
    _check(fmt, q, d.view(np.float16), xh, yh)
    x[5] = np.inf
    yn = m.matvec(torch.from_numpy(x).cuda(), activations="q8_1").cpu().numpy()
    assert np.isnan(yn).all()
    with pytest.raises(ValueError):
        m.matvec(torch.zeros(2, K, device="cuda"), activations="q8_1")
    k2 = 992  # a multiple of 32 but not of 256: the q8_1 kernel does not take it
    q2 = m.q[:, :k2 if fmt == "q8_0" else k2 // 2].contiguous()
    with pytest.raises(_lib.QGemvError):
        qg.qgemv(fmt, q2, m.d[:, :k2 // 32].contiguous(), torch.zeros(k2, device="cuda"),
                 activations="q8_1")


@pytest.mark.gpu
def test_q8_1_deterministic_and_capturable():
    torch, qg = _gpu()
    rng = np.random.default_rng(5)
    M, K = 8192, 4096
    W = torch.from_numpy((rng.standard_normal((M, K)) * 0.02).astype(np.float32)).cuda()
    m = qg.QuantizedMatrix.from_float(W, "q4_0")
    x = torch.randn(K, device="cuda")
    y1 = m.matvec(x, activations="q8_1").clone()
    y2 = m.matvec(x, activations="q8_1").clone()
    assert torch.equal(y1, y2)
    out = torch.empty(M, device="cuda")
    s = torch.cuda.Stream()
    with torch.cuda.stream(s):
        m.matvec(x, out, activations="q8_1")
    s.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        m.matvec(x, out, activations="q8_1")
    out.zero_()
    g.replay()
    torch.cuda.synchronize()
    assert torch.equal(out, y1)
    del g
