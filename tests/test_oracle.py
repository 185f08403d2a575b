"""The oracle against the reference's own outputs (CPU only).

Pins oracle/qformats_oracle.py to golden vectors produced by the reference's
python/qformats.py and its C++ quantizers / float64 matvec (src/bench.cu),
then restates the reference's CPU format checks (tests/test_quant_cpu.py)
against the oracle.
"""

import numpy as np
import pytest

from oracle import qformats_oracle as o
from oracle import ref_lib


def test_golden_cases_present(golden):
    assert {"ref_uniform_64x512", "normal_64x1024_n3", "normal_5x11008", "odd_3x96_n2",
            "edge_8x256"} <= set(golden)


@pytest.mark.parametrize("fmt", ["q8_0", "q4_0"])
def test_oracle_quantizer_matches_reference_bytes(golden, fmt):
    key = "8" if fmt == "q8_0" else "4"
    for name, g in golden.items():
        q, d = o.quantize(fmt, g["W"])
        assert np.array_equal(q, g["q" + key]), name
        assert np.array_equal(d.view(np.uint16), g["d" + key]), name


@pytest.mark.parametrize("fmt", ["q8_0", "q4_0"])
def test_oracle_aos_layout_matches_reference_blocks(golden, fmt):
    key = "8" if fmt == "q8_0" else "4"
    for name, g in golden.items():
        if "aos" + key not in g:
            pytest.skip("golden file has no C++ reference blocks")
        q, d = o.quantize(fmt, g["W"])
        blocks = o.to_aos(fmt, q, d)
        assert np.array_equal(blocks, g["aos" + key]), name
        q2, d2 = o.from_aos(fmt, blocks)
        assert np.array_equal(q2, q) and np.array_equal(d2.view(np.uint16), d.view(np.uint16))


@pytest.mark.parametrize("fmt", ["q8_0", "q4_0"])
def test_oracle_matvec_matches_reference_f64(golden, fmt):
    key = "8" if fmt == "q8_0" else "4"
    for name, g in golden.items():
        d = g["d" + key].view(np.float16)
        y = o.matvec_ref(fmt, g["q" + key], d, g["X"])
        ref = g["y%s_f64" % key]
        assert np.allclose(y, ref, rtol=1e-12, atol=1e-12 * np.abs(ref).max()), name
        # the reference's fp32 torch path is inside the reference gate
        ok, _, rel = o.check_gate(g["y%s_f32" % key], ref)
        assert ok, (name, rel)


@pytest.mark.parametrize("fmt", ["q8_0", "q4_0"])
def test_oracle_dequant_matches_reference_fp32_path(golden, fmt):
    """dequant(q, d) @ x in fp32 (the reference's CPU GEMV) within the gate."""
    key = "8" if fmt == "q8_0" else "4"
    for name, g in golden.items():
        d = g["d" + key].view(np.float16)
        Wd = o.dequant(fmt, g["q" + key], d)
        y = np.stack([Wd @ g["X"][n] for n in range(g["X"].shape[0])])
        ok, _, rel = o.check_gate(y, g["y%s_f64" % key])
        assert ok, (name, rel)


@pytest.mark.parametrize("fmt", ["q8_0", "q4_0"])
def test_torch_cpu_dequant_matches_reference(golden, fmt):
    """The torch restatement of the reference's CPU path (the timed CPU
    baseline): dequantized weights equal the numpy oracle's bit for bit, and
    dequant(q, d) @ x agrees with the reference's own torch fp32 outputs."""
    import torch
    key = "8" if fmt == "q8_0" else "4"
    for name, g in golden.items():
        q, d = g["q" + key], g["d" + key].view(np.float16)
        Wt = o.dequant_torch(fmt, torch.from_numpy(q), torch.from_numpy(d))
        assert np.array_equal(Wt.numpy(), o.dequant(fmt, q, d)), name
        y = (Wt @ torch.from_numpy(g["X"]).T).T.numpy()
        ok, _, rel = o.check_gate(y, g["y%s_f32" % key], 1e-6)
        assert ok, (name, rel)


def test_reference_cpu_checks_on_oracle(golden):
    """tests/test_quant_cpu.py:59-110 of the reference, run on the oracle with
    the reference's own input (torch seed 1234, U(-1, 1), [64, 512])."""
    W = golden["ref_uniform_64x512"]["W"]
    M, K = W.shape
    q8, d8 = o.quantize_q8_0(W)
    r8 = o.dequant_q8_0(q8, d8)
    step8 = np.repeat(d8.astype(np.float32), o.QK, axis=1)
    e8 = np.abs(W - r8)
    assert (e8 <= step8 + 1e-6).all()
    assert (e8 <= step8 * 0.5 + 1e-6).mean() > 0.99
    q4, d4 = o.quantize_q4_0(W)
    r4 = o.dequant_q4_0(q4, d4)
    step4 = np.repeat(np.abs(d4.astype(np.float32)), o.QK, axis=1)
    e4 = np.abs(W - r4)
    assert (e4 <= step4 * (1 + 2 ** -8) + 1e-6).all()
    assert int((e4 > step4 * 0.5 + 1e-6).sum()) <= M * (K // o.QK)
    # ggml nibble order: low nibble = weights 0-15, high = 16-31
    p = q4.reshape(M, K // 32, 16).astype(np.int32)
    dd = d4.astype(np.float32)[:, :, None]
    ref = r4.reshape(M, K // 32, 32)
    assert np.allclose(((p & 15) - 8) * dd, ref[:, :, :16], atol=1e-6)
    assert np.allclose(((p >> 4) - 8) * dd, ref[:, :, 16:], atol=1e-6)
    # byte counts
    assert q8.size + d8.size * 2 == M * (K // 32) * 34
    assert q4.size + d4.size * 2 == M * (K // 32) * 18


def test_check_functions_detect_errors():
    y_ref = np.array([1.0, -2.0, 3.0])
    assert o.check_gate(y_ref + 1e-7, y_ref)[0]
    assert not o.check_gate(y_ref + 1e-3, y_ref)[0]
    wn = np.ones(3)
    x = np.ones(4)
    assert o.check_rowwise(y_ref + 1e-6, y_ref, wn, x)[0]
    bad = y_ref.copy()
    bad[1] += 1e-3  # a planted mistake must be caught
    assert not o.check_rowwise(bad, y_ref, wn, x)[0]


@pytest.mark.skipif(ref_lib.load() is None, reason="oracle/_ref not built")
@pytest.mark.parametrize("fmt", ["q8_0", "q4_0"])
def test_oracle_vs_reference_cpp_random(fmt):
    """Broader sweep against the reference's compiled C++ quantizer and matvec."""
    rng = np.random.default_rng(42)
    for M, K, scale in ((7, 96, 1.0), (33, 320, 0.02), (4, 4096, 1e-4), (16, 256, 3e3)):
        W = (rng.standard_normal((M, K)) * scale).astype(np.float32)
        x = rng.standard_normal(K).astype(np.float32)
        q, d = o.quantize(fmt, W)
        blocks = ref_lib.quantize_aos(fmt, W)
        assert np.array_equal(o.to_aos(fmt, q, d), blocks)
        y = o.matvec_ref(fmt, q, d, x)
        ref = ref_lib.matvec(fmt, blocks, x)
        assert np.allclose(y, ref, rtol=1e-12, atol=1e-12 * np.abs(ref).max())
