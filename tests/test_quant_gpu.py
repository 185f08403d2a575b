"""GPU quantizer / dequantizer / repack: bit-exact against the reference's
bytes (golden vectors from python/qformats.py) and the oracle."""

import numpy as np
import pytest
import torch

import qgemv_roofline_b200 as qg
from oracle import qformats_oracle as o

pytestmark = pytest.mark.gpu
DEV = "cuda"


def quant(fmt, W):
    return (qg.quantize_q8_0 if fmt == "q8_0" else qg.quantize_q4_0)(W)


@pytest.mark.parametrize("fmt", ["q8_0", "q4_0"])
def test_golden_bytes(golden, fmt):
    k = "8" if fmt == "q8_0" else "4"
    for name, g in golden.items():
        q, d = quant(fmt, torch.from_numpy(g["W"]).to(DEV))
        assert np.array_equal(q.cpu().numpy(), g["q" + k]), name
        assert np.array_equal(d.cpu().numpy().view(np.uint16), g["d" + k]), name
        if "aos" + k in g:
            blocks = (qg.quantize_q8_0_aos if fmt == "q8_0" else qg.quantize_q4_0_aos)(
                torch.from_numpy(g["W"]).to(DEV))
            assert np.array_equal(blocks.cpu().numpy(), g["aos" + k]), name


def distributions():
    rng = np.random.default_rng(77)
    yield "uniform", (rng.random((64, 512)) * 2 - 1).astype(np.float32)
    yield "normal", (rng.standard_normal((128, 1024)) * 0.02).astype(np.float32)
    scales = 10.0 ** rng.uniform(-8, 4, size=(96, 1))
    yield "wide", (rng.standard_normal((96, 256)) * scales).astype(np.float32)
    W = (rng.standard_normal((32, 256)) * 0.5).astype(np.float32)
    W[:, ::3] = 0.0
    W[::2, :32] = 0.0
    yield "zeros", W
    W = np.round(rng.standard_normal((32, 256)) * 4) / 4  # many exact ties
    yield "ties", W.astype(np.float32)
    W = (rng.standard_normal((16, 128)) * 1e-6).astype(np.float32)  # fp16 subnormal / zero d
    yield "tiny", W
    yield "ragged", (rng.standard_normal((7, 96))).astype(np.float32)


@pytest.mark.parametrize("fmt", ["q8_0", "q4_0"])
def test_random_distributions_bit_exact(fmt):
    for name, W in distributions():
        q, d = quant(fmt, torch.from_numpy(W).to(DEV))
        qo, do = o.quantize(fmt, W)
        assert np.array_equal(q.cpu().numpy(), qo), name
        assert np.array_equal(d.cpu().numpy().view(np.uint16), do.view(np.uint16)), name


@pytest.mark.parametrize("fmt", ["q8_0", "q4_0"])
def test_strided_input_rows(fmt):
    rng = np.random.default_rng(3)
    Wbig = rng.standard_normal((40, 320)).astype(np.float32)
    Wt = torch.from_numpy(Wbig).to(DEV)[:, :256]  # row stride 320
    q, d = quant(fmt, Wt)
    qo, do = o.quantize(fmt, np.ascontiguousarray(Wbig[:, :256]))
    assert np.array_equal(q.cpu().numpy(), qo)
    assert np.array_equal(d.cpu().numpy().view(np.uint16), do.view(np.uint16))


@pytest.mark.parametrize("fmt", ["q8_0", "q4_0"])
def test_dequant_bit_exact(fmt):
    for name, W in distributions():
        qo, do = o.quantize(fmt, W)
        qt, dt = torch.from_numpy(qo).to(DEV), torch.from_numpy(do).to(DEV)
        w = (qg.dequant_q8_0 if fmt == "q8_0" else qg.dequant_q4_0)(qt, dt).cpu().numpy()
        assert np.array_equal(w.view(np.uint32), o.dequant(fmt, qo, do).view(np.uint32)), name


@pytest.mark.parametrize("fmt", ["q8_0", "q4_0"])
def test_repack_round_trip(fmt):
    for name, W in distributions():
        qo, do = o.quantize(fmt, W)
        blocks = qg.to_aos(fmt, torch.from_numpy(qo).to(DEV), torch.from_numpy(do).to(DEV))
        assert np.array_equal(blocks.cpu().numpy(), o.to_aos(fmt, qo, do)), name
        q2, d2 = qg.from_aos(fmt, blocks)
        assert np.array_equal(q2.cpu().numpy(), qo) and torch.equal(d2.cpu(), torch.from_numpy(do))


def test_cpu_tensors_round_trip_through_gpu(golden):
    g = golden["ref_uniform_64x512"]
    q, d = qg.quantize_q8_0(torch.from_numpy(g["W"]))
    assert q.device.type == "cpu" and d.device.type == "cpu"
    assert np.array_equal(q.numpy(), g["q8"])
    w = qg.dequant_q8_0(q, d)
    assert w.device.type == "cpu"
    assert np.array_equal(w.numpy(), o.dequant_q8_0(g["q8"], g["d8"].view(np.float16)))


@pytest.mark.parametrize("fmt", ["q8_0", "q4_0"])
def test_full_size_quantizer_checksum(fmt):
    """98304 x 4096 quantized on the GPU: equal row subsets to the oracle, and
    AoS == to_aos(SoA) over the whole matrix (a checksum of checksums)."""
    M, K = 98304, 4096
    g = torch.Generator(device=DEV).manual_seed(11)
    W = torch.randn(M, K, generator=g, device=DEV) * 0.02
    q, d = quant(fmt, W)
    blocks = (qg.quantize_q8_0_aos if fmt == "q8_0" else qg.quantize_q4_0_aos)(W)
    assert torch.equal(qg.to_aos(fmt, q, d), blocks)
    rows = torch.arange(0, M, 997, device=DEV)
    qo, do = o.quantize(fmt, W[rows].cpu().numpy())
    assert np.array_equal(q[rows].cpu().numpy(), qo)
    assert np.array_equal(d[rows].cpu().numpy().view(np.uint16), do.view(np.uint16))
