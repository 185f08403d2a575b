"""Generate the golden q8_0 / q4_0 fixtures from the reference itself.

Run in a checkout where the reference project is present (by default the
directory ``reference`` beside this repository's root; set QGEMV_REFERENCE to
point elsewhere):

    python tests/golden/make_golden.py

For every case it stores the fp32 weights W and activations X, and the
reference's outputs on them:

* ``q8``, ``d8``, ``q4``, ``d4``: bytes from the reference's
  python/qformats.py (``quantize_q8_0`` / ``quantize_q4_0``), d as raw fp16
  bits (uint16);
* ``y8_f32``, ``y4_f32``: the reference's CPU GEMV, ``dequant(q, d) @ x`` in
  torch float32 (python/triton_qgemv.py:135,154), one row per column of X;
* ``aos8``, ``aos4``, ``y8_f64``, ``y4_f64`` (when oracle/_ref is built): the
  reference's C++ quantizer blocks (src/bench.cu:32-69) and float64 matvec
  (src/bench.cu:75-111).

The script also asserts that the Python and C++ quantizers of the reference
agree byte for byte on every case.  Output: tests/golden/golden.npz.
"""

from __future__ import annotations

import os
import sys

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(os.path.dirname(HERE))
REF = os.environ.get("QGEMV_REFERENCE", os.path.join(REPO, os.pardir, "reference"))
sys.path.insert(0, os.path.join(REF, "python"))
sys.path.insert(0, REPO)

import qformats  # noqa: E402  (the reference's own module)

from oracle import ref_lib  # noqa: E402


def edge_matrix() -> np.ndarray:
    """8 rows x 8 blocks of hand-made edge blocks (all finite)."""
    blocks = []
    z = np.zeros(32, np.float32)
    blocks.append(z.copy())                                   # all zero -> d = +0 / -0
    b = z.copy(); b[5] = 0.5; b[9] = -0.5; blocks.append(b)   # tie, positive first
    b = z.copy(); b[3] = -0.25; b[30] = 0.25; blocks.append(b)  # tie, negative first
    blocks.append(np.full(32, 1e-7, np.float32))              # d underflows in fp16
    b = np.linspace(-1e-3, 1e-3, 32).astype(np.float32); blocks.append(b)  # subnormal d
    b = np.linspace(-1e5, 3e4, 32).astype(np.float32); blocks.append(b)    # large values
    # exact rounding ties for q8 (d = 1 -> id = 1): 2.5, -3.5, 0.5, ...
    b = (np.arange(32, dtype=np.float32) - 16) + np.float32(0.5); b[0] = 127.0
    blocks.append(b)
    b = z.copy(); b[31] = -3.0; blocks.append(b)              # single nonzero, last, negative
    b = np.where(np.arange(32) % 2 == 0, 1.0, -1.0).astype(np.float32) * 0.75
    blocks.append(b)                                          # alternating, all ties
    # q4 ties: mx = 8 -> d = -1 -> id = -1; w*id + 8.5 hits exact .0/.5 values
    b = (np.arange(32, dtype=np.float32) * 0.5 - 8.0); b[16] = 8.0; blocks.append(b)
    b = np.full(32, -2.0, np.float32); b[7] = 2.0; blocks.append(b)  # first max negative
    b = np.full(32, 5.0e5, np.float32); b[1] = -5.2e5; blocks.append(b)  # large d, both formats finite
    rng = np.random.default_rng(99)
    while len(blocks) < 64:
        s = 10.0 ** rng.uniform(-6, 3)
        blocks.append((rng.standard_normal(32) * s).astype(np.float32))
    return np.stack(blocks).reshape(8, 8 * 32)


def cases():
    torch.manual_seed(1234)                       # tests/test_quant_cpu.py:39-41, :96
    W = torch.rand(64, 512) * 2 - 1
    x = torch.rand(512) * 2 - 1
    yield "ref_uniform_64x512", W.numpy(), x.numpy()[None, :]

    g = torch.Generator().manual_seed(20240601)
    W = torch.randn(64, 1024, generator=g) * 0.02
    X = torch.randn(3, 1024, generator=g)
    yield "normal_64x1024_n3", W.numpy(), X.numpy()

    g = torch.Generator().manual_seed(7)
    W = torch.randn(5, 11008, generator=g) * 0.02
    X = torch.randn(1, 11008, generator=g)
    yield "normal_5x11008", W.numpy(), X.numpy()

    g = torch.Generator().manual_seed(3)
    W = torch.randn(3, 96, generator=g)
    X = torch.randn(2, 96, generator=g)
    yield "odd_3x96_n2", W.numpy(), X.numpy()

    W = edge_matrix()
    g = torch.Generator().manual_seed(11)
    X = torch.randn(1, W.shape[1], generator=g)
    yield "edge_8x256", W, X.numpy()


def main():
    out = {}
    have_ref = ref_lib.load() is not None
    for name, W, X in cases():
        W = np.ascontiguousarray(W, np.float32)
        X = np.ascontiguousarray(X, np.float32)
        Wt = torch.from_numpy(W)
        q8, d8 = qformats.quantize_q8_0(Wt)
        q4, d4 = qformats.quantize_q4_0(Wt)
        Xt = torch.from_numpy(X)
        y8 = torch.stack([qformats.dequant_q8_0(q8, d8) @ Xt[n] for n in range(X.shape[0])])
        y4 = torch.stack([qformats.dequant_q4_0(q4, d4) @ Xt[n] for n in range(X.shape[0])])
        rec = {
            "W": W, "X": X,
            "q8": q8.numpy(), "d8": d8.view(torch.int16).numpy().view(np.uint16),
            "q4": q4.numpy(), "d4": d4.view(torch.int16).numpy().view(np.uint16),
            "y8_f32": y8.numpy(), "y4_f32": y4.numpy(),
        }
        if have_ref:
            a8 = ref_lib.quantize_aos("q8_0", W)
            a4 = ref_lib.quantize_aos("q4_0", W)
            # the reference's two quantizers must agree byte for byte
            assert (a8[:, :, 2:].reshape(q8.shape).view(np.int8) == rec["q8"]).all(), name
            assert (a8[:, :, :2].copy().view(np.uint16).reshape(d8.shape) == rec["d8"]).all(), name
            assert (a4[:, :, 2:].reshape(q4.shape) == rec["q4"]).all(), name
            assert (a4[:, :, :2].copy().view(np.uint16).reshape(d4.shape) == rec["d4"]).all(), name
            rec["aos8"], rec["aos4"] = a8, a4
            rec["y8_f64"] = np.stack([ref_lib.matvec("q8_0", a8, X[n]) for n in range(X.shape[0])])
            rec["y4_f64"] = np.stack([ref_lib.matvec("q4_0", a4, X[n]) for n in range(X.shape[0])])
        for k, v in rec.items():
            out[f"{name}/{k}"] = v
        print(f"{name}: W{W.shape} X{X.shape} ref_cpp={'yes' if have_ref else 'no'}")
    out["meta/torch"] = np.array(torch.__version__)
    path = os.path.join(HERE, "golden.npz")
    np.savez_compressed(path, **out)
    print(f"wrote {path} ({os.path.getsize(path)} bytes)")


if __name__ == "__main__":
    main()
