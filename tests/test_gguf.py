"""GGUF read / write: q8_0 / q4_0 blocks, f32 / f16 arrays and metadata round
trip through a file (CPU); loading onto the GPU as ggml blocks, SoA planes
and batch tiles gives GEMVs within the oracle's bound (GPU)."""

import numpy as np
import pytest

from oracle import qformats_oracle as o
from qgemv_roofline_b200 import gguf


def _blocks(fmt, M, K, seed):
    rng = np.random.default_rng(seed)
    W = (rng.standard_normal((M, K)) * 0.02).astype(np.float32)
    q, d = o.quantize(fmt, W)
    return q, d, o.to_aos(fmt, q, d)


def _file(tmp_path):
    q8, d8, b8 = _blocks("q8_0", 48, 256, 1)
    q4, d4, b4 = _blocks("q4_0", 33, 1024, 2)
    f32 = np.arange(12, dtype=np.float32).reshape(3, 4)
    f16 = np.linspace(-1, 1, 8).astype(np.float16)
    meta = {"general.name": "unit", "n_layer": 2, "rope.theta": 1e4, "flag": True,
            "neg": -5, "tokens": ["a", "bc", ""], "ids": [1, 2, 3]}
    p = str(tmp_path / "t.gguf")
    gguf.write_gguf(p, {"blk.0.q8": ("q8_0", b8), "blk.0.q4": ("q4_0", b4), "norm": f32,
                        "half": f16}, meta)
    return p, (q8, d8, b8), (q4, d4, b4), f32, f16, meta


def test_round_trip(tmp_path):
    p, (q8, d8, b8), (q4, d4, b4), f32, f16, meta = _file(tmp_path)
    r = gguf.GGUFReader(p)
    assert r.version == 3
    for k, v in meta.items():
        assert r.metadata[k] == v, k
    t8, t4 = r.tensors["blk.0.q8"], r.tensors["blk.0.q4"]
    assert (t8.type_name, t8.shape, t8.nbytes) == ("q8_0", (48, 256), 48 * 8 * 34)
    assert (t4.type_name, t4.shape, t4.nbytes) == ("q4_0", (33, 1024), 33 * 32 * 18)
    assert (r.blocks("blk.0.q8") == b8).all() and (r.blocks("blk.0.q4") == b4).all()
    assert (r.array("norm") == f32).all() and (r.array("half") == f16).all()
    assert (r.data_offset + t4.offset) % 32 == 0
    # the file's blocks are the reference's bytes: back to planes
    q, d = o.from_aos("q8_0", r.blocks("blk.0.q8"))
    assert (q == q8).all() and (d.view(np.uint16) == d8.view(np.uint16)).all()


def test_rejects_bad_files(tmp_path):
    bad = tmp_path / "bad.gguf"
    bad.write_bytes(b"GGML" + b"\0" * 60)
    with pytest.raises(ValueError):
        gguf.GGUFReader(str(bad))
    bad.write_bytes(b"GGUF" + (9).to_bytes(4, "little") + b"\0" * 60)
    with pytest.raises(ValueError):
        gguf.GGUFReader(str(bad))
    p, *_ = _file(tmp_path)
    r = gguf.GGUFReader(p)
    with pytest.raises(ValueError):
        r.blocks("norm")
    with pytest.raises(ValueError):
        r.array("blk.0.q8")


@pytest.mark.gpu
@pytest.mark.parametrize("layout", ["aos", "soa", "tiled"])
def test_load_and_gemv(tmp_path, layout):
    import torch
    p, (q8, d8, _), (q4, d4, _), *_ = _file(tmp_path)
    r = gguf.GGUFReader(p)
    for name, fmt, q, d in (("blk.0.q8", "q8_0", q8, d8), ("blk.0.q4", "q4_0", q4, d4)):
        m = r.load(name, "cuda", layout=layout)
        X = np.random.default_rng(5).standard_normal((3, m.K)).astype(np.float32)
        Y = m.matvec(torch.from_numpy(X).cuda()).cpu().numpy().astype(np.float64)
        y_ref = o.matvec_ref(fmt, q, d.view(np.float16), X)
        ok, worst = o.check_rowwise(Y, y_ref, o.row_norms(fmt, q, d.view(np.float16)), X, 1e-5)
        assert ok, (name, layout, worst)
