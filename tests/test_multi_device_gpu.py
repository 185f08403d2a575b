"""One process, several GPUs: the C-ABI multi-GPU handle (qgemv_mg_*) through
MultiDeviceQGemv, against the single-GPU entry points and the float64
oracle.  With one GPU the handle holds the whole matrix on it; with more
(when the box has them) every device holds a row shard and the all-gather
brings every row to every device."""

import numpy as np
import pytest
import torch

import qgemv_roofline_b200 as qg
from qgemv_roofline_b200 import _lib
from qgemv_roofline_b200.shard import MultiDeviceQGemv, row_range
from oracle import qformats_oracle as o

pytestmark = pytest.mark.gpu


def make(fmt, M, K, N, seed):
    rng = np.random.default_rng(seed)
    W = (rng.standard_normal((M, K)) * 0.02).astype(np.float32)
    X = rng.standard_normal((N, K)).astype(np.float32)
    q, d = o.quantize(fmt, W)
    return q, d.view(np.float16), X


def matrix(fmt, q, d, layout):
    qt = torch.from_numpy(np.ascontiguousarray(q)).to("cuda:0")
    dt = torch.from_numpy(np.ascontiguousarray(d)).to("cuda:0")
    M, K = q.shape[0], d.shape[1] * 32
    if layout == "soa":
        return qg.QuantizedMatrix(fmt, M, K, "soa", q=qt, d=dt)
    return qg.QuantizedMatrix(fmt, M, K, "aos", blocks=qg.to_aos(fmt, qt, dt))


def check(fmt, q, d, X, Y):
    y64 = o.matvec_ref(fmt, q, d, X)
    bound = 1e-5 * o.row_norms(fmt, q, d)[None, :] * np.linalg.norm(X.astype(np.float64), axis=1)[:, None]
    assert (np.abs(Y.astype(np.float64).reshape(y64.shape) - y64) <= bound).all()


@pytest.mark.parametrize("fmt", ["q8_0", "q4_0"])
@pytest.mark.parametrize("layout", ["soa", "aos"])
@pytest.mark.parametrize("N", [1, 4])
def test_one_device_matches_single_gpu_call(fmt, layout, N):
    M, K = 1000, 4096
    q, d, X = make(fmt, M, K, N, seed=M + N)
    W = matrix(fmt, q, d, layout)
    Xt = torch.from_numpy(X).to("cuda:0")
    x = Xt[0] if N == 1 else Xt
    mg = MultiDeviceQGemv(W, [0])
    (y,) = mg([x])
    torch.cuda.synchronize()
    assert torch.equal(y, W.matvec(x))   # the same kernel on the same rows
    check(fmt, q, d, X, y.cpu().numpy())
    mg.close()
    assert _lib.lib().qgemv_check_device_error(0, None) == 0


def test_reshard_and_streams():
    """A second shard replaces the first; the caller's own streams order the work."""
    M, K = 777, 2048
    q, d, X = make("q8_0", M, K, 2, seed=5)
    W = matrix("q8_0", q, d, "soa")
    mg = MultiDeviceQGemv(W, [0])
    q4, d4, _ = make("q4_0", M, K, 1, seed=6)
    W4 = matrix("q4_0", q4, d4, "soa")
    mg2 = MultiDeviceQGemv(W4, [0])
    s = torch.cuda.Stream(device="cuda:0")
    Xt = torch.from_numpy(X).to("cuda:0")
    with torch.cuda.stream(s):
        (y,) = mg([Xt])
        (y4,) = mg2([Xt])
    s.synchronize()
    assert torch.equal(y, W.matvec(Xt))
    assert torch.equal(y4, W4.matvec(Xt))
    mg.close()
    mg2.close()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 or more GPUs")
@pytest.mark.parametrize("fmt", ["q8_0", "q4_0"])
@pytest.mark.parametrize("N", [1, 3])
def test_row_shards_and_allgather_on_every_device(fmt, N):
    P = min(torch.cuda.device_count(), 8)
    M, K = 12289, 4096   # not a multiple of P
    q, d, X = make(fmt, M, K, N, seed=11 * N)
    W = matrix(fmt, q, d, "soa")
    mg = MultiDeviceQGemv(W, list(range(P)))
    assert mg.row_ranges == [row_range(M, g, P) for g in range(P)]
    Xt = torch.from_numpy(X)
    xs = [(Xt[0] if N == 1 else Xt).to(f"cuda:{g}") for g in range(P)]
    ys = mg(xs, allgather=True)
    for g in range(P):
        torch.cuda.synchronize(g)
    ref = ys[0].cpu()
    for g in range(P):
        assert torch.equal(ys[g].cpu(), ref)   # every device holds the same rows
        r0, r1 = row_range(M, g, P)
        # a device's own rows: the single-GPU call on the same shard
        part = W.rows(r0, r1).to(f"cuda:{g}")
        own = part.matvec(xs[g])
        torch.cuda.synchronize(g)
        assert torch.equal(ys[g][..., r0:r1].cpu(), own.cpu())
    check(fmt, q, d, X, ref.numpy())
    # without the gather each device holds only its rows; the others keep their values
    ys2 = [torch.full_like(y, 7.0) for y in ys]
    mg(xs, ys2, allgather=False)
    for g in range(P):
        torch.cuda.synchronize(g)
        r0, r1 = row_range(M, g, P)
        yg = ys2[g].cpu()
        assert torch.equal(yg[..., r0:r1], ref[..., r0:r1])
        assert (yg[..., :r0] == 7.0).all() and (yg[..., r1:] == 7.0).all()
    mg.close()
