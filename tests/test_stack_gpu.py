"""The decode layer stack on one GPU: every GEMV of a step against the
float64 oracle (given the input that GEMV actually received), the CUDA-graph
replay against the eager step, the fused and persistent paths on one rank
(every row of a full 7B layer is in test_full_rows_gpu.py)."""

import numpy as np
import pytest
import torch

from oracle import qformats_oracle as o
from qgemv_roofline_b200 import stack

pytestmark = pytest.mark.gpu
SMALL = (("qkv", 384, 256), ("o", 256, 256), ("gate_up", 704, 256), ("down", 256, 352))


def check_trace(fmt, st, trace, rows=None):
    for (m, xin, yout), (q, d) in zip(trace, st.full):
        qh = q.cpu().numpy()
        dh = d.cpu().numpy()
        X = xin.cpu().numpy()[None, :].astype(np.float32)
        r = slice(None) if rows is None else rows
        y_ref = o.matvec_ref(fmt, qh[r], dh[r], X)
        wn = o.row_norms(fmt, qh[r], dh[r])
        Y = yout.cpu().numpy()[None, :][:, r]
        ok, worst = o.check_rowwise(Y.astype(np.float64), y_ref, wn, X, 1e-5)
        assert ok, (m.name, m.layer, worst)


@pytest.mark.parametrize("fmt", ["q8_0", "q4_0"])
@pytest.mark.parametrize("layout", ["soa", "tiled"])
def test_small_stack_every_gemv(fmt, layout):
    st = stack.DecodeStack.from_random(fmt, n_layers=2, shapes=SMALL, seed=3, device="cuda",
                                       layout=layout, keep_full=True)
    x = torch.randn(256, device="cuda", generator=torch.Generator(device="cuda").manual_seed(1))
    trace = []
    y = st(x, trace=trace)
    assert len(trace) == 8 and tuple(y.shape) == (256,)
    check_trace(fmt, st, trace)


@pytest.mark.parametrize("fmt", ["q8_0", "q4_0"])
def test_graph_replay_matches_eager(fmt):
    st = stack.DecodeStack.from_random(fmt, n_layers=3, shapes=SMALL, seed=4, device="cuda")
    x = torch.randn(256, device="cuda")
    y_eager = st(x).clone()
    g, out = st.capture(x)
    out.zero_()
    g.replay()
    torch.cuda.synchronize()
    assert torch.equal(out, y_eager)


def _init_single_rank_group():
    import os
    import socket
    import torch.distributed as dist
    if dist.is_initialized():
        return
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("nccl", rank=0, world_size=1, device_id=torch.device("cuda", 0))


@pytest.mark.parametrize("fmt", ["q8_0", "q4_0"])
def test_fused_stack_one_rank_matches_plain(fmt):
    """The fused path (kernel-side stores and counters, token fence) on one
    rank: same bits as the plain stack, over several graph replays (the
    counters keep growing from token to token)."""
    _init_single_rank_group()
    shapes = (("qkv", 768, 512), ("o", 512, 512), ("gate_up", 1280, 512), ("down", 512, 768))
    plain = stack.DecodeStack.from_random(fmt, n_layers=2, shapes=shapes, seed=6, device="cuda")
    fused = stack.DecodeStack.from_random(fmt, n_layers=2, shapes=shapes, seed=6, device="cuda",
                                          fused=True)
    x = torch.randn(512, device="cuda")
    y_plain = plain(x).clone()
    y_fused = fused(x).clone()
    torch.cuda.synchronize()
    assert torch.equal(y_plain, y_fused)
    g, out = fused.capture(x)
    for _ in range(3):
        out.zero_()
        g.replay()
        torch.cuda.synchronize()
        assert torch.equal(out, y_plain)
    from qgemv_roofline_b200 import _lib
    assert _lib.lib().qgemv_check_device_error(0, None) == 0
    del g



@pytest.mark.parametrize("fmt", ["q8_0", "q4_0"])
def test_persistent_stack_matches_per_launch_stack(fmt):
    """All GEMVs of a token in one cooperative launch: the same output as the
    per-launch stack (within the oracle's bound, in practice the same bits),
    eagerly and over CUDA-graph replays, with the grid-wide counters reset
    between tokens."""
    shapes = (("qkv", 1536, 1024), ("o", 1024, 1024), ("gate_up", 2816, 1024), ("down", 1024, 1536))
    plain = stack.DecodeStack.from_random(fmt, n_layers=3, shapes=shapes, seed=9, device="cuda",
                                          keep_full=True)
    pers = stack.DecodeStack.from_random(fmt, n_layers=3, shapes=shapes, seed=9, device="cuda",
                                         persistent=True)
    x = torch.randn(1024, device="cuda")
    trace = []
    y_plain = plain(x, trace=trace).clone()
    y_pers = pers(x).clone()
    torch.cuda.synchronize()
    m, _, _ = trace[-1]
    q, d = plain.full[-1]
    y_ref = o.matvec_ref(fmt, q.cpu().numpy(), d.cpu().numpy(),
                         trace[-1][1].cpu().numpy()[None, :].astype(np.float32))
    wn = o.row_norms(fmt, q.cpu().numpy(), d.cpu().numpy())
    ok, worst = o.check_rowwise(y_pers.cpu().numpy()[None, :].astype(np.float64), y_ref, wn,
                                trace[-1][1].cpu().numpy()[None, :], 1e-5)
    assert ok, worst
    assert torch.allclose(y_pers, y_plain, rtol=1e-6, atol=0)
    g, out = pers.capture(x)
    for _ in range(3):
        out.zero_()
        g.replay()
        torch.cuda.synchronize()
        assert torch.equal(out, y_pers)
    from qgemv_roofline_b200 import _lib
    assert _lib.lib().qgemv_check_device_error(0, None) == 0
    del g


def test_persistent_stack_7b_layer_spot_rows():
    st = stack.DecodeStack.from_random("q8_0", n_layers=2, seed=10, device="cuda",
                                       persistent=True)
    plain = stack.DecodeStack.from_random("q8_0", n_layers=2, seed=10, device="cuda")
    x = torch.randn(4096, device="cuda")
    assert torch.allclose(st(x), plain(x), rtol=1e-6, atol=0)
