"""Tiles claimed at run time by the single-column kernel (a counter per stream
and per captured launch): results must not depend on how launches from
several streams, from captured graphs and from plain calls interleave."""

import numpy as np
import pytest
import torch

import qgemv_roofline_b200 as qg
from qgemv_roofline_b200 import _lib
from oracle import qformats_oracle as o

pytestmark = pytest.mark.gpu
DEV = "cuda"


def matrix(fmt, M, K, seed):
    g = torch.Generator(device=DEV).manual_seed(seed)
    W = torch.randn(M, K, generator=g, device=DEV) * 0.02
    q, d = (qg.quantize_q8_0 if fmt == "q8_0" else qg.quantize_q4_0)(W)
    return q, d


def reference(fmt, q, d, x):
    """Float64 oracle of y for planes on the GPU."""
    qh, dh = q.cpu().numpy(), d.cpu().numpy()
    return o.matvec_ref(fmt, qh, dh, x.cpu().numpy()[None, :])[0], o.row_norms(fmt, qh, dh)


def check(fmt, y, ref, wn, x):
    ok, worst = o.check_rowwise(y.cpu().numpy()[None, :], ref[None, :], wn,
                                x.cpu().numpy()[None, :])
    assert ok, f"{fmt}: outside 1e-5 ||w|| ||x|| (worst ratio {worst:.3g})"


@pytest.mark.parametrize("fmt", ["q8_0", "q4_0"])
def test_concurrent_streams_each_exact(fmt):
    # four streams, each a chain of dependent GEMVs on its own matrix, issued
    # interleaved so that launches of different streams overlap on the GPU
    M, K, nstreams, chain = 24576, 4096, 4, 6
    mats = [matrix(fmt, M, K, 100 + i) for i in range(nstreams)]
    x0 = torch.randn(K, device=DEV)
    streams = [torch.cuda.Stream() for _ in range(nstreams)]
    outs = [[torch.empty(M, device=DEV) for _ in range(chain)] for _ in range(nstreams)]
    torch.cuda.synchronize()
    for j in range(chain):
        for i, st in enumerate(streams):
            with torch.cuda.stream(st):
                xin = x0 if j == 0 else outs[i][j - 1][:K]
                qg.qgemv(fmt, mats[i][0], mats[i][1], xin, y=outs[i][j])
    torch.cuda.synchronize()
    for i in range(nstreams):
        for j in (0, chain - 1):
            xin = x0 if j == 0 else outs[i][j - 1][:K]
            ref, wn = reference(fmt, mats[i][0], mats[i][1], xin)
            check(fmt, outs[i][j], ref, wn, xin)
    assert _lib.lib().qgemv_check_device_error(0, None) == 0


@pytest.mark.parametrize("fmt", ["q8_0", "q4_0"])
def test_graph_replays_between_plain_calls(fmt):
    M, K = 49152, 4096
    q, d = matrix(fmt, M, K, 7)
    x = torch.randn(K, device=DEV)
    y_plain = qg.qgemv(fmt, q, d, x)
    torch.cuda.synchronize()
    yg = torch.empty(M, device=DEV)
    st = torch.cuda.Stream()
    st.wait_stream(torch.cuda.current_stream())
    g = torch.cuda.CUDAGraph()
    with torch.cuda.stream(st):
        qg.qgemv(fmt, q, d, x, y=yg)  # warm-up outside capture
        torch.cuda.synchronize()
        with torch.cuda.graph(g, stream=st):
            qg.qgemv(fmt, q, d, x, y=yg)
            qg.qgemv(fmt, q, d, x, y=yg)
    for _ in range(3):
        yg.zero_()
        g.replay()
        y2 = qg.qgemv(fmt, q, d, x)  # plain calls on the same stream in between
        torch.cuda.synchronize()
        assert torch.equal(yg, y_plain)
        assert torch.equal(y2, y_plain)
    assert _lib.lib().qgemv_check_device_error(0, None) == 0


@pytest.mark.parametrize("fmt", ["q8_0", "q4_0"])
@pytest.mark.parametrize("M", [1, 17, 300, 4096, 98304 + 16])
def test_grid_sizes_and_ragged_tiles(fmt, M):
    # a few rows (fewer tiles than CTAs) and ragged last tiles
    K = 4096
    q, d = matrix(fmt, M, K, M)
    x = torch.randn(K, device=DEV)
    ref, wn = reference(fmt, q, d, x)
    for _ in range(3):  # the counter is reset by every launch's last claim
        y = qg.qgemv(fmt, q, d, x)
        check(fmt, y, ref, wn, x)
    assert _lib.lib().qgemv_check_device_error(0, None) == 0
