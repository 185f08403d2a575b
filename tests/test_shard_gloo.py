"""Row sharding and the y all-gather with two gloo ranks on the CPU.

The per-rank GEMV is the oracle's float64 matvec here (the host-side
partition / gather logic is what is under test; the kernels are tested on the
GPU elsewhere)."""

import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from oracle import qformats_oracle as o
from qgemv_roofline_b200 import shard


def test_row_range_partitions_exactly():
    for M in (1, 7, 98304, 98305, 11008):
        for P in (1, 2, 3, 8):
            ranges = [shard.row_range(M, g, P) for g in range(P)]
            assert ranges[0][0] == 0 and ranges[-1][1] == M
            assert all(a[1] == b[0] for a, b in zip(ranges, ranges[1:]))
            sizes = [r1 - r0 for r0, r1 in ranges]
            assert max(sizes) - min(sizes) <= 1
    with pytest.raises(ValueError):
        shard.row_range(10, 2, 2)


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, world, port, M, K, N, fmt, out_q):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        rng = np.random.default_rng(5)  # same full matrix on every rank
        W = (rng.standard_normal((M, K)) * 0.02).astype(np.float32)
        X = rng.standard_normal((N, K)).astype(np.float32)
        q, d = o.quantize(fmt, W)
        r0, r1 = shard.row_range(M, rank, world)
        ql, dl = q[r0:r1], d[r0:r1]

        def local_gemv(x, y=None):
            xx = x.numpy()
            return torch.from_numpy(o.matvec_ref(fmt, ql, dl, xx).astype(np.float32))

        sh = shard.ShardedQGemv(None, M, K, fmt, local_gemv=local_gemv)
        assert (sh.r0, sh.r1) == (r0, r1)
        y_vec = sh(torch.from_numpy(X[0]), gather=True)
        y_mat = sh(torch.from_numpy(X), gather=True)
        y_loc = sh(torch.from_numpy(X[0]), gather=False)
        ref = o.matvec_ref(fmt, q, d, X).astype(np.float32)
        ok = (tuple(y_vec.shape) == (M,) and tuple(y_mat.shape) == (N, M)
              and np.allclose(y_vec.numpy(), ref[0], rtol=0, atol=1e-6)
              and np.allclose(y_mat.numpy(), ref, rtol=0, atol=1e-6)
              and np.allclose(y_loc.numpy(), ref[0, r0:r1], rtol=0, atol=1e-6))
        out_q.put((rank, bool(ok)))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("M,world", [(96, 2), (97, 2), (50, 3)])
def test_sharded_gemv_gathers_full_y(M, world):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, M, 64, 3, "q4_0", q))
             for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
    results = dict(q.get(timeout=5) for _ in range(world))
    assert all(p.exitcode == 0 for p in procs)
    assert all(results[r] for r in range(world)), results
