"""The sharded decode stack with two and three gloo ranks on the CPU: every
rank's final output equals the single-process chain.  The per-rank GEMV is
the oracle's float64 matvec (the partition and gather plumbing is under
test; the kernels are tested on the GPU elsewhere)."""

import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from oracle import qformats_oracle as o
from qgemv_roofline_b200 import stack
from qgemv_roofline_b200.shard import row_range

SHAPES = (("qkv", 96, 64), ("o", 64, 64), ("gate_up", 130, 64), ("down", 64, 96))


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _matrices(fmt, layers):
    rng = np.random.default_rng(11)
    out = []
    for _ in range(layers):
        for name, M, K in SHAPES:
            W = (rng.standard_normal((M, K)) * 0.05).astype(np.float32)
            out.append((name, M, K) + tuple(o.quantize(fmt, W)))
    return out


def _chain(fmt, full, x):
    cur = x.astype(np.float32)
    for name, M, K, q, d in full:
        cur = o.matvec_ref(fmt, q, d, cur[None, :K])[0].astype(np.float32)
    return cur


def _worker(rank, world, port, fmt, layers, out_q):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        full = _matrices(fmt, layers)
        mats = []
        for j, (name, M, K, q, d) in enumerate(full):
            r0, r1 = row_range(M, rank, world)
            mats.append(stack.StackMatrix(name, j // len(SHAPES), M, K, r0, r1, (q[r0:r1], d[r0:r1])))

        def local_gemv(m, x, y):
            q, d = m.local
            return torch.from_numpy(o.matvec_ref(fmt, q, d, x.numpy()[None, :])[0].astype(np.float32))

        st = stack.DecodeStack(fmt, mats, layers, SHAPES, local_gemv=local_gemv)
        x = np.random.default_rng(3).standard_normal(64).astype(np.float32)
        y = st(torch.from_numpy(x)).numpy()
        ref = _chain(fmt, full, x)
        out_q.put((rank, bool(y.shape == ref.shape and np.allclose(y, ref, rtol=1e-6, atol=0))))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 3])
def test_sharded_stack_matches_single_process(world):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, "q8_0", 2, q)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
    res = dict(q.get(timeout=5) for _ in range(world))
    assert all(res[r] for r in range(world)), res
