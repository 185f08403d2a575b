"""The all-gather inside the kernels on several GPUs of one box (one process
per GPU, NCCL process group, symmetric memory): every rank's output of a
sharded decode stack whose kernels store their rows into the peers' buffers
-- one GEMV launch per matrix (fused) or one persistent launch per token --
equals the stack that all-gathers with NCCL, eagerly and over CUDA-graph
replays, token after token.  Skipped with fewer than two GPUs."""

import os
import socket

import pytest
import torch
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu
SHAPES = (("qkv", 1536, 1024), ("o", 1024, 1024), ("gate_up", 2816, 1024), ("down", 1024, 1536))


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, world, port, fmt, mode, out_q):
    import torch.distributed as dist
    from datetime import timedelta
    from qgemv_roofline_b200 import _lib, stack

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=dev,
                            timeout=timedelta(seconds=60))
    ok = False
    try:
        plain = stack.DecodeStack.from_random(fmt, n_layers=2, shapes=SHAPES, seed=8, device=dev)
        fused = stack.DecodeStack.from_random(fmt, n_layers=2, shapes=SHAPES, seed=8, device=dev,
                                              fused=mode == "fused",
                                              persistent=mode == "persistent")
        x = torch.randn(1024, device=dev, generator=torch.Generator(device=dev).manual_seed(2))
        y_plain = plain(x).clone()
        y_fused = fused(x).clone()
        torch.cuda.synchronize()
        ok = torch.equal(y_plain, y_fused)
        for _ in range(3):  # eager tokens: the counters keep growing
            ok = ok and torch.equal(fused(x), y_plain)
        g, out = fused.capture(x)
        for _ in range(3):
            out.zero_()
            g.replay()
            torch.cuda.synchronize()
            ok = ok and torch.equal(out, y_plain)
        del g
        ok = ok and _lib.lib().qgemv_check_device_error(0, None) == 0
        torch.cuda.synchronize()
        dist.barrier()
    finally:
        out_q.put((rank, bool(ok)))
        dist.destroy_process_group()


@pytest.mark.parametrize("fmt", ["q8_0", "q4_0"])
@pytest.mark.parametrize("mode", ["fused", "persistent"])
def test_fused_stack_matches_nccl_stack(fmt, mode):
    world = min(torch.cuda.device_count(), 8)
    if world < 2:
        pytest.skip("needs two or more GPUs")
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, fmt, mode, q))
             for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=300)
    res = dict(q.get(timeout=10) for _ in range(world))
    assert all(res[r] for r in range(world)), res
