#!/usr/bin/env python3
"""Benchmark of the q8_0 / q4_0 GEMV hot path on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

Workload (the large, L2-safe configuration the headline target is quoted on):
W [98304, 4096] ~ N(0, 0.02) fp32, quantized on the GPU to q8_0 and to q4_0
(SoA planes), x fp32 [4096] ~ N(0, 1), batch 1.  One *step* = one q8_0 GEMV
plus one q4_0 GEMV.  With N GPUs (one process per GPU, torchrun) the rows of a
[N * 98304, 4096] matrix are sharded: rank g owns rows [g*98304, (g+1)*98304)
of both formats, resident in its HBM; x is replicated; the step needs no
collective.  Work per GPU is fixed as N grows ("weak" scaling, the default;
rows are independent, so the path partitions).  Beside it, under N > 1, the
line reports the same 98304-row matrix sharded N ways (98304 / N rows per
rank, "row_sharded_fixed_M": total work fixed) and an NCCL all-gather of y,
each timed separately.  --scaling strong makes the fixed-M sharding the value.

Every rank keeps C_f copies of each format's weight slice and call i of that
format reads copy i % C_f, with C_f chosen so that the bytes streamed between
two reads of the same copy are >= 4x the 126 MB L2 (the weights are never
timed from L2).  The K timed steps are issued as K q8_0 calls back to back,
then K q4_0 calls back to back (events only at the start, between the two
groups and at the end), so each group's launches overlap the previous
launch's tail the way a caller's stream of GEMVs does.

Printed (rank 0, one JSON line): the whole-job algorithmic GB/s (weights
M*K*(34|18)/32 + x 4*K + y 4*M per call) over the max-over-ranks device time
of the K timed steps, with the roofline of the dominant kernel, the CPU
baseline, the end-to-end figure through the public API with host buffers, and
the SM clocks sampled during the timed region.
"""

from __future__ import annotations

import argparse
import json
import math
import os
import sys
import time

REPO = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, REPO)

METRIC = ("q8_0/q4_0 GEMV HBM GB/s as % of measured B200 read roof; "
          "µs/call at 1–8 GPUs")
M_FULL, K_FULL = 98304, 4096
SEED = 20260101
L2_BYTES = 126 * 1000 * 1000
BLOCK = {"q8_0": 34, "q4_0": 18}


def parse():
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawTextHelpFormatter)
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20000)
    ap.add_argument("--warmup", type=int, default=50)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--M", type=int, default=M_FULL)
    ap.add_argument("--K", type=int, default=K_FULL)
    ap.add_argument("--layout", choices=["soa", "aos"], default="soa")
    ap.add_argument("--scaling", choices=["weak", "strong"], default="weak",
                    help="xl workload under N > 1 GPUs: weak = 98304 rows per GPU (a [N*98304, "
                         "4096] matrix row-sharded); strong = the 98304-row matrix sharded N ways")
    ap.add_argument("--no-extras", action="store_true",
                    help="skip roofs, e2e and the CPU baseline (profiling runs)")
    ap.add_argument("--cpu-seconds", type=float, default=10.0,
                    help="CPU-baseline sample size, in seconds of CPU work")
    ap.add_argument("--workload", choices=["xl", "stack", "batch"], default="xl",
                    help="xl: the headline 98304x4096 GEMV (default); stack: the 32-layer "
                         "decode GEMV stack; batch: 28672x8192 with 1..16 columns")
    ap.add_argument("--layers", type=int, default=32, help="stack workload: layers")
    ap.add_argument("--persistent", action="store_true",
                    help="stack workload, one GPU: all GEMVs of a token in one cooperative launch")
    ap.add_argument("--fused", action="store_true",
                    help="stack workload: all-gather inside the GEMV kernels (peer stores, "
                         "symmetric memory) instead of NCCL")
    args = ap.parse_args()
    if args.workload != "xl" and args.steps == 20000:
        args.steps = 30 if args.workload == "stack" else 200
    return args


def wbytes(fmt, M, K):
    return M * (K // 32) * BLOCK[fmt]


def alg_bytes(fmt, M, K, N=1):
    return wbytes(fmt, M, K) + 4 * K * N + 4 * M * N


def workload_config(args, world, rows, copies=None):
    Mtot = rows * world
    cfg = {
        "workload": f"q8_0 + q4_0 GEMV, W [{Mtot}, {args.K}], x fp32 [{args.K}], batch 1"
                    + (f", rows sharded over {world} GPUs ({rows} per GPU)" if world > 1 else ""),
        "M": Mtot, "K": args.K, "batch": 1, "formats": ["q8_0", "q4_0"],
        "layout": args.layout, "rows_per_gpu": rows,
        "weights": "W ~ N(0, 0.02) fp32 (seeded per rank), quantized on the GPU; x ~ N(0, 1)",
        "parallelism": f"row-shard x{world}" if world > 1 else "single GPU",
    }
    if copies is not None:
        cfg["weight_copies_rotated"] = copies
        cfg["l2"] = ("inputs larger than L2: rotated weight copies per format, >= 4x the "
                     "126 MB L2 streamed between reads of one copy; no flush")
        cfg["timed_order"] = "K q8_0 calls back to back, then K q4_0 calls"
    return cfg


def measured_peak():
    p = os.path.join(REPO, "MEASURED_PEAKS.json")
    try:
        with open(p) as f:
            j = json.load(f)
        return float(j["hbm_gbs"]), "of measured (MEASURED_PEAKS.json hbm_gbs, copy)"
    except Exception:
        return 6650.0, "of fallback (6.65 TB/s)"


def dram_traffic(kernel_key):
    """Per-launch DRAM bytes (read + write) of a kernel from a committed ncu
    summary, or None when no capture exists for this workload."""
    p = os.path.join(REPO, "profiles", "dram_traffic.json")
    try:
        with open(p) as f:
            return json.load(f).get(kernel_key)
    except Exception:
        return None


# ------------------------------------------------------- stack / batch workloads

def _timed(torch, dist, dev, world, fn, warmup, steps):
    """Device time (ms, max over ranks) of `steps` calls of fn after `warmup`."""
    for _ in range(warmup):
        fn()
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record()
    for _ in range(steps):
        fn()
    b.record()
    b.synchronize()
    t = torch.tensor([a.elapsed_time(b)], dtype=torch.float64, device=dev)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return t.item()


def stack_workload(args, rank, world, dev):
    """32 decode layers x {QKV 12288x4096, O 4096x4096, gate+up 22016x4096,
    down 4096x11008}, batch 1, q8_0 then q4_0; rows sharded over the ranks
    with an NCCL all-gather of every y; one step = one token through all
    layers, replayed from a CUDA graph."""
    import torch
    import torch.distributed as dist

    import qgemv_roofline_b200 as qg
    from qgemv_roofline_b200 import stack
    from qgemv_roofline_b200.clocks import ClockSampler

    res, graphs, total_bytes, total_ms = {}, [], 0, 0.0
    if args.fused and not dist.is_initialized():
        # the fused path addresses buffers through a process group, even of one
        import socket
        sk = socket.socket()
        sk.bind(("127.0.0.1", 0))
        os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
        os.environ["MASTER_PORT"] = str(sk.getsockname()[1])
        sk.close()
        dist.init_process_group("nccl", rank=0, world_size=1, device_id=dev)
    x = torch.randn(4096, generator=torch.Generator(device=dev).manual_seed(SEED), device=dev)
    uuid = None
    try:
        uuid = str(torch.cuda.get_device_properties(dev).uuid)
        uuid = uuid if uuid.startswith("GPU-") else "GPU-" + uuid
    except Exception:
        pass
    with ClockSampler(uuid) as sampler:
        for fmt in ("q8_0", "q4_0"):
            st = stack.DecodeStack.from_random(fmt, n_layers=args.layers, seed=SEED, device=dev,
                                               fused=args.fused,
                                               persistent=args.persistent and world == 1)
            g, out = st.capture(x)
            graphs.append(g)
            ms = _timed(torch, dist, dev, world, g.replay, args.warmup, args.steps)
            per = ms / args.steps
            res[fmt] = {"us_per_token": per * 1e3, "weight_bytes": st.weight_bytes,
                        "gbps_aggregate": st.weight_bytes / (per * 1e-3) / 1e9,
                        "gemv_launches_per_token": 1 if st.persistent is not None else len(st.mats),
                        "allgathers_per_token": (0 if args.fused else len(st.mats))
                        if world > 1 else 0}
            total_bytes += st.weight_bytes * args.steps
            total_ms += ms
            del st, out
            torch.cuda.empty_cache()
    graphs.clear()  # graphs holding NCCL calls go before the process group
    value = total_bytes / (total_ms * 1e-3) / 1e9
    peak, note = measured_peak()
    if rank == 0:
        line = {"metric": "32-layer q8_0/q4_0 decode GEMV stack: weight GB/s (µs/token per format)",
                "value": value, "unit": "GB/s", "n_gpus": world, "steps": args.steps,
                "warmup": args.warmup, "ms_per_step": total_ms / args.steps,
                "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
                "dtype": "fp32", "data": "synthetic (seeded N(0, 0.02) weights, N(0, 1) x)",
                "config": {"workload": f"{args.layers} layers x (QKV 12288x4096, O 4096x4096, "
                                       f"gate+up 22016x4096, down 4096x11008), batch 1",
                           "parallelism": (f"row-shard x{world} + " +
                                           ("all-gather of every y inside the GEMV kernels "
                                            "(peer stores, counters)" if args.fused else
                                            "NCCL all-gather of every y"))
                           if world > 1 else "single GPU" + (", fused path" if args.fused else "")
                           + (", one persistent launch per token" if args.persistent else ""),
                           "step": "one token through all layers, q8_0 stack then q4_0 stack, "
                                   "each a CUDA graph replay",
                           "l2": "inputs larger than L2 (3.6-6.9 GB of weights per stack)"},
                "per_format": res, "frac_of_peak_per_gpu": value / world / peak,
                "peak_note": note, "clocks": sampler.summary(),
                "gpu_launches": args.steps * world * sum(r["gemv_launches_per_token"]
                                                         for r in res.values())}
        print(json.dumps(line), flush=True)
    return 0


def batch_workload(args, rank, world, dev):
    """W [28672, 8192] (rows sharded) with X [N, 8192], N in 1..16, from SoA
    planes and from batch tiles."""
    import torch
    import torch.distributed as dist

    import qgemv_roofline_b200 as qg
    from qgemv_roofline_b200 import _lib

    M, K = 28672, 8192
    r0, r1 = M * rank // world, M * (rank + 1) // world
    rows = r1 - r0
    out = []
    lib = _lib.lib()
    for fmt in ("q8_0", "q4_0"):
        g = torch.Generator(device=dev).manual_seed(SEED + 7919 * rank)
        W = torch.randn(rows, K, generator=g, device=dev) * 0.02
        q, d = (qg.quantize_q8_0 if fmt == "q8_0" else qg.quantize_q4_0)(W)
        del W
        copies = max(2, math.ceil(4 * L2_BYTES / wbytes(fmt, rows, K)))
        soa = [(q, d)] + [(q.clone(), d.clone()) for _ in range(copies - 1)]
        tiles = [qg.tile_weights(fmt, q=a, d=b) for a, b in soa]
        fid = 8 if fmt == "q8_0" else 4
        for N in (1, 2, 4, 8, 16):
            X = torch.randn(N, K, device=dev)
            Y = torch.empty(N, rows, device=dev)
            nb = max(lib.qgemv_tiled_workspace_bytes(K, N), 16)
            ws = torch.empty(nb, dtype=torch.uint8, device=dev)
            sp = torch.cuda.current_stream().cuda_stream
            it = [0]

            def soa_call():
                a, b = soa[it[0] % copies]
                it[0] += 1
                _lib.call("qgemv_soa_ws", fid, a.data_ptr(), b.data_ptr(), X.data_ptr(),
                          Y.data_ptr(), rows, K, N, K, rows, ws.data_ptr(), nb, sp)

            def tiled_call():
                t = tiles[it[0] % copies]
                it[0] += 1
                _lib.call("qgemv_tiled_gemv", fid, t.data_ptr(), rows, K, X.data_ptr(),
                          Y.data_ptr(), N, K, rows, ws.data_ptr(), nb, sp)

            for layout, fn in (("soa", soa_call), ("tiled", tiled_call)):
                ms = _timed(torch, dist, dev, world, fn, args.warmup, args.steps)
                per = ms / args.steps
                b = alg_bytes(fmt, rows, K, N)
                out.append({"fmt": fmt, "layout": layout, "N": N, "us_per_call": per * 1e3,
                            "gbps_aggregate": world * b / (per * 1e-3) / 1e9})
        del soa, tiles, q, d
        torch.cuda.empty_cache()
    if rank == 0:
        peak, note = measured_peak()
        print(json.dumps({"metric": "small-batch GEMV 28672x8192, N columns: GB/s",
                          "value": max(r["gbps_aggregate"] for r in out if r["N"] == 16),
                          "unit": "GB/s", "n_gpus": world, "steps": args.steps,
                          "warmup": args.warmup, "higher_is_better": True, "scaling": "strong",
                          "vs_baseline": None, "dtype": "fp32",
                          "data": "synthetic (seeded N(0, 0.02) weights, N(0, 1) X)",
                          "config": {"workload": "W [28672, 8192], X [N, 8192], N in 1..16",
                                     "rows_per_gpu": rows, "l2": "rotated weight copies, >= 4x L2"},
                          "peak": peak, "peak_note": note, "results": out}), flush=True)
    return 0


# ----------------------------------------------------------------- reference arm

def reference_arm(args, rank, world):
    """The reference's own CPU implementation of the path, on the host cores.

    The reference's C++ GEMV (src/bench.cu:75-111, compiled from the reference
    tree into oracle/_ref) run on all host threads over a bounded row sample
    of the same workload; falls back to the oracle's restatement of the
    reference's CPU path (dequantize, then matvec) when oracle/_ref is absent.
    """
    if rank != 0:
        return 0
    import numpy as np

    from oracle import qformats_oracle as o
    from oracle import ref_lib

    cores = len(os.sched_getaffinity(0)) if hasattr(os, "sched_getaffinity") else os.cpu_count()
    rng = np.random.default_rng(SEED)
    K = args.K
    x = rng.standard_normal(K).astype(np.float32)
    have_ref = ref_lib.load() is not None

    def build(rows):
        W = (rng.standard_normal((rows, K)) * 0.02).astype(np.float32)
        if have_ref:
            plans = [ref_lib.Plan(f, ref_lib.quantize_aos(f, W), cores) for f in ("q8_0", "q4_0")]
            return lambda: [p.run(x) for p in plans]
        qd = [o.quantize(f, W) for f in ("q8_0", "q4_0")]
        return lambda: [o.dequant(f, q, d) @ x for f, (q, d) in zip(("q8_0", "q4_0"), qd)]

    # size the sample so warm-up + timed steps take about a minute of CPU time
    probe_rows = min(args.M, 1024)
    fn = build(probe_rows)
    fn()
    t0 = time.perf_counter()
    fn()
    t_probe = max(time.perf_counter() - t0, 1e-6)
    budget = 60.0 / max(1, args.steps + args.warmup)
    rows = int(max(32, min(args.M, probe_rows * budget / t_probe)))
    rows -= rows % 32 if rows > 32 else 0
    fn = build(rows)
    for _ in range(args.warmup):
        fn()
    t0 = time.perf_counter()
    for _ in range(args.steps):
        fn()
    dt = time.perf_counter() - t0
    step_bytes = alg_bytes("q8_0", rows, K) + alg_bytes("q4_0", rows, K)
    value = step_bytes * args.steps / dt / 1e9
    kind = "reference" if have_ref else "port"
    sample = (f"{rows} of {args.M} rows x {K}, q8_0 + q4_0 per step, "
              + ("reference C++ float64 matvec (src/bench.cu:75-111)" if have_ref else
                 "oracle restatement of dequant(q, d) @ x (python/qformats.py:43-56)")
              + f" on {cores} threads")
    line = {
        "impl": "reference", "metric": METRIC, "value": value, "unit": "GB/s",
        "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": dt / args.steps * 1e3, "higher_is_better": True,
        "scaling": args.scaling, "vs_baseline": None, "dtype": "fp64" if have_ref else "fp32",
        "data": "synthetic (seeded)",
        "config": workload_config(args, world,
                                  args.M if args.scaling == "weak" else args.M // world),
        "cpu_baseline": {"value": value, "unit": "GB/s", "cores": cores, "kind": kind,
                         "sample": sample},
        "e2e": {"value": value, "unit": "GB/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
        "gpu_launches": 0,
    }
    print(json.dumps(line), flush=True)
    return 0


# ------------------------------------------------------------------ CPU baseline

def cpu_baseline(qg, mats, x, K, seconds):
    """The reference's CPU GEMV on a bounded row sample of this workload."""
    import numpy as np
    import torch

    from oracle import qformats_oracle as o
    from oracle import ref_lib

    cores = len(os.sched_getaffinity(0)) if hasattr(os, "sched_getaffinity") else os.cpu_count()
    have_ref = ref_lib.load() is not None
    xh = x.cpu().numpy()

    def runner(rows):
        fns = []
        for fmt in ("q8_0", "q4_0"):
            q, d = mats[fmt][0]
            if have_ref:
                blocks = qg.to_aos(fmt, q[:rows], d[:rows]).cpu().numpy()
                p = ref_lib.Plan(fmt, blocks, cores)
                fns.append(lambda p=p: p.run(xh))
            else:
                qh, dh = q[:rows].cpu().numpy(), d[:rows].cpu().numpy()
                fns.append(lambda f=fmt, qh=qh, dh=dh: o.dequant(f, qh, dh) @ xh)
        return lambda: [f() for f in fns]

    probe = runner(2048)
    probe()
    t0 = time.perf_counter()
    probe()
    t1 = max(time.perf_counter() - t0, 1e-6)
    M = mats["q8_0"][0][0].shape[0]
    reps = 5
    rows = int(min(M, max(2048, 2048 * seconds / (reps * t1))))
    rows -= rows % 32
    fn = runner(rows)
    fn()
    t0 = time.perf_counter()
    for _ in range(reps):
        fn()
    dt = (time.perf_counter() - t0) / reps
    step_bytes = alg_bytes("q8_0", rows, K) + alg_bytes("q4_0", rows, K)
    torch.cuda.synchronize()
    return {
        "value": step_bytes / dt / 1e9, "unit": "GB/s", "cores": cores,
        "kind": "reference" if have_ref else "port",
        "sample": (f"{rows} of {M} rows x {K}, one q8_0 + one q4_0 matvec, {reps} reps; "
                   + ("the reference's C++ float64 matvec (src/bench.cu:75-111)"
                      if have_ref else "oracle restatement of dequant(q, d) @ x")),
        "us_per_step_full_shape_est": dt * 1e6 * M / rows,
    }


# ---------------------------------------------------------------------- our arm

def main():
    args = parse()
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if args.impl == "reference":
        return reference_arm(args, rank, world)

    import torch
    import torch.distributed as dist

    import qgemv_roofline_b200 as qg
    from qgemv_roofline_b200 import roof
    from qgemv_roofline_b200.clocks import ClockSampler
    from qgemv_roofline_b200.timing import summarize, time_steps

    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        from datetime import timedelta
        dist.init_process_group("nccl", timeout=timedelta(seconds=180), device_id=dev)

    if args.workload != "xl":
        fn = stack_workload if args.workload == "stack" else batch_workload
        rc = fn(args, rank, world, dev)
        if dist.is_initialized():
            dist.barrier()
            dist.destroy_process_group()
        return rc

    def barrier():
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()

    def max_over_ranks(vals):
        t = torch.tensor(vals, dtype=torch.float64, device=dev)
        if world > 1:
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return t.tolist()

    M, K = args.M, args.K
    weak = args.scaling == "weak"
    rows = M if weak else M * (rank + 1) // world - M * rank // world
    step_bytes_rank = alg_bytes("q8_0", rows, K) + alg_bytes("q4_0", rows, K)
    ncopies = {f: max(2, math.ceil(4 * L2_BYTES / wbytes(f, rows, K))) for f in ("q8_0", "q4_0")}

    # weights: this rank's rows of W, generated and quantized on the GPU
    g = torch.Generator(device=dev).manual_seed(SEED + 7919 * rank)
    W = torch.randn(rows, K, generator=g, device=dev) * 0.02
    x = torch.randn(K, generator=torch.Generator(device=dev).manual_seed(SEED), device=dev)
    mats = {}
    for fmt in ("q8_0", "q4_0"):
        c = ncopies[fmt]
        if args.layout == "soa":
            q, d = (qg.quantize_q8_0 if fmt == "q8_0" else qg.quantize_q4_0)(W)
            mats[fmt] = [(q, d)] + [(q.clone(), d.clone()) for _ in range(c - 1)]
        else:
            b = (qg.quantize_q8_0_aos if fmt == "q8_0" else qg.quantize_q4_0_aos)(W)
            mats[fmt] = [b] + [b.clone() for _ in range(c - 1)]
    del W
    ys = {f: torch.empty(rows, device=dev) for f in mats}
    calls = [{"fmt": f, "layout": args.layout, "copies": mats[f], "M": rows, "K": K,
              "x": x, "y": ys[f]} for f in ("q8_0", "q4_0")]
    torch.cuda.synchronize()

    extras = {}
    if not args.no_extras:
        r = roof.measure(nbytes=1 << 30, batches=10, calls=5, device=dev)
        extras["roofs"] = {k: (round(v, 1) if isinstance(v, float) else v) for k, v in r.items()}
        cub = roof.cublas_fp16_mv(rows, K, copies=max(1, math.ceil(4 * L2_BYTES / (rows * K * 2))),
                                  batches=5, calls=10, device=dev)
        extras["roofs"]["cublas_fp16_mv_gbps"] = round(cub["gbps"], 1)
        extras["roofs"]["cublas_fp16_mv_shape"] = [rows, K]

    # ------------------------------------------------------------- timed region
    uuid = None
    try:
        uuid = str(torch.cuda.get_device_properties(dev).uuid)
        uuid = uuid if uuid.startswith("GPU-") else "GPU-" + uuid
    except Exception:
        pass
    barrier()
    with ClockSampler(uuid) as sampler:
        total_ms, per_ms = time_steps(calls, args.warmup, args.steps, grouped=True)
        barrier()
    clocks = sampler.summary()
    total_ms, q8_ms, q4_ms = max_over_ranks([total_ms, per_ms[0], per_ms[1]])

    # ------------------------- the fixed 98304-row matrix sharded N ways (N > 1)
    # Rank slices of M / N rows taken from the resident copies at distinct row
    # offsets (views, no new memory): copies x N distinct slices per format,
    # >= 4x L2 streamed between two reads of one slice.
    if world > 1 and weak:
        rs = M // world
        scalls = []
        for f in ("q8_0", "q4_0"):
            views = []
            for cp in mats[f]:
                for j in range(world):
                    if args.layout == "soa":
                        views.append((cp[0][j * rs:(j + 1) * rs], cp[1][j * rs:(j + 1) * rs]))
                    else:
                        views.append(cp[j * rs:(j + 1) * rs])
            scalls.append({"fmt": f, "layout": args.layout, "copies": views, "M": rs, "K": K,
                           "x": x, "y": ys[f][:rs]})
        barrier()
        s_total, s_per = time_steps(scalls, args.warmup, args.steps, grouped=True)
        barrier()
        s_total, s_q8, s_q4 = max_over_ranks([s_total, s_per[0], s_per[1]])
        s_bytes = alg_bytes("q8_0", rs, K) + alg_bytes("q4_0", rs, K)
        extras["row_sharded_fixed_M"] = {
            "M": M, "rows_per_gpu": rs, "scaling": "strong",
            "value": world * s_bytes * args.steps / (s_total * 1e-3) / 1e9, "unit": "GB/s",
            "ms_per_step": s_total / args.steps,
            "slices_rotated": {f: len(c["copies"]) for f, c in zip(("q8_0", "q4_0"), scalls)},
            "per_format": {f: {"us_per_call": ms / args.steps * 1e3,
                               "gbps_aggregate": world * alg_bytes(f, rs, K)
                               / (ms / args.steps * 1e-3) / 1e9}
                           for f, ms in (("q8_0", s_q8), ("q4_0", s_q4))}}
    K_steps = args.steps
    value = world * step_bytes_rank * K_steps / (total_ms * 1e-3) / 1e9
    peak, peak_note = measured_peak()

    def fmt_stats(fmt, ms):
        per = ms / K_steps
        b = alg_bytes(fmt, rows, K)
        return {"us_per_call": per * 1e3, "gbps_per_gpu": b / (per * 1e-3) / 1e9,
                "gbps_weight_only_per_gpu": wbytes(fmt, rows, K) / (per * 1e-3) / 1e9,
                "gbps_aggregate": world * b / (per * 1e-3) / 1e9,
                "frac_of_peak": b / (per * 1e-3) / 1e9 / peak}

    per_format = {"q8_0": fmt_stats("q8_0", q8_ms), "q4_0": fmt_stats("q4_0", q4_ms)}
    if "roofs" in extras:
        sr = extras["roofs"]["stream_read_gbps"]
        for f in per_format:
            per_format[f]["frac_of_stream_read_roof"] = per_format[f]["gbps_per_gpu"] / sr
    dom = "q8_0" if q8_ms >= q4_ms else "q4_0"
    # the configuration the library dispatches for this slice (csrc/gemv_tma.cu)
    if dom == "q4_0":
        targs = "4,1,8,16" if rows * (K // 2 + K // 16) >= (150 << 20) else "4,1,8,8"
    else:
        targs = "8,1,4,8" if rows * (K + K // 16) < (256 << 20) else "8,1,4,16"
    kname = f"k_gemv_tma<{targs},{'false' if args.layout == 'soa' else 'true'}"
    kname += ",4096>" if args.layout == "soa" and K == 4096 else ">"
    ach = per_format[dom]["gbps_per_gpu"]
    traffic = dram_traffic(f"{dom}_{args.layout}_{rows}x{K}")
    roofline = {"bound": "hbm", "achieved": ach, "peak": peak, "unit": "GB/s",
                "frac": ach / peak, "traffic": traffic, "kernel": kname,
                "note": f"peak {peak_note}; achieved = algorithmic bytes per launch "
                        f"({alg_bytes(dom, rows, K)}) / mean launch time (CUDA events)"}

    # ------------------------------------- opt-in q8_1 activations (not the metric)
    # x rounded to int8 per 32-element block inside the kernel (ggml's q8_1
    # route): reported beside the exact path, never as its value.
    calls81 = [dict(c, activations="q8_1") for c in calls]
    n81 = min(args.steps, 2000)
    _, per81 = time_steps(calls81, min(args.warmup, 20), n81, grouped=True)
    q8_81, q4_81 = max_over_ranks(per81)
    extras["opt_in_q8_1"] = {
        f: {"us_per_call": ms / n81 * 1e3,
            "gbps_per_gpu": alg_bytes(f, rows, K) / (ms / n81 * 1e-3) / 1e9,
            "frac_of_peak": alg_bytes(f, rows, K) / (ms / n81 * 1e-3) / 1e9 / peak}
        for f, ms in (("q8_0", q8_81), ("q4_0", q4_81))}
    extras["opt_in_q8_1"]["numerics"] = ("x rounded to int8 per 32-element block (q8_1); "
                                         "outside the exact path's 1e-5 bound; "
                                         f"{n81} calls per format, after the timed region")

    # ---------------------------------------------------------- NCCL all-gather
    if world > 1:
        yfull = torch.empty(rows * world, device=dev)
        yl = ys["q8_0"]
        for _ in range(5):
            dist.all_gather_into_tensor(yfull, yl)
        barrier()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        n_ag = 200
        for _ in range(n_ag):
            dist.all_gather_into_tensor(yfull, yl)
        b.record()
        b.synchronize()
        (ag_ms,) = max_over_ranks([a.elapsed_time(b) / n_ag])
        extras["allgather_y"] = {"us_per_call": ag_ms * 1e3, "bytes": rows * world * 4,
                                 "backend": "nccl"}

    # --------------------------------------------------------------- end to end
    e2e = None
    if not args.no_extras:
        mq = {f: qg.QuantizedMatrix(f, rows, K, "soa", q=mats[f][0][0], d=mats[f][0][1])
              if args.layout == "soa" else qg.QuantizedMatrix(f, rows, K, "aos", blocks=mats[f][0])
              for f in mats}
        mq = {f: [m] for f, m in mq.items()}
        for f in mats:
            for c in range(1, ncopies[f]):
                if args.layout == "soa":
                    mq[f].append(qg.QuantizedMatrix(f, rows, K, "soa", q=mats[f][c][0],
                                                    d=mats[f][c][1]))
                else:
                    mq[f].append(qg.QuantizedMatrix(f, rows, K, "aos", blocks=mats[f][c]))
        xh = x.cpu().pin_memory()
        yh = {f: torch.empty(rows, pin_memory=True) for f in mats}
        xd = torch.empty_like(x)
        st = torch.cuda.current_stream()
        n_e2e = min(args.steps, 2000)

        # results are read back on a copy stream, so the q8_0 read-back overlaps
        # the q4_0 GEMV and the two GEMVs stay adjacent on the compute stream
        cst = torch.cuda.Stream(device=dev)
        done = {f: torch.cuda.Event() for f in mats}

        def e2e_step(i):
            xd.copy_(xh, non_blocking=True)
            for f in ("q8_0", "q4_0"):
                y = mq[f][i % ncopies[f]].matvec(xd, ys[f])
                done[f].record(st)
                cst.wait_event(done[f])
                with torch.cuda.stream(cst):
                    yh[f].copy_(y, non_blocking=True)
            cst.synchronize()
            st.synchronize()

        for i in range(min(args.warmup, 20)):
            e2e_step(i)
        barrier()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        for i in range(n_e2e):
            e2e_step(i)
        b.record()
        b.synchronize()
        (e2e_ms,) = max_over_ranks([a.elapsed_time(b)])
        e2e = {"value": world * step_bytes_rank * n_e2e / (e2e_ms * 1e-3) / 1e9, "unit": "GB/s",
               "h2d_bytes_per_step": world * 4 * K, "d2h_bytes_per_step": world * 2 * 4 * rows,
               "steps": n_e2e, "us_per_step": e2e_ms * 1e3 / n_e2e,
               "path": "QuantizedMatrix.matvec -> qgemv -> C ABI, pinned host x/y "
                       "(read back on a copy stream), host sync every step"}

    cpu = None
    if rank == 0 and world == 1 and not args.no_extras:
        cpu = cpu_baseline(qg, mats if args.layout == "soa" else
                           {f: [qg.from_aos(f, mats[f][0])] for f in mats}, x, K, args.cpu_seconds)

    if rank == 0:
        dinfo = qg.device_info(local)
        line = {
            "metric": METRIC, "value": value, "unit": "GB/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": total_ms / K_steps,
            "higher_is_better": True, "scaling": args.scaling, "vs_baseline": None,
            "dtype": "fp32", "data": "synthetic (seeded N(0, 0.02) weights, N(0, 1) x)",
            "config": workload_config(args, world, rows, ncopies),
            "roofline": roofline, "cpu_baseline": cpu, "e2e": e2e,
            "gpu_launches": 2 * K_steps * world, "clocks": clocks,
            "per_format": per_format, **extras,
            "device": {"name": dinfo["name"], "sms": dinfo["sms"], "l2_bytes": dinfo["l2_bytes"],
                       "datasheet_gbps": round(dinfo["datasheet_gbps"], 1)},
        }
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    return 0


if __name__ == "__main__":
    sys.exit(main())
