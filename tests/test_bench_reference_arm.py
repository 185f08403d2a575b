"""The reference arm of bench.py on the CPU: `bench.py --impl reference` times
the reference's own CPU GEMV (src/bench.cu:75-111, built into oracle/_ref; the
oracle's restatement when it is absent) and prints one JSON line with the
same metric, unit and config as the GPU arm, a cpu_baseline describing the
run and an e2e record with no host<->device bytes.  Under torchrun only rank 0
prints; the other ranks exit 0 without work.  Small shapes keep it to seconds."""

import json
import os
import subprocess
import sys

import pytest

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, REPO)

import bench  # noqa: E402

ARGS = ["--impl", "reference", "--steps", "2", "--warmup", "1", "--M", "1024", "--K", "4096"]


def _lines(out):
    return [json.loads(l) for l in out.splitlines() if l.startswith("{")]


def test_reference_arm_line():
    p = subprocess.run([sys.executable, os.path.join(REPO, "bench.py"), *ARGS], cwd=REPO,
                       capture_output=True, text=True, timeout=300)
    assert p.returncode == 0, p.stderr[-2000:]
    lines = _lines(p.stdout)
    assert len(lines) == 1
    line = lines[0]
    assert line["impl"] == "reference"
    assert line["metric"] == bench.METRIC and line["unit"] == "GB/s"
    assert line["higher_is_better"] is True and line["n_gpus"] == 1
    assert line["steps"] == 2 and line["warmup"] == 1
    assert line["value"] > 0 and line["gpu_launches"] == 0
    # the same workload description as the GPU arm's line for these arguments
    sys_argv = sys.argv
    try:
        sys.argv = ["bench.py", *ARGS]
        args = bench.parse()
    finally:
        sys.argv = sys_argv
    assert line["config"] == bench.workload_config(args, 1, 1024, bench.xl_copies(1024, 4096))
    cpu = line["cpu_baseline"]
    assert cpu["value"] == line["value"] and cpu["cores"] >= 1
    assert cpu["kind"] in ("reference", "port") and cpu["sample"]
    e2e = line["e2e"]
    assert e2e["value"] == line["value"] and e2e["unit"] == line["unit"]
    assert e2e["h2d_bytes_per_step"] == 0 and e2e["d2h_bytes_per_step"] == 0


def test_reference_arm_under_torchrun_prints_once():
    cmd = [sys.executable, "-m", "torch.distributed.run", "--nnodes", "1", "--nproc-per-node", "2",
           "--master-addr", "127.0.0.1", "--master-port", "29561",
           os.path.join(REPO, "bench.py"), *ARGS, "--gpus", "2"]
    p = subprocess.run(cmd, cwd=REPO, capture_output=True, text=True, timeout=300)
    assert p.returncode == 0, p.stderr[-2000:]
    lines = _lines(p.stdout)
    assert len(lines) == 1 and lines[0]["impl"] == "reference" and lines[0]["n_gpus"] == 2
