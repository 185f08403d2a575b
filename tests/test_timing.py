"""The timing harness (the reference's time_kernel / summarize,
src/bench.cu:115-156) and the clock sampler: statistics on the CPU, and the
native timed loop qgemv_time_steps on the GPU (its outputs are the GEMVs'
own results, its times are positive and consistent between the interleaved
and the grouped order)."""

import math

import pytest
import torch

from qgemv_roofline_b200.clocks import ClockSampler
from qgemv_roofline_b200.timing import summarize


def test_summarize_six_statistics():
    s = summarize([4.0, 1.0, 3.0, 2.0, 5.0])
    assert (s["median"], s["min"], s["max"], s["mean"], s["n"]) == (3.0, 1.0, 5.0, 3.0, 5)
    assert math.isclose(s["sd"], math.sqrt(2.0))
    assert s["p95"] == 4.0  # element int(0.95 * (n - 1)) of the sorted samples
    e = summarize([])
    assert e["n"] == 0 and math.isnan(e["median"])


def test_clock_sampler_summary_from_rows():
    cs = ClockSampler()
    # index, uuid, sm, max sm, power, active, hw, hw thermal, sw thermal, sw power cap
    cs.rows = [["0", "GPU-x", "1965", "1965", "700", "0x0", "Not Active", "Not Active",
                "Not Active", "Not Active"],
               ["0", "GPU-x", "1600", "1965", "990", "0x4", "Not Active", "Not Active",
                "Not Active", "Active"],
               ["0", "GPU-x", "300", "1965", "100", "0x1", "Not Active", "Not Active",
                "Not Active", "Not Active"]]
    s = cs.summary()
    assert s["sm_max_mhz"] == 1965.0 and s["samples"] == 3
    assert s["sm_mhz"] in (1600.0, 1965.0)       # idle samples (300) are not "under load"
    assert s["reasons"] == ["sw_power_cap"]
    assert ClockSampler().summary() is None
    assert ClockSampler().keep_busy(lambda: None) == 0  # no nvidia-smi process started


@pytest.mark.gpu
def test_time_steps_results_and_orders():
    import qgemv_roofline_b200 as qg
    from qgemv_roofline_b200.timing import time_steps

    dev = torch.device("cuda", 0)
    g = torch.Generator(device=dev).manual_seed(11)
    M, K = 2048, 4096
    W = torch.randn(M, K, generator=g, device=dev) * 0.02
    x = torch.randn(K, generator=g, device=dev)
    calls = []
    for fmt in ("q8_0", "q4_0"):
        q, d = (qg.quantize_q8_0 if fmt == "q8_0" else qg.quantize_q4_0)(W)
        cps = [(q, d), (q.clone(), d.clone()), (q.clone(), d.clone())]
        calls.append({"fmt": fmt, "layout": "soa", "M": M, "K": K, "x": x,
                      "y": torch.full((M,), float("nan"), device=dev), "copies": cps})
    for grouped in (False, True):
        total, per = time_steps(calls, 3, 50, grouped=grouped)
        assert total > 0 and all(p > 0 for p in per)
        assert sum(per) <= total * 1.05 + 1e-3       # the calls fit in the timed region
        for c in calls:
            want = qg.qgemv(c["fmt"], c["copies"][0][0], c["copies"][0][1], x)
            assert torch.equal(c["y"], want)         # every copy holds the same bytes
    # the GGUF-block layout goes through the same harness
    blocks = qg.to_aos("q8_0", calls[0]["copies"][0][0], calls[0]["copies"][0][1])
    y = torch.empty(M, device=dev)
    total, per = time_steps([{"fmt": "q8_0", "layout": "aos", "M": M, "K": K, "x": x, "y": y,
                              "copies": [blocks]}], 2, 20)
    assert total > 0
    assert torch.equal(y, qg.qgemv_aos("q8_0", blocks, x))
    qg._lib.call("qgemv_check_device_error", 0, None)
