"""Event timing and summary statistics.

The reference bracketed every launch with its own event pair and reported
median/min/max/mean/sd/p95 over the samples (src/bench.cu:115-156).  For
microsecond-scale calls that per-launch bracket measures launch gaps, so here
a *sample* is a batch of back-to-back calls between one event pair, divided
by the number of calls; the same six statistics are reported over batches.
"""

from __future__ import annotations

import math
from typing import Callable

import torch


def summarize(samples):
    """median/min/max/mean/sd/p95 of a list of numbers (src/bench.cu:117-132)."""
    s = sorted(samples)
    n = len(s)
    if n == 0:
        return {"median": math.nan, "min": math.nan, "max": math.nan, "mean": math.nan,
                "sd": math.nan, "p95": math.nan, "n": 0}
    mean = sum(s) / n
    var = sum((v - mean) ** 2 for v in s) / n
    return {"median": s[n // 2], "min": s[0], "max": s[-1], "mean": mean,
            "sd": math.sqrt(var), "p95": s[int(0.95 * (n - 1))], "n": n}


def time_calls(fn: Callable[[int], None], calls_per_batch: int, batches: int,
               warmup_calls: int = 3, stream: torch.cuda.Stream | None = None):
    """Times ``fn(i)`` (i = running call index, for rotating buffers).

    Returns per-call milliseconds, one sample per batch of ``calls_per_batch``
    back-to-back calls timed with CUDA events recorded on ``stream``.
    """
    st = stream or torch.cuda.current_stream()
    i = 0
    with torch.cuda.stream(st):
        for _ in range(warmup_calls):
            fn(i)
            i += 1
        st.synchronize()
        out = []
        for _ in range(batches):
            a = torch.cuda.Event(enable_timing=True)
            b = torch.cuda.Event(enable_timing=True)
            a.record(st)
            for _ in range(calls_per_batch):
                fn(i)
                i += 1
            b.record(st)
            b.synchronize()
            out.append(a.elapsed_time(b) / calls_per_batch)
    return out


def time_steps(calls, warmup: int, steps: int, stream: int | None = None,
               grouped: bool = False):
    """Native timed loop (qgemv_time_steps in include/qgemv_b200.h).

    ``calls``: list of dicts with keys fmt ("q8_0"/"q4_0"), layout ("soa"/"aos"),
    optional activations ("exact", default, or "q8_1": one column, the opt-in
    int8-activation kernel), copies (list of (q, d) tensor pairs for SoA, or
    block tensors for AoS),
    M, K, x [N, K] or [K], y.  Step i runs every call once on copy
    i % len(copies).  grouped=False: steps in order, an event after every
    call; grouped=True: each call's launches back to back as one group, events
    only between groups.  Returns (total_ms, [ms of call j summed over steps]).
    """
    import ctypes

    from . import _lib

    descs = (_lib.CallDesc * len(calls))()
    keep = []
    for j, c in enumerate(calls):
        copies = c["copies"]
        n = len(copies)
        qs = (ctypes.c_void_p * n)()
        ds = (ctypes.c_void_p * n)()
        for k, cp in enumerate(copies):
            if c.get("layout", "soa") == "soa":
                qs[k], ds[k] = cp[0].data_ptr(), cp[1].data_ptr()
            else:
                qs[k] = cp.data_ptr()
        keep += [qs, ds]
        x, y = c["x"], c["y"]
        N = 1 if x.dim() == 1 else x.shape[0]
        descs[j].format = _lib.FORMAT_CODE[c["fmt"]]
        descs[j].layout = ((0 if c.get("layout", "soa") == "soa" else 1)
                           + (2 if c.get("activations", "exact") == "q8_1" else 0))
        descs[j].ncopies = n
        descs[j].ncols = N
        descs[j].M, descs[j].K = c["M"], c["K"]
        descs[j].ldx = c["K"] if N == 1 else x.stride(0)
        descs[j].ldy = c["M"] if N == 1 else y.stride(0)
        descs[j].q = ctypes.cast(qs, ctypes.POINTER(ctypes.c_void_p))
        descs[j].d = ctypes.cast(ds, ctypes.POINTER(ctypes.c_void_p))
        descs[j].x, descs[j].y = x.data_ptr(), y.data_ptr()
    out = (ctypes.c_float * (len(calls) + 1))()
    st = torch.cuda.current_stream().cuda_stream if stream is None else stream
    _lib.call("qgemv_time_steps", descs, len(calls), warmup, steps, int(grouped), st, out)
    return float(out[0]), [float(out[1 + j]) for j in range(len(calls))]
