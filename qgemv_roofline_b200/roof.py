"""The HBM read roof, measured three ways on the device (src/bench.cu:162-206,
python/triton_qgemv.py:171-185): a streaming-read kernel (128-bit loads; and
a TMA bulk-copy variant), a device-to-device copy, and a cuBLAS fp16 matvec
of the GEMV's shape.  The read roof is the better of the two read probes.
"""

from __future__ import annotations

import torch

from . import _lib
from .timing import summarize, time_calls


def stream_read(buf: torch.Tensor, sink: torch.Tensor, blocks_per_sm: int = 4,
                stream: int | None = None) -> None:
    st = torch.cuda.current_stream(buf.device).cuda_stream if stream is None else stream
    _lib.call("qgemv_roof_stream_read", buf.data_ptr(), buf.numel() * buf.element_size(),
              sink.data_ptr(), blocks_per_sm, st)


def bulk_read(buf: torch.Tensor, sink: torch.Tensor, status: torch.Tensor,
              stream: int | None = None) -> None:
    st = torch.cuda.current_stream(buf.device).cuda_stream if stream is None else stream
    _lib.call("qgemv_roof_bulk_read", buf.data_ptr(), buf.numel() * buf.element_size(),
              sink.data_ptr(), status.data_ptr(), st)


def d2d(dst: torch.Tensor, src: torch.Tensor, stream: int | None = None) -> None:
    st = torch.cuda.current_stream(src.device).cuda_stream if stream is None else stream
    _lib.call("qgemv_roof_d2d", dst.data_ptr(), src.data_ptr(),
              src.numel() * src.element_size(), st)


def measure(nbytes: int = 1 << 30, batches: int = 10, calls: int = 5,
            blocks_per_sm: int = 4, device=None) -> dict:
    """GB/s (1e9 B/s) of the three device roofs on a buffer of ``nbytes``
    (>= 4x the 126 MB L2 by default)."""
    device = device or torch.device("cuda", torch.cuda.current_device())
    buf = torch.empty(nbytes, dtype=torch.uint8, device=device).fill_(1)
    sink = torch.zeros(4, dtype=torch.int32, device=device)
    status = torch.zeros(1, dtype=torch.int32, device=device)
    out = {"bytes": nbytes}
    # the 128-bit stream read at several CTAs per SM (more bytes in flight per
    # SM with more CTAs); the best configuration is the probe's figure
    sweep = {}
    for bps in sorted({blocks_per_sm, 8, 16}):
        ms = time_calls(lambda i, b=bps: stream_read(buf, sink, b), calls, batches)
        sweep[bps] = nbytes / (summarize(ms)["median"] * 1e-3) / 1e9
    best = max(sweep, key=sweep.get)
    out["stream_read_gbps"] = sweep[best]
    out["stream_read_blocks_per_sm"] = best
    out["stream_read_sweep_gbps"] = {str(k): round(v, 1) for k, v in sweep.items()}
    ms = time_calls(lambda i: bulk_read(buf, sink, status), calls, batches)
    s = summarize(ms)
    torch.cuda.synchronize(device)
    out["bulk_read_gbps"] = nbytes / (s["median"] * 1e-3) / 1e9
    out["bulk_read_status"] = int(status.item())
    half = nbytes // 2
    ms = time_calls(lambda i: d2d(buf[half:], buf[:half]), calls, batches)
    s = summarize(ms)
    out["d2d_gbps"] = 2 * half / (s["median"] * 1e-3) / 1e9  # read + write
    # the read roof: the best of the two read probes
    out["read_roof_gbps"] = max(out["stream_read_gbps"], out["bulk_read_gbps"])
    del buf
    return out


def cublas_fp16_mv(M: int, K: int, copies: int, batches: int = 10, calls: int = 10,
                   device=None) -> dict:
    """torch.mv (cuBLAS) on fp16 [M, K] weights, rotating ``copies`` weight
    copies so the working set exceeds L2.  GB/s counts M*K*2 weight bytes."""
    device = device or torch.device("cuda", torch.cuda.current_device())
    g = torch.Generator(device=device).manual_seed(5)
    Ws = [torch.randn(M, K, generator=g, device=device, dtype=torch.float16) for _ in range(copies)]
    x = torch.randn(K, generator=g, device=device, dtype=torch.float16)
    y = torch.empty(M, device=device, dtype=torch.float16)
    ms = time_calls(lambda i: torch.mv(Ws[i % copies], x, out=y), calls, batches)
    s = summarize(ms)
    return {"M": M, "K": K, "copies": copies, "us": s["median"] * 1e3,
            "gbps": M * K * 2 / (s["median"] * 1e-3) / 1e9}
