"""Roof probes run and report plausible B200 bandwidths."""

import pytest
import torch

from qgemv_roofline_b200 import roof

pytestmark = pytest.mark.gpu


def test_roof_measure_small():
    r = roof.measure(nbytes=256 << 20, batches=3, calls=2)
    assert r["bulk_read_status"] == 0
    for k in ("stream_read_gbps", "bulk_read_gbps", "d2d_gbps"):
        assert 500 < r[k] < 20000, (k, r[k])


def test_cublas_mv_reference_point():
    r = roof.cublas_fp16_mv(4096, 4096, copies=4, batches=3, calls=4)
    assert r["gbps"] > 100
    torch.cuda.synchronize()
