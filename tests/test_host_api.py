"""Host-side API behaviour that needs no GPU: shape/dtype errors and the
absence of any CPU fallback."""

import pytest
import torch

import qgemv_roofline_b200 as qg
from qgemv_roofline_b200 import gemv


def test_reference_names_exported():
    for name in ("QK", "quantize_q8_0", "quantize_q4_0", "dequant_q8_0", "dequant_q4_0"):
        assert hasattr(qg, name)
    assert qg.QK == 32


def test_shape_and_dtype_errors_match_reference_style():
    with pytest.raises(RuntimeError, match="invalid for input of size"):
        qg.quantize_q8_0(torch.zeros(4, 40))
    with pytest.raises(RuntimeError):
        qg.quantize_q4_0(torch.zeros(40))
    with pytest.raises(TypeError):
        qg.quantize_q8_0(torch.zeros(4, 64, dtype=torch.float16))


@pytest.mark.skipif(torch.cuda.is_available(), reason="checks the no-GPU behaviour")
def test_no_cpu_fallback_without_gpu():
    with pytest.raises(RuntimeError, match="CUDA"):
        qg.quantize_q8_0(torch.zeros(4, 64))
    with pytest.raises(RuntimeError, match="CUDA"):
        qg.dequant_q4_0(torch.zeros(4, 32, dtype=torch.uint8), torch.zeros(4, 2, dtype=torch.float16))
    with pytest.raises(ValueError, match="CUDA"):
        qg.qgemv("q8_0", torch.zeros(4, 64, dtype=torch.int8), torch.zeros(4, 2, dtype=torch.float16),
                 torch.zeros(64))


def test_algorithmic_bytes():
    assert gemv.algorithmic_bytes("q8_0", 98304, 4096) == 98304 * 128 * 34 + 4 * 4096 + 4 * 98304
    assert qg.weight_bytes("q4_0", 11008, 4096) == 25362432
    assert qg.weight_bytes("q8_0", 4096, 4096) == 17825792
