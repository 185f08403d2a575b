"""qgemv_roofline_b200: ggml q8_0 / q4_0 quantized GEMV for NVIDIA B200 (sm_100a).

Public API (torch tensors as buffers; compute in libqgemv_b200.so):

* format API mirroring the reference's python/qformats.py:
  ``QK``, ``quantize_q8_0``, ``quantize_q4_0``, ``dequant_q8_0``,
  ``dequant_q4_0``, plus ``to_aos`` / ``from_aos`` and ``quantize_*_aos``;
* GEMV: ``qgemv(fmt, q, d, x)``, ``qgemv_aos(fmt, blocks, x)``,
  ``qgemv_tiled(fmt, tile_weights(fmt, q, d), M, K, X)`` (batch tiles),
  ``qgemv_tc(tile_weights_tc(q, d, fmt=fmt), M, K, X, fmt=fmt)`` (the tcgen05 tensor cores),
  ``QuantizedMatrix``;
* GGUF files: ``gguf.GGUFReader`` (load q8_0 / q4_0 tensors onto a GPU), ``gguf.write_gguf``;
* roof probes: ``roof.measure``, ``roof.cublas_fp16_mv``;
* multi-GPU row sharding: ``shard.ShardedQGemv``; the decode layer stack:
  ``stack.DecodeStack``.
"""

from . import _lib, gemv, gguf, qformats, roof, shard, stack, timing  # noqa: F401
from ._lib import QGemvError, device_info  # noqa: F401
from .gemv import (QuantizedMatrix, algorithmic_bytes, qgemv, qgemv_aos,  # noqa: F401
                   qgemv_tc, qgemv_tiled, tile_weights, tile_weights_tc)
from .qformats import (QK, dequant_q4_0, dequant_q8_0, from_aos, quantize_q4_0,  # noqa: F401
                       quantize_q4_0_aos, quantize_q8_0, quantize_q8_0_aos, to_aos, weight_bytes)

__version__ = "1.0.0"
