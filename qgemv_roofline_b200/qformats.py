"""ggml q8_0 / q4_0 block formats on the GPU: the reference's format API.

Same names, signatures and outputs as the reference's python/qformats.py
(``QK``, ``quantize_q8_0``, ``quantize_q4_0``, ``dequant_q8_0``,
``dequant_q4_0``; python/qformats.py:14-56): the quantizers return the SoA
planes ``(q int8 [M, K], d float16 [M, K/32])`` and
``(packed uint8 [M, K/2], d float16 [M, K/32])``, byte-identical to the
reference.  Added: ``to_aos`` / ``from_aos`` (ggml block bytes, so a row is
a row of a GGUF tensor) and ``quantize_*_aos``.

All work runs in the sm_100a kernels of libqgemv_b200.so.  CUDA tensors stay
on their device; CPU tensors are copied to the current CUDA device, processed
there and copied back (results are still CPU tensors, as the reference
returns).  Without a CUDA device every function raises: there is no CPU
implementation in this package.
"""

from __future__ import annotations

import torch

from . import _lib

QK = 32
BLOCK_BYTES = {"q8_0": 34, "q4_0": 18}


def _stream_ptr(t: torch.Tensor) -> int:
    return torch.cuda.current_stream(t.device).cuda_stream


def _to_device(t: torch.Tensor):
    """(tensor on CUDA, original device)."""
    if t.is_cuda:
        return t, t.device
    if not torch.cuda.is_available():
        raise RuntimeError("qgemv_roofline_b200 runs on CUDA (sm_100a) only; no GPU is available")
    return t.cuda(), t.device


def _check_w(W: torch.Tensor):
    if W.dim() != 2:
        raise RuntimeError(f"W must be 2-D [M, K], got shape {tuple(W.shape)}")
    M, K = W.shape
    if K % QK:
        raise RuntimeError(f"shape '[{M}, {K // QK}, {QK}]' is invalid for input of size {M * K}")
    if W.dtype != torch.float32:
        raise TypeError(f"W must be float32, got {W.dtype}")
    return M, K


def _quantize(fmt: str, W: torch.Tensor, aos: bool):
    M, K = _check_w(W)
    Wd, home = _to_device(W)
    if Wd.stride(1) != 1:
        Wd = Wd.contiguous()
    dev = Wd.device
    with torch.cuda.device(dev):
        if aos:
            blocks = torch.empty((M, K // QK, BLOCK_BYTES[fmt]), dtype=torch.uint8, device=dev)
            _lib.call("qgemv_quantize_aos", _lib.FORMAT_CODE[fmt], Wd.data_ptr(), M, K,
                      Wd.stride(0), blocks.data_ptr(), _stream_ptr(Wd))
            return blocks.to(home)
        qcols = K if fmt == "q8_0" else K // 2
        q = torch.empty((M, qcols), dtype=torch.int8 if fmt == "q8_0" else torch.uint8, device=dev)
        d = torch.empty((M, K // QK), dtype=torch.float16, device=dev)
        _lib.call("qgemv_quantize_soa", _lib.FORMAT_CODE[fmt], Wd.data_ptr(), M, K,
                  Wd.stride(0), q.data_ptr(), d.data_ptr(), _stream_ptr(Wd))
        return q.to(home), d.to(home)


def quantize_q8_0(W: torch.Tensor):
    """ggml q8_0 (qformats.py:17-25): per 32-weight block d = amax/127, q = round(w/d)."""
    return _quantize("q8_0", W, aos=False)


def quantize_q4_0(W: torch.Tensor):
    """ggml q4_0 (qformats.py:28-40): d = (signed value of largest magnitude)/-8,
    q = clamp(trunc(w/d + 8.5), 0, 15), packed low nibble = weights 0-15."""
    return _quantize("q4_0", W, aos=False)


def quantize_q8_0_aos(W: torch.Tensor) -> torch.Tensor:
    """q8_0 straight to ggml blocks, uint8 [M, K/32, 34]."""
    return _quantize("q8_0", W, aos=True)


def quantize_q4_0_aos(W: torch.Tensor) -> torch.Tensor:
    """q4_0 straight to ggml blocks, uint8 [M, K/32, 18]."""
    return _quantize("q4_0", W, aos=True)


def _dequant(fmt: str, q: torch.Tensor, d: torch.Tensor) -> torch.Tensor:
    if q.dim() != 2 or d.dim() != 2:
        raise RuntimeError("q and d must be 2-D")
    M = q.shape[0]
    K = q.shape[1] if fmt == "q8_0" else q.shape[1] * 2
    if K % QK or tuple(d.shape) != (M, K // QK):
        raise RuntimeError(f"shape mismatch: q {tuple(q.shape)}, d {tuple(d.shape)}")
    if d.dtype != torch.float16:
        raise TypeError(f"d must be float16, got {d.dtype}")
    qd, home = _to_device(q)
    dd = d.to(qd.device).contiguous()
    qd = qd.contiguous()
    with torch.cuda.device(qd.device):
        w = torch.empty((M, K), dtype=torch.float32, device=qd.device)
        _lib.call("qgemv_dequant_soa", _lib.FORMAT_CODE[fmt], qd.data_ptr(), dd.data_ptr(),
                  w.data_ptr(), M, K, _stream_ptr(qd))
    return w.to(home)


def dequant_q8_0(q: torch.Tensor, d: torch.Tensor) -> torch.Tensor:
    """fp32 weights q * d (qformats.py:43-46)."""
    return _dequant("q8_0", q, d)


def dequant_q4_0(packed: torch.Tensor, d: torch.Tensor) -> torch.Tensor:
    """fp32 weights (nibble - 8) * d (qformats.py:49-56)."""
    return _dequant("q4_0", packed, d)


def to_aos(fmt: str, q: torch.Tensor, d: torch.Tensor) -> torch.Tensor:
    """SoA planes -> ggml blocks uint8 [M, K/32, 34|18] (src/bench.cu:300-314, inverse)."""
    M = q.shape[0]
    K = q.shape[1] if fmt == "q8_0" else q.shape[1] * 2
    qd, home = _to_device(q)
    qd = qd.contiguous()
    dd = d.to(qd.device).contiguous()
    with torch.cuda.device(qd.device):
        blocks = torch.empty((M, K // QK, BLOCK_BYTES[fmt]), dtype=torch.uint8, device=qd.device)
        _lib.call("qgemv_repack", _lib.FORMAT_CODE[fmt], 0, blocks.data_ptr(), qd.data_ptr(),
                  dd.data_ptr(), M, K, _stream_ptr(qd))
    return blocks.to(home)


def from_aos(fmt: str, blocks: torch.Tensor):
    """ggml blocks uint8 [M, K/32, 34|18] -> SoA planes (q, d) (src/bench.cu:300-314)."""
    if blocks.dim() != 3 or blocks.shape[2] != BLOCK_BYTES[fmt] or blocks.dtype != torch.uint8:
        raise RuntimeError(f"blocks must be uint8 [M, K/32, {BLOCK_BYTES[fmt]}]")
    M, nb, _ = blocks.shape
    K = nb * QK
    bd, home = _to_device(blocks)
    bd = bd.contiguous()
    with torch.cuda.device(bd.device):
        qcols = K if fmt == "q8_0" else K // 2
        q = torch.empty((M, qcols), dtype=torch.int8 if fmt == "q8_0" else torch.uint8,
                        device=bd.device)
        d = torch.empty((M, nb), dtype=torch.float16, device=bd.device)
        _lib.call("qgemv_repack", _lib.FORMAT_CODE[fmt], 1, bd.data_ptr(), q.data_ptr(),
                  d.data_ptr(), M, K, _stream_ptr(bd))
    return q.to(home), d.to(home)


def weight_bytes(fmt: str, M: int, K: int) -> int:
    """Bytes of a quantized [M, K] matrix: M * K * (34 | 18) / 32."""
    return M * (K // QK) * BLOCK_BYTES[fmt]
