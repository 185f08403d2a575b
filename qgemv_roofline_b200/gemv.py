"""Quantized GEMV entry points: ``y = W x`` and ``Y = X W^T`` for N <= 16 columns.

The reference's kernels took ``(Q, D, x, y, M, K)`` for one fp32 column
(src/qgemv_kernels.cuh); these wrappers take torch tensors, validate them,
and call the C ABI (include/qgemv_b200.h) with their device pointers on the
current CUDA stream.  ``x`` is ``[K]`` (returns ``[M]``) or ``[N, K]`` (returns
``[N, M]``; row n of X is activation vector n).  Tensors must already be on
the GPU: this is the hot path and it does no implicit copies.
"""

from __future__ import annotations

import functools
from dataclasses import dataclass

import torch

from . import _lib
from .qformats import BLOCK_BYTES, QK

_SOA_FN = {"q8_0": "qgemv_q8_0_soa", "q4_0": "qgemv_q4_0_soa"}
_AOS_FN = {"q8_0": "qgemv_q8_0_aos", "q4_0": "qgemv_q4_0_aos"}


def _on_tensor_device(fn):
    """Runs ``fn`` with the device of its first CUDA tensor argument current:
    the C ABI launches on the current device, and the per-device state it
    keeps (workspaces, tile counters) belongs to that device too."""
    @functools.wraps(fn)
    def wrapper(*args, **kwargs):
        for a in (*args, *kwargs.values()):
            if isinstance(a, torch.Tensor) and a.is_cuda:
                with torch.cuda.device(a.device):
                    return fn(*args, **kwargs)
        return fn(*args, **kwargs)
    return wrapper


def _check_fmt(fmt: str):
    if fmt not in _SOA_FN:
        raise ValueError(f"format must be 'q8_0' or 'q4_0', got {fmt!r}")


def _xy(x: torch.Tensor, M: int, K: int, y: torch.Tensor | None, device):
    if not x.is_cuda or x.device != device:
        raise ValueError(f"x must be a CUDA tensor on {device}")
    if x.dtype != torch.float32:
        raise TypeError(f"x must be float32, got {x.dtype}")
    vec = x.dim() == 1
    X = x.unsqueeze(0) if vec else x
    if X.dim() != 2 or X.shape[1] != K:
        raise ValueError(f"x must be [K={K}] or [N, K={K}], got {tuple(x.shape)}")
    if X.stride(1) != 1:
        X = X.contiguous()
    N = X.shape[0]
    if y is None:
        Y = torch.empty((N, M), dtype=torch.float32, device=device)
        y = Y[0] if vec else Y
    else:
        if y.dtype != torch.float32 or y.device != device:
            raise ValueError("y must be a float32 tensor on the weights' device")
        Y = y.unsqueeze(0) if y.dim() == 1 else y
        if tuple(Y.shape) != (N, M) or Y.stride(1) != 1:
            raise ValueError(f"y must be [{M}] or [N, {M}] with unit last stride")
    ldx = X.stride(0) if N > 1 else K
    ldy = Y.stride(0) if N > 1 else M
    return X, Y, y, N, ldx, ldy


# Workspaces of the batched calls, one per (device, torch stream), grown on
# demand: calls on one stream are ordered, so they may share it.
_WS: dict = {}


def _workspace(device, nbytes: int, stream) -> torch.Tensor:
    """A device buffer of at least ``nbytes`` for a call on the current torch
    stream (``stream`` None).  Under stream capture, or for a raw stream
    handle, a fresh buffer from torch's caching allocator (stream-ordered; a
    captured graph keeps its own)."""
    nbytes = max(int(nbytes), 16)
    cur = torch.cuda.current_stream(device)
    if stream is not None or torch.cuda.is_current_stream_capturing():
        return torch.empty(nbytes, dtype=torch.uint8, device=device)
    key = (device.index, cur.stream_id, cur.cuda_stream)
    ws = _WS.get(key)
    if ws is None or ws.numel() < nbytes:
        ws = torch.empty(nbytes, dtype=torch.uint8, device=device)
        _WS[key] = ws
    return ws


def _check_act(activations: str, N: int):
    if activations not in ("exact", "q8_1"):
        raise ValueError(f"activations must be 'exact' or 'q8_1', got {activations!r}")
    if activations == "q8_1" and N != 1:
        raise ValueError("q8_1 activations are a single-column path (x must be [K])")


@_on_tensor_device
def qgemv(fmt: str, q: torch.Tensor, d: torch.Tensor, x: torch.Tensor,
          y: torch.Tensor | None = None, stream: int | None = None,
          activations: str = "exact") -> torch.Tensor:
    """SoA GEMV: q (int8 [M, K] | uint8 [M, K/2]), d fp16 [M, K/32], x [K] or [N, K].

    ``activations="q8_1"`` (one column) rounds x to int8 per 32-element block
    inside the kernel (ggml's q8_1 route): faster, but y then carries that
    rounding and is outside the exact path's 1e-5 bound.
    """
    _check_fmt(fmt)
    if not q.is_cuda:
        raise ValueError("q must be a CUDA tensor (weights stay resident on the GPU)")
    M = q.shape[0]
    K = q.shape[1] if fmt == "q8_0" else q.shape[1] * 2
    if q.dim() != 2 or not q.is_contiguous() or q.element_size() != 1:
        raise ValueError("q must be a contiguous 1-byte 2-D tensor")
    if d.dtype != torch.float16 or tuple(d.shape) != (M, K // QK) or not d.is_contiguous():
        raise ValueError(f"d must be contiguous float16 [{M}, {K // QK}]")
    X, Y, y, N, ldx, ldy = _xy(x, M, K, y, q.device)
    _check_act(activations, N)
    st = torch.cuda.current_stream(q.device).cuda_stream if stream is None else stream
    if activations == "q8_1":
        _lib.call("qgemv_soa_q8_1", 8 if fmt == "q8_0" else 4, q.data_ptr(), d.data_ptr(),
                  X.data_ptr(), Y.data_ptr(), M, K, st)
        return y
    if N >= 2:
        fid = 8 if fmt == "q8_0" else 4
        nbytes = _lib.lib().qgemv_soa_workspace_bytes(fid, M, K, N)
        ws = _workspace(q.device, nbytes, stream)
        _lib.call("qgemv_soa_ws", fid, q.data_ptr(), d.data_ptr(), X.data_ptr(), Y.data_ptr(),
                  M, K, N, ldx, ldy, ws.data_ptr(), nbytes, st)
        return y
    _lib.call(_SOA_FN[fmt], q.data_ptr(), d.data_ptr(), X.data_ptr(), Y.data_ptr(),
              M, K, N, ldx, ldy, st)
    return y


@_on_tensor_device
def qgemv_aos(fmt: str, blocks: torch.Tensor, x: torch.Tensor,
              y: torch.Tensor | None = None, stream: int | None = None,
              activations: str = "exact") -> torch.Tensor:
    """GEMV over ggml blocks uint8 [M, K/32, 34|18] (GGUF layout, no repack);
    ``activations`` as in ``qgemv``."""
    _check_fmt(fmt)
    if not blocks.is_cuda:
        raise ValueError("blocks must be a CUDA tensor")
    if (blocks.dim() != 3 or blocks.shape[2] != BLOCK_BYTES[fmt] or blocks.dtype != torch.uint8
            or not blocks.is_contiguous()):
        raise ValueError(f"blocks must be contiguous uint8 [M, K/32, {BLOCK_BYTES[fmt]}]")
    M, nb, _ = blocks.shape
    K = nb * QK
    X, Y, y, N, ldx, ldy = _xy(x, M, K, y, blocks.device)
    _check_act(activations, N)
    st = torch.cuda.current_stream(blocks.device).cuda_stream if stream is None else stream
    if activations == "q8_1":
        _lib.call("qgemv_aos_q8_1", 8 if fmt == "q8_0" else 4, blocks.data_ptr(), X.data_ptr(),
                  Y.data_ptr(), M, K, st)
        return y
    _lib.call(_AOS_FN[fmt], blocks.data_ptr(), X.data_ptr(), Y.data_ptr(), M, K, N, ldx, ldy, st)
    return y


@_on_tensor_device
def tile_weights(fmt: str, q: torch.Tensor | None = None, d: torch.Tensor | None = None,
                 blocks: torch.Tensor | None = None, stream: int | None = None) -> torch.Tensor:
    """Batch tiles (uint8, 1-D) of a matrix given as SoA planes (q, d) or ggml
    blocks [M, K/32, 34|18]: the layout the tensor-core batch kernel streams
    with one bulk copy per 16 rows x 512 columns.  Made once per matrix."""
    _check_fmt(fmt)
    fid = _lib.FORMAT_CODE[fmt]
    if blocks is not None:
        if not blocks.is_cuda or blocks.dim() != 3 or not blocks.is_contiguous():
            raise ValueError("blocks must be a contiguous CUDA tensor [M, K/32, bytes]")
        M, K, src, dsrc, layout, dev = blocks.shape[0], blocks.shape[1] * QK, blocks, None, 1, blocks.device
    else:
        if q is None or d is None or not q.is_cuda or not q.is_contiguous() or not d.is_contiguous():
            raise ValueError("q and d must be contiguous CUDA tensors")
        M = q.shape[0]
        K = q.shape[1] if fmt == "q8_0" else q.shape[1] * 2
        src, dsrc, layout, dev = q, d, 0, q.device
    out = torch.empty(_lib.lib().qgemv_tiled_bytes(fid, M, K), dtype=torch.uint8, device=dev)
    st = torch.cuda.current_stream(dev).cuda_stream if stream is None else stream
    _lib.call("qgemv_tile_weights", fid, layout, src.data_ptr(),
              None if dsrc is None else dsrc.data_ptr(), M, K, out.data_ptr(), st)
    return out


@_on_tensor_device
def qgemv_tiled(fmt: str, tiled: torch.Tensor, M: int, K: int, x: torch.Tensor,
                y: torch.Tensor | None = None, stream: int | None = None) -> torch.Tensor:
    """GEMV over batch tiles (tile_weights); x [K] or [N, K] for any N."""
    _check_fmt(fmt)
    if not tiled.is_cuda or tiled.dtype != torch.uint8:
        raise ValueError("tiled must be a uint8 CUDA tensor")
    fid = _lib.FORMAT_CODE[fmt]
    if tiled.numel() != _lib.lib().qgemv_tiled_bytes(fid, M, K):
        raise ValueError(f"tiles hold {tiled.numel()} bytes, not those of a [{M}, {K}] {fmt} matrix")
    X, Y, y, N, ldx, ldy = _xy(x, M, K, y, tiled.device)
    st = torch.cuda.current_stream(tiled.device).cuda_stream if stream is None else stream
    nbytes = _lib.lib().qgemv_tiled_workspace_bytes(K, N)
    ws = _workspace(tiled.device, nbytes, stream)
    _lib.call("qgemv_tiled_gemv", fid, tiled.data_ptr(), M, K, X.data_ptr(), Y.data_ptr(), N,
              ldx, ldy, ws.data_ptr(), ws.numel(), st)
    return y


@_on_tensor_device
def tile_weights_tc(q: torch.Tensor | None = None, d: torch.Tensor | None = None,
                    blocks: torch.Tensor | None = None, stream: int | None = None,
                    fmt: str = "q8_0") -> torch.Tensor:
    """tc tiles (uint8, 1-D) of a ``fmt`` matrix given as SoA planes (q, d) or
    ggml blocks [M, K/32, 34|18]: the layout the tcgen05 batch kernel streams,
    one bulk copy per 128 rows x 256 columns.  Made once per matrix."""
    _check_fmt(fmt)
    fid = _lib.FORMAT_CODE[fmt]
    if blocks is not None:
        if not blocks.is_cuda or blocks.dim() != 3 or not blocks.is_contiguous() \
                or blocks.shape[2] != BLOCK_BYTES[fmt]:
            raise ValueError(f"blocks must be a contiguous CUDA tensor [M, K/32, {BLOCK_BYTES[fmt]}]")
        M, K, src, dsrc, layout, dev = blocks.shape[0], blocks.shape[1] * QK, blocks, None, 1, blocks.device
    else:
        if q is None or d is None or not q.is_cuda or not q.is_contiguous() or not d.is_contiguous():
            raise ValueError("q and d must be contiguous CUDA tensors")
        M = q.shape[0]
        K = q.shape[1] if fmt == "q8_0" else q.shape[1] * 2
        src, dsrc, layout, dev = q, d, 0, q.device
    out = torch.empty(_lib.lib().qgemv_tc_bytes(fid, M, K), dtype=torch.uint8, device=dev)
    st = torch.cuda.current_stream(dev).cuda_stream if stream is None else stream
    _lib.call("qgemv_tc_tile", fid, layout, src.data_ptr(),
              None if dsrc is None else dsrc.data_ptr(), M, K, out.data_ptr(), st)
    return out


@_on_tensor_device
def qgemv_tc(tiles: torch.Tensor, M: int, K: int, x: torch.Tensor, y: torch.Tensor | None = None,
             stream: int | None = None, fmt: str = "q8_0") -> torch.Tensor:
    """GEMV over tc tiles (tile_weights_tc) on the tcgen05 tensor cores;
    x [K] or [N, K] for any N."""
    _check_fmt(fmt)
    fid = _lib.FORMAT_CODE[fmt]
    if not tiles.is_cuda or tiles.dtype != torch.uint8:
        raise ValueError("tiles must be a uint8 CUDA tensor")
    if tiles.numel() != _lib.lib().qgemv_tc_bytes(fid, M, K):
        raise ValueError(f"tiles hold {tiles.numel()} bytes, not those of a [{M}, {K}] {fmt} matrix")
    X, Y, y, N, ldx, ldy = _xy(x, M, K, y, tiles.device)
    st = torch.cuda.current_stream(tiles.device).cuda_stream if stream is None else stream
    nbytes = _lib.lib().qgemv_tc_workspace_bytes(M, K)  # on the tiles' device
    ws = _workspace(tiles.device, nbytes, stream)
    _lib.call("qgemv_tc_gemv", fid, tiles.data_ptr(), M, K, X.data_ptr(), Y.data_ptr(), N, ldx,
              ldy, ws.data_ptr(), ws.numel(), st)
    return y


@dataclass
class QuantizedMatrix:
    """A quantized [M, K] weight matrix resident on one GPU.

    ``layout`` is "soa" (planes ``q``, ``d``), "aos" (ggml ``blocks``),
    "tiled" (batch tiles, ``tiled``: the layout of the tensor-core batch
    kernel, see ``to_tiled``) or "tc" (q8_0 tc tiles, ``tiled``: the layout
    of the tcgen05 batch kernel, see ``to_tc``).
    """

    fmt: str
    M: int
    K: int
    layout: str = "soa"
    q: torch.Tensor | None = None
    d: torch.Tensor | None = None
    blocks: torch.Tensor | None = None
    tiled: torch.Tensor | None = None

    @classmethod
    def from_float(cls, W: torch.Tensor, fmt: str, layout: str = "soa") -> "QuantizedMatrix":
        from . import qformats
        M, K = W.shape
        if layout == "soa":
            q, d = (qformats.quantize_q8_0 if fmt == "q8_0" else qformats.quantize_q4_0)(W)
            return cls(fmt, M, K, "soa", q=q, d=d)
        blocks = (qformats.quantize_q8_0_aos if fmt == "q8_0" else qformats.quantize_q4_0_aos)(W)
        return cls(fmt, M, K, "aos", blocks=blocks)

    @property
    def nbytes(self) -> int:
        return self.M * (self.K // QK) * BLOCK_BYTES[self.fmt]

    @property
    def device(self):
        return {"soa": self.q, "aos": self.blocks, "tiled": self.tiled,
                "tc": self.tiled}[self.layout].device

    def to_tiled(self) -> "QuantizedMatrix":
        """The same matrix as batch tiles (for calls with several columns)."""
        if self.layout == "tiled":
            return self
        if self.layout == "soa":
            t = tile_weights(self.fmt, q=self.q, d=self.d)
        else:
            t = tile_weights(self.fmt, blocks=self.blocks)
        return QuantizedMatrix(self.fmt, self.M, self.K, "tiled", tiled=t)

    def to_tc(self) -> "QuantizedMatrix":
        """The same matrix as tc tiles (the tcgen05 batch kernel)."""
        if self.layout == "tc":
            return self
        if self.layout == "soa":
            t = tile_weights_tc(q=self.q, d=self.d, fmt=self.fmt)
        elif self.layout == "aos":
            t = tile_weights_tc(blocks=self.blocks, fmt=self.fmt)
        else:
            raise ValueError("make tc tiles from the SoA or ggml-block matrix")
        return QuantizedMatrix(self.fmt, self.M, self.K, "tc", tiled=t)

    def matvec(self, x: torch.Tensor, y: torch.Tensor | None = None,
               stream: int | None = None, activations: str = "exact") -> torch.Tensor:
        """y = W x; ``activations="q8_1"`` selects the opt-in int8-activation
        kernel (one column; SoA or AoS layout)."""
        if self.layout == "soa":
            return qgemv(self.fmt, self.q, self.d, x, y, stream, activations)
        if self.layout == "tiled":
            if activations != "exact":
                raise ValueError("batch tiles run the exact path only")
            return qgemv_tiled(self.fmt, self.tiled, self.M, self.K, x, y, stream)
        if self.layout == "tc":
            if activations != "exact":
                raise ValueError("tc tiles run the exact path only")
            return qgemv_tc(self.tiled, self.M, self.K, x, y, stream, fmt=self.fmt)
        return qgemv_aos(self.fmt, self.blocks, x, y, stream, activations)

    __call__ = matvec

    def rows(self, r0: int, r1: int) -> "QuantizedMatrix":
        """Row slice [r0, r1) as a new matrix (copies; used for row sharding)."""
        if self.layout in ("tiled", "tc"):
            raise ValueError("slice the SoA or ggml-block matrix, then tile the slice")
        if self.layout == "soa":
            return QuantizedMatrix(self.fmt, r1 - r0, self.K, "soa",
                                   q=self.q[r0:r1].contiguous(), d=self.d[r0:r1].contiguous())
        return QuantizedMatrix(self.fmt, r1 - r0, self.K, "aos",
                               blocks=self.blocks[r0:r1].contiguous())

    def to(self, device) -> "QuantizedMatrix":
        if self.layout in ("tiled", "tc"):
            return QuantizedMatrix(self.fmt, self.M, self.K, self.layout, tiled=self.tiled.to(device))
        if self.layout == "soa":
            return QuantizedMatrix(self.fmt, self.M, self.K, "soa", q=self.q.to(device),
                                   d=self.d.to(device))
        return QuantizedMatrix(self.fmt, self.M, self.K, "aos", blocks=self.blocks.to(device))


def algorithmic_bytes(fmt: str, M: int, K: int, N: int = 1) -> int:
    """Bytes a call must move: weights M*K*(34|18)/32 + x 4*K*N + y 4*M*N."""
    return M * (K // QK) * BLOCK_BYTES[fmt] + 4 * K * N + 4 * M * N
