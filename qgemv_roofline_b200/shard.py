"""Row-sharded quantized GEMV across the GPUs of one node (one process per GPU).

The reference is single-GPU.  For the large shapes the rows of W are split
over the ranks of a ``torch.distributed`` process group: rank g owns rows
``[row_range(M, g, P)]`` of W, resident in its own HBM as SoA planes (or
ggml blocks); x is replicated (it is the caller's input, or the all-gathered
y of the previous layer).  Each rank computes its y slice with no
communication; an NCCL all-gather assembles the full y only when the caller
asks for it.

``local_gemv`` is the per-rank kernel call (default: the sm_100a C-ABI through
``QuantizedMatrix.matvec``); it is a parameter so the host-side partition and
gather logic can be exercised without a GPU.
"""

from __future__ import annotations

from typing import Callable

import torch
import torch.distributed as dist

from .gemv import QuantizedMatrix


def row_range(M: int, rank: int, world: int) -> tuple[int, int]:
    """Rows [r0, r1) of rank ``rank``: contiguous, sizes differ by at most one."""
    if world < 1 or not 0 <= rank < world:
        raise ValueError(f"rank {rank} out of range for world size {world}")
    return M * rank // world, M * (rank + 1) // world


class ShardedQGemv:
    """This rank's row slice of a quantized [M, K] matrix.

    ``forward(x, gather=False)`` returns this rank's y slice ``[rows]`` (or
    ``[N, rows]``); ``gather=True`` returns the full ``[M]`` (``[N, M]``) y on
    every rank, assembled with one all-gather (rank-major, padded to equal
    slice sizes when M is not a multiple of the world size).
    """

    def __init__(self, local: QuantizedMatrix | None, M: int, K: int, fmt: str,
                 group=None, local_gemv: Callable | None = None):
        self.group = group
        self.world = dist.get_world_size(group) if dist.is_initialized() else 1
        self.rank = dist.get_rank(group) if dist.is_initialized() else 0
        self.M, self.K, self.fmt = M, K, fmt
        self.r0, self.r1 = row_range(M, self.rank, self.world)
        self.local = local
        if local is not None and (local.M != self.r1 - self.r0 or local.K != K):
            raise ValueError(f"local slice is [{local.M}, {local.K}], expected "
                             f"[{self.r1 - self.r0}, {K}]")
        self.local_gemv = local_gemv or (lambda x, y=None: self.local.matvec(x, y))
        self.slice_max = -(-M // self.world)  # ceil: padded slice for the gather

    @classmethod
    def from_full(cls, full: QuantizedMatrix, device=None, group=None) -> "ShardedQGemv":
        """Takes this rank's rows of a full matrix (held on any device) to ``device``."""
        world = dist.get_world_size(group) if dist.is_initialized() else 1
        rank = dist.get_rank(group) if dist.is_initialized() else 0
        r0, r1 = row_range(full.M, rank, world)
        part = full.rows(r0, r1)
        if device is not None:
            part = part.to(device)
        return cls(part, full.M, full.K, full.fmt, group=group)

    def forward(self, x: torch.Tensor, gather: bool = False) -> torch.Tensor:
        y = self.local_gemv(x)
        if not gather or self.world == 1:
            return y
        return self.all_gather(y)

    __call__ = forward

    def all_gather(self, y_local: torch.Tensor) -> torch.Tensor:
        """[rows] or [N, rows] slices of every rank -> full [M] or [N, M].

        One all-gather into a [P, N, S] buffer (S = the largest slice).  When
        every rank holds S rows (M divisible by P) a vector needs nothing more
        (the buffer is y in row order) and N columns one transposing copy;
        otherwise the slices are padded to S before the gather and the
        padding dropped after it."""
        vec = y_local.dim() == 1
        Y = y_local.unsqueeze(0) if vec else y_local
        N, rows = Y.shape
        P, S = self.world, self.slice_max
        even = self.M == P * S
        if rows == S:
            send = Y.contiguous()
        else:
            send = torch.zeros((N, S), dtype=Y.dtype, device=Y.device)
            send[:, :rows] = Y
        out = torch.empty((P * N, S), dtype=Y.dtype, device=Y.device)
        dist.all_gather_into_tensor(out, send, group=self.group)
        out = out.view(P, N, S)
        if even:
            if vec:
                return out.view(self.M)
            return out.permute(1, 0, 2).reshape(N, self.M)
        sizes = [row_range(self.M, g, P)[1] - row_range(self.M, g, P)[0] for g in range(P)]
        full = torch.cat([out[g, :, :sizes[g]] for g in range(P)], dim=1)  # [N, M]
        return full[0] if vec else full


class MultiDeviceQGemv:
    """One process, several GPUs: a quantized matrix sharded by rows over
    ``devices`` (the same ``row_range`` partition) through the C-ABI
    multi-GPU handle (``qgemv_mg_*``), with the all-gather of y done by peer
    copies between the devices instead of NCCL.

    ``forward(xs, allgather=True)`` takes one X per device (``[K]`` or
    ``[N, K]``, on that device) and returns one Y per device (``[M]`` or
    ``[N, M]``): the device's own rows, and with ``allgather`` every row.
    Each device's work runs on its current torch stream.
    """

    def __init__(self, full: QuantizedMatrix, devices):
        import ctypes

        from . import _lib

        if full.layout not in ("soa", "aos"):
            raise ValueError("shard a matrix held as SoA planes or ggml blocks")
        self._lib = _lib
        self.devices = [torch.device("cuda", d) if isinstance(d, int) else torch.device(d)
                        for d in devices]
        n = len(self.devices)
        ids = (ctypes.c_int32 * n)(*[d.index for d in self.devices])
        h = ctypes.c_void_p()
        _lib.call("qgemv_mg_init", n, ids, ctypes.byref(h))
        self._h = h
        self.M, self.K, self.fmt = full.M, full.K, full.fmt
        soa = full.layout == "soa"
        src = full.q if soa else full.blocks
        if src.is_cuda:
            torch.cuda.synchronize(src.device)  # the shards are copied from finished bytes
        try:
            _lib.call("qgemv_mg_shard", self._h, _lib.FORMAT_CODE[self.fmt], 0 if soa else 1,
                      src.data_ptr(), full.d.data_ptr() if soa else None, self.M, self.K)
            self.row_ranges = []
            for g in range(n):
                r0, rows = ctypes.c_int64(), ctypes.c_int64()
                _lib.call("qgemv_mg_rows", self._h, g, ctypes.byref(r0), ctypes.byref(rows))
                self.row_ranges.append((r0.value, r0.value + rows.value))
        except Exception:
            self.close()
            raise

    def forward(self, xs, ys=None, allgather: bool = True):
        import ctypes

        n = len(self.devices)
        if len(xs) != n:
            raise ValueError(f"one x per device: {n} expected, {len(xs)} given")
        one = xs[0].dim() == 1
        N = 1 if one else xs[0].shape[0]
        for x, dev in zip(xs, self.devices):
            if x.device != dev or x.dtype != torch.float32 or not x.is_contiguous() \
                    or x.shape[-1] != self.K or (1 if x.dim() == 1 else x.shape[0]) != N:
                raise ValueError(f"x must be contiguous fp32 [{'' if one else 'N, '}K] on {dev}")
        if ys is None:
            ys = [torch.empty((self.M,) if one else (N, self.M), device=dev)
                  for dev in self.devices]
        xp = (ctypes.c_void_p * n)(*[x.data_ptr() for x in xs])
        yp = (ctypes.c_void_p * n)(*[y.data_ptr() for y in ys])
        sp = (ctypes.c_void_p * n)(*[torch.cuda.current_stream(dev).cuda_stream
                                     for dev in self.devices])
        self._lib.call("qgemv_mg_gemv", self._h, xp, yp, N, int(allgather), sp)
        return ys

    __call__ = forward

    def close(self):
        if getattr(self, "_h", None) is not None and self._h.value:
            self._lib.call("qgemv_mg_destroy", self._h)
        self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass
