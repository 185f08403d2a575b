"""Decode-time layer stack of quantized GEMVs, row-sharded across the GPUs of
one node.

The 7B-style decode configuration: ``n_layers`` layers, each four GEMVs at
batch 1 -- QKV [12288, 4096], O [4096, 4096], gate+up [22016, 4096] and down
[4096, 11008] -- with W ~ N(0, 0.02) quantized to q8_0 or q4_0.  Only the
GEMVs are on this path: the attention, the gated activation and the residual
are outside it, so each GEMV reads the leading K entries of the previous
output (QKV -> O reads its first 4096, gate+up -> down its first 11008, down
feeds the next layer's QKV).

With P ranks (one process per GPU, ``torch.distributed``) every matrix is
row-sharded: rank g holds rows ``row_range(M, g, P)`` of each of the
4 * n_layers matrices and computes that slice of every y; an all-gather (NCCL
``all_gather_into_tensor`` into a preallocated buffer when P divides M)
assembles the full y that the next GEMV needs.  One decode step is therefore
4 * n_layers GEMV launches and, at P > 1, as many all-gathers; ``capture``
records the whole step as one CUDA graph.

``local_gemv(mat, x, y)`` is the per-rank kernel call (default: the sm_100a
C ABI through ``QuantizedMatrix.matvec``); it is a parameter so the sharding
and gather plumbing can be exercised without a GPU.
"""

from __future__ import annotations

from dataclasses import dataclass
from typing import Callable, Sequence

import torch
import torch.distributed as dist

from .gemv import QuantizedMatrix
from .shard import row_range

# (name, M, K) of the four GEMVs of a 7B-style decode layer
LAYER_7B = (("qkv", 12288, 4096), ("o", 4096, 4096), ("gate_up", 22016, 4096),
            ("down", 4096, 11008))


@dataclass
class StackMatrix:
    name: str
    layer: int
    M: int
    K: int
    r0: int
    r1: int
    local: object  # this rank's rows (a QuantizedMatrix, or whatever local_gemv takes)


def weight_bytes(fmt: str, shapes: Sequence = LAYER_7B, n_layers: int = 32) -> int:
    per = {"q8_0": 34, "q4_0": 18}[fmt]
    return n_layers * sum(M * (K // 32) * per for _, M, K in shapes)


class DecodeStack:
    """``n_layers`` x ``shapes`` quantized GEMVs, this rank's row slices.

    ``make_local(layer, index, name, M, K, r0, r1)`` returns the rank's slice
    of one matrix; ``from_random`` builds them on the GPU from seeded
    N(0, 0.02) weights (identical for every world size).
    """

    def __init__(self, fmt: str, matrices: list[StackMatrix], n_layers: int,
                 shapes: Sequence = LAYER_7B, device=None, group=None,
                 local_gemv: Callable | None = None, fused: bool = False,
                 persistent: bool = False):
        self.fmt, self.n_layers, self.shapes = fmt, n_layers, tuple(shapes)
        self.group = group
        self.world = dist.get_world_size(group) if dist.is_initialized() else 1
        self.rank = dist.get_rank(group) if dist.is_initialized() else 0
        self.mats = matrices
        self.device = torch.device(device) if device is not None else torch.device("cpu")
        self.local_gemv = local_gemv or (lambda m, x, y: m.local.matvec(x, y))
        # one local and one gathered output buffer per matrix kind (reused by every layer)
        self.y_local, self.y_full = [], []
        for _, M, _ in self.shapes:
            r0, r1 = row_range(M, self.rank, self.world)
            self.y_local.append(torch.empty(r1 - r0, dtype=torch.float32, device=self.device))
            self.y_full.append(torch.empty(M, dtype=torch.float32, device=self.device)
                               if self.world > 1 else None)
        self.nccl = self.world > 1 and dist.get_backend(group) == "nccl"
        self.fused = None
        if fused:
            self.fused = _FusedGather(self)
        self.persistent = None
        if persistent:
            if fused:
                raise ValueError("choose one of fused and persistent")
            self.persistent = _PersistentStack(self)

    @classmethod
    def from_random(cls, fmt: str, n_layers: int = 32, shapes: Sequence = LAYER_7B,
                    seed: int = 0, device=None, group=None, layout: str = "soa",
                    keep_full: bool = False, fused: bool = False,
                    persistent: bool = False) -> "DecodeStack":
        """Seeded weights W ~ N(0, 0.02), generated and quantized on ``device``;
        each rank keeps its rows (``keep_full`` also keeps the full matrices on
        ``.full``, for tests)."""
        from . import qformats
        dev = torch.device(device) if device is not None else torch.device("cuda")
        world = dist.get_world_size(group) if dist.is_initialized() else 1
        rank = dist.get_rank(group) if dist.is_initialized() else 0
        quant = qformats.quantize_q8_0 if fmt == "q8_0" else qformats.quantize_q4_0
        mats, full = [], []
        for layer in range(n_layers):
            for i, (name, M, K) in enumerate(shapes):
                g = torch.Generator(device=dev).manual_seed(seed * 100003 + layer * 16 + i)
                W = torch.randn(M, K, generator=g, device=dev) * 0.02
                q, d = quant(W)
                del W
                r0, r1 = row_range(M, rank, world)
                part = QuantizedMatrix(fmt, r1 - r0, K, "soa", q=q[r0:r1].contiguous(),
                                       d=d[r0:r1].contiguous())
                if layout == "tiled":
                    part = part.to_tiled()
                mats.append(StackMatrix(name, layer, M, K, r0, r1, part))
                if keep_full:
                    full.append((q, d))
                del q, d
        st = cls(fmt, mats, n_layers, shapes, device=dev, group=group, fused=fused,
                 persistent=persistent)
        st.full = full
        return st

    @property
    def weight_bytes(self) -> int:
        return weight_bytes(self.fmt, self.shapes, self.n_layers)

    def _gather(self, i: int, y_local: torch.Tensor, M: int) -> torch.Tensor:
        if self.world == 1:
            return y_local
        out = self.y_full[i]
        if self.nccl and M % self.world == 0:
            dist.all_gather_into_tensor(out, y_local, group=self.group)
            return out
        S = -(-M // self.world)
        pad = torch.zeros(S, dtype=y_local.dtype, device=y_local.device)
        pad[:y_local.numel()] = y_local
        parts = [torch.empty_like(pad) for _ in range(self.world)]
        dist.all_gather(parts, pad, group=self.group)
        cols = []
        for g in range(self.world):
            a, b = row_range(M, g, self.world)
            cols.append(parts[g][:b - a])
        out.copy_(torch.cat(cols))
        return out

    def forward(self, x: torch.Tensor, trace: list | None = None) -> torch.Tensor:
        """One decode step: x [K of the first matrix] -> the last matrix's y.

        ``trace``, when given, receives (matrix, input, full output) per GEMV."""
        if self.fused is not None:
            return self.fused.forward(x, trace)
        if self.persistent is not None:
            return self.persistent.forward(x, trace)
        cur = x
        nk = len(self.shapes)
        for j, m in enumerate(self.mats):
            i = j % nk
            xin = cur[:m.K]
            y_loc = self.local_gemv(m, xin, self.y_local[i])
            cur = self._gather(i, y_loc, m.M)
            if trace is not None:
                trace.append((m, xin.clone(), cur.clone()))
        return cur

    __call__ = forward

    def capture(self, x_static: torch.Tensor, warmup: int = 2):
        """A CUDA graph of one ``forward`` on ``x_static`` (returns the graph
        and the output tensor it writes)."""
        s = torch.cuda.Stream(self.device)
        s.wait_stream(torch.cuda.current_stream(self.device))
        with torch.cuda.stream(s):
            for _ in range(warmup):
                self.forward(x_static)
        torch.cuda.current_stream(self.device).wait_stream(s)
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            out = self.forward(x_static)
        return g, out


class _FusedGather:
    """Symmetric buffers, counters and call descriptors of a fused stack.

    Every rank holds one full-y buffer per matrix kind and a counter array
    (one counter per GEMV of a token plus one for the token fence) in
    symmetric memory, so each GEMV kernel stores its rows into every rank's
    buffer itself and signals with a counter (``qgemv_soa_fused``); a token
    ends with ``qgemv_token_fence``.  No NCCL call is left on the path.
    """

    def __init__(self, st: "DecodeStack"):
        import ctypes

        import torch.distributed._symmetric_memory as symm_mem

        from . import _lib

        if not dist.is_initialized():
            raise RuntimeError("the fused stack needs an initialised process group")
        try:
            symm_mem.set_backend("CUDA")
        except Exception:
            pass
        self.st, self.lib = st, _lib.lib()
        dev, world, rank = st.device, st.world, st.rank
        group = st.group or dist.group.WORLD
        n = len(st.mats)
        self.y = [symm_mem.empty(M, dtype=torch.float32, device=dev) for _, M, _ in st.shapes]
        self.y_h = [symm_mem.rendezvous(t, group) for t in self.y]
        self.sig = symm_mem.empty(n + 1, dtype=torch.int32, device=dev)
        self.sig.zero_()
        self.sig_h = symm_mem.rendezvous(self.sig, group)
        self.cta = torch.zeros(n, dtype=torch.int32, device=dev)
        self.tok = torch.zeros(1, dtype=torch.int32, device=dev)
        torch.cuda.synchronize(dev)
        dist.barrier(group)
        sig_ptrs = list(self.sig_h.buffer_ptrs)
        nk = len(st.shapes)
        self.desc = []
        for j, m in enumerate(st.mats):
            i = j % nk
            d = _lib.FuseDesc()
            peers = [k for k in range(world) if k != rank]
            for slot, k in enumerate(peers):
                d.peer_y[slot] = self.y_h[i].buffer_ptrs[k] + 4 * m.r0
            for k in range(world):
                d.sig_out[k] = sig_ptrs[k] + 4 * j
            d.cta_count = self.cta.data_ptr() + 4 * j
            d.sig_in = self.sig.data_ptr() + 4 * (j - 1) if j > 0 else None
            d.tok = self.tok.data_ptr()
            d.npeer, d.nranks = len(peers), world
            self.desc.append(d)
        self.done = (ctypes.c_void_p * world)(*[p + 4 * n for p in sig_ptrs])
        self.done_local = self.sig.data_ptr() + 4 * n
        self.fid = _lib.FORMAT_CODE[st.fmt]

    def reset(self):
        """Recovery after a timed-out token (QGEMV_ERR_TIMEOUT): clears this
        device's error word and zeroes the counters, the per-call CTA counts
        and the token count on every rank (a collective: every rank calls it,
        with no fused call in flight)."""
        from . import _lib

        st = self.st
        group = st.group or dist.group.WORLD
        torch.cuda.synchronize(st.device)
        dist.barrier(group)
        self.lib.qgemv_check_device_error(1, None)
        self.sig.zero_()
        self.cta.zero_()
        self.tok.zero_()
        torch.cuda.synchronize(st.device)
        dist.barrier(group)
        _lib.call("qgemv_check_device_error", 0, None)

    def forward(self, x, trace=None):
        """One token; returns this rank's full output buffer of the last GEMV
        (complete once the token fence has run)."""
        import ctypes

        from . import _lib

        if trace is not None:
            raise ValueError("the fused stack keeps no per-GEMV outputs to trace")
        st = self.st
        nk = len(st.shapes)
        s = torch.cuda.current_stream(st.device).cuda_stream
        cur = x
        for j, m in enumerate(st.mats):
            i = j % nk
            q = m.local
            if q.layout != "soa":
                raise ValueError("the fused stack runs on SoA planes")
            _lib.call("qgemv_soa_fused", self.fid, q.q.data_ptr(), q.d.data_ptr(),
                      cur[:m.K].data_ptr(), self.y[i][m.r0:m.r1].data_ptr(), m.r1 - m.r0, m.K,
                      ctypes.byref(self.desc[j]), s)
            cur = self.y[i]
        _lib.call("qgemv_token_fence", self.done, st.world, self.done_local, self.tok.data_ptr(), s)
        return cur


class _PersistentStack:
    """All GEMVs of a token in one cooperative launch per rank
    (``qgemv_stack_create`` on one GPU, ``qgemv_stack_create_ranks`` on P):
    one CTA per SM streams the next matrices' weights while the current GEMV
    waits for its input.  Outputs are 8-byte slots (fp32 value, tag); with P
    ranks every GEMV stores its rows into every rank's slots (symmetric
    memory, NVLink) and readers wait for the tag of the current token, so no
    collective call is left on the path.  The last GEMV's full output is on
    every rank when the launch completes."""

    def __init__(self, st: "DecodeStack"):
        import ctypes

        from . import _lib

        self.st, self.lib = st, _lib.lib()
        nk = len(st.shapes)
        n = len(st.mats)
        K0 = st.mats[0].K
        dev, world, rank = st.device, st.world, st.rank
        self.x_in = torch.empty(K0, dtype=torch.float32, device=dev)
        for m in st.mats:
            if m.local.layout != "soa":
                raise ValueError("the persistent stack runs on SoA planes")
        if world > 1:
            import torch.distributed._symmetric_memory as symm_mem
            try:
                symm_mem.set_backend("CUDA")
            except Exception:
                pass
            group = st.group or dist.group.WORLD
            self.slots = [symm_mem.empty(M, dtype=torch.int64, device=dev) for _, M, _ in st.shapes]
            for t in self.slots:
                t.zero_()
            handles = [symm_mem.rendezvous(t, group) for t in self.slots]
            torch.cuda.synchronize(dev)
            dist.barrier(group)
        else:
            self.slots = [torch.zeros(M, dtype=torch.int64, device=dev) for _, M, _ in st.shapes]
        descs = (_lib.StackGemvDesc * n)()
        peers = [k for k in range(world) if k != rank]
        self._peer_y = (ctypes.c_void_p * max(1, n * (world - 1)))()
        for j, m in enumerate(st.mats):
            q = m.local
            y = self.slots[j % nk]
            descs[j] = _lib.StackGemvDesc(q.q.data_ptr(), q.d.data_ptr(), self.x_in.data_ptr(),
                                          y.data_ptr(), m.r0, m.r1 - m.r0, m.M, m.K)
            for i, k in enumerate(peers):
                self._peer_y[j * (world - 1) + i] = handles[j % nk].buffer_ptrs[k]
        h = ctypes.c_void_p()
        fid = _lib.FORMAT_CODE[st.fmt]
        if world > 1:
            rk = _lib.StackRanksDesc()
            rk.nranks, rk.rank = world, rank
            rk.peer_y = ctypes.cast(self._peer_y, ctypes.c_void_p)
            _lib.call("qgemv_stack_create_ranks", fid, descs, n, ctypes.byref(rk), ctypes.byref(h))
        else:
            _lib.call("qgemv_stack_create", fid, descs, n, ctypes.byref(h))
        self.handle = h
        # y of the last GEMV: the low 32-bit words of its slots
        self.out = self.slots[(n - 1) % nk].view(torch.float32)[0::2]

    def forward(self, x, trace=None):
        from . import _lib

        if trace is not None:
            raise ValueError("the persistent stack keeps no per-GEMV outputs to trace")
        st = self.st
        if x.data_ptr() != self.x_in.data_ptr():
            self.x_in.copy_(x[:self.x_in.numel()])
        _lib.call("qgemv_stack_run", self.handle,
                  torch.cuda.current_stream(st.device).cuda_stream)
        return self.out

    def reset(self):
        """Recovery after a timed-out token: clears the device error word,
        zeroes the output slots and the token count (on every rank: a
        collective when P > 1)."""
        from . import _lib

        st = self.st
        torch.cuda.synchronize(st.device)
        if st.world > 1:
            dist.barrier(st.group or dist.group.WORLD)
        self.lib.qgemv_check_device_error(1, None)
        for t in self.slots:
            t.zero_()
        _lib.call("qgemv_stack_reset", self.handle, None)
        torch.cuda.synchronize(st.device)
        if st.world > 1:
            dist.barrier(st.group or dist.group.WORLD)

    def __del__(self):
        h = getattr(self, "handle", None)
        if h is not None and h.value:
            try:
                self.lib.qgemv_stack_destroy(h)
            except Exception:
                pass
