"""GGUF files: read q8_0 / q4_0 (and f32 / f16) tensors, write them back.

A q8_0 / q4_0 weight in a GGUF file is exactly the ggml block array this
library calls AoS: ``[rows][K/32]`` blocks of 34 / 18 bytes (fp16 d first).
``GGUFReader`` maps the file (numpy memmap, no copy on the host) and loads a
tensor onto a GPU as ggml blocks, as SoA planes (split on the GPU by the
repack kernel) or as batch tiles.  ``write_gguf`` writes such tensors (and
metadata) as a GGUF version 3 file.

File layout (GGUF version 2/3, little endian): magic ``GGUF``, uint32
version, uint64 tensor count, uint64 metadata count, the metadata key/value
pairs, the tensor infos (name, uint32 n_dims, uint64 dims with dims[0] the
contiguous one, uint32 ggml type, uint64 offset into the data section), then
the data section, aligned to ``general.alignment`` (default 32) bytes.
"""

from __future__ import annotations

import struct
from dataclasses import dataclass

import numpy as np

# ggml tensor types handled here (ggml's enum values)
GGML_F32, GGML_F16, GGML_Q4_0, GGML_Q8_0 = 0, 1, 2, 8
_TYPE_NAME = {GGML_F32: "f32", GGML_F16: "f16", GGML_Q4_0: "q4_0", GGML_Q8_0: "q8_0"}
_BLOCK = {GGML_Q4_0: (32, 18), GGML_Q8_0: (32, 34), GGML_F32: (1, 4), GGML_F16: (1, 2)}

# metadata value types
(T_U8, T_I8, T_U16, T_I16, T_U32, T_I32, T_F32, T_BOOL, T_STR, T_ARR, T_U64, T_I64,
 T_F64) = range(13)
_SCALAR = {T_U8: "<B", T_I8: "<b", T_U16: "<H", T_I16: "<h", T_U32: "<I", T_I32: "<i",
           T_F32: "<f", T_BOOL: "<?", T_U64: "<Q", T_I64: "<q", T_F64: "<d"}
MAGIC = b"GGUF"


@dataclass
class TensorInfo:
    name: str
    dims: tuple          # ggml order: dims[0] is the contiguous (K) dimension
    ggml_type: int
    offset: int          # into the data section
    nbytes: int

    @property
    def type_name(self) -> str:
        return _TYPE_NAME.get(self.ggml_type, f"ggml_type_{self.ggml_type}")

    @property
    def shape(self) -> tuple:
        """(rows, K) for a matrix: the torch/numpy order of ``dims`` reversed."""
        return tuple(reversed(self.dims))


class _Cursor:
    def __init__(self, buf):
        self.buf, self.pos = buf, 0

    def take(self, fmt):
        v = struct.unpack_from(fmt, self.buf, self.pos)
        self.pos += struct.calcsize(fmt)
        return v[0]

    def string(self):
        n = self.take("<Q")
        s = bytes(self.buf[self.pos:self.pos + n]).decode("utf-8")
        self.pos += n
        return s

    def value(self, t):
        if t in _SCALAR:
            return self.take(_SCALAR[t])
        if t == T_STR:
            return self.string()
        if t == T_ARR:
            et, n = self.take("<I"), self.take("<Q")
            return [self.value(et) for _ in range(n)]
        raise ValueError(f"unknown GGUF metadata type {t}")


def _nbytes(ggml_type: int, dims) -> int:
    if ggml_type not in _BLOCK:
        return -1
    per, size = _BLOCK[ggml_type]
    n = int(np.prod(dims, dtype=np.int64))
    if dims and dims[0] % per:
        raise ValueError(f"row length {dims[0]} is not a multiple of the block size {per}")
    return n // per * size


class GGUFReader:
    """Metadata and tensors of a GGUF file (mapped, read lazily)."""

    def __init__(self, path: str):
        self.path = path
        self._mm = np.memmap(path, dtype=np.uint8, mode="r")
        c = _Cursor(self._mm)
        if bytes(self._mm[:4]) != MAGIC:
            raise ValueError(f"{path}: not a GGUF file")
        c.pos = 4
        self.version = c.take("<I")
        if self.version not in (2, 3):
            raise ValueError(f"{path}: GGUF version {self.version} is not supported")
        n_tensors, n_kv = c.take("<Q"), c.take("<Q")
        self.metadata = {}
        for _ in range(n_kv):
            key = c.string()
            self.metadata[key] = c.value(c.take("<I"))
        self.tensors: dict[str, TensorInfo] = {}
        for _ in range(n_tensors):
            name = c.string()
            nd = c.take("<I")
            dims = tuple(c.take("<Q") for _ in range(nd))
            t, off = c.take("<I"), c.take("<Q")
            self.tensors[name] = TensorInfo(name, dims, t, off, _nbytes(t, dims))
        align = int(self.metadata.get("general.alignment", 32))
        self.data_offset = (c.pos + align - 1) // align * align

    def raw(self, name: str) -> np.ndarray:
        """The tensor's bytes (a view of the mapped file)."""
        ti = self.tensors[name]
        if ti.nbytes < 0:
            raise ValueError(f"{name}: ggml type {ti.ggml_type} is not handled")
        a = self.data_offset + ti.offset
        if a + ti.nbytes > self._mm.size:
            raise ValueError(f"{name}: data runs past the end of the file")
        return self._mm[a:a + ti.nbytes]

    def blocks(self, name: str) -> np.ndarray:
        """q8_0 / q4_0 tensor as ggml blocks uint8 [rows, K/32, 34|18] (host view)."""
        ti = self.tensors[name]
        if ti.ggml_type not in (GGML_Q8_0, GGML_Q4_0):
            raise ValueError(f"{name} is {ti.type_name}, not q8_0 / q4_0")
        K = ti.dims[0]
        rows = int(np.prod(ti.dims[1:], dtype=np.int64)) if len(ti.dims) > 1 else 1
        return self.raw(name).reshape(rows, K // 32, _BLOCK[ti.ggml_type][1])

    def array(self, name: str) -> np.ndarray:
        """f32 / f16 tensor as a numpy array in torch order (host view)."""
        ti = self.tensors[name]
        dt = {GGML_F32: np.float32, GGML_F16: np.float16}.get(ti.ggml_type)
        if dt is None:
            raise ValueError(f"{name} is {ti.type_name}, not f32 / f16")
        return self.raw(name).view(dt).reshape(ti.shape)

    def load(self, name: str, device="cuda", layout: str = "soa"):
        """A q8_0 / q4_0 tensor as a ``QuantizedMatrix`` on ``device``: "aos"
        keeps the file's blocks, "soa" splits them into planes on the GPU,
        "tiled" re-lays them as batch tiles."""
        import torch

        from .gemv import QuantizedMatrix
        from .qformats import from_aos

        ti = self.tensors[name]
        blk = self.blocks(name)
        M, nb, _ = blk.shape
        fmt = ti.type_name
        host = torch.from_numpy(np.array(blk))  # one host copy out of the read-only map
        dev_blocks = host.pin_memory().to(device, non_blocking=True) if torch.cuda.is_available() \
            else host.to(device)
        m = QuantizedMatrix(fmt, M, nb * 32, "aos", blocks=dev_blocks)
        if layout == "aos":
            return m
        if layout == "tiled":
            return m.to_tiled()
        if layout != "soa":
            raise ValueError(f"layout must be 'aos', 'soa' or 'tiled', got {layout!r}")
        q, d = from_aos(fmt, dev_blocks)
        return QuantizedMatrix(fmt, M, nb * 32, "soa", q=q, d=d)


def _put_value(out: bytearray, v):
    if isinstance(v, bool):
        out += struct.pack("<I?", T_BOOL, v)
    elif isinstance(v, int):
        out += struct.pack("<Iq", T_I64, v) if v < 0 else struct.pack("<IQ", T_U64, v)
    elif isinstance(v, float):
        out += struct.pack("<Id", T_F64, v)
    elif isinstance(v, str):
        b = v.encode("utf-8")
        out += struct.pack("<IQ", T_STR, len(b)) + b
    elif isinstance(v, (list, tuple)):
        if not v:
            out += struct.pack("<IIQ", T_ARR, T_U8, 0)
            return
        probe = bytearray()
        _put_value(probe, v[0])
        et = struct.unpack_from("<I", probe)[0]
        out += struct.pack("<IIQ", T_ARR, et, len(v))
        for e in v:
            item = bytearray()
            _put_value(item, e)
            if struct.unpack_from("<I", item)[0] != et:
                raise TypeError("GGUF arrays hold one element type")
            out += item[4:]
    else:
        raise TypeError(f"unsupported metadata value {v!r}")


def write_gguf(path: str, tensors: dict, metadata: dict | None = None, alignment: int = 32):
    """Writes a GGUF version 3 file.

    ``tensors`` maps names to ``("q8_0" | "q4_0", blocks uint8 [rows, K/32, 34|18])`` or to
    float32 / float16 numpy arrays (torch order).  ``metadata`` values may be bool, int,
    float, str or lists of one of those.
    """
    meta = dict(metadata or {})
    meta.setdefault("general.alignment", alignment)
    items = []
    for name, v in tensors.items():
        if isinstance(v, tuple):
            fmt, blk = v
            blk = np.ascontiguousarray(blk, dtype=np.uint8)
            t = {"q8_0": GGML_Q8_0, "q4_0": GGML_Q4_0}[fmt]
            if blk.ndim != 3 or blk.shape[2] != _BLOCK[t][1]:
                raise ValueError(f"{name}: blocks must be [rows, K/32, {_BLOCK[t][1]}]")
            dims = (blk.shape[1] * 32, blk.shape[0])
            data = blk.tobytes()
        else:
            arr = np.ascontiguousarray(v)
            t = {np.dtype(np.float32): GGML_F32, np.dtype(np.float16): GGML_F16}[arr.dtype]
            dims = tuple(reversed(arr.shape))
            data = arr.tobytes()
        items.append((name, dims, t, data))
    head = bytearray(MAGIC) + struct.pack("<IQQ", 3, len(items), len(meta))
    for k, v in meta.items():
        kb = k.encode("utf-8")
        head += struct.pack("<Q", len(kb)) + kb
        _put_value(head, v)
    off, offsets = 0, []
    for name, dims, t, data in items:
        offsets.append(off)
        off = (off + len(data) + alignment - 1) // alignment * alignment
    for (name, dims, t, data), o in zip(items, offsets):
        nb = name.encode("utf-8")
        head += struct.pack("<Q", len(nb)) + nb + struct.pack("<I", len(dims))
        head += b"".join(struct.pack("<Q", d) for d in dims) + struct.pack("<IQ", t, o)
    pad = (-len(head)) % alignment
    with open(path, "wb") as f:
        f.write(head + b"\0" * pad)
        pos = 0
        for (name, dims, t, data), o in zip(items, offsets):
            f.write(b"\0" * (o - pos))
            f.write(data)
            pos = o + len(data)
