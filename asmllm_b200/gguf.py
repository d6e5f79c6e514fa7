"""GGUF files: read, write, and upload Q4_0 / Q8_0 tensors into HBM.

The reference parses GGUF v3 in Python (THRISHAL12345/asmllm
src/runtime/generate.py:38-88: header, metadata, tensor table, 32-byte
aligned data section) and splits each Q4_0 / Q8_0 tensor into a quant plane
and fp32 scales on the host (generate.py:91-119).  Here the file is parsed
the same way (plus the metadata values and `general.alignment`), the raw
blocks of a tensor are copied to the GPU once, and the split runs on the
device (asm_gguf_split_async) into the resident layout: quant plane + fp16
scales, 18 / 34 bytes per block as in the file.

Format (GGUF v3, little endian): "GGUF", uint32 version, uint64 tensor
count, uint64 metadata count; metadata = (string key, uint32 type, value);
tensor info = (string name, uint32 n_dims, uint64 dims[n_dims] innermost
first, uint32 ggml type, uint64 offset into the data section); the data
section starts at the next multiple of the alignment.
"""
from __future__ import annotations

import struct
from dataclasses import dataclass

import numpy as np

GGUF_MAGIC = b"GGUF"
GGML_F32, GGML_F16, GGML_Q4_0, GGML_Q5_0, GGML_Q8_0 = 0, 1, 2, 6, 8
BLOCK_BYTES = {GGML_Q4_0: 18, GGML_Q8_0: 34, GGML_Q5_0: 22}
ELEM_BYTES = {GGML_F32: 4, GGML_F16: 2}

# metadata value types
_U8, _I8, _U16, _I16, _U32, _I32, _F32, _BOOL, _STR, _ARR, _U64, _I64, _F64 = range(13)
_SCALAR = {_U8: "<B", _I8: "<b", _U16: "<H", _I16: "<h", _U32: "<I", _I32: "<i", _F32: "<f", _BOOL: "<?",
           _U64: "<Q", _I64: "<q", _F64: "<d"}


@dataclass
class TensorInfo:
    name: str
    dims: tuple  # innermost first (ne[0] = columns)
    type: int
    offset: int  # into the data section

    @property
    def rows(self) -> int:
        return int(np.prod(self.dims[1:])) if len(self.dims) > 1 else 1

    @property
    def cols(self) -> int:
        return int(self.dims[0])

    @property
    def nbytes(self) -> int:
        n = int(np.prod(self.dims))
        if self.type in BLOCK_BYTES:
            return n // 32 * BLOCK_BYTES[self.type]
        return n * ELEM_BYTES[self.type]


class _Reader:
    def __init__(self, buf):
        self.buf, self.pos = buf, 0

    def take(self, fmt):
        v = struct.unpack_from(fmt, self.buf, self.pos)
        self.pos += struct.calcsize(fmt)
        return v[0] if len(v) == 1 else v

    def string(self):
        n = self.take("<Q")
        s = bytes(self.buf[self.pos:self.pos + n]).decode("utf-8", errors="replace")
        self.pos += n
        return s

    def value(self, t):
        if t in _SCALAR:
            return self.take(_SCALAR[t])
        if t == _STR:
            return self.string()
        if t == _ARR:
            et, n = self.take("<I"), self.take("<Q")
            return [self.value(et) for _ in range(n)]
        raise ValueError(f"unknown GGUF metadata type {t}")


class GGUFFile:
    """A parsed GGUF file (memory-mapped)."""

    def __init__(self, path):
        self.path = str(path)
        self._map = np.memmap(self.path, dtype=np.uint8, mode="r")
        r = _Reader(self._map)
        if bytes(self._map[:4]) != GGUF_MAGIC:
            raise ValueError(f"{self.path}: not a GGUF file")
        r.pos = 4
        self.version = r.take("<I")
        if self.version not in (2, 3):
            raise ValueError(f"{self.path}: GGUF version {self.version} (2 or 3 supported)")
        n_tensors, n_kv = r.take("<Q"), r.take("<Q")
        self.metadata = {}
        for _ in range(n_kv):
            key = r.string()
            self.metadata[key] = r.value(r.take("<I"))
        self.tensors = {}
        for _ in range(n_tensors):
            name = r.string()
            nd = r.take("<I")
            dims = tuple(r.take("<Q") for _ in range(nd))
            ttype, off = r.take("<I"), r.take("<Q")
            self.tensors[name] = TensorInfo(name, dims, ttype, off)
        self.alignment = int(self.metadata.get("general.alignment", 32))
        self.data_offset = (r.pos + self.alignment - 1) // self.alignment * self.alignment

    def raw(self, name) -> np.ndarray:
        t = self.tensors[name]
        start = self.data_offset + t.offset
        if start + t.nbytes > self._map.size:
            raise ValueError(f"{self.path}: tensor {name} runs past the end of the file")
        return self._map[start:start + t.nbytes]

    def array(self, name) -> np.ndarray:
        """F32 / F16 tensors as float32, shape (rows, cols)."""
        t = self.tensors[name]
        if t.type == GGML_F32:
            a = self.raw(name).view(np.float32)
        elif t.type == GGML_F16:
            a = self.raw(name).view(np.float16).astype(np.float32)
        else:
            raise ValueError(f"{name}: type {t.type} is not F32/F16")
        return a.reshape(t.rows, t.cols) if len(t.dims) > 1 else a.copy()


def write_gguf(path, metadata: dict, tensors: list, alignment: int = 32) -> None:
    """Writes a GGUF v3 file.  metadata: {key: int | float | str | list[str|int|float]}
    (ints as int32/uint64 by sign and size, floats as float32); tensors: [(name,
    dims innermost first, ggml type, raw bytes)]."""

    def s(x: str) -> bytes:
        b = x.encode()
        return struct.pack("<Q", len(b)) + b

    def val(v):
        if isinstance(v, bool):
            return struct.pack("<I?", _BOOL, v)
        if isinstance(v, int):
            return struct.pack("<Ii", _I32, v) if -2**31 <= v < 2**31 else struct.pack("<IQ", _U64, v)
        if isinstance(v, float):
            return struct.pack("<If", _F32, v)
        if isinstance(v, str):
            return struct.pack("<I", _STR) + s(v)
        if isinstance(v, (list, tuple)):
            if all(isinstance(e, str) for e in v):
                return struct.pack("<IIQ", _ARR, _STR, len(v)) + b"".join(s(e) for e in v)
            if all(isinstance(e, int) for e in v):
                return struct.pack("<IIQ", _ARR, _I32, len(v)) + b"".join(struct.pack("<i", e) for e in v)
            return struct.pack("<IIQ", _ARR, _F32, len(v)) + b"".join(struct.pack("<f", float(e)) for e in v)
        raise TypeError(f"metadata value {v!r}")

    md = dict(metadata)
    if alignment != 32:
        md["general.alignment"] = alignment
    out = bytearray(GGUF_MAGIC + struct.pack("<IQQ", 3, len(tensors), len(md)))
    for k, v in md.items():
        out += s(k) + val(v)
    off = 0
    offsets = []
    for name, dims, ttype, raw in tensors:
        offsets.append(off)
        out += s(name) + struct.pack("<I", len(dims)) + b"".join(struct.pack("<Q", d) for d in dims)
        out += struct.pack("<IQ", ttype, off)
        off = (off + len(raw) + alignment - 1) // alignment * alignment
    out += b"\0" * ((-len(out)) % alignment)
    data_start = len(out)
    for (name, dims, ttype, raw), o in zip(tensors, offsets):
        out += b"\0" * (data_start + o - len(out))  # alignment padding before each tensor
        out += bytes(raw)
    with open(path, "wb") as f:
        f.write(out)


def blocks_from_planes(qs: np.ndarray, scales: np.ndarray) -> np.ndarray:
    """GGUF blocks (fp16 d, then the quants) from a quant plane [M, nb, 16 | 32]
    and scales [M, nb] (converted to fp16)."""
    nblk = scales.size
    qb = np.ascontiguousarray(qs).reshape(nblk, -1).view(np.uint8)
    d = np.ascontiguousarray(scales, dtype=np.float32).reshape(nblk).astype(np.float16).view(np.uint8).reshape(nblk, 2)
    return np.ascontiguousarray(np.concatenate([d, qb], axis=1)).reshape(-1)


def upload(gg: GGUFFile, name: str, device=None):
    """A Q4_0 / Q8_0 tensor in HBM: (quant plane [rows, cols/32, 16 | 32], fp16
    scales [rows, cols/32]), split on the device from one copy of the raw blocks."""
    import torch

    from . import ops
    from .native import FMT_Q4_0, FMT_Q8_0

    t = gg.tensors[name]
    if t.type not in (GGML_Q4_0, GGML_Q8_0):
        raise ValueError(f"{name}: GGML type {t.type} is not Q4_0 / Q8_0")
    fmt = FMT_Q4_0 if t.type == GGML_Q4_0 else FMT_Q8_0
    dev = torch.device(device) if device is not None else torch.device("cuda", torch.cuda.current_device())
    raw = torch.from_numpy(np.ascontiguousarray(gg.raw(name))).pin_memory().to(dev, non_blocking=True)
    nblk = t.rows * (t.cols // 32)
    qs, d = ops.gguf_split_dev(fmt, raw, nblk)
    per = 16 if fmt == FMT_Q4_0 else 32
    return qs.view(t.rows, t.cols // 32, per), d.view(t.rows, t.cols // 32)
