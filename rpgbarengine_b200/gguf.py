"""Minimal GGUF v3 writer and reader (host side, numpy only).

The on-disk format is ggml's GGUF as the reference reads it
(src/gguf.h:3-15, src/gguf.cc:69-160):

    magic u32 'GGUF' | version u32 | n_tensors u64 | n_kv u64
    kv[]      key (u64 len + bytes) | value type u32 | value
    tensor[]  name | n_dims u32 | dims u64[n_dims] | ggml type u32 | offset u64
    padding to general.alignment (default 32)
    data      each tensor's raw bytes at its offset (offsets 32-byte aligned)

dims[0] is the fastest axis, so a weight matrix is row-major
[rows = dims[1], cols = dims[0]].  Block payloads are written unchanged.
"""
from __future__ import annotations

import struct
from dataclasses import dataclass, field

import numpy as np

GGUF_MAGIC = 0x46554747
ALIGN = 32

# ggml type ids used on the hot path (src/quant.h:22-38)
F32, F16, Q8_0, Q4_K, Q6_K = 0, 1, 8, 12, 14
TYPE_BLOCK = {F32: (1, 4), F16: (1, 2), Q8_0: (32, 34), Q4_K: (256, 144), Q6_K: (256, 210)}
TYPE_NAME = {F32: "F32", F16: "F16", Q8_0: "Q8_0", Q4_K: "Q4_K", Q6_K: "Q6_K"}

# metadata value types (gguf_metadata_value_type)
_U8, _I8, _U16, _I16, _U32, _I32, _F32, _BOOL, _STR, _ARR, _U64, _I64, _F64 = range(13)


def row_bytes(ggml_type: int, n: int) -> int:
    be, bb = TYPE_BLOCK[ggml_type]
    if n % be:
        raise ValueError(f"{n} elements is not a whole number of {TYPE_NAME[ggml_type]} blocks")
    return (n // be) * bb


@dataclass
class Tensor:
    name: str
    ggml_type: int
    dims: tuple  # dims[0] fastest
    data: np.ndarray  # uint8, raw block bytes

    @property
    def n_bytes(self) -> int:
        return int(self.data.nbytes)


@dataclass
class GgufFile:
    meta: dict = field(default_factory=dict)
    tensors: list = field(default_factory=list)

    def tensor(self, name: str) -> Tensor:
        for t in self.tensors:
            if t.name == name:
                return t
        raise KeyError(name)


def _w_str(f, s: str):
    b = s.encode("utf-8")
    f.write(struct.pack("<Q", len(b)))
    f.write(b)


def _w_value(f, v):
    if isinstance(v, bool):
        f.write(struct.pack("<IB", _BOOL, int(v)))
    elif isinstance(v, int):
        if -(2**31) <= v < 2**31:
            f.write(struct.pack("<Ii", _I32, v))
        else:
            f.write(struct.pack("<Iq", _I64, v))
    elif isinstance(v, float):
        f.write(struct.pack("<If", _F32, v))
    elif isinstance(v, str):
        f.write(struct.pack("<I", _STR))
        _w_str(f, v)
    elif isinstance(v, (list, tuple)):
        f.write(struct.pack("<I", _ARR))
        if len(v) and isinstance(v[0], str):
            f.write(struct.pack("<IQ", _STR, len(v)))
            for s in v:
                _w_str(f, s)
        elif len(v) and isinstance(v[0], float):
            f.write(struct.pack("<IQ", _F32, len(v)))
            f.write(np.asarray(v, dtype="<f4").tobytes())
        else:
            f.write(struct.pack("<IQ", _I32, len(v)))
            f.write(np.asarray(v, dtype="<i4").tobytes())
    else:
        raise TypeError(f"unsupported metadata value {type(v)}")


def write(path: str, meta: dict, tensors: list, version: int = 3) -> None:
    """Write a GGUF file (v3 by default; v1 differs only in its two 32-bit
    counts).  meta values: bool/int/float/str or lists of them."""
    offsets, off = [], 0
    for t in tensors:
        offsets.append(off)
        off += t.n_bytes
        off = (off + ALIGN - 1) // ALIGN * ALIGN
    with open(path, "wb") as f:
        if version == 1:
            f.write(struct.pack("<IIII", GGUF_MAGIC, 1, len(tensors), len(meta)))
        else:
            f.write(struct.pack("<IIQQ", GGUF_MAGIC, version, len(tensors), len(meta)))
        for k, v in meta.items():
            _w_str(f, k)
            _w_value(f, v)
        for t, o in zip(tensors, offsets):
            _w_str(f, t.name)
            f.write(struct.pack("<I", len(t.dims)))
            f.write(struct.pack(f"<{len(t.dims)}Q", *t.dims))
            f.write(struct.pack("<IQ", t.ggml_type, o))
        pos = f.tell()
        f.write(b"\0" * ((pos + ALIGN - 1) // ALIGN * ALIGN - pos))
        base = f.tell()
        for t, o in zip(tensors, offsets):
            cur = f.tell() - base
            if cur < o:
                f.write(b"\0" * (o - cur))
            f.write(memoryview(np.ascontiguousarray(t.data)).cast("B"))


class _Reader:
    def __init__(self, buf):
        self.buf, self.pos = buf, 0

    def take(self, fmt):
        v = struct.unpack_from(fmt, self.buf, self.pos)
        self.pos += struct.calcsize(fmt)
        return v if len(v) > 1 else v[0]

    def string(self):
        n = self.take("<Q")
        s = bytes(self.buf[self.pos:self.pos + n]).decode("utf-8", "replace")
        self.pos += n
        return s

    def value(self, vt):
        simple = {_U8: "<B", _I8: "<b", _U16: "<H", _I16: "<h", _U32: "<I", _I32: "<i",
                  _F32: "<f", _U64: "<Q", _I64: "<q", _F64: "<d"}
        if vt in simple:
            return self.take(simple[vt])
        if vt == _BOOL:
            return bool(self.take("<B"))
        if vt == _STR:
            return self.string()
        if vt == _ARR:
            et, n = self.take("<I"), self.take("<Q")
            return [self.value(et) for _ in range(n)]
        raise ValueError(f"unknown metadata type {vt}")


def read(path: str, load_data: bool = True) -> GgufFile:
    """Parse a GGUF file; tensor data are zero-copy views of a memory map."""
    mm = np.memmap(path, dtype=np.uint8, mode="r")
    r = _Reader(mm)
    magic, version = r.take("<I"), r.take("<I")
    if magic != GGUF_MAGIC or version not in (1, 2, 3):
        raise ValueError(f"{path}: not a GGUF v1-3 file")
    n_t, n_kv = (r.take("<I"), r.take("<I")) if version == 1 else (r.take("<Q"), r.take("<Q"))
    out = GgufFile()
    for _ in range(n_kv):
        k = r.string()
        out.meta[k] = r.value(r.take("<I"))
    infos = []
    for _ in range(n_t):
        name = r.string()
        nd = r.take("<I")
        dims = tuple(r.take("<Q") for _ in range(nd))
        infos.append((name, dims, r.take("<I"), r.take("<Q")))
    align = int(out.meta.get("general.alignment", ALIGN))
    base = (r.pos + align - 1) // align * align
    for name, dims, ty, off in infos:
        n = int(np.prod(dims))
        nb = row_bytes(ty, n) if ty in TYPE_BLOCK else 0
        data = mm[base + off: base + off + nb] if load_data else np.empty(0, np.uint8)
        out.tensors.append(Tensor(name, ty, dims, data))
    return out
