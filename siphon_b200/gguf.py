"""Minimal GGUF v3 writer and reader for synthetic models.

Follows the public GGUF layout (little-endian): "GGUF", u32 version,
u64 tensor count, u64 key-value count; key-value pairs (string key, u32 value
type, value); tensor infos (string name, u32 n_dims, u64 dims, u32 ggml type,
u64 offset into the data section); padding to `general.alignment`; tensor
data, each tensor aligned. Strings are u64 length + bytes. The reference
reads the same layout (its src/gguf.c).
"""

from __future__ import annotations

import struct
from dataclasses import dataclass
from pathlib import Path
from typing import Callable, Union

import numpy as np

from . import quant as Q

U8, I8, U16, I16, U32, I32, F32, BOOL, STRING, ARRAY, U64, I64, F64 = range(13)
ALIGN = 32
_FMT = {U8: "<B", I8: "<b", U16: "<H", I16: "<h", U32: "<I", I32: "<i", F32: "<f", BOOL: "<B",
        U64: "<Q", I64: "<q", F64: "<d"}

# tensor payload: the raw bytes, or a function returning them (called once,
# while the file is written, so large models never sit in memory whole)
Payload = Union[np.ndarray, Callable[[], np.ndarray]]


def _str(s: str) -> bytes:
    b = s.encode()
    return struct.pack("<Q", len(b)) + b


def _value(vtype: int, v) -> bytes:
    if vtype == STRING:
        return _str(v)
    if vtype == ARRAY:
        etype, items = v
        return struct.pack("<IQ", etype, len(items)) + b"".join(_value(etype, x) for x in items)
    return struct.pack(_FMT[vtype], v)


def tensor_bytes(ttype: int, dims: tuple[int, ...]) -> int:
    n = 1
    for d in dims[1:]:
        n *= d
    return n * Q.row_bytes(ttype, dims[0])


def write(path: str | Path, kvs: list[tuple[str, int, object]],
          tensors: list[tuple[str, tuple[int, ...], int, Payload]]) -> Path:
    """kvs: (key, value type, value); tensors: (name, dims with dims[0] the
    row length, ggml type id, raw bytes as uint8 or a function making them)."""
    path = Path(path)
    head = bytearray(b"GGUF" + struct.pack("<IQQ", 3, len(tensors), len(kvs)))
    for key, vt, v in kvs:
        head += _str(key) + struct.pack("<I", vt) + _value(vt, v)
    offset = 0
    sizes = []
    for name, dims, ttype, _ in tensors:
        nbytes = tensor_bytes(ttype, dims)
        sizes.append(nbytes)
        head += _str(name) + struct.pack("<I", len(dims)) + b"".join(struct.pack("<Q", d) for d in dims)
        head += struct.pack("<IQ", ttype, offset)
        offset += (nbytes + ALIGN - 1) // ALIGN * ALIGN
    head += b"\0" * ((ALIGN - len(head) % ALIGN) % ALIGN)
    with open(path, "wb") as f:
        f.write(head)
        for (name, dims, ttype, data), nbytes in zip(tensors, sizes):
            if callable(data):
                data = data()
            b = np.ascontiguousarray(data).view(np.uint8).reshape(-1)
            if b.size != nbytes:
                raise ValueError(f"{name}: {b.size} bytes for a {Q.NAMES[ttype]} tensor of dims {dims} "
                                 f"({nbytes} expected)")
            b.tofile(f)
            f.write(b"\0" * ((ALIGN - b.size % ALIGN) % ALIGN))
    return path


@dataclass(frozen=True)
class TensorInfo:
    name: str
    dims: tuple[int, ...]
    type: int
    offset: int      # from the start of the file
    nbytes: int


class Reader:
    """Read-only view of a GGUF file: key-values, tensor infos, and each
    tensor's bytes as a slice of a memory map."""

    def __init__(self, path: str | Path):
        self.path = Path(path)
        self.map = np.memmap(self.path, dtype=np.uint8, mode="r")
        buf = self.map
        pos = 0

        def take(fmt: str):
            nonlocal pos
            size = struct.calcsize(fmt)
            v = struct.unpack_from(fmt, buf, pos)
            pos += size
            return v[0] if len(v) == 1 else v

        def string() -> str:
            nonlocal pos
            n = take("<Q")
            s = bytes(buf[pos:pos + n]).decode()
            pos += n
            return s

        def value(vt: int):
            if vt == STRING:
                return string()
            if vt == ARRAY:
                et, n = take("<I"), take("<Q")
                return [value(et) for _ in range(n)]
            return take(_FMT[vt])

        if bytes(buf[:4]) != b"GGUF":
            raise ValueError(f"{path}: not a GGUF file")
        pos = 4
        version, n_tensors, n_kv = take("<I"), take("<Q"), take("<Q")
        if version != 3:
            raise ValueError(f"{path}: GGUF version {version} (3 expected)")
        self.kv: dict[str, object] = {}
        for _ in range(n_kv):
            key = string()
            self.kv[key] = value(take("<I"))
        infos = []
        for _ in range(n_tensors):
            name = string()
            nd = take("<I")
            dims = tuple(take("<Q") for _ in range(nd))
            ttype, off = take("<I"), take("<Q")
            infos.append((name, dims, ttype, off))
        align = int(self.kv.get("general.alignment", ALIGN))
        base = (pos + align - 1) // align * align
        self.tensors = {n: TensorInfo(n, d, t, base + o, tensor_bytes(t, d)) for n, d, t, o in infos}

    def data(self, name: str) -> np.ndarray:
        t = self.tensors[name]
        return self.map[t.offset:t.offset + t.nbytes]
