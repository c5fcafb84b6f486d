"""Minimal GGUF v3 writer for synthetic models.

Follows the public GGUF layout (little-endian): "GGUF", u32 version,
u64 tensor count, u64 key-value count; key-value pairs (string key, u32 value
type, value); tensor infos (string name, u32 n_dims, u64 dims, u32 ggml type,
u64 offset into the data section); padding to `general.alignment`; tensor
data, each tensor aligned. Strings are u64 length + bytes. The reference
reads the same layout (its src/gguf.c).
"""

from __future__ import annotations

import struct
from pathlib import Path

import numpy as np

U8, I8, U16, I16, U32, I32, F32, BOOL, STRING, ARRAY, U64, I64, F64 = range(13)
ALIGN = 32


def _str(s: str) -> bytes:
    b = s.encode()
    return struct.pack("<Q", len(b)) + b


def _value(vtype: int, v) -> bytes:
    fmt = {U8: "<B", I8: "<b", U16: "<H", I16: "<h", U32: "<I", I32: "<i", F32: "<f", BOOL: "<B",
           U64: "<Q", I64: "<q", F64: "<d"}
    if vtype == STRING:
        return _str(v)
    if vtype == ARRAY:
        etype, items = v
        return struct.pack("<IQ", etype, len(items)) + b"".join(_value(etype, x) for x in items)
    return struct.pack(fmt[vtype], v)


def write(path: str | Path, kvs: list[tuple[str, int, object]],
          tensors: list[tuple[str, tuple[int, ...], int, np.ndarray]]) -> Path:
    """kvs: (key, value type, value); tensors: (name, dims with dims[0] the
    row length, ggml type id, raw bytes as uint8)."""
    path = Path(path)
    head = bytearray(b"GGUF" + struct.pack("<IQQ", 3, len(tensors), len(kvs)))
    for key, vt, v in kvs:
        head += _str(key) + struct.pack("<I", vt) + _value(vt, v)
    offset = 0
    offsets = []
    for name, dims, ttype, data in tensors:
        offsets.append(offset)
        head += _str(name) + struct.pack("<I", len(dims)) + b"".join(struct.pack("<Q", d) for d in dims)
        head += struct.pack("<IQ", ttype, offset)
        offset += (data.nbytes + ALIGN - 1) // ALIGN * ALIGN
    head += b"\0" * ((ALIGN - len(head) % ALIGN) % ALIGN)
    with open(path, "wb") as f:
        f.write(head)
        for (name, dims, ttype, data), off in zip(tensors, offsets):
            b = np.ascontiguousarray(data).view(np.uint8).tobytes()
            f.write(b)
            f.write(b"\0" * ((ALIGN - len(b) % ALIGN) % ALIGN))
    return path
