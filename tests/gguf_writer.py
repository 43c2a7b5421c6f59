"""Minimal GGUF v3 writer for the tests (any tensor type, given its packed bytes).

Layout (the GGUF format): "GGUF", u32 version 3, u64 tensor count, u64 metadata
count; metadata (u64-length string key, u32 value type, value); tensor infos
(name, u32 n_dims, u64 dims innermost first, u32 ggml type, u64 offset from the
data start); padding to the alignment; tensor data, each tensor at an aligned
offset.
"""
from __future__ import annotations

import struct

import numpy as np

U8, I8, U16, I16, U32, I32, F32, BOOL, STRING, ARRAY, U64, I64, F64 = range(13)
_FMT = {U8: "<B", I8: "<b", U16: "<H", I16: "<h", U32: "<I", I32: "<i", F32: "<f", BOOL: "<?",
        U64: "<Q", I64: "<q", F64: "<d"}

# ggml tensor types used by the tests
GGML_F32, GGML_F16, GGML_Q4_0, GGML_Q8_0, GGML_Q4_K, GGML_Q6_K, GGML_I32 = 0, 1, 2, 8, 12, 14, 26
GGML_OF_FMT = {0: 0, 1: 1, 7: 2, 8: 3, 9: 6, 10: 7, 11: 8, 12: 10, 13: 11, 14: 12, 15: 13, 16: 14}


def _str(s: str) -> bytes:
    b = s.encode()
    return struct.pack("<Q", len(b)) + b


def _value(t: int, v) -> bytes:
    if t == STRING:
        return _str(v)
    if t == ARRAY:
        et, items = v
        out = struct.pack("<IQ", et, len(items))
        return out + b"".join(_str(x) if et == STRING else struct.pack(_FMT[et], x) for x in items)
    return struct.pack(_FMT[t], v)


def write_gguf(path, kv, tensors, alignment: int = 32, version: int = 3) -> list[int]:
    """kv: [(key, type, value)]; tensors: [(name, ggml_type, shape outermost first, bytes)].
    Returns each tensor's offset in the file."""
    head = b"GGUF" + struct.pack("<IQQ", version, len(tensors), len(kv))
    for key, t, v in kv:
        head += _str(key) + struct.pack("<I", t) + _value(t, v)
    offs, off = [], 0
    for name, gt, shape, data in tensors:
        offs.append(off)
        head += _str(name) + struct.pack("<I", len(shape))
        head += b"".join(struct.pack("<Q", d) for d in reversed(shape))
        head += struct.pack("<IQ", gt, off)
        off += (len(data) + alignment - 1) // alignment * alignment
    data_start = (len(head) + alignment - 1) // alignment * alignment
    body = bytearray(head + b"\0" * (data_start - len(head)))
    for (name, gt, shape, data), o in zip(tensors, offs):
        assert len(body) == data_start + o
        body += bytes(data) + b"\0" * ((-len(data)) % alignment)
    with open(path, "wb") as f:
        f.write(body)
    return [data_start + o for o in offs]


def as_bytes(a: np.ndarray) -> bytes:
    return np.ascontiguousarray(a).tobytes()
