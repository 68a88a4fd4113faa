"""GGUF v3 writer: metadata and tensors in the layout GgufModelFile.Open
reads (header, typed key/value pairs, tensor descriptors, data aligned to
general.alignment). Used to save synthetic models and by the tests; reading
is the library's si_gguf_* (native.GgufFile).
"""
from __future__ import annotations

import struct
from pathlib import Path

import numpy as np

MAGIC = 0x46554747
VERSION = 3
# GgufMetadataType (GgufModelFile.cs:7-22)
U8, I8, U16, I16, U32, I32, F32, BOOL, STRING, ARRAY, U64, I64, F64 = range(13)
_PACK = {U8: "<B", I8: "<b", U16: "<H", I16: "<h", U32: "<I", I32: "<i", F32: "<f", BOOL: "<B", U64: "<Q",
         I64: "<q", F64: "<d"}


def _string(s: str) -> bytes:
    b = s.encode("utf-8")
    return struct.pack("<Q", len(b)) + b


def _value(v) -> bytes:
    """A typed value: (type, value) tuples are written as given; Python
    bool/int/float/str map to Bool/Int32 (Int64 when out of range)/Float32/
    String; lists and numpy arrays to Array."""
    if isinstance(v, tuple):
        t, x = v
        if t == STRING:
            return struct.pack("<I", STRING) + _string(x)
        if t == ARRAY:
            et, items = x
            body = struct.pack("<IIQ", ARRAY, et, len(items))
            if et == STRING:
                return body + b"".join(_string(i) for i in items)
            return body + b"".join(struct.pack(_PACK[et], i) for i in items)
        return struct.pack("<I", t) + struct.pack(_PACK[t], x)
    if isinstance(v, bool):
        return _value((BOOL, int(v)))
    if isinstance(v, int):
        return _value((I32, v) if -2**31 <= v < 2**31 else (I64, v))
    if isinstance(v, float):
        return _value((F32, v))
    if isinstance(v, str):
        return _value((STRING, v))
    if isinstance(v, (list, np.ndarray)):
        arr = list(v)
        if arr and isinstance(arr[0], str):
            return _value((ARRAY, (STRING, arr)))
        if arr and isinstance(arr[0], (float, np.floating)):
            return _value((ARRAY, (F32, [float(a) for a in arr])))
        return _value((ARRAY, (I32, [int(a) for a in arr])))
    raise TypeError(f"unsupported metadata value {v!r}")


def write(path, metadata: dict, tensors: list, alignment: int = 32) -> None:
    """tensors: (name, gguf type id, dims fastest-first, data as a numpy array or bytes)."""
    tensors = [(n, t, d, np.frombuffer(bytes(x), dtype=np.uint8) if isinstance(x, (bytes, bytearray))
                else np.ascontiguousarray(x).view(np.uint8).reshape(-1)) for n, t, d, x in tensors]
    head = struct.pack("<IIQQ", MAGIC, VERSION, len(tensors), len(metadata))
    for k, v in metadata.items():
        head += _string(k) + _value(v)
    offsets, off = [], 0
    for _, _, _, data in tensors:
        off = (off + alignment - 1) // alignment * alignment
        offsets.append(off)
        off += len(data)
    for (name, t, dims, _), o in zip(tensors, offsets):
        head += _string(name) + struct.pack("<I", len(dims)) + b"".join(struct.pack("<Q", d) for d in dims)
        head += struct.pack("<IQ", t, o)
    start = (len(head) + alignment - 1) // alignment * alignment
    with open(Path(path), "wb") as f:
        f.write(head + b"\0" * (start - len(head)))
        pos = 0
        for (_, _, _, data), o in zip(tensors, offsets):
            f.write(b"\0" * (o - pos))
            f.write(data.tobytes())
            pos = o + len(data)
