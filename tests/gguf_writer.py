"""A minimal GGUF (version 3) writer for the tests: metadata key/values and F32 tensors, in
the published layout (magic, version, counts, key/values, tensor infos, data aligned to 32
bytes). It stands in for the reference's converters (tools/convert_*.py), which need the
models' checkpoints; the files it writes carry the keys those converters write."""
from __future__ import annotations

import struct

import numpy as np

U8, I8, U16, I16, U32, I32, F32, BOOL, STRING, ARRAY, U64, I64, F64 = range(13)
_FMT = {U8: "<B", I8: "<b", U16: "<H", I16: "<h", U32: "<I", I32: "<i", F32: "<f", BOOL: "<B",
        U64: "<Q", I64: "<q", F64: "<d"}


def _str(s: str) -> bytes:
    b = s.encode()
    return struct.pack("<Q", len(b)) + b


def _value(t, v) -> bytes:
    if t == STRING:
        return _str(v)
    return struct.pack(_FMT[t], v)


def write(path, kv, tensors=None, alignment=32):
    """kv: {key: (type, value)} with type one of the constants above, or (ARRAY, elem_type,
    [values]); tensors: {name: float32 array}."""
    tensors = tensors or {}
    out = bytearray(b"GGUF" + struct.pack("<IQQ", 3, len(tensors), len(kv)))
    for k, spec in kv.items():
        out += _str(k)
        if spec[0] == ARRAY:
            _, et, vals = spec
            out += struct.pack("<IIQ", ARRAY, et, len(vals))
            for v in vals:
                out += _value(et, v)
        else:
            t, v = spec
            out += struct.pack("<I", t) + _value(t, v)
    blobs, off = [], 0
    for name, arr in tensors.items():
        a = np.ascontiguousarray(arr, np.float32)
        out += _str(name) + struct.pack("<I", a.ndim)
        for d in a.shape[::-1]:
            out += struct.pack("<Q", d)
        out += struct.pack("<IQ", 0, off)
        blob = a.tobytes()
        pad = (-len(blob)) % alignment
        blobs.append(blob + b"\0" * pad)
        off += len(blob) + pad
    out += b"\0" * ((-len(out)) % alignment)
    for b in blobs:
        out += b
    with open(path, "wb") as f:
        f.write(bytes(out))
