"""Minimal GGUF v3 writer for hand-built test fixtures.

The reference's tests assemble GGUF images byte by byte (e.g.
crates/ramforge-runtime/src/inference.rs:2148-2300); this helper does the same
for the parity tests: metadata (scalars, strings, arrays), tensor infos with
32-byte aligned offsets and the data section (gguf.rs:196-330 reads it back).
"""
from __future__ import annotations

import struct

import numpy as np

U8, I8, U16, I16, U32, I32, F32, BOOL, STR, ARR, U64, I64, F64 = range(13)
_FMT = {U8: "<B", I8: "<b", U16: "<H", I16: "<h", U32: "<I", I32: "<i", F32: "<f", BOOL: "<B", U64: "<Q",
        I64: "<q", F64: "<d"}


def _s(b: bytearray, s: str):
    e = s.encode()
    b += struct.pack("<Q", len(e)) + e


def _val(b: bytearray, t: int, v):
    if t == STR:
        _s(b, v)
    else:
        b += struct.pack(_FMT[t], v)


def write_gguf(meta: list, tensors: list, alignment: int = 32, version: int = 3) -> bytes:
    """meta: [(key, type, value)] (ARR value = (elem_type, [values]));
    tensors: [(name, dims, ggml_type, raw_bytes)] with dims = [ne0, ne1, ...]."""
    b = bytearray(b"GGUF")
    b += struct.pack("<I", version) + struct.pack("<Q", len(tensors)) + struct.pack("<Q", len(meta))
    for key, t, v in meta:
        _s(b, key)
        b += struct.pack("<I", t)
        if t == ARR:
            et, vals = v
            b += struct.pack("<I", et) + struct.pack("<Q", len(vals))
            for x in vals:
                _val(b, et, x)
        else:
            _val(b, t, v)
    off = 0
    offsets = []
    for name, dims, gt, raw in tensors:
        offsets.append(off)
        off += (len(raw) + alignment - 1) // alignment * alignment
    for (name, dims, gt, raw), o in zip(tensors, offsets):
        _s(b, name)
        b += struct.pack("<I", len(dims))
        for d in dims:
            b += struct.pack("<Q", d)
        b += struct.pack("<I", gt) + struct.pack("<Q", o)
    while len(b) % alignment:
        b.append(0)
    for (name, dims, gt, raw), o in zip(tensors, offsets):
        b += bytes(raw)
        while len(b) % alignment:
            b.append(0)
    return bytes(b)


def f32_bytes(a) -> bytes:
    return np.ascontiguousarray(a, np.float32).tobytes()
