"""Minimal GGUF reader for tests: tensor infos and payload slices of an in-memory
image (layout per crates/ramforge-core/src/gguf.rs:196-330)."""
from __future__ import annotations

import struct

import numpy as np

_SCALAR = {0: "<B", 1: "<b", 2: "<H", 3: "<h", 4: "<I", 5: "<i", 6: "<f", 7: "<B", 10: "<Q", 11: "<q", 12: "<d"}
_BLOCK = {0: (1, 4), 1: (1, 2), 2: (32, 18), 6: (32, 22), 8: (32, 34), 10: (256, 84), 11: (256, 110),
          12: (256, 144), 13: (256, 176), 14: (256, 210), 15: (256, 292)}


def read_tensors(img) -> dict:
    b = bytes(np.asarray(img, np.uint8)) if not isinstance(img, bytes) else img
    pos = 0

    def take(fmt):
        nonlocal pos
        v = struct.unpack_from(fmt, b, pos)[0]
        pos += struct.calcsize(fmt)
        return v

    def string():
        nonlocal pos
        n = take("<Q")
        s = b[pos:pos + n].decode()
        pos += n
        return s

    def value(t):
        if t == 8:
            return string()
        if t == 9:
            et, n = take("<I"), take("<Q")
            return [value(et) for _ in range(n)]
        return take(_SCALAR[t])

    assert b[:4] == b"GGUF"
    pos = 4
    take("<I")
    nt, nkv = take("<Q"), take("<Q")
    meta = {}
    for _ in range(nkv):
        k = string()
        meta[k] = value(take("<I"))
    align = meta.get("general.alignment", 32)
    infos = []
    for _ in range(nt):
        name = string()
        nd = take("<I")
        dims = [take("<Q") for _ in range(nd)]
        infos.append((name, dims, take("<I"), take("<Q")))
    ds = (pos + align - 1) // align * align
    out = {}
    for name, dims, t, off in infos:
        ne = int(np.prod(dims))
        qk, bs = _BLOCK[t]
        n = (ne + qk - 1) // qk * bs
        out[name] = {"dims": dims, "type": t, "data": np.frombuffer(b, np.uint8, n, ds + off)}
    return out


def tensor_bytes(img, name) -> np.ndarray:
    return read_tensors(img)[name]["data"]
