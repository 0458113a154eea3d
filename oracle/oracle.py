"""ctypes wrapper over liboracle.so - the CPU restatement of RAMforge's
legacy decode hot path.

TEST INFRASTRUCTURE ONLY: imported by tests/, by __graft_entry__.smoke() and
by the cpu_baseline / --impl reference legs of bench.py, always as the checker
or the timed CPU baseline, never as the product path.
"""
from __future__ import annotations

import ctypes
import os
import subprocess

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
_LIB_PATH = os.path.join(_HERE, "liboracle.so")
_lib = None

F32, F16, Q4_0, Q5_0, Q8_0, Q4_K, Q6_K = 0, 1, 2, 6, 8, 12, 14
Q2_K, Q3_K, Q5_K, Q8_K = 10, 11, 13, 15

_f32p = ctypes.POINTER(ctypes.c_float)
_u8p = ctypes.POINTER(ctypes.c_uint8)
_u32p = ctypes.POINTER(ctypes.c_uint32)


class OracleError(RuntimeError):
    pass


def build() -> str:
    """Compile liboracle.so with the committed Makefile."""
    subprocess.run(["make", "-s", "-C", _HERE], check=True)
    return _LIB_PATH


class _Config(ctypes.Structure):
    _fields_ = [(n, ctypes.c_uint32) for n in (
        "vocab_size", "context_length", "n_embd", "n_layers", "n_ff", "n_heads",
        "n_kv_heads", "head_dim")] + [("rms_eps", ctypes.c_float), ("rope_theta", ctypes.c_float)]


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(_LIB_PATH):
            build()
        L = ctypes.CDLL(_LIB_PATH)
        sz = ctypes.c_size_t
        L.orc_f16_to_f32.restype = ctypes.c_float
        L.orc_f16_to_f32.argtypes = [ctypes.c_uint16]
        L.orc_f32_to_f16.restype = ctypes.c_uint16
        L.orc_f32_to_f16.argtypes = [ctypes.c_float]
        L.orc_row_bytes.restype = sz
        L.orc_row_bytes.argtypes = [ctypes.c_int, sz]
        L.orc_dequant_row.argtypes = [ctypes.c_int, _u8p, sz, sz, _f32p]
        L.orc_matvec.argtypes = [ctypes.c_int, _u8p, sz, sz, sz, _f32p, _f32p, ctypes.c_int]
        L.orc_matvec_reference.argtypes = [ctypes.c_int, _u8p, sz, sz, sz, _f32p, _f32p]
        L.orc_rmsnorm.argtypes = [_f32p, _f32p, ctypes.c_float, sz, _f32p]
        L.orc_rope.argtypes = [_f32p, _f32p, sz, sz, sz, sz, ctypes.c_float]
        L.orc_attention.argtypes = [_f32p] * 5 + [sz] * 4 + [_f32p]
        L.orc_softmax.argtypes = [_f32p, sz]
        L.orc_silu.argtypes = [_f32p, _f32p, sz]
        L.orc_swiglu.argtypes = [_f32p, _f32p, _f32p, sz]
        L.orc_argmax.restype = ctypes.c_uint32
        L.orc_argmax.argtypes = [_f32p, sz]
        L.orc_model_open.restype = ctypes.c_void_p
        L.orc_model_open.argtypes = [ctypes.c_void_p, sz, ctypes.c_int, ctypes.c_uint32, ctypes.c_int]
        L.orc_model_close.argtypes = [ctypes.c_void_p]
        L.orc_last_error.restype = ctypes.c_char_p
        L.orc_model_config.argtypes = [ctypes.c_void_p, ctypes.POINTER(_Config)]
        L.orc_forward.argtypes = [ctypes.c_void_p, ctypes.c_uint32, ctypes.c_uint32, _f32p]
        L.orc_logits.argtypes = [ctypes.c_void_p, _f32p, _f32p]
        L.orc_last_layer_hiddens.argtypes = [ctypes.c_void_p, _f32p]
        L.orc_layer_step.argtypes = [ctypes.c_void_p, ctypes.c_uint32, ctypes.c_uint32, _f32p]
        L.orc_logits_rows.argtypes = [ctypes.c_void_p, _f32p, ctypes.c_uint32, ctypes.c_uint32, _f32p]
        L.orc_kv_len.restype = ctypes.c_uint32
        L.orc_kv_len.argtypes = [ctypes.c_void_p]
        L.orc_kv_reset.argtypes = [ctypes.c_void_p]
        L.orc_kv_fill_synthetic.argtypes = [ctypes.c_void_p, ctypes.c_uint32, ctypes.c_uint32]
        L.orc_kv_read.argtypes = [ctypes.c_void_p, ctypes.c_uint32, ctypes.c_int, ctypes.c_uint32,
                                  ctypes.c_uint32, _f32p]
        L.orc_generate.argtypes = [ctypes.c_void_p, _u32p, ctypes.c_uint32, ctypes.c_uint32, _u32p,
                                   _f32p, _f32p]
        _lib = L
    return _lib


def _fp(a):
    return a.ctypes.data_as(_f32p)


def _check(rc):
    if rc != 0:
        raise OracleError(lib().orc_last_error().decode())


def f16_to_f32(bits: int) -> float:
    return lib().orc_f16_to_f32(bits)


def f32_to_f16(v: float) -> int:
    return lib().orc_f32_to_f16(v)


def row_bytes(gtype: int, n: int) -> int:
    return lib().orc_row_bytes(gtype, n)


def dequant_row(gtype: int, raw: bytes | np.ndarray, n: int) -> np.ndarray:
    b = np.frombuffer(bytes(raw), dtype=np.uint8) if not isinstance(raw, np.ndarray) else raw
    b = np.ascontiguousarray(b, dtype=np.uint8)
    out = np.empty(n, np.float32)
    _check(lib().orc_dequant_row(gtype, b.ctypes.data_as(_u8p), b.size, n, _fp(out)))
    return out


def matvec(gtype: int, raw, n_in: int, n_out: int, x: np.ndarray, threads: int = 1,
           reference: bool = False) -> np.ndarray:
    b = np.ascontiguousarray(np.frombuffer(bytes(raw), np.uint8) if not isinstance(raw, np.ndarray) else raw,
                             dtype=np.uint8)
    x = np.ascontiguousarray(x, np.float32)
    if x.size != n_in:  # TensorData::matvec refuses, never reinterprets (tensor.rs:1205-1218)
        raise OracleError(f"matvec arity mismatch: x has {x.size} elements, the matrix takes {n_in}")
    y = np.empty(n_out, np.float32)
    if reference:
        _check(lib().orc_matvec_reference(gtype, b.ctypes.data_as(_u8p), b.size, n_in, n_out, _fp(x), _fp(y)))
    else:
        _check(lib().orc_matvec(gtype, b.ctypes.data_as(_u8p), b.size, n_in, n_out, _fp(x), _fp(y), threads))
    return y


def rmsnorm(x, w, eps) -> np.ndarray:
    x = np.ascontiguousarray(x, np.float32)
    w = np.ascontiguousarray(w, np.float32)
    y = np.empty_like(x)
    _check(lib().orc_rmsnorm(_fp(x), _fp(w), eps, x.size, _fp(y)))
    return y


def rope(q, k, pos, head_dim, n_heads, n_kv_heads, theta):
    q = np.array(q, np.float32)
    k = np.array(k, np.float32)
    _check(lib().orc_rope(_fp(q), _fp(k), pos, head_dim, n_heads, n_kv_heads, theta))
    return q, k


def attention(q, k_hist, v_hist, k_cur, v_cur, hist, n_heads, n_kv_heads, head_dim):
    arrs = [np.ascontiguousarray(a, np.float32).reshape(-1) for a in (q, k_hist, v_hist, k_cur, v_cur)]
    for i in (1, 2):  # ctypes needs a valid pointer even for empty history
        if arrs[i].size == 0:
            arrs[i] = np.zeros(1, np.float32)
    out = np.empty(n_heads * head_dim, np.float32)
    _check(lib().orc_attention(*[_fp(a) for a in arrs], hist, n_heads, n_kv_heads, head_dim, _fp(out)))
    return out


def softmax(v):
    v = np.array(v, np.float32)
    _check(lib().orc_softmax(_fp(v), v.size))
    return v


def swiglu(g, u):
    g = np.ascontiguousarray(g, np.float32)
    u = np.ascontiguousarray(u, np.float32)
    y = np.empty_like(g)
    lib().orc_swiglu(_fp(g), _fp(u), _fp(y), g.size)
    return y


def argmax(v) -> int:
    v = np.ascontiguousarray(v, np.float32)
    return int(lib().orc_argmax(_fp(v), v.size))


class OracleModel:
    """The reference executor over a GGUF image held in memory.

    kv_f16=True rounds committed K/V history to f16 (the GPU cache format);
    False is the reference's f32 cache.  `threads` partitions matvec rows
    only and never changes a result.
    """

    def __init__(self, gguf: bytes | np.ndarray | memoryview, kv_f16: bool = True, max_seq: int = 0,
                 threads: int = 1):
        if isinstance(gguf, np.ndarray):
            self._buf = np.ascontiguousarray(gguf, np.uint8)
        else:
            self._buf = np.frombuffer(gguf, dtype=np.uint8)
        self._h = lib().orc_model_open(self._buf.ctypes.data, self._buf.size, int(kv_f16), max_seq, threads)
        if not self._h:
            raise OracleError(lib().orc_last_error().decode())
        c = _Config()
        lib().orc_model_config(self._h, ctypes.byref(c))
        self.config = {f: getattr(c, f) for f, _ in _Config._fields_}

    def close(self):
        if self._h:
            lib().orc_model_close(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    @property
    def kv_len(self) -> int:
        return lib().orc_kv_len(self._h)

    def reset(self):
        lib().orc_kv_reset(self._h)

    def kv_fill_synthetic(self, n: int, seed: int = 0) -> None:
        """Timing support only: history length n with seeded values, so a layer
        step can be timed at a long decode's context without n forwards."""
        _check(lib().orc_kv_fill_synthetic(self._h, n, seed))

    def forward(self, token: int, pos: int) -> np.ndarray:
        out = np.empty(self.config["n_embd"], np.float32)
        _check(lib().orc_forward(self._h, token, pos, _fp(out)))
        return out

    def logits(self, final_hidden) -> np.ndarray:
        fh = np.ascontiguousarray(final_hidden, np.float32)
        out = np.empty(self.config["vocab_size"], np.float32)
        _check(lib().orc_logits(self._h, _fp(fh), _fp(out)))
        return out

    def layer_step(self, layer: int, pos: int, hidden: np.ndarray) -> None:
        """One layer of a token forward on `hidden` in place (no KV commit)."""
        _check(lib().orc_layer_step(self._h, layer, pos, _fp(hidden)))

    def logits_rows(self, final_hidden, r0: int, r1: int) -> np.ndarray:
        fh = np.ascontiguousarray(final_hidden, np.float32)
        out = np.empty(r1 - r0, np.float32)
        _check(lib().orc_logits_rows(self._h, _fp(fh), r0, r1, _fp(out)))
        return out

    def layer_hiddens(self) -> np.ndarray:
        out = np.empty((self.config["n_layers"], self.config["n_embd"]), np.float32)
        lib().orc_last_layer_hiddens(self._h, _fp(out))
        return out

    def kv_read(self, layer: int, which_v: bool, start: int, end: int) -> np.ndarray:
        kvd = self.config["n_kv_heads"] * self.config["head_dim"]
        out = np.empty((end - start, kvd), np.float32)
        _check(lib().orc_kv_read(self._h, layer, int(which_v), start, end, _fp(out)))
        return out

    def generate(self, prompt, n_new: int, want_logits: bool = False):
        p = np.ascontiguousarray(prompt, np.uint32)
        toks = np.empty(max(n_new, 1), np.uint32)
        margins = np.empty(max(n_new, 1), np.float32)
        logits = np.empty((max(n_new, 1), self.config["vocab_size"]), np.float32) if want_logits else None
        _check(lib().orc_generate(self._h, p.ctypes.data_as(_u32p), p.size, n_new, toks.ctypes.data_as(_u32p),
                                  _fp(logits) if logits is not None else None, _fp(margins)))
        return toks[:n_new], (logits[:n_new] if logits is not None else None), margins[:n_new]
