"""Seeded synthetic Llama GGUF models for the benchmark configurations.

The benchmark configurations are synthetic models (weights N(0, 0.02) from a seed,
quantised to GGUF block formats, f32 ones for norms); there is no public
checkpoint or dataset on this path.  The images are produced by
librfsynth.so (counter-based normal generator + the build's own GGUF writer
and block encoders), in memory, in a few seconds for an 8B-shaped model.
"""
from __future__ import annotations

import ctypes
import os
from dataclasses import dataclass, field, replace

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
SYNTH_PATH = os.path.join(_HERE, "librfsynth.so")

F32, F16, Q4_0, Q8_0, Q4_K, Q6_K = 0, 1, 2, 8, 12, 14
Q5_0, Q2_K, Q3_K, Q5_K, Q8_K = 6, 10, 11, 13, 15  # no encoder here: random_blocks
TYPE_NAMES = {F32: "F32", F16: "F16", Q4_0: "Q4_0", Q8_0: "Q8_0", Q4_K: "Q4_K", Q6_K: "Q6_K"}


class _Spec(ctypes.Structure):
    _fields_ = [("arch", ctypes.c_char_p)] + [(n, ctypes.c_uint32) for n in (
        "vocab_size", "context_length", "n_embd", "n_layers", "n_ff", "n_heads", "n_kv_heads")] + [
        ("rms_eps", ctypes.c_float), ("rope_theta", ctypes.c_float), ("layer_type", ctypes.c_int),
        ("embd_type", ctypes.c_int), ("out_type", ctypes.c_int), ("seed", ctypes.c_uint64),
        ("weight_std", ctypes.c_float), ("v_type", ctypes.c_int), ("down_type", ctypes.c_int),
        ("qkv_bias_std", ctypes.c_float)]


_lib = None


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(SYNTH_PATH):
            from . import build
            build.build_synth()
        L = ctypes.CDLL(SYNTH_PATH)
        L.rfs_llama_gguf_size.restype = ctypes.c_uint64
        L.rfs_llama_gguf_size.argtypes = [ctypes.POINTER(_Spec)]
        L.rfs_llama_gguf_write.restype = ctypes.c_int
        L.rfs_llama_gguf_write.argtypes = [ctypes.POINTER(_Spec), ctypes.c_void_p, ctypes.c_uint64, ctypes.c_int]
        L.rfs_fill_normal.restype = None
        L.rfs_fill_normal.argtypes = [ctypes.c_uint64, ctypes.c_uint64, ctypes.c_float, ctypes.c_uint64,
                                      ctypes.c_void_p, ctypes.c_size_t]
        L.rfs_row_bytes.restype = ctypes.c_size_t
        L.rfs_row_bytes.argtypes = [ctypes.c_int, ctypes.c_size_t]
        L.rfs_quantize.restype = ctypes.c_int
        L.rfs_quantize.argtypes = [ctypes.c_int, ctypes.c_void_p, ctypes.c_size_t, ctypes.c_size_t, ctypes.c_void_p,
                                   ctypes.c_int]
        _lib = L
    return _lib


@dataclass(frozen=True)
class LlamaSpec:
    name: str
    vocab_size: int
    n_embd: int
    n_layers: int
    n_ff: int
    n_heads: int
    n_kv_heads: int
    rope_theta: float = 10000.0
    rms_eps: float = 1e-5
    context_length: int = 4096
    layer_type: int = Q8_0
    embd_type: int = Q8_0
    out_type: int = Q8_0  # -1: tied to token_embd
    seed: int = 0
    weight_std: float = 0.02
    arch: str = "llama"
    v_type: int = -1        # attn_v type; -1: layer_type (Q4_K_M-style mixes use Q6_K)
    down_type: int = -1     # ffn_down type; -1: layer_type
    qkv_bias_std: float = 0.0  # > 0: qwen2 Q/K/V biases of N(0, qkv_bias_std)

    @property
    def head_dim(self) -> int:
        return self.n_embd // self.n_heads


# TinyLlama-1.1B shape, Q8_0 everywhere, seed 0.  The reference derives
# head_dim = n_embd / n_heads = 64 (runtime/src/model.rs:148), so a head_dim of
# 128 at this width cannot run on its CPU executor; 64 is used.
TINYLLAMA = LlamaSpec("tinyllama-1.1b-q8_0", vocab_size=32000, n_embd=2048, n_layers=22, n_ff=5632, n_heads=32,
                      n_kv_heads=4, rope_theta=10000.0, context_length=2048, layer_type=Q8_0, embd_type=Q8_0,
                      out_type=Q8_0, seed=0)
# Llama-3-8B shape, Q4_K layers, Q8_0 embedding/output, seed 3.
LLAMA3_8B = LlamaSpec("llama-3-8b-q4_k", vocab_size=128256, n_embd=4096, n_layers=32, n_ff=14336, n_heads=32,
                      n_kv_heads=8, rope_theta=500000.0, context_length=8192, layer_type=Q4_K, embd_type=Q8_0,
                      out_type=Q8_0, seed=3)
# Llama-3-70B shape, Q4_K everywhere, seed 4 (out-of-core workload).
LLAMA3_70B = LlamaSpec("llama-3-70b-q4_k", vocab_size=128256, n_embd=8192, n_layers=80, n_ff=28672, n_heads=64,
                       n_kv_heads=8, rope_theta=500000.0, context_length=8192, layer_type=Q4_K, embd_type=Q4_K,
                       out_type=Q4_K, seed=4)

CONFIGS = {s.name: s for s in (TINYLLAMA, LLAMA3_8B, LLAMA3_70B)}


def scaled(spec: LlamaSpec, **kw) -> LlamaSpec:
    """Same architecture family with some dimensions changed (test-size models)."""
    return replace(spec, **kw)


def gguf_bytes(spec: LlamaSpec, threads: int | None = None) -> np.ndarray:
    """Generate the GGUF image of `spec` in memory (uint8 array)."""
    s = _Spec(spec.arch.encode(), spec.vocab_size, spec.context_length, spec.n_embd, spec.n_layers, spec.n_ff,
              spec.n_heads, spec.n_kv_heads, spec.rms_eps, spec.rope_theta, spec.layer_type, spec.embd_type,
              spec.out_type, spec.seed, spec.weight_std, spec.v_type, spec.down_type, spec.qkv_bias_std)
    n = lib().rfs_llama_gguf_size(ctypes.byref(s))
    if n == 0:
        raise ValueError(f"invalid synthetic spec {spec}")
    buf = np.empty(n, np.uint8)
    t = threads or min(64, os.cpu_count() or 8)
    rc = lib().rfs_llama_gguf_write(ctypes.byref(s), buf.ctypes.data, n, t)
    if rc != 0:
        raise RuntimeError(f"rfs_llama_gguf_write failed ({rc})")
    return buf


def normal(seed: int, stream: int, n: int, std: float = 1.0, start: int = 0) -> np.ndarray:
    out = np.empty(n, np.float32)
    lib().rfs_fill_normal(seed, stream, std, start, out.ctypes.data, n)
    return out


def quantize(gtype: int, x: np.ndarray, threads: int | None = None) -> np.ndarray:
    """Quantise a 2-D f32 array [rows, cols] into GGUF block bytes."""
    x = np.ascontiguousarray(x, np.float32)
    if x.ndim == 1:
        x = x[None, :]
    rows, cols = x.shape
    rb = lib().rfs_row_bytes(gtype, cols)
    if rb == 0:
        raise ValueError(f"{cols} columns do not fit type {gtype}")
    out = np.empty(rows * rb, np.uint8)
    rc = lib().rfs_quantize(gtype, x.ctypes.data, rows, cols, out.ctypes.data, threads or min(32, os.cpu_count() or 4))
    if rc != 0:
        raise RuntimeError("quantize failed")
    return out


def row_bytes(gtype: int, n: int) -> int:
    return lib().rfs_row_bytes(gtype, n)


# Block layouts of the formats without an encoder here: (elements, bytes, offsets of
# the f16 super-scales that must be finite).
_RANDOM_BLOCKS = {Q5_0: (32, 22, (0,)), Q2_K: (256, 84, (80, 82)), Q3_K: (256, 110, (108,)),
                  Q5_K: (256, 176, (0, 2)), Q8_K: (256, 292, ())}


def random_blocks(gtype: int, rows: int, k: int, seed: int) -> np.ndarray:
    """rows x k weights of ggml type gtype (Q5_0, Q2_K, Q3_K, Q5_K, Q8_K) as GGUF blocks of
    random quant and scale bytes, with normal f16 super-scales in [2^-12, 2^-10)
    (Q8_K: an f32 d in [1e-3, 3e-3)).  Every byte pattern of the other fields is a
    valid block, so these are well-formed weights of the format's full value range."""
    qk, bs, dpos = _RANDOM_BLOCKS[gtype]
    rng = np.random.default_rng(seed)
    nb = rows * k // qk
    b = rng.integers(0, 256, (nb, bs), dtype=np.uint8)
    for o in dpos:
        b[:, o:o + 2] = rng.integers(0x0C00, 0x1400, nb).astype("<u2").view(np.uint8).reshape(nb, 2)
    if gtype == Q8_K:
        b[:, 0:4] = rng.uniform(1e-3, 3e-3, nb).astype("<f4").view(np.uint8).reshape(nb, 4)
    return b.reshape(-1)
