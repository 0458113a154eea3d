"""ramforge_b200 - a B200 (sm_100a) decode engine for RAMforge's legacy executor.

The compute path is librfcuda.so (hand-written CUDA kernels + a C ABI,
include/rfcuda.h); this package holds its Python host mirror (engine.py),
ctypes bindings (_lib.py), the synthetic model generator (synth.py) and the
build script (build.py).
"""
from .engine import DecodeEngine, QMatrix, RfError, decode_attention, selftest_wait, tp_unique_id  # noqa: F401

__all__ = ["DecodeEngine", "QMatrix", "RfError", "decode_attention", "selftest_wait", "tp_unique_id"]
