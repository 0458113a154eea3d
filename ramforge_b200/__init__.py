"""ramforge_b200 - a B200 (sm_100a) decode engine for RAMforge's legacy executor.

The compute path is librfcuda.so (hand-written CUDA kernels + a C ABI,
include/rfcuda.h); this package holds its Python host mirror (engine.py),
ctypes bindings (_lib.py), the synthetic model generator (synth.py) and the
build script (build.py).
"""
from .engine import (DecodeEngine, QMatrix, RfError, decode_attention, layer_read_plan,  # noqa: F401
                     selftest_wait, should_keep_resident, tp_unique_id)

__all__ = ["DecodeEngine", "QMatrix", "RfError", "decode_attention", "layer_read_plan", "selftest_wait",
           "should_keep_resident", "tp_unique_id"]
