"""ctypes bindings of librfcuda.so (include/rfcuda.h).

The library is loaded from this package directory only; a missing or stale
build raises ImportError instead of falling back to anything else.
"""
from __future__ import annotations

import ctypes
import os

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "librfcuda.so")

RF_OK = 0
RF_EINVAL, RF_ENOMEM, RF_ECUDA, RF_EFORMAT, RF_ESTATE, RF_EUNSUPPORTED, RF_ENCCL, RF_ETIMEOUT = range(-1, -9, -1)
ERROR_NAMES = {
    -1: "RF_EINVAL", -2: "RF_ENOMEM", -3: "RF_ECUDA", -4: "RF_EFORMAT", -5: "RF_ESTATE",
    -6: "RF_EUNSUPPORTED", -7: "RF_ENCCL", -8: "RF_ETIMEOUT",
}

TYPE_F32, TYPE_F16, TYPE_Q4_0, TYPE_Q8_0, TYPE_Q4_K, TYPE_Q5_K, TYPE_Q6_K = 0, 1, 2, 8, 12, 13, 14
TYPE_Q2_K, TYPE_Q3_K = 10, 11
TYPE_Q5_0, TYPE_Q8_K = 6, 15  # stored as f32
ROLE_NAMES = ["attn_norm", "attn_q", "attn_k", "attn_v", "attn_output", "ffn_norm", "ffn_gate", "ffn_up", "ffn_down"]
# rf_layer_load roles 0-11: the nine weights, then the optional qwen2 Q/K/V biases
LAYER_VIEW_NAMES = ROLE_NAMES + ["attn_q.bias", "attn_k.bias", "attn_v.bias"]
ROLE_TOKEN_EMBD, ROLE_OUTPUT_NORM, ROLE_OUTPUT = 16, 17, 18

# Every symbol include/rfcuda.h declares (checked by tests/test_synth_and_abi.py).
EXPORTS = [
    "rf_last_error", "rf_abi_version", "rf_gguf_read_config", "rf_tp_shard_plan", "rf_engine_create", "rf_engine_create_from_gguf",
    "rf_engine_create_from_file", "rf_engine_destroy", "rf_engine_config", "rf_persistent_load",
    "rf_layer_load", "rf_layer_load_gguf", "rf_layer_release", "rf_layer_is_resident", "rf_layer_compute",
    "rf_embed", "rf_hidden_write", "rf_hidden_read", "rf_kv_commit", "rf_forward_token", "rf_prefill",
    "rf_compute_logits",
    "rf_decode_step", "rf_generate", "rf_kv_reset", "rf_kv_seq_len", "rf_kv_read", "rf_budget_total",
    "rf_budget_used", "rf_budget_available", "rf_set_residency_plan", "rf_residency_stats_get",
    "rf_step_kernel_count", "rf_selftest_wait", "rf_decode_timed",
    "rf_bench_layer_kernels", "rf_tp_unique_id", "rf_tp_peer_sum", "rf_matrix_create", "rf_matrix_destroy", "rf_matrix_device_bytes",
    "rf_qmatvec", "rf_qgemm", "rf_qgemm_error_word", "rf_decode_attention", "rf_decode_attention_noalloc",
    "rf_should_keep_resident", "rf_layer_read_plan", "rf_plan_residency", "rf_set_layer_cache",
]


class RfError(RuntimeError):
    def __init__(self, code: int, msg: str):
        super().__init__(f"{ERROR_NAMES.get(code, code)}: {msg}")
        self.code = code


class ModelConfig(ctypes.Structure):
    _fields_ = [(n, ctypes.c_uint32) for n in (
        "vocab_size", "context_length", "n_embd", "n_layers", "n_ff", "n_heads", "n_kv_heads", "head_dim")] + [
        ("rms_eps", ctypes.c_float), ("rope_theta", ctypes.c_float)]

    def as_dict(self):
        return {f: getattr(self, f) for f, _ in self._fields_}


class RuntimeConfig(ctypes.Structure):
    _fields_ = [("device", ctypes.c_int), ("tp_rank", ctypes.c_int), ("tp_size", ctypes.c_int),
                ("nccl_id", ctypes.c_void_p), ("max_seq_len", ctypes.c_uint32),
                ("vram_budget_bytes", ctypes.c_uint64), ("ring_slots", ctypes.c_int), ("kv_f32", ctypes.c_int),
                ("disable_graphs", ctypes.c_int)]


class TensorView(ctypes.Structure):
    _fields_ = [("role", ctypes.c_int), ("ggml_type", ctypes.c_int), ("ne0", ctypes.c_uint64),
                ("ne1", ctypes.c_uint64), ("host", ctypes.c_void_p), ("bytes", ctypes.c_uint64)]


class TpShard(ctypes.Structure):
    _fields_ = [(n, ctypes.c_uint32) for n in ("q_heads", "q_head_offset", "kv_heads", "kv_head_offset", "ff_rows",
                                               "ff_offset", "vocab_rows", "vocab_offset")]


class TensorExtent(ctypes.Structure):
    _fields_ = [("file_offset", ctypes.c_uint64), ("byte_length", ctypes.c_uint64)]


class ReadRange(ctypes.Structure):
    _fields_ = [("file_offset", ctypes.c_uint64), ("byte_length", ctypes.c_uint64), ("logical_bytes", ctypes.c_uint64),
                ("gap_bytes", ctypes.c_uint64), ("first", ctypes.c_uint32), ("count", ctypes.c_uint32)]


class PlannedTensor(ctypes.Structure):
    _fields_ = [("index", ctypes.c_uint32), ("range", ctypes.c_uint32), ("offset_in_range", ctypes.c_uint64)]


class ReadPlanTotals(ctypes.Structure):
    _fields_ = [(n, ctypes.c_uint64) for n in ("logical_tensor_count", "logical_bytes", "physical_bytes", "gap_bytes",
                                               "reusable_group_buffer_bytes")]


class ResidencyStats(ctypes.Structure):
    _fields_ = [(n, ctypes.c_uint64) for n in ("layer_loads", "layer_releases", "cache_hits", "cache_misses",
                                               "evictions", "peak_bytes", "h2d_bytes", "ring_copies",
                                               "host_image_bytes", "file_reads", "file_read_bytes",
                                               "file_gap_bytes", "host_mapped_bytes")]


_lib = None


def lib():
    """Load librfcuda.so; raises ImportError when the native build is missing."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise ImportError(f"{LIB_PATH} is not built; run `python -m ramforge_b200.build`")
        L = ctypes.CDLL(LIB_PATH)
        c_int, c_u32, c_u64, vp = ctypes.c_int, ctypes.c_uint32, ctypes.c_uint64, ctypes.c_void_p
        f32p, u32p, u64p = ctypes.POINTER(ctypes.c_float), ctypes.POINTER(c_u32), ctypes.POINTER(c_u64)
        sig = {
            "rf_last_error": (ctypes.c_char_p, []),
            "rf_abi_version": (c_int, []),
            "rf_gguf_read_config": (c_int, [vp, c_u64, ctypes.POINTER(ModelConfig)]),
            "rf_tp_shard_plan": (c_int, [ctypes.POINTER(ModelConfig), c_int, c_int, c_int, ctypes.POINTER(TpShard)]),
            "rf_engine_create": (c_int, [ctypes.POINTER(ModelConfig), ctypes.POINTER(RuntimeConfig), ctypes.POINTER(vp)]),
            "rf_engine_create_from_gguf": (c_int, [vp, c_u64, ctypes.POINTER(RuntimeConfig), ctypes.POINTER(vp)]),
            "rf_engine_create_from_file": (c_int, [ctypes.c_char_p, ctypes.POINTER(RuntimeConfig), ctypes.POINTER(vp)]),
            "rf_engine_destroy": (None, [vp]),
            "rf_engine_config": (c_int, [vp, ctypes.POINTER(ModelConfig)]),
            "rf_persistent_load": (c_int, [vp, ctypes.POINTER(TensorView)]),
            "rf_layer_load": (c_int, [vp, c_int, ctypes.POINTER(TensorView), c_int]),
            "rf_layer_load_gguf": (c_int, [vp, c_int]),
            "rf_layer_release": (c_int, [vp, c_int]),
            "rf_layer_is_resident": (c_int, [vp, c_int]),
            "rf_layer_compute": (c_int, [vp, c_int, c_u32]),
            "rf_embed": (c_int, [vp, c_u32]),
            "rf_hidden_write": (c_int, [vp, f32p, c_u32]),
            "rf_hidden_read": (c_int, [vp, f32p, c_u32]),
            "rf_kv_commit": (c_int, [vp]),
            "rf_forward_token": (c_int, [vp, c_u32, c_u32, f32p]),
            "rf_prefill": (c_int, [vp, u32p, c_u32]),
            "rf_compute_logits": (c_int, [vp, f32p, u32p]),
            "rf_decode_step": (c_int, [vp, c_u32, u32p]),
            "rf_generate": (c_int, [vp, u32p, c_u32, c_u32, u32p]),
            "rf_kv_reset": (c_int, [vp]),
            "rf_kv_seq_len": (c_int, [vp, u32p]),
            "rf_kv_read": (c_int, [vp, c_int, c_int, c_u32, c_u32, f32p]),
            "rf_budget_total": (c_int, [vp, u64p]),
            "rf_budget_used": (c_int, [vp, u64p]),
            "rf_budget_available": (c_int, [vp, u64p]),
            "rf_set_residency_plan": (c_int, [vp, ctypes.POINTER(ctypes.c_uint8), c_int, c_u64]),
            "rf_residency_stats_get": (c_int, [vp, ctypes.POINTER(ResidencyStats)]),
            "rf_tp_unique_id": (c_int, [ctypes.POINTER(ctypes.c_uint8)]),
            "rf_should_keep_resident": (c_int, [c_u64, c_u64]),
            "rf_plan_residency": (c_int, [vp, c_u64, c_int, ctypes.POINTER(ctypes.c_uint8)]),
            "rf_set_layer_cache": (c_int, [vp, c_u64]),
            "rf_layer_read_plan": (c_int, [ctypes.POINTER(TensorExtent), c_u32, ctypes.POINTER(ReadRange), c_u32, u32p,
                                           ctypes.POINTER(PlannedTensor), ctypes.POINTER(ReadPlanTotals)]),
            "rf_tp_peer_sum": (c_int, [vp, ctypes.POINTER(c_int)]),
            "rf_step_kernel_count": (c_int, [vp, u32p]),
            "rf_selftest_wait": (c_int, [c_int, u32p]),
            "rf_decode_timed": (c_int, [vp, c_u32, c_u32, u32p, f32p]),
            "rf_bench_layer_kernels": (c_int, [vp, c_u32, f32p]),
            "rf_matrix_create": (c_int, [c_int, vp, c_u64, c_int, c_u32, c_u32, ctypes.POINTER(vp)]),
            "rf_matrix_destroy": (None, [vp]),
            "rf_matrix_device_bytes": (c_u64, [vp]),
            "rf_qmatvec": (c_int, [vp, vp, vp, c_int, vp]),
            "rf_qgemm": (c_int, [vp, vp, vp, c_int, vp]),
            "rf_qgemm_error_word": (c_int, [u32p]),
            "rf_decode_attention": (c_int, [vp, vp, vp, c_int, c_int, c_int, c_int, c_int, vp, vp]),
            "rf_decode_attention_noalloc": (c_int, [vp, vp, vp, c_int, c_int, c_int, c_int, c_int, vp, vp]),
        }
        for name, (res, args) in sig.items():
            fn = getattr(L, name)
            fn.restype = res
            fn.argtypes = args
        _lib = L
    return _lib


def check(rc: int) -> None:
    if rc != RF_OK:
        raise RfError(rc, lib().rf_last_error().decode(errors="replace"))
