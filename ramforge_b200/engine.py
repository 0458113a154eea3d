"""Host-side mirror of RAMforge's legacy executor API over librfcuda.so.

The names follow the reference (crates/ramforge-runtime/src/streaming_model.rs,
inference.rs, kv_cache.rs, memory.rs) so that parity tests read like its own:
`load_layer` / `release_layer` / `forward_single_streaming` /
`compute_logits` / `generate`, a KV cache with `seq_len`, `append`-free
deferred commits and `get_k_range`, and a byte budget.  Every call goes through
the C ABI in include/rfcuda.h; there is no CPU fallback.
"""
from __future__ import annotations

import ctypes
from typing import Iterable, Sequence

import numpy as np

from . import _lib
from ._lib import RfError, check, lib

_f32p = ctypes.POINTER(ctypes.c_float)
_u32p = ctypes.POINTER(ctypes.c_uint32)


def _fp(a: np.ndarray):
    return a.ctypes.data_as(_f32p)


def tp_unique_id() -> bytes:
    """128-byte NCCL id for rank 0 to distribute to the other ranks."""
    buf = (ctypes.c_uint8 * 128)()
    check(lib().rf_tp_unique_id(buf))
    return bytes(buf)


def should_keep_resident(resident_bytes: int, budget_total: int) -> bool:
    """should_keep_resident (persistent.rs:468): resident when at most a quarter of the budget."""
    return bool(lib().rf_should_keep_resident(resident_bytes, budget_total))


def layer_read_plan(extents):
    """build_layer_read_plan (layer_read.rs:50) over [(file_offset, byte_length), ...]:
    returns (ranges, placements, totals) as dicts; ranges hold file_offset,
    byte_length, logical_bytes, gap_bytes and the plan indices of their tensors."""
    from ._lib import PlannedTensor, ReadPlanTotals, ReadRange, TensorExtent
    n = len(extents)
    ext = (TensorExtent * max(1, n))(*[TensorExtent(o, b) for o, b in extents])
    cap = max(1, n)
    ranges = (ReadRange * cap)()
    placed = (PlannedTensor * cap)()
    tot = ReadPlanTotals()
    nr = ctypes.c_uint32()
    check(lib().rf_layer_read_plan(ext, n, ranges, cap, ctypes.byref(nr), placed, ctypes.byref(tot)))
    rs = [{"file_offset": r.file_offset, "byte_length": r.byte_length, "logical_bytes": r.logical_bytes,
           "gap_bytes": r.gap_bytes, "tensors": [placed[r.first + i].index for i in range(r.count)]}
          for r in ranges[:nr.value]]
    pl = [{"index": p.index, "range": p.range, "offset_in_range": p.offset_in_range} for p in placed[:n]]
    totals = {f: getattr(tot, f) for f, _ in tot._fields_}
    return rs, pl, totals


class DecodeEngine:
    """One GPU (one tensor-parallel rank) running the legacy decoder.

    gguf: a GGUF image (bytes / uint8 array, kept alive by the engine) or a path.
    """

    def __init__(self, gguf, device: int = 0, max_seq_len: int = 0, kv_f32: bool = False, tp_rank: int = 0,
                 tp_size: int = 1, nccl_id: bytes | None = None, ring_slots: int = 0, vram_budget_bytes: int = 0,
                 disable_graphs: bool = False):
        self._h = ctypes.c_void_p()
        self._id_buf = None
        rt = _lib.RuntimeConfig()
        rt.device = device
        rt.tp_rank = tp_rank
        rt.tp_size = tp_size
        if nccl_id is not None:
            self._id_buf = (ctypes.c_uint8 * 128).from_buffer_copy(nccl_id)
            rt.nccl_id = ctypes.cast(self._id_buf, ctypes.c_void_p)
        rt.max_seq_len = max_seq_len
        rt.vram_budget_bytes = vram_budget_bytes
        rt.ring_slots = ring_slots
        rt.kv_f32 = int(kv_f32)
        rt.disable_graphs = int(disable_graphs)
        self.tp_size = max(1, tp_size)
        self.tp_rank = tp_rank
        if isinstance(gguf, (str, bytes)) and not isinstance(gguf, bytes):
            self._src = None
            check(lib().rf_engine_create_from_file(gguf.encode(), ctypes.byref(rt), ctypes.byref(self._h)))
        else:
            src = np.frombuffer(gguf, np.uint8) if isinstance(gguf, (bytes, bytearray, memoryview)) else gguf
            self._src = np.ascontiguousarray(src, np.uint8)
            check(lib().rf_engine_create_from_gguf(self._src.ctypes.data, self._src.size, ctypes.byref(rt),
                                                   ctypes.byref(self._h)))
        c = _lib.ModelConfig()
        check(lib().rf_engine_config(self._h, ctypes.byref(c)))
        self.config = c.as_dict()

    # ---- lifecycle ---------------------------------------------------------
    def close(self):
        if self._h:
            lib().rf_engine_destroy(self._h)
            self._h = ctypes.c_void_p()

    def __enter__(self):
        return self

    def __exit__(self, *a):
        self.close()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    # ---- layers (load_layer / release_layer / execute_layer) -----------------
    def load_layer(self, layer: int):
        check(lib().rf_layer_load_gguf(self._h, layer))

    def load_layer_views(self, layer: int, tensors: dict):
        """rf_layer_load with host tensors: {role_name: (ggml_type, ne0, ne1, uint8 array)}; role names
        are the nine weights ("attn_q", ...) and the optional biases ("attn_q.bias", ...)."""
        views = (_lib.TensorView * len(tensors))()
        keep = []
        for i, (name, (gtype, ne0, ne1, data)) in enumerate(tensors.items()):
            arr = np.ascontiguousarray(data, np.uint8)
            keep.append(arr)
            views[i] = _lib.TensorView(_lib.LAYER_VIEW_NAMES.index(name), gtype, ne0, ne1, arr.ctypes.data, arr.size)
        check(lib().rf_layer_load(self._h, layer, views, len(tensors)))

    def release_layer(self, layer: int):
        check(lib().rf_layer_release(self._h, layer))

    def layer_is_resident(self, layer: int) -> bool:
        return bool(lib().rf_layer_is_resident(self._h, layer))

    def execute_layer(self, layer: int, pos: int):
        check(lib().rf_layer_compute(self._h, layer, pos))

    def embed(self, token: int):
        check(lib().rf_embed(self._h, token))

    def hidden(self) -> np.ndarray:
        out = np.empty(self.config["n_embd"], np.float32)
        check(lib().rf_hidden_read(self._h, _fp(out), out.size))
        return out

    def set_hidden(self, x: np.ndarray):
        x = np.ascontiguousarray(x, np.float32)
        check(lib().rf_hidden_write(self._h, _fp(x), x.size))

    def kv_commit(self):
        check(lib().rf_kv_commit(self._h))

    # ---- token forward / logits / generation -----------------------------------
    def forward_single_streaming(self, token: int, pos: int, want_hidden: bool = True) -> np.ndarray | None:
        out = np.empty(self.config["n_embd"], np.float32) if want_hidden else None
        check(lib().rf_forward_token(self._h, token, pos, _fp(out) if want_hidden else None))
        return out

    def compute_logits(self, want_logits: bool = True):
        logits = np.empty(self.config["vocab_size"], np.float32) if want_logits else None
        am = ctypes.c_uint32()
        check(lib().rf_compute_logits(self._h, _fp(logits) if want_logits else None, ctypes.byref(am)))
        return logits, am.value

    def decode_step(self, token: int) -> int:
        nxt = ctypes.c_uint32()
        check(lib().rf_decode_step(self._h, token, ctypes.byref(nxt)))
        return nxt.value

    def prefill(self, tokens: Sequence[int]):
        """The prompt tokens at positions [kv_seq_len, kv_seq_len + n) as batched
        tensor-core passes (rf_prefill); afterwards compute_logits() gives the last
        token's logits, as after forward_single_streaming of each token in turn."""
        t = np.ascontiguousarray(tokens, np.uint32)
        check(lib().rf_prefill(self._h, t.ctypes.data_as(_u32p), t.size))

    def generate(self, prompt: Sequence[int], n_new: int, batched_prefill: bool = False) -> np.ndarray:
        """Greedy generation (rf_generate).  With batched_prefill, every prompt token
        but the last goes through rf_prefill first, then the last one starts the
        decode loop."""
        p = np.ascontiguousarray(prompt, np.uint32)
        if batched_prefill and p.size > 1:
            self.prefill(p[:-1])
            p = p[-1:]
        out = np.zeros(max(1, n_new), np.uint32)
        check(lib().rf_generate(self._h, p.ctypes.data_as(_u32p), p.size, n_new, out.ctypes.data_as(_u32p)))
        return out[:n_new]

    # ---- measurement hooks ------------------------------------------------------------
    @property
    def step_kernel_count(self) -> int:
        v = ctypes.c_uint32()
        check(lib().rf_step_kernel_count(self._h, ctypes.byref(v)))
        return v.value

    @property
    def tp_peer_sum(self) -> bool:
        """True when tensor-parallel sums run over NVLink peer memory (else NCCL)."""
        v = ctypes.c_int()
        check(lib().rf_tp_peer_sum(self._h, ctypes.byref(v)))
        return bool(v.value)

    def decode_timed(self, token: int, n_steps: int):
        """n greedy decode steps timed on the device; returns (tokens, device_ms)."""
        out = np.zeros(max(1, n_steps), np.uint32)
        ms = ctypes.c_float()
        check(lib().rf_decode_timed(self._h, token, n_steps, out.ctypes.data_as(_u32p), ctypes.byref(ms)))
        return out[:n_steps], ms.value

    def bench_layer_kernels(self, iters: int = 3) -> list:
        """Average ms per launch of [qkv_rope, attention, wo_residual, gateup_swiglu, down_residual]."""
        out = np.zeros(5, np.float32)
        check(lib().rf_bench_layer_kernels(self._h, iters, _fp(out)))
        return out.tolist()

    # ---- KV cache ------------------------------------------------------------------
    @property
    def kv_seq_len(self) -> int:
        v = ctypes.c_uint32()
        check(lib().rf_kv_seq_len(self._h, ctypes.byref(v)))
        return v.value

    def kv_reset(self):
        check(lib().rf_kv_reset(self._h))

    def kv_read(self, layer: int, which_v: bool, start: int, end: int) -> np.ndarray:
        kvd = self.config["n_kv_heads"] // self.tp_size * self.config["head_dim"]
        out = np.empty((max(0, end - start), kvd), np.float32)
        check(lib().rf_kv_read(self._h, layer, int(which_v), start, end, _fp(out)))
        return out

    # ---- budget / residency -------------------------------------------------------------
    def _u64(self, fn) -> int:
        v = ctypes.c_uint64()
        check(fn(self._h, ctypes.byref(v)))
        return v.value

    @property
    def budget_total(self) -> int:
        return self._u64(lib().rf_budget_total)

    @property
    def budget_used(self) -> int:
        return self._u64(lib().rf_budget_used)

    @property
    def budget_available(self) -> int:
        return self._u64(lib().rf_budget_available)

    def set_residency_plan(self, resident: Iterable[bool], ring_slots: int = 0, vram_weight_budget_bytes: int = 0):
        mask = np.ascontiguousarray([1 if r else 0 for r in resident], np.uint8)
        check(lib().rf_set_residency_plan(self._h, mask.ctypes.data_as(ctypes.POINTER(ctypes.c_uint8)), ring_slots,
                                          vram_weight_budget_bytes))

    def plan_residency(self, vram_weight_budget_bytes: int, ring_slots: int = 0) -> list:
        """rf_plan_residency: resident layers chosen for the weight budget; returns the mask."""
        mask = (ctypes.c_uint8 * self.config["n_layers"])()
        check(lib().rf_plan_residency(self._h, vram_weight_budget_bytes, ring_slots, mask))
        return [bool(m) for m in mask]

    def set_layer_cache(self, capacity_bytes: int):
        """rf_set_layer_cache: LRU byte capacity for streamed layers kept after their step."""
        check(lib().rf_set_layer_cache(self._h, capacity_bytes))

    def residency_stats(self) -> dict:
        s = _lib.ResidencyStats()
        check(lib().rf_residency_stats_get(self._h, ctypes.byref(s)))
        return {f: getattr(s, f) for f, _ in s._fields_}


class QMatrix:
    """A packed GGUF matrix on the current device (rf_matrix_create)."""

    def __init__(self, gtype: int, gguf_bytes, n_out: int, n_in: int, on_device_ptr: int | None = None,
                 nbytes: int | None = None):
        self._h = ctypes.c_void_p()
        if on_device_ptr is not None:
            check(lib().rf_matrix_create(gtype, on_device_ptr, nbytes, 1, n_out, n_in, ctypes.byref(self._h)))
        else:
            b = np.ascontiguousarray(gguf_bytes, np.uint8)
            check(lib().rf_matrix_create(gtype, b.ctypes.data, b.size, 0, n_out, n_in, ctypes.byref(self._h)))
        self.gtype, self.n_out, self.n_in = gtype, n_out, n_in

    @property
    def device_bytes(self) -> int:
        return lib().rf_matrix_device_bytes(self._h)

    def matvec(self, x_ptr: int, y_ptr: int, batch: int = 1, stream: int = 0):
        """y[b] = W x[b] on device pointers (e.g. torch tensor .data_ptr())."""
        check(lib().rf_qmatvec(self._h, x_ptr, y_ptr, batch, stream))

    def gemm(self, x_ptr: int, y_ptr: int, n_tokens: int, stream: int = 0):
        """Y[t] = W X[t] for n_tokens rows on the tensor cores (rf_qgemm); device pointers."""
        check(lib().rf_qgemm(self._h, x_ptr, y_ptr, n_tokens, stream))

    def close(self):
        if self._h:
            lib().rf_matrix_destroy(self._h)
            self._h = ctypes.c_void_p()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


def selftest_wait(device: int = 0) -> int:
    """Runs one peer sum whose second rank never arrives (rf_selftest_wait);
    returns its error word (1: the bounded wait gave up, as it must)."""
    w = ctypes.c_uint32()
    check(lib().rf_selftest_wait(device, ctypes.byref(w)))
    return w.value


def decode_attention(q_ptr: int, k_ptr: int, v_ptr: int, ctx: int, n_heads: int, n_kv_heads: int, head_dim: int,
                     batch: int, out_ptr: int, stream: int = 0):
    """GQA decode attention on device pointers (rf_decode_attention)."""
    check(lib().rf_decode_attention(q_ptr, k_ptr, v_ptr, ctx, n_heads, n_kv_heads, head_dim, batch, out_ptr, stream))


__all__ = ["DecodeEngine", "QMatrix", "decode_attention", "selftest_wait", "tp_unique_id", "RfError"]
