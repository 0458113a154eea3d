#!/usr/bin/env python3
"""Decode benchmark: batch-1 greedy decode tokens/s of the Llama-3-8B-shaped
Q4_K model (32 layers, dim 4096, 32/8 heads, FFN 14336, vocab 128256, Q8_0
embedding/output) on 1..8 B200s (tensor parallel).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

A step is one greedy decode token (embedding, 32 layers, output norm, LM head,
argmax, token advance) at context 512 + W + i.  The model is synthetic
(seeded N(0, 0.02) weights quantised to Q4_K, Q8_0 embedding/output; there is
no checkpoint or dataset on this path).  Every step reads the whole 4.5 GB of
weights, far larger than the 126 MB L2, so no flush is needed between steps.

Prints one JSON line on rank 0.  `value` is device-timed (CUDA events on the
engine stream, max over ranks); `e2e` goes through the public C ABI call
rf_decode_step with the token in pinned host memory every step; `roofline` is
the dominant kernel (the fused gate/up + SwiGLU Q4_K GEMV) timed with events
over every layer in turn; `cpu_baseline` is the reference's CPU path (the
oracle port, reference threading) on a bounded sample.
"""
from __future__ import annotations

import argparse
import json
import os
import sys
import threading
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

METRIC = "batch-1 decode tokens/s (Llama-3-8B Q4_K)"
UNIT = "tokens/s"
PROMPT_LEN = 512


def dist_env():
    ws = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", str(rank)))
    return ws, rank, local


def measured_peaks():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            p = json.load(f)
        return float(p["hbm_gbs"]), "measured"
    except Exception:
        return 6650.0, "fallback"


class ClockSampler:
    """SM clocks, power and clock-event (throttle) reasons of this rank's GPU,
    read through NVML every 5 ms by a thread while the timed region runs (the
    same fields as nvidia-smi's clocks.sm / clocks_event_reasons.*)."""

    REASONS = (("hw_slowdown", 0x8), ("hw_thermal_slowdown", 0x40), ("sw_thermal_slowdown", 0x20),
               ("sw_power_cap", 0x4))

    def __init__(self, device_index: int, period_s: float = 0.005):
        self.dev = device_index
        self.period = period_s
        self.rows = []
        self.err = None
        self.nvml = None
        self.handle = None
        self.thread = None
        self.stop = None

    def _handle(self):
        import pynvml
        import torch
        pynvml.nvmlInit()
        self.nvml = pynvml
        p = torch.cuda.get_device_properties(self.dev)
        bus = f"{p.pci_domain_id:08x}:{p.pci_bus_id:02x}:{p.pci_device_id:02x}.0"
        try:
            return pynvml.nvmlDeviceGetHandleByPciBusId(bus)
        except Exception:
            return pynvml.nvmlDeviceGetHandleByIndex(self.dev)

    def _sample(self):
        n = self.nvml
        sm = n.nvmlDeviceGetClockInfo(self.handle, n.NVML_CLOCK_SM)
        mask = n.nvmlDeviceGetCurrentClocksEventReasons(self.handle)
        watts = n.nvmlDeviceGetPowerUsage(self.handle) / 1e3
        self.rows.append((sm, mask, watts))

    def _loop(self):
        while not self.stop.is_set():
            try:
                self._sample()
            except Exception as e:  # keep what was read; report the failure
                self.err = str(e)
                return
            self.stop.wait(self.period)

    def __enter__(self):
        try:
            self.handle = self._handle()
            self.max_mhz = self.nvml.nvmlDeviceGetMaxClockInfo(self.handle, self.nvml.NVML_CLOCK_SM)
        except Exception as e:
            self.err = f"nvml: {e}"
            return self
        self.stop = threading.Event()
        self.thread = threading.Thread(target=self._loop, daemon=True)
        self.thread.start()
        return self

    def __exit__(self, *a):
        if self.thread:
            self.stop.set()
            self.thread.join(timeout=5)
        if self.nvml and self.handle is not None:
            try:
                self._sample()  # one more at the end of the timed region
            except Exception:
                pass

    def summary(self):
        if not self.rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": [self.err or "no samples"]}
        sm = [r[0] for r in self.rows]
        reasons = sorted({name for _, mask, _ in self.rows for name, bit in self.REASONS if mask & bit})
        return {"sm_mhz": float(np.median(sm)), "sm_max_mhz": float(self.max_mhz), "reasons": reasons,
                "samples": len(self.rows), "power_w_median": float(np.median([r[2] for r in self.rows])),
                "source": "nvml, 5 ms period, during the timed region"}


# DRAM bytes of one gate/up launch at TP1, from an ncu capture (dram__bytes_read.sum
# 66,170,624 + dram__bytes_write.sum 577,024) of
#   ncu --set full --clock-control none -k regex:EpiSwiGLU ... python bench.py --profile --layers 2
# A rank of a TP-N run holds 1/N of the rows, so its launch moves 1/N of it.
GATEUP_DRAM_BYTES_NCU = 66_747_648


def algorithmic_bytes(spec, tp: int, ctx: float):
    """Weight + activation bytes one decode token must move (per rank): matrices
    M*K*b (b = GGUF bytes/element), KV f16 at context ctx, vectors 4 bytes/elem."""
    from ramforge_b200 import synth
    bpe = {synth.Q4_K: 144 / 256, synth.Q8_0: 34 / 32, synth.Q4_0: 18 / 32}
    d, ff, hd = spec.n_embd, spec.n_ff, spec.head_dim
    q, kv = spec.n_heads * hd, spec.n_kv_heads * hd
    b = bpe[spec.layer_type]
    layer_w = (d * (q + 2 * kv) + q * d + 2 * d * ff + ff * d) * b / tp
    lm = spec.vocab_size * d * bpe[spec.out_type] / tp
    kv_bytes = spec.n_layers * 2 * (kv / tp) * 2 * ctx
    gateup = 2 * (ff / tp) * d * b + 4 * d + 4 * ff / tp
    return spec.n_layers * layer_w + lm + kv_bytes, gateup


def make_model(spec, world, rank):
    """GGUF image of the benchmark model: in memory for 1 rank; shared through
    /dev/shm for several ranks (rank 0 writes, the others map it)."""
    from ramforge_b200 import synth
    if world == 1:
        return synth.gguf_bytes(spec)
    import torch.distributed as dist
    path = f"/dev/shm/ramforge_b200_{spec.name}_s{spec.seed}.gguf"
    if rank == 0 and not os.path.exists(path):
        g = synth.gguf_bytes(spec)
        tmp = path + f".tmp{os.getpid()}"
        g.tofile(tmp)
        os.replace(tmp, path)
    dist.barrier()
    return path


def cpu_baseline(gguf, spec, ctx: int, threads: int = 1):
    """Reference CPU path (oracle port): one full decode token (32 layers + LM head +
    argmax) at position `ctx`, the context the GPU arm decodes at, over a seeded
    synthetic KV history of that length.  threads=1 is the reference's own
    dispatch (Q4_K/Q8_0 matvecs single-threaded, compute_dispatch.rs:219-254);
    more threads split every matvec's rows over host cores (not the reference's
    dispatch for these formats; the rows' arithmetic is unchanged)."""
    from oracle import oracle as orc
    m = orc.OracleModel(gguf, kv_f16=True, max_seq=ctx + 2, threads=threads)
    m.kv_fill_synthetic(ctx)
    t0 = time.perf_counter()
    fh = m.forward(1, ctx)
    orc.argmax(m.logits(fh))
    dt = time.perf_counter() - t0
    m.close()
    what = ("the reference's threading (Q4_K/Q8_0 matvecs single-threaded)" if threads == 1 else
            f"every matvec's rows split over {threads} host threads (all cores, row-parallel; the reference "
            "itself runs Q4_K/Q8_0 single-threaded)")
    return {"value": 1.0 / dt, "unit": UNIT, "cores": threads, "kind": "port",
            "sample": f"1 greedy decode token of the same model (32 layers + LM head + argmax) at position {ctx} "
                      f"over a synthetic KV history, oracle port with {what}",
            "seconds": dt}


def host_cores() -> int:
    try:
        return len(os.sched_getaffinity(0))
    except Exception:
        return os.cpu_count() or 1


def run_reference(args, spec):
    """--impl reference: the reference's CPU implementation (oracle port, its own
    threading: Q4_K/Q8_0 matvecs single-threaded, compute_dispatch.rs:219-254) on
    this workload, at the contexts the GPU arm decodes at (step i attends over
    PROMPT_LEN + warmup + i positions of a seeded synthetic KV history).  A step is
    a bounded sample: one layer of a decode token (layer i mod 32, no commit) plus
    1/32 of the LM-head rows, so tokens/s = 1 / (32 * mean step time)."""
    from oracle import oracle as orc
    from ramforge_b200 import synth
    t_gen = time.perf_counter()
    g = synth.gguf_bytes(spec)
    gen_s = time.perf_counter() - t_gen
    ctx0 = PROMPT_LEN + args.warmup
    m = orc.OracleModel(g, kv_f16=True, max_seq=ctx0 + args.steps + 2, threads=1)
    m.kv_fill_synthetic(ctx0 + args.steps)
    L, V = spec.n_layers, spec.vocab_size
    hidden = np.asarray(synth.normal(9, 9, spec.n_embd), np.float32)

    def step(i, pos):
        layer = i % L
        m.layer_step(layer, pos, hidden)
        r0 = layer * V // L
        m.logits_rows(hidden, r0, (layer + 1) * V // L)

    for i in range(args.warmup):
        step(i, PROMPT_LEN + i)
    t0 = time.perf_counter()
    for i in range(args.steps):
        step(args.warmup + i, ctx0 + i)
    dt = time.perf_counter() - t0
    per_step = dt / args.steps
    value = 1.0 / (per_step * L)
    sample = (f"per step: one layer of a decode token (layer i mod 32) at context {ctx0}+i over a synthetic KV "
              "history + 1/32 of the LM-head rows; reference threading (Q4_K/Q8_0 single-threaded)")
    line = {
        "impl": "reference", "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": per_step * 1e3, "higher_is_better": True,
        "scaling": "strong", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": workload_config(spec, args, 1),
        "cpu_baseline": {"value": value, "unit": UNIT, "cores": 1, "kind": "port", "sample": sample,
                         "host_cores": host_cores()},
        "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        "model_generation_s": gen_s,
    }
    m.close()
    emit(line)


def run_profile(args, spec):
    """--profile: the same model shape (optionally fewer layers) run eagerly for a
    handful of launches, so an ncu capture of it stays small and ends by itself:
    4 prompt tokens, then 2 greedy decode steps (5 kernels per layer + 4)."""
    import torch
    from ramforge_b200 import DecodeEngine, synth
    if args.layers:
        spec = synth.scaled(spec, name=f"{spec.name}-{args.layers}l", n_layers=args.layers)
    torch.cuda.set_device(0)
    g = synth.gguf_bytes(spec)
    if args.prefill:  # one batched prefill (tensor-core GEMMs) after a warm-up one
        eng = DecodeEngine(g, device=0, max_seq_len=args.prefill + 8)
        prompt = np.random.default_rng(3).integers(0, spec.vocab_size, args.prefill).tolist()
        eng.prefill(prompt)
        eng.kv_reset()
        t0 = time.perf_counter()
        eng.prefill(prompt)
        emit({"profile_run": spec.name, "layers": spec.n_layers, "prefill_tokens": args.prefill,
              "ms": (time.perf_counter() - t0) * 1e3})
        eng.close()
        return
    eng = DecodeEngine(g, device=0, max_seq_len=64, disable_graphs=True)
    first = int(eng.generate([11, 22, 33, 44], 1)[0])
    toks, ms = eng.decode_timed(first, 2)
    torch.cuda.synchronize()
    emit({"profile_run": spec.name, "layers": spec.n_layers, "tokens": toks.tolist(), "ms": ms})
    eng.close()


def run_attn_profile(args):
    """--profile-attn CTX,BATCH: benchmark configuration 3's inputs at one shape,
    three rf_decode_attention calls (an ncu capture takes the last)."""
    import torch
    from ramforge_b200 import decode_attention
    ctx, batch = (int(v) for v in args.profile_attn.split(","))
    H, KV, hd = 32, 8, 128
    torch.cuda.set_device(0)
    g = torch.Generator(device="cuda").manual_seed(2)
    q = torch.randn(batch, H, hd, device="cuda", generator=g)
    k = torch.randn(batch, KV, ctx, hd, device="cuda", generator=g).half()
    v = torch.randn(batch, KV, ctx, hd, device="cuda", generator=g).half()
    o = torch.empty(batch, H, hd, device="cuda")
    for _ in range(3):
        decode_attention(q.data_ptr(), k.data_ptr(), v.data_ptr(), ctx, H, KV, hd, batch, o.data_ptr())
    torch.cuda.synchronize()
    emit({"profile_attn": {"ctx": ctx, "batch": batch}, "finite": bool(torch.isfinite(o).all().item())})


def pinned_h2d_gbs():
    """Pinned host-to-device copy rate of this box (1 GiB, 5 copies, CUDA events)."""
    import torch
    h = torch.empty(1 << 30, dtype=torch.uint8).pin_memory()
    d = torch.empty(1 << 30, dtype=torch.uint8, device="cuda")
    d.copy_(h, non_blocking=True)
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(5):
        d.copy_(h, non_blocking=True)
    e1.record()
    torch.cuda.synchronize()
    gbs = 5 * (1 << 30) / (e0.elapsed_time(e1) / 1e3) / 1e9
    del h, d
    return gbs


def out_of_core(eng, spec, first_token, steps):
    """The benchmark engine re-planned for a weight budget of three quarters of its
    layer images plus two ring slots (rf_plan_residency): the last quarter of the
    layers streams every step from pinned host images through the ring.  tokens/s against
    the bound the measured pinned host-to-device rate sets for the streamed bytes."""
    h2d = pinned_h2d_gbs()
    d, kv, ff = spec.n_embd, spec.n_kv_heads * spec.head_dim, spec.n_ff
    layer_est = ((d + 2 * kv) * d + d * d + 2 * ff * d + d * ff) * 144 // 256 + 8 * d  # Q4_K image, norms
    budget = int((spec.n_layers * 3 // 4 + 2) * layer_est * 1.001)
    mask = eng.plan_residency(budget, ring_slots=2)
    n = mask.count(False)
    eng.kv_reset()
    t0 = time.perf_counter()
    eng.generate([first_token], 1)  # builds the streamed layers' pinned images
    setup_s = time.perf_counter() - t0
    toks, dev_ms = eng.decode_timed(int(first_token), steps)
    st = eng.residency_stats()
    layer_bytes = st["host_image_bytes"] / max(1, n)
    value = steps / (dev_ms / 1e3)
    bound = h2d * 1e9 / (n * layer_bytes) if n else float("inf")
    return {"api": "rf_plan_residency + rf_decode_timed", "weight_budget_bytes": budget,
            "streamed_layers": n, "layers": spec.n_layers, "ring_slots": 2, "tokens_per_s": value,
            "steps": steps, "layer_image_bytes": layer_bytes, "h2d_gbs": h2d,
            "h2d_bound_tokens_per_s": bound, "frac_of_h2d_bound": value / bound, "setup_s": setup_s,
            "ring_copies": st["ring_copies"]}


def config5(steps):
    """Benchmark configuration 5: the 70B shape (dim 8192, 80 layers, 64/8 heads, FFN
    28672, vocab 128256, Q4_K layers and output, seed 4) under a 4 GiB per-GPU
    weight budget: rf_plan_residency keeps the layers that fit beside 2 ring slots
    and streams the rest from pinned host images every step.  Returns tokens/s
    against the bound of the pinned host-to-device rate measured here."""
    import torch
    from ramforge_b200 import DecodeEngine, synth
    spec = synth.scaled(synth.LLAMA3_8B, name="llama-70b-shape-q4k", n_embd=8192, n_layers=80, n_heads=64,
                        n_kv_heads=8, n_ff=28672, seed=4, out_type=synth.Q4_K, context_length=4096)
    h2d = pinned_h2d_gbs()
    t0 = time.perf_counter()
    g = synth.gguf_bytes(spec)
    gen_s = time.perf_counter() - t0
    t0 = time.perf_counter()
    eng = DecodeEngine(g, device=torch.cuda.current_device(), max_seq_len=64, ring_slots=2)
    mask = eng.plan_residency(4 << 30, ring_slots=2)
    load_s = time.perf_counter() - t0
    n = mask.count(False)
    t0 = time.perf_counter()
    first = int(eng.generate([11, 22], 1)[0])  # also packs every streamed layer into pinned memory once
    first_s = time.perf_counter() - t0
    toks, dev_ms = eng.decode_timed(first, steps)
    st = eng.residency_stats()
    eng.close()
    del g
    layer_bytes = st["host_image_bytes"] / max(1, n)
    value = steps / (dev_ms / 1e3)
    bound = h2d * 1e9 / (n * layer_bytes)
    return {"metric": "out-of-core decode tokens/s (70B shape Q4_K, 4 GiB weight budget)", "value": value,
            "unit": "tokens/s", "steps": steps, "api": "rf_plan_residency + rf_decode_timed",
            "workload": "70B-shape Q4_K greedy decode, 4 GiB of device weights, 2 ring slots",
            "resident_layers": spec.n_layers - n, "streamed_layers": n, "layer_image_bytes": layer_bytes,
            "roofline": {"bound": "h2d", "achieved": n * layer_bytes * value / 1e9, "peak": h2d, "unit": "GB/s",
                         "frac": value / bound, "peak_source": "pinned host-to-device copy measured in this run"},
            "tokens": toks.tolist(), "setup_s": {"generation": gen_s, "engine": load_s, "first_token": first_s},
            "ring_copies": st["ring_copies"]}


def run_config5(args):
    """--config5: configuration 5 alone, as its own line."""
    import torch
    torch.cuda.set_device(0)
    emit(config5(args.steps))


def run_ring(args, spec):
    """--ring N: out-of-core decode through the residency ring.  The last N
    layers of the same model are left out of the residency plan and stream every
    step from pinned host images through 2 device ring slots; the line reports
    tokens/s against the bound the measured pinned host-to-device bandwidth sets
    (N layer images per token)."""
    import torch
    from ramforge_b200 import DecodeEngine
    torch.cuda.set_device(0)
    h = torch.empty(1 << 30, dtype=torch.uint8).pin_memory()
    d = torch.empty(1 << 30, dtype=torch.uint8, device="cuda")
    d.copy_(h, non_blocking=True)
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(5):
        d.copy_(h, non_blocking=True)
    e1.record()
    torch.cuda.synchronize()
    h2d_gbs = 5 * (1 << 30) / (e0.elapsed_time(e1) / 1e3) / 1e9
    del h, d
    n = max(1, min(args.ring, spec.n_layers))
    eng = DecodeEngine(make_model(spec, 1, 0), device=0, max_seq_len=PROMPT_LEN + args.warmup + args.steps + 16)
    eng.set_residency_plan([i < spec.n_layers - n for i in range(spec.n_layers)], ring_slots=2)
    prompt = np.random.default_rng(3).integers(0, spec.vocab_size, 8).tolist()
    first = int(eng.generate(prompt, 1)[0])
    toks, _ = eng.decode_timed(first, args.warmup)
    toks, dev_ms = eng.decode_timed(int(toks[-1]), args.steps)
    st = eng.residency_stats()
    layer_bytes = st["host_image_bytes"] / n
    value = args.steps / (dev_ms / 1e3)
    bound = h2d_gbs * 1e9 / (n * layer_bytes)
    emit({
        "metric": "out-of-core decode tokens/s (Llama-3-8B Q4_K shape, streamed layers)", "value": value,
        "unit": "tokens/s", "n_gpus": 1, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": dev_ms / args.steps, "higher_is_better": True, "data": "synthetic",
        "config": {"workload": f"{n} of {spec.n_layers} layers streamed through 2 ring slots per token",
                   "layer_image_bytes": layer_bytes, "prompt_tokens": len(prompt)},
        "roofline": {"bound": "h2d", "achieved": n * layer_bytes * value / 1e9, "peak": h2d_gbs, "unit": "GB/s",
                     "frac": value / bound, "peak_source": "pinned host-to-device copy measured in this run"},
        "residency_stats": st})
    eng.close()


# GGUF bytes per 256 weights (quant.rs block sizes)
GGUF_BYTES_PER_256 = {"Q8_0": 272, "Q4_0": 144, "Q4_K": 144, "Q5_K": 176, "Q6_K": 210, "Q3_K": 110, "Q2_K": 84}


def run_gemv_sweep(args):
    """--gemv-sweep: benchmark configuration 2, the standalone quantized GEMV
    (rf_qmatvec) of every tiled format on the four config-2 shapes at the --batches
    sizes (default 1), one JSON line each; past batch 1, Q4_K and Q8_0 lines also time
    the tensor-core GEMM (rf_qgemm) on the same inputs.  Time: CUDA events on the launching stream around 100 calls
    after 3 warm-up calls, rotating over distinct copies of the matrix that
    together exceed 4x the 126 MB L2.  `gbs` is algorithmic bytes (GGUF bytes
    M*K*b plus 4K + 4M) over that time; `moved_bytes` is the packed matrix."""
    import torch
    from ramforge_b200 import QMatrix, synth
    peak, peak_kind = measured_peaks()
    names = {synth.Q8_0: "Q8_0", synth.Q4_0: "Q4_0", synth.Q4_K: "Q4_K", synth.Q5_K: "Q5_K", synth.Q6_K: "Q6_K",
             synth.Q3_K: "Q3_K", synth.Q2_K: "Q2_K"}
    shapes = [(4096, 4096), (14336, 4096), (4096, 14336), (128256, 4096)]
    stream = torch.cuda.current_stream()
    want = set(f for f in args.formats.split(",") if f) or set(names.values())
    batches = [int(b) for b in args.batches.split(",") if b]
    for gtype, name in names.items():
        if name not in want:
            continue
        for M, K in shapes:
            if gtype in (synth.Q5_K, synth.Q3_K, synth.Q2_K):
                raw = synth.random_blocks(gtype, M, K, seed=M)
            else:
                raw = synth.quantize(gtype, synth.normal(1, 100 + gtype, M * K, std=0.02).reshape(M, K))
            first = QMatrix(gtype, raw, M, K)
            copies = [first] + [QMatrix(gtype, raw, M, K)
                                for _ in range(min(63, -(-4 * 126_000_000 // first.device_bytes) - 1))]
            del raw
            def timed(fn, n):
                for i in range(3):
                    fn(i)
                e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                torch.cuda.synchronize()
                e0.record(stream)
                for i in range(n):
                    fn(i)
                e1.record(stream)
                torch.cuda.synchronize()
                return e0.elapsed_time(e1) * 1e3 / n

            for batch in batches:
                x = torch.randn(batch, K, device="cuda")
                y = torch.empty(batch, M, device="cuda")
                n = max(10, 100 // batch)
                def gemv(i):  # rf_qmatvec takes up to 8 vectors a call
                    for b0 in range(0, batch, 8):
                        nb = min(8, batch - b0)
                        copies[i % len(copies)].matvec(x[b0].data_ptr(), y[b0].data_ptr(), nb, stream.cuda_stream)

                us = timed(gemv, n)
                alg = M * K * GGUF_BYTES_PER_256[name] / 256 + 4 * K * batch + 4 * M * batch
                line = {"metric": "standalone GEMV GB/s (benchmark configuration 2)", "format": name, "M": M,
                        "K": K, "batch": batch, "us_per_call": us, "gbs": alg / us / 1e3, "unit": "GB/s",
                        "frac": alg / us / 1e3 / peak, "peak": peak, "peak_source": f"{peak_kind} hbm_gbs",
                        "algorithmic_bytes": alg, "moved_bytes": first.device_bytes, "copies": len(copies),
                        "calls": n, "api": "rf_qmatvec (CUDA cores, one pass over the weights per vector, 8 vectors a call)"}
                if batch > 1 and gtype in (synth.Q4_K, synth.Q8_0):
                    # the tensor-core GEMM of the prompt path on the same inputs: where it starts to pay
                    gus = timed(lambda i: copies[i % len(copies)].gemm(x.data_ptr(), y.data_ptr(), batch,
                                                                       stream.cuda_stream), n)
                    line["tensor_core"] = {"api": "rf_qgemm (tcgen05, one pass per 128 vectors)", "us_per_call": gus,
                                           "gbs": alg / gus / 1e3, "tflops": 2.0 * M * K * batch / gus / 1e6,
                                           "faster_than_gemv": gus < us}
                emit(line)
                del x, y
            for m in copies:
                m.close()
            del copies
            torch.cuda.empty_cache()


ATTN_SHAPES = [(b, c) for b in (1, 8) for c in (512, 2048, 8192, 32768)]


def attention_sweep(peak: float, peak_kind: str, iters: int = 50):
    """Benchmark configuration 3: rf_decode_attention (32 query heads over 8 KV
    heads of head_dim 128, f16 K/V, one query token per sequence) at batch 1/8 x
    context 512/2048/8192/32768.  Time: CUDA events around the replay of one CUDA
    graph holding `iters` calls (captured after 3 warm-up calls, so the figure is
    device time, not the host's launch rate), rotating over distinct K/V buffers
    that together exceed 4x the 126 MB L2 (one buffer when a single one does).
    Algorithmic bytes per call: batch*ctx*KV*hd*2*2 (K and V f16) + batch*H*hd*4*2
    (query in, output out)."""
    import torch
    from ramforge_b200 import decode_attention
    H, KV, hd = 32, 8, 128
    stream = torch.cuda.current_stream()
    rows = []
    for batch, ctx in ATTN_SHAPES:
        kv_elems = batch * KV * ctx * hd
        per_copy = kv_elems * 2 * 2
        copies = max(1, min(256, -(-4 * 126_000_000 // per_copy)))
        k = torch.empty(copies, kv_elems, dtype=torch.float16, device="cuda").normal_()
        v = torch.empty(copies, kv_elems, dtype=torch.float16, device="cuda").normal_()
        q = torch.randn(batch, H, hd, device="cuda")
        o = torch.empty(batch, H, hd, device="cuda")

        def call(i, st):
            j = i % copies
            decode_attention(q.data_ptr(), k[j].data_ptr(), v[j].data_ptr(), ctx, H, KV, hd, batch, o.data_ptr(),
                             st.cuda_stream)

        for i in range(3):  # also creates the library's workspace, before the capture
            call(i, stream)
        torch.cuda.synchronize()
        # the timed calls replay from one captured graph: device time, not the host's launch rate
        side = torch.cuda.Stream()
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=side):
            for i in range(iters):
                call(i, side)
        graph.replay()  # warm
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        torch.cuda.synchronize()
        e0.record(stream)
        graph.replay()
        e1.record(stream)
        torch.cuda.synchronize()
        us = e0.elapsed_time(e1) * 1e3 / iters
        del graph
        alg = per_copy + batch * H * hd * 4 * 2
        rows.append({"batch": batch, "ctx": ctx, "us_per_call": us, "gbs": alg / us / 1e3,
                     "frac": alg / us / 1e3 / peak, "algorithmic_bytes": alg, "copies": copies})
        del k, v, q, o
        torch.cuda.empty_cache()
    return {"kernel": "attn_kernel (rf_decode_attention)", "peak": peak, "peak_source": f"{peak_kind} hbm_gbs",
            "unit": "GB/s", "rows": rows}


def run_attn_sweep(args):
    """--attn-sweep: benchmark configuration 3 on its own, one JSON line per shape."""
    import torch
    torch.cuda.set_device(0)
    peak, peak_kind = measured_peaks()
    res = attention_sweep(peak, peak_kind)
    for r in res["rows"]:
        emit({"metric": "decode attention GB/s (benchmark configuration 3)", "unit": "GB/s", "value": r["gbs"],
              "heads": "32q/8kv", "head_dim": 128, "kv": "f16", "peak": peak,
              "peak_source": res["peak_source"], **r})


def token_digest(tokens) -> str:
    import hashlib
    return hashlib.sha256(np.ascontiguousarray(tokens, np.uint32).tobytes()).hexdigest()[:16]


def workload_config(spec, args, tp):
    return {"workload": "llama-3-8b-shape Q4_K batch-1 greedy decode after a 512-token prompt",
            "layers": spec.n_layers, "dim": spec.n_embd, "heads": f"{spec.n_heads}q/{spec.n_kv_heads}kv",
            "ffn": spec.n_ff, "vocab": spec.vocab_size, "weights": "Q4_K layers, Q8_0 token_embd/output",
            "kv_cache": "f16", "prompt_tokens": PROMPT_LEN, "decode_context": f"{PROMPT_LEN + args.warmup}.."
            f"{PROMPT_LEN + args.warmup + args.steps}", "parallelism": f"tp{tp}",
            "l2": "no flush: every step streams 4.5 GB of weights (> 126 MB L2)"}


_RESULT_FD = None


def emit(obj):
    """Write one result line (JSON) to the process's real stdout."""
    sys.stdout.flush()
    os.write(_RESULT_FD if _RESULT_FD is not None else 1, (json.dumps(obj) + "\n").encode())


def json_only_stdout():
    """Point file descriptor 1 at stderr for the rest of the run, so that nothing
    but the result line reaches stdout: libraries print there at the C level (NCCL's
    version banner when the environment sets NCCL_DEBUG, for one)."""
    global _RESULT_FD
    sys.stdout.flush()
    _RESULT_FD = os.dup(1)
    os.dup2(2, 1)


def batched_prefill(eng, spec, prompt, first_tbt, tbt_s):
    """The 512-token prompt through rf_prefill (tensor-core GEMMs in 256-token
    chunks) against the token-by-token prompt of rf_generate (one decode-graph
    forward per token, the reference's loop): host time around the synchronous
    calls, best of 3 after one warm-up; `tflops` counts 2 flops per layer weight
    and prompt token (the three split-bf16 products are not counted)."""
    n = len(prompt)
    times = []
    for _ in range(4):
        eng.kv_reset()
        t0 = time.perf_counter()
        eng.prefill(prompt)
        times.append(time.perf_counter() - t0)
    _, first = eng.compute_logits(want_logits=False)
    best = min(times[1:])
    d, q, kv, ff = spec.n_embd, spec.n_embd, spec.n_kv_heads * spec.head_dim, spec.n_ff
    layer_params = spec.n_layers * ((q + 2 * kv) * d + d * q + 2 * ff * d + d * ff)
    return {"api": "rf_prefill", "prompt_tokens": n, "tokens_per_s": n / best, "ms": best * 1e3,
            "token_by_token_tokens_per_s": n / tbt_s, "speedup": tbt_s / best,
            "tflops": 2.0 * layer_params * n / best / 1e12,
            "first_token_equals_token_by_token": int(first) == int(first_tbt),
            "timing": "host clock around the synchronous call (best of 3 after a warm-up)"}


def main():
    json_only_stdout()
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=256)
    ap.add_argument("--warmup", type=int, default=8)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--profile", action="store_true", help="small eager run for ncu captures")
    ap.add_argument("--layers", type=int, default=0, help="with --profile: layer count of the model")
    ap.add_argument("--prefill", type=int, default=0, help="with --profile: batched prefill of this many tokens")
    ap.add_argument("--profile-attn", default="", help="CTX,BATCH: a few rf_decode_attention calls (ncu capture)")
    ap.add_argument("--config5", action="store_true", help="70B-shape model, 4 GiB weight budget, ring (benchmark configuration 5)")
    ap.add_argument("--no-ring", action="store_true", help="leave the out-of-core measurements off the main line")
    ap.add_argument("--ring", type=int, default=0, help="out-of-core run: stream this many layers per step")
    ap.add_argument("--gemv-sweep", action="store_true", help="benchmark configuration 2: GEMV per format and shape")
    ap.add_argument("--formats", default="", help="with --gemv-sweep: comma-separated subset, e.g. Q4_K,Q6_K")
    ap.add_argument("--batches", default="1", help="with --gemv-sweep: batch sizes, e.g. 1,4,8,16,32")
    ap.add_argument("--attn-sweep", action="store_true", help="benchmark configuration 3: decode attention GB/s")
    ap.add_argument("--no-attn-sweep", action="store_true", help="leave the attention sweep off the main line")
    args = ap.parse_args()
    args.warmup = max(args.warmup, 3)
    world, rank, local = dist_env()

    from ramforge_b200 import synth
    spec = synth.LLAMA3_8B

    if args.impl == "reference":
        if rank == 0:
            run_reference(args, spec)
        return
    if args.profile:
        run_profile(args, spec)
        return
    if args.profile_attn:
        run_attn_profile(args)
        return
    if args.config5:
        run_config5(args)
        return
    if args.ring:
        run_ring(args, spec)
        return
    if args.gemv_sweep:
        run_gemv_sweep(args)
        return
    if args.attn_sweep:
        run_attn_sweep(args)
        return

    import torch
    torch.cuda.set_device(local)
    if world > 1:
        import torch.distributed as dist
        from datetime import timedelta
        dist.init_process_group("nccl", device_id=torch.device("cuda", local), timeout=timedelta(seconds=600))
    from ramforge_b200 import DecodeEngine, tp_unique_id

    t0 = time.perf_counter()
    gguf = make_model(spec, world, rank)
    gen_s = time.perf_counter() - t0
    nccl_id = None
    if world > 1:
        import torch.distributed as dist
        obj = [tp_unique_id() if rank == 0 else None]
        dist.broadcast_object_list(obj, src=0)
        nccl_id = obj[0]
    e2e_steps = args.steps
    max_seq = PROMPT_LEN + args.warmup + max(args.steps, e2e_steps) + 16
    t0 = time.perf_counter()
    eng = DecodeEngine(gguf, device=local, max_seq_len=max_seq, tp_rank=rank, tp_size=world, nccl_id=nccl_id)
    load_s = time.perf_counter() - t0
    prompt = np.random.default_rng(3).integers(0, spec.vocab_size, PROMPT_LEN).tolist()

    def barrier():
        torch.cuda.synchronize()
        if world > 1:
            import torch.distributed as dist
            dist.barrier()

    def max_over_ranks(x: float) -> float:
        if world == 1:
            return x
        import torch.distributed as dist
        t = torch.tensor([x], device="cuda", dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    # prefill (token by token, like the reference: inference.rs:578-592) + warm-up
    t0 = time.perf_counter()
    first = int(eng.generate(prompt, 1)[0])
    tbt_s = time.perf_counter() - t0
    toks, _ = eng.decode_timed(first, args.warmup)
    nxt = int(toks[-1])
    barrier()
    with ClockSampler(local) as clk:
        toks, dev_ms = eng.decode_timed(nxt, args.steps)
        barrier()
    dev_ms = max_over_ranks(dev_ms)
    clocks = clk.summary()
    timed_tokens = toks.copy()
    value = args.steps / (dev_ms / 1e3)

    # e2e: same positions again through rf_decode_step (pinned H2D token+pos, D2H token, sync)
    eng.kv_reset()
    first = int(eng.generate(prompt, 1)[0])
    tok = first
    for _ in range(args.warmup):
        tok = eng.decode_step(tok)
    barrier()
    e2e_tokens = np.zeros(e2e_steps, np.uint32)
    t0 = time.perf_counter()
    for i in range(e2e_steps):
        tok = eng.decode_step(tok)
        e2e_tokens[i] = tok
    barrier()
    e2e_s = max_over_ranks(time.perf_counter() - t0)
    e2e = {"value": e2e_steps / e2e_s, "unit": UNIT, "h2d_bytes_per_step": 8, "d2h_bytes_per_step": 4,
           "api": "rf_decode_step (token + position in, next token out)"}
    # Greedy tokens of both runs: identical on every rank count when the
    # tensor-parallel decode reproduces the single-GPU one (same prompt, positions).
    tokens = {"timed_sha256_16": token_digest(timed_tokens), "e2e_sha256_16": token_digest(e2e_tokens),
              "timed_first8": timed_tokens[:8].tolist(), "first_after_prompt": first,
              "timed_equals_e2e": bool(np.array_equal(timed_tokens, e2e_tokens))}

    prefill = batched_prefill(eng, spec, prompt, first, tbt_s) if world == 1 else None

    # dominant kernel: gate/up + SwiGLU GEMV, timed over every layer (weights >> L2)
    kms = eng.bench_layer_kernels(iters=3)
    kms = [max_over_ranks(k) for k in kms]
    ctx_mean = PROMPT_LEN + args.warmup + args.steps / 2
    step_bytes, gateup_bytes = algorithmic_bytes(spec, world, ctx_mean)
    peak, peak_kind = measured_peaks()
    achieved = gateup_bytes / (kms[3] / 1e3) / 1e9
    roofline = {"bound": "hbm", "kernel": "qgemv_kernel<Q4_K, EpiSwiGLU> (ffn gate/up + SwiGLU)",
                "achieved": achieved, "peak": peak, "unit": "GB/s", "frac": achieved / peak,
                "peak_source": f"{peak_kind} hbm_gbs", "bytes_per_launch": gateup_bytes,
                "ms_per_launch": kms[3], "traffic": GATEUP_DRAM_BYTES_NCU / world,
                "traffic_source": "ncu dram__bytes_read.sum + dram__bytes_write.sum of one TP1 launch "
                                  "(bench.py --profile --layers 2), divided by the ranks"}
    step_gbs = step_bytes / (dev_ms / args.steps / 1e3) / 1e9

    line = {
        "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": dev_ms / args.steps, "higher_is_better": True,
        "scaling": "strong", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": workload_config(spec, args, world), "clocks": clocks, "e2e": e2e,
        "gpu_launches": args.steps * eng.step_kernel_count, "roofline": roofline,
        "step_roofline": {"bytes_per_token_per_gpu": step_bytes, "achieved_gbs": step_gbs, "frac": step_gbs / peak},
        "kernel_ms": dict(zip(["qkv_rope", "attention", "wo_residual", "gateup_swiglu", "down_residual"], kms)),
        "tokens": tokens, "tp_peer_sum": eng.tp_peer_sum if world > 1 else None, "prefill": prefill,
        "setup_s": {"model_generation": gen_s, "engine_load": load_s},
    }
    if world == 1 and not args.no_ring:
        line["out_of_core"] = out_of_core(eng, spec, first, max(4, args.steps // 4))
    eng.close()
    if world > 1:
        import torch.distributed as dist
        dist.barrier()
        dist.destroy_process_group()
    if rank == 0:
        if world == 1 and not args.no_attn_sweep:
            line["attention_sweep"] = attention_sweep(peak, peak_kind)
        if world == 1 and not args.no_ring:
            line["config5"] = config5(2)
        if world == 1 and not args.no_cpu_baseline:
            ctx = PROMPT_LEN + args.warmup
            line["cpu_baseline"] = cpu_baseline(gguf, spec, ctx, threads=1)
            line["cpu_baseline_all_cores"] = cpu_baseline(gguf, spec, ctx, threads=host_cores())
        emit(line)


if __name__ == "__main__":
    main()
