"""Tensor-parallel partitioning on CPU: two gloo ranks run one transformer layer
and the LM head of a small Q4_K model on the shards rf_tp_shard_plan gives them
(the same plan the GPU engine uses), with the oracle's arithmetic, and must
reproduce the single-rank oracle:

  * Q/K/V and gate/up are split by rows (KV-head groups, FFN rows), Wo and Wdown
    by columns on quant-block boundaries; each row-parallel projection ends in a
    sum all-reduce with the residual added by rank 0 only;
  * greedy argmax over vocab shards keeps the first-maximum rule (sampling.rs:48-53).
"""
import ctypes
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))

SPEC_KW = dict(name="tp-q4k", vocab_size=512, n_embd=512, n_layers=1, n_ff=1024, n_heads=8, n_kv_heads=4, seed=31,
               context_length=64)


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _slice_cols(raw: np.ndarray, n_rows: int, row_bytes: int, blk_bytes: int, qk: int, c0: int, ncols: int):
    """Columns [c0, c0+ncols) of every row of a GGUF block matrix (block aligned)."""
    rows = raw[: n_rows * row_bytes].reshape(n_rows, row_bytes)
    return np.ascontiguousarray(rows[:, c0 // qk * blk_bytes:(c0 + ncols) // qk * blk_bytes]).reshape(-1)


def _worker(rank, world, port, out_q):
    import sys
    sys.path.insert(0, ROOT)
    from oracle import oracle as orc
    from ramforge_b200 import _lib, synth
    from tests.gguf_reader import read_tensors

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        spec = synth.scaled(synth.LLAMA3_8B, **SPEC_KW)
        g = synth.gguf_bytes(spec, threads=2)
        ts = read_tensors(g)
        ref = orc.OracleModel(g, kv_f16=False, max_seq=8)
        cfg = ref.config
        c = _lib.ModelConfig(**{k: cfg[k] for k, _ in _lib.ModelConfig._fields_})
        sh = _lib.TpShard()
        _lib.check(_lib.lib().rf_tp_shard_plan(ctypes.byref(c), world, rank, synth.Q4_K, ctypes.byref(sh)))
        d, hd, ff = cfg["n_embd"], cfg["head_dim"], cfg["n_ff"]
        qk, bb = 256, 144
        rb = lambda n: n // qk * bb  # noqa: E731

        def W(name):
            return ts[name]["data"]

        tok = 17
        hidden = orc.dequant_row(orc.Q8_0, W("token_embd.weight")[tok * orc.row_bytes(orc.Q8_0, d):], d)
        # single-rank reference for the layer and the logits
        want = hidden.copy()
        ref.layer_step(0, 0, want)
        # ---- attention block on this rank's heads
        x = orc.rmsnorm(hidden, np.ones(d, np.float32), cfg["rms_eps"])
        q0, nq = sh.q_head_offset * hd, sh.q_heads * hd
        k0, nk = sh.kv_head_offset * hd, sh.kv_heads * hd
        q = orc.matvec(orc.Q4_K, W("blk.0.attn_q.weight")[q0 * rb(d):(q0 + nq) * rb(d)], d, nq, x)
        k = orc.matvec(orc.Q4_K, W("blk.0.attn_k.weight")[k0 * rb(d):(k0 + nk) * rb(d)], d, nk, x)
        v = orc.matvec(orc.Q4_K, W("blk.0.attn_v.weight")[k0 * rb(d):(k0 + nk) * rb(d)], d, nk, x)
        q, k = orc.rope(q, k, 0, hd, sh.q_heads, sh.kv_heads, cfg["rope_theta"])
        att = orc.attention(q, [], [], k, v, 0, sh.q_heads, sh.kv_heads, hd)
        wo = _slice_cols(W("blk.0.attn_output.weight"), d, rb(cfg["n_heads"] * hd), bb, qk, q0, nq)
        part = orc.matvec(orc.Q4_K, wo, nq, d, att) + (hidden if rank == 0 else 0.0)
        t = torch.from_numpy(part.astype(np.float32))
        dist.all_reduce(t)
        hidden = t.numpy()
        # ---- FFN block on this rank's rows / columns
        x = orc.rmsnorm(hidden, np.ones(d, np.float32), cfg["rms_eps"])
        f0, nf = sh.ff_offset, sh.ff_rows
        gte = orc.matvec(orc.Q4_K, W("blk.0.ffn_gate.weight")[f0 * rb(d):(f0 + nf) * rb(d)], d, nf, x)
        up = orc.matvec(orc.Q4_K, W("blk.0.ffn_up.weight")[f0 * rb(d):(f0 + nf) * rb(d)], d, nf, x)
        act = orc.swiglu(gte, up)
        dn = _slice_cols(W("blk.0.ffn_down.weight"), d, rb(ff), bb, qk, f0, nf)
        part = orc.matvec(orc.Q4_K, dn, nf, d, act) + (hidden if rank == 0 else 0.0)
        t = torch.from_numpy(part.astype(np.float32))
        dist.all_reduce(t)
        hidden = t.numpy()
        layer_err = float(np.abs(hidden - want).max() / np.abs(want).max())
        # ---- LM head on this rank's vocab rows, greedy argmax over ranks
        fh = orc.rmsnorm(want, np.ones(d, np.float32), cfg["rms_eps"])
        full = ref.logits(fh)
        full[100] = full[300] = full.max() + 1.0  # a tie across the two vocab shards
        v0, nv = sh.vocab_offset, sh.vocab_rows
        local = full[v0:v0 + nv]
        li = int(np.argmax(local))
        pairs = [None] * world
        dist.all_gather_object(pairs, (float(local[li]), v0 + li))
        best = max(pairs, key=lambda p: (p[0], -p[1]))
        out_q.put((rank, layer_err, best[1], orc.argmax(full), (sh.vocab_offset, sh.vocab_rows)))
    finally:
        dist.destroy_process_group()


def test_two_rank_layer_and_argmax_match_single_rank():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = [q.get(timeout=300) for _ in range(2)]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    res.sort()
    for rank, layer_err, best, want, (v0, nv) in res:
        assert layer_err < 1e-4, (rank, layer_err)
        assert best == want == 100
    assert res[0][4] == (0, 256) and res[1][4] == (256, 256)
