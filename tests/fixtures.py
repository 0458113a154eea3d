"""Test fixtures restated from the reference's own tests.

gqa_*: the GQA forward fixture of crates/ramforge-runtime/src/inference.rs:2111-2337
(qwen2 arch, n_embd 8, 4 query heads, 2 KV heads, head_dim 2, FFN 16, vocab 16,
f32 weights from a small LCG, tied output) and a numpy float32 restatement of
its scalar reference forward (inference.rs:2338-2476).
"""
from __future__ import annotations

import numpy as np

from tests.gguf_writer import ARR, F32, STR, U32, f32_bytes, write_gguf

GQA_N_EMBD, GQA_N_HEADS, GQA_N_KV_HEADS, GQA_HEAD_DIM, GQA_FFN, GQA_VOCAB = 8, 4, 2, 2, 16, 16


def lcg_weights(n: int, seed: int) -> np.ndarray:
    """w(n, seed) of inference.rs:2119-2128: s = seed*2654435761 + i*224682251 (u32 wrap),
    value 0.01 * ((s & 63) - 20) in f32."""
    i = np.arange(n, dtype=np.uint64)
    s = (np.uint64(seed) * np.uint64(2654435761) + i * np.uint64(224682251)) & np.uint64(0xFFFFFFFF)
    v = (s & np.uint64(0x3F)).astype(np.float32) - np.float32(20.0)
    return (np.float32(0.01) * v).astype(np.float32)


def gqa_weights() -> dict:
    q_dim, kv_dim = GQA_N_HEADS * GQA_HEAD_DIM, GQA_N_KV_HEADS * GQA_HEAD_DIM
    return {
        "embd": lcg_weights(GQA_VOCAB * GQA_N_EMBD, 1),
        "output_norm": np.ones(GQA_N_EMBD, np.float32),
        "attn_norm": np.ones(GQA_N_EMBD, np.float32),
        "attn_q": lcg_weights(GQA_N_EMBD * q_dim, 2),
        "attn_k": lcg_weights(GQA_N_EMBD * kv_dim, 3),
        "attn_v": lcg_weights(GQA_N_EMBD * kv_dim, 4),
        "attn_output": lcg_weights(q_dim * GQA_N_EMBD, 5),
        "ffn_norm": np.ones(GQA_N_EMBD, np.float32),
        "ffn_gate": lcg_weights(GQA_N_EMBD * GQA_FFN, 6),
        "ffn_up": lcg_weights(GQA_N_EMBD * GQA_FFN, 7),
        "ffn_down": lcg_weights(GQA_FFN * GQA_N_EMBD, 8),
    }


def gqa_gguf() -> bytes:
    """The fixture GGUF of inference.rs:2148-2337 (11 f32 tensors, tokenizer metadata)."""
    w = gqa_weights()
    q_dim, kv_dim = GQA_N_HEADS * GQA_HEAD_DIM, GQA_N_KV_HEADS * GQA_HEAD_DIM
    toks = ["<unk>", "<s>", "</s>", "▁hi", "▁there", "a", "b", "c", "d", "e", "f", "g", "h", "i", "j", "k"]
    meta = [
        ("general.architecture", STR, "qwen2"),
        ("qwen2.vocab_size", U32, GQA_VOCAB),
        ("qwen2.context_length", U32, 64),
        ("qwen2.embedding_length", U32, GQA_N_EMBD),
        ("qwen2.block_count", U32, 1),
        ("qwen2.feed_forward_length", U32, GQA_FFN),
        ("qwen2.attention.head_count", U32, GQA_N_HEADS),
        ("qwen2.attention.head_count_kv", U32, GQA_N_KV_HEADS),
        ("qwen2.attention.layer_norm_rms_epsilon", F32, 1e-5),
        ("qwen2.rope.freq_base", F32, 10000.0),
        ("tokenizer.ggml.model", STR, "llama"),
        ("tokenizer.ggml.tokens", ARR, (STR, toks)),
        ("tokenizer.ggml.scores", ARR, (F32, [0.0] * GQA_VOCAB)),
        ("tokenizer.ggml.token_type", ARR, (U32, [2, 3, 3] + [1] * 13)),
        ("tokenizer.ggml.bos_token_id", U32, 1),
    ]
    tensors = [
        ("token_embd.weight", [GQA_N_EMBD, GQA_VOCAB], 0, f32_bytes(w["embd"])),
        ("output_norm.weight", [GQA_N_EMBD], 0, f32_bytes(w["output_norm"])),
        ("blk.0.attn_norm.weight", [GQA_N_EMBD], 0, f32_bytes(w["attn_norm"])),
        ("blk.0.attn_q.weight", [GQA_N_EMBD, q_dim], 0, f32_bytes(w["attn_q"])),
        ("blk.0.attn_k.weight", [GQA_N_EMBD, kv_dim], 0, f32_bytes(w["attn_k"])),
        ("blk.0.attn_v.weight", [GQA_N_EMBD, kv_dim], 0, f32_bytes(w["attn_v"])),
        ("blk.0.attn_output.weight", [q_dim, GQA_N_EMBD], 0, f32_bytes(w["attn_output"])),
        ("blk.0.ffn_norm.weight", [GQA_N_EMBD], 0, f32_bytes(w["ffn_norm"])),
        ("blk.0.ffn_gate.weight", [GQA_N_EMBD, GQA_FFN], 0, f32_bytes(w["ffn_gate"])),
        ("blk.0.ffn_up.weight", [GQA_N_EMBD, GQA_FFN], 0, f32_bytes(w["ffn_up"])),
        ("blk.0.ffn_down.weight", [GQA_FFN, GQA_N_EMBD], 0, f32_bytes(w["ffn_down"])),
    ]
    return write_gguf(meta, tensors)


def gqa_reference_forward(w, token, pos, k_hist: list, v_hist: list, eps=1e-5):
    """numpy float32 restatement of reference_forward_gqa (inference.rs:2338-2476)."""
    f = np.float32
    hd, nh, nkv, d = GQA_HEAD_DIM, GQA_N_HEADS, GQA_N_KV_HEADS, GQA_N_EMBD
    q_dim, kv_dim = nh * hd, nkv * hd

    def rmsnorm(x, wt):
        mean = f(np.sum(x * x, dtype=np.float32)) / f(x.size)
        rms = np.sqrt(f(mean + f(eps)), dtype=np.float32)
        return (x / rms * wt).astype(np.float32)

    def matvec(wt, n_in, n_out, x):
        return (wt.reshape(n_out, n_in) @ x).astype(np.float32)

    def rope(x):
        half = hd // 2
        for j in range(half):
            th = np.float32(np.power(np.float32(10000.0), np.float32(-2.0 * j / hd), dtype=np.float32)) * f(pos)
            c, s = np.cos(th, dtype=np.float32), np.sin(th, dtype=np.float32)
            a, b = x[j], x[j + half]
            x[j], x[j + half] = a * c - b * s, a * s + b * c

    hidden = w["embd"][token * d:(token + 1) * d].copy()
    tmp = rmsnorm(hidden, w["attn_norm"])
    q = matvec(w["attn_q"], d, q_dim, tmp)
    k = matvec(w["attn_k"], d, kv_dim, tmp)
    v = matvec(w["attn_v"], d, kv_dim, tmp)
    for h in range(nh):
        rope(q[h * hd:(h + 1) * hd])
    for h in range(nkv):
        rope(k[h * hd:(h + 1) * hd])
    keys = k_hist + [k]
    vals = v_hist + [v]
    out = np.zeros(q_dim, np.float32)
    for h in range(nh):
        kvh = h * nkv // nh
        sc = np.array([np.dot(q[h * hd:(h + 1) * hd], kk[kvh * hd:(kvh + 1) * hd]) / np.sqrt(f(hd)) for kk in keys],
                      np.float32)
        e = np.exp(sc - sc.max()).astype(np.float32)
        p = e / e.sum(dtype=np.float32)
        for pi, vv in zip(p, vals):
            out[h * hd:(h + 1) * hd] += pi * vv[kvh * hd:(kvh + 1) * hd]
    hidden = hidden + matvec(w["attn_output"], q_dim, d, out)
    k_hist.append(k)
    v_hist.append(v)
    tmp = rmsnorm(hidden, w["ffn_norm"])
    g = matvec(w["ffn_gate"], d, GQA_FFN, tmp)
    u = matvec(w["ffn_up"], d, GQA_FFN, tmp)
    gu = (g / (f(1.0) + np.exp(-g))) * u
    hidden = hidden + matvec(w["ffn_down"], GQA_FFN, d, gu.astype(np.float32))
    return rmsnorm(hidden.astype(np.float32), w["output_norm"])
