"""Test fixtures restated from the reference's own tests.

gqa_*: the GQA forward fixture of crates/ramforge-runtime/src/inference.rs:2111-2337
(qwen2 arch, n_embd 8, 4 query heads, 2 KV heads, head_dim 2, FFN 16, vocab 16,
f32 weights from a small LCG, tied output) and a numpy float32 restatement of
its scalar reference forward (inference.rs:2338-2476).

qwen2_bias_*: the biased qwen2 fixture of inference.rs:1620-1845 (n_embd 8, 2
heads of head_dim 4, 2 KV heads, FFN 16, vocab 16, closed-form f32 weight tables,
Q/K/V biases, tied output) and its reference forward (inference.rs:1846-1993):
the same restatement with the biases added after the projections, before RoPE.
"""
from __future__ import annotations

import numpy as np

from tests.gguf_writer import ARR, F32, I32, STR, U32, f32_bytes, write_gguf

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
    return reference_forward(w, token, pos, k_hist, v_hist, eps, GQA_N_EMBD, GQA_N_HEADS, GQA_N_KV_HEADS,
                             GQA_HEAD_DIM, GQA_FFN)


def reference_forward(w, token, pos, k_hist: list, v_hist: list, eps, d, nh, nkv, hd, ffn):
    """One-layer scalar forward of the reference's fixture tests: RMSNorm, ggml
    [in,out] matvecs, Q/K/V biases after the projections when w has them
    (inference.rs:1899-1912), half-split RoPE, attention over history + current,
    SwiGLU FFN, output RMSNorm."""
    f = np.float32
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
    if "bias_q" in w:
        q = (q + w["bias_q"]).astype(np.float32)
        k = (k + w["bias_k"]).astype(np.float32)
        v = (v + w["bias_v"]).astype(np.float32)
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
    g = matvec(w["ffn_gate"], d, ffn, tmp)
    u = matvec(w["ffn_up"], d, ffn, tmp)
    gu = (g / (f(1.0) + np.exp(-g))) * u
    hidden = hidden + matvec(w["ffn_down"], ffn, d, gu.astype(np.float32))
    return rmsnorm(hidden.astype(np.float32), w["output_norm"])


QB_N_EMBD, QB_N_HEADS, QB_N_KV_HEADS, QB_HEAD_DIM, QB_FFN, QB_VOCAB = 8, 2, 2, 4, 16, 16


def qwen2_bias_weights() -> dict:
    """qwen2_weights (inference.rs:1644-1670): every entry a closed form of its flat
    index i, evaluated in f32 (a + b * k with k a small integer)."""
    f = np.float32
    i = np.arange(128)

    def w(n, a, b, k):
        return (f(a) + f(b) * k[:n].astype(np.float32)).astype(np.float32)

    t, c = np.arange(16 * 8) // 8, np.arange(16 * 8) % 8
    embd = (f(0.02) * (t + 1).astype(np.float32) + f(0.003) * c.astype(np.float32)).astype(np.float32)
    r, m = i // 8, i % 8
    return {
        "embd": embd,
        "output_norm": np.ones(8, np.float32),
        "attn_norm": np.ones(8, np.float32),
        "attn_q": w(64, 0.03, 0.01, (r + 2 * m) % 5),
        "attn_k": w(64, 0.02, 0.01, (r + 3 * m) % 7),
        "attn_v": w(64, 0.01, 0.02, (2 * r + m) % 5),
        "attn_output": w(64, 0.03, 0.01, (r + m) % 4),
        "ffn_norm": np.ones(8, np.float32),
        "ffn_gate": w(128, 0.02, 0.01, (r + m) % 6),
        "ffn_up": w(128, 0.01, 0.015, (r + 2 * m) % 5),
        "ffn_down": w(128, 0.02, 0.01, (r + 3 * m) % 7),
        "bias_q": w(8, 0.05, 0.01, i),
        "bias_k": w(8, 0.04, 0.02, i),
        "bias_v": w(8, 0.03, 0.03, i),
    }


def qwen2_bias_gguf(mode: str = "full") -> bytes:
    """create_qwen2_biased_gguf (inference.rs:1672-1844): 14 f32 tensors, the biases
    beside their matrices, tied output.  mode "only_q" keeps the Q bias alone and
    "wrong_dim" gives it 4 elements (the partial-set and shape cases of
    create_model_with_qkv_bias, streaming_model.rs:2075-2100)."""
    w = qwen2_bias_weights()
    toks = ["<unk>", "<s>", "</s>", "\u2581hello", "\u2581world", "hello", "world", "!", "\u2581", "a", "b", "c",
            "d", "e", "f", "g"]
    meta = [
        ("general.architecture", STR, "qwen2"),
        ("qwen2.vocab_size", U32, QB_VOCAB),
        ("qwen2.context_length", U32, 64),
        ("qwen2.embedding_length", U32, QB_N_EMBD),
        ("qwen2.block_count", U32, 1),
        ("qwen2.feed_forward_length", U32, QB_FFN),
        ("qwen2.attention.head_count", U32, QB_N_HEADS),
        ("qwen2.attention.head_count_kv", U32, QB_N_KV_HEADS),
        ("qwen2.attention.layer_norm_rms_epsilon", F32, 1e-5),
        ("qwen2.rope.freq_base", F32, 10000.0),
        ("tokenizer.ggml.model", STR, "llama"),
        ("tokenizer.ggml.tokens", ARR, (STR, toks)),
        ("tokenizer.ggml.scores", ARR, (F32, [0.0] * QB_VOCAB)),
        ("tokenizer.ggml.token_type", ARR, (I32, [2, 3, 3] + [1] * 13)),
        ("tokenizer.ggml.bos_token_id", U32, 1),
        ("tokenizer.ggml.eos_token_id", U32, 2),
    ]
    bq = w["bias_q"][:4] if mode == "wrong_dim" else w["bias_q"]
    tensors = [
        ("token_embd.weight", [8, 16], 0, f32_bytes(w["embd"])),
        ("output_norm.weight", [8], 0, f32_bytes(w["output_norm"])),
        ("blk.0.attn_norm.weight", [8], 0, f32_bytes(w["attn_norm"])),
        ("blk.0.attn_q.weight", [8, 8], 0, f32_bytes(w["attn_q"])),
        ("blk.0.attn_q.bias", [bq.size], 0, f32_bytes(bq)),
        ("blk.0.attn_k.weight", [8, 8], 0, f32_bytes(w["attn_k"])),
        ("blk.0.attn_k.bias", [8], 0, f32_bytes(w["bias_k"])),
        ("blk.0.attn_v.weight", [8, 8], 0, f32_bytes(w["attn_v"])),
        ("blk.0.attn_v.bias", [8], 0, f32_bytes(w["bias_v"])),
        ("blk.0.attn_output.weight", [8, 8], 0, f32_bytes(w["attn_output"])),
        ("blk.0.ffn_norm.weight", [8], 0, f32_bytes(w["ffn_norm"])),
        ("blk.0.ffn_gate.weight", [8, 16], 0, f32_bytes(w["ffn_gate"])),
        ("blk.0.ffn_up.weight", [8, 16], 0, f32_bytes(w["ffn_up"])),
        ("blk.0.ffn_down.weight", [16, 8], 0, f32_bytes(w["ffn_down"])),
    ]
    if mode == "only_q":
        tensors = [t for t in tensors if t[0] not in ("blk.0.attn_k.bias", "blk.0.attn_v.bias")]
    return write_gguf(meta, tensors)


def qwen2_bias_reference_forward(w, token, pos, k_hist: list, v_hist: list, eps=1e-5):
    """reference_forward_biased (inference.rs:1846-1993)."""
    return reference_forward(w, token, pos, k_hist, v_hist, eps, QB_N_EMBD, QB_N_HEADS, QB_N_KV_HEADS, QB_HEAD_DIM,
                             QB_FFN)


def random_blocks(gtype: int, rows: int, k: int, seed: int) -> np.ndarray:
    """Random well-formed GGUF blocks of a format without a synthetic encoder
    (ramforge_b200.synth.random_blocks)."""
    from ramforge_b200 import synth
    return synth.random_blocks(gtype, rows, k, seed)
