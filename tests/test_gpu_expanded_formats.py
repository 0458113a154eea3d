"""Q5_0 and Q8_K, formats the engine decodes to f32 at load, and a model mixing
every supported format.

The reference decodes each block of Q5_0 and Q8_K and sums deq[j]*x[j]
(matvec_q5_0/_q8_k, quant.rs:1050-1490), so the engine keeps the decoded rows
(the reference's dequantize, value for value, on the host) and runs its F32 GEMV.
Bars: matvec within 2e-4*max|y| of the oracle (f32 reassociation only);
embedding rows bit-exact (the host decode against the oracle's); a model mixing
these with the tiled formats (Q5_K, Q3_K, Q2_K among them, a V of its own type,
a Q2_K LM head) gives the oracle's greedy tokens and logits within 1e-3.
"""
import os

import numpy as np
import pytest

from oracle import oracle as orc
from ramforge_b200 import DecodeEngine, QMatrix, synth
from tests import fixtures as fx
from tests.gguf_writer import F32, STR, U32, f32_bytes, write_gguf

pytestmark = pytest.mark.gpu
THREADS = min(32, os.cpu_count() or 8)
EXPANDED = [orc.Q5_0, orc.Q8_K]
RANDOM = EXPANDED + [orc.Q5_K, orc.Q3_K, orc.Q2_K]  # formats without a synthetic encoder


def _y(m, x, M):
    import torch
    dx = torch.from_numpy(x).cuda()
    dy = torch.empty(M, device="cuda")
    m.matvec(dx.data_ptr(), dy.data_ptr())
    torch.cuda.synchronize()
    return dy.cpu().numpy()


@pytest.mark.parametrize("gtype", EXPANDED)
@pytest.mark.parametrize("M,K", [(1, 256), (33, 768), (130, 2304), (1024, 4096)])
def test_qmatvec_matches_oracle(gtype, M, K):
    raw = fx.random_blocks(gtype, M, K, seed=M + gtype)
    x = synth.normal(3, 7, K, std=1.0)
    m = QMatrix(gtype, raw, M, K)
    assert m.device_bytes >= 4 * M * K  # stored as f32
    y = _y(m, x, M)
    ref = orc.matvec(gtype, raw, K, M, x, threads=THREADS)
    assert np.abs(y - ref).max() <= 2e-4 * np.abs(ref).max() + 1e-6
    m.close()


@pytest.mark.parametrize("gtype", EXPANDED)
def test_device_bytes_equal_host_bytes(gtype):
    import torch
    M, K = 77, 1024
    raw = fx.random_blocks(gtype, M, K, seed=9)
    x = synth.normal(4, 7, K, std=1.0)
    draw = torch.from_numpy(np.ascontiguousarray(raw)).cuda()
    a = QMatrix(gtype, raw, M, K)
    b = QMatrix(gtype, None, M, K, on_device_ptr=draw.data_ptr(), nbytes=raw.size)
    assert np.array_equal(_y(a, x, M), _y(b, x, M))
    a.close()
    b.close()


D, H, KV, FF, V, L = 256, 4, 2, 512, 300, 2
HD = D // H
# per layer: the ggml type of q, k, v, o, gate, up, down (layer 0: Q5_K Q/K beside a
# Q3_K V, f32-stored gate/up and down; layer 1: Q4_K Q/K, a Q6_K V, Q5_K down)
LAYER_TYPES = [(orc.Q5_K, orc.Q5_K, orc.Q3_K, orc.Q2_K, orc.Q8_K, orc.Q8_K, orc.Q5_0),
               (orc.Q4_K, orc.Q4_K, orc.Q6_K, orc.Q8_0, orc.Q4_0, orc.Q4_0, orc.Q5_K)]


def _matrix(gtype, rows, k, seed):
    if gtype in RANDOM:
        return fx.random_blocks(gtype, rows, k, seed)
    return synth.quantize(gtype, synth.normal(seed, 1, rows * k, std=0.05).reshape(rows, k))


def _mixed_gguf(embd_type=orc.Q5_0):
    meta = [("general.architecture", STR, "llama"), ("llama.vocab_size", U32, V), ("llama.context_length", U32, 128),
            ("llama.embedding_length", U32, D), ("llama.block_count", U32, L), ("llama.feed_forward_length", U32, FF),
            ("llama.attention.head_count", U32, H), ("llama.attention.head_count_kv", U32, KV),
            ("llama.attention.layer_norm_rms_epsilon", F32, 1e-5), ("llama.rope.freq_base", F32, 10000.0)]
    ones = f32_bytes(np.ones(D, np.float32))
    ts = [("token_embd.weight", [D, V], embd_type, _matrix(embd_type, V, D, 1).tobytes())]
    shapes = [(D, H * HD), (D, KV * HD), (D, KV * HD), (H * HD, D), (D, FF), (D, FF), (FF, D)]
    names = ["attn_q", "attn_k", "attn_v", "attn_output", "ffn_gate", "ffn_up", "ffn_down"]
    for l in range(L):
        ts.append((f"blk.{l}.attn_norm.weight", [D], 0, ones))
        ts.append((f"blk.{l}.ffn_norm.weight", [D], 0, ones))
        for j, (name, (k, rows), gt) in enumerate(zip(names, shapes, LAYER_TYPES[l])):
            ts.append((f"blk.{l}.{name}.weight", [k, rows], gt, _matrix(gt, rows, k, 100 * l + j).tobytes()))
    ts.append(("output_norm.weight", [D], 0, ones))
    ts.append(("output.weight", [D, V], orc.Q2_K, fx.random_blocks(orc.Q2_K, V, D, 2).tobytes()))
    return write_gguf(meta, ts)


@pytest.fixture(scope="module")
def mixed_model():
    return _mixed_gguf()


def test_mixed_model_embedding_rows_are_exact(mixed_model):
    from tests.gguf_reader import tensor_bytes
    eng = DecodeEngine(mixed_model, max_seq_len=16)
    rb = orc.row_bytes(orc.Q5_0, D)
    emb = tensor_bytes(mixed_model, "token_embd.weight")
    for tok in (0, 7, 123, V - 1):
        eng.embed(tok)
        assert np.array_equal(eng.hidden(), orc.dequant_row(orc.Q5_0, emb[tok * rb:(tok + 1) * rb], D)), tok
    eng.close()


def test_mixed_model_stepwise_parity_and_generation(mixed_model):
    eng = DecodeEngine(mixed_model, max_seq_len=64)
    ref = orc.OracleModel(mixed_model, kv_f16=True, max_seq=64, threads=THREADS)
    for pos, tok in enumerate([3, 150, 42, 299]):
        h = eng.forward_single_streaming(tok, pos)
        hr = ref.forward(tok, pos)
        assert np.abs(h - hr).max() <= 1e-3 * np.abs(hr).max(), pos
        lg, am = eng.compute_logits()
        lr = ref.logits(hr)
        assert np.abs(lg - lr).max() <= 1e-3 * np.abs(lr).max(), pos
        assert am == orc.argmax(lr)
    eng.close()
    prompt = [5, 17, 260]
    want, _, margins = orc.OracleModel(mixed_model, kv_f16=True, max_seq=64, threads=THREADS).generate(prompt, 20)
    eng = DecodeEngine(mixed_model, max_seq_len=64)
    assert eng.generate(prompt, 20).tolist() == want.tolist(), margins
    eng.close()


@pytest.mark.parametrize("embd_type", [orc.Q2_K, orc.Q3_K, orc.Q5_K, orc.Q6_K, orc.Q8_K])
def test_embedding_rows_of_every_format_are_exact(embd_type):
    # token_embd in each format: the row the engine decodes on the device (tiled
    # formats) or on the host (f32-held ones) equals the reference's dequantize
    from tests.gguf_reader import tensor_bytes
    g = _mixed_gguf(embd_type)
    eng = DecodeEngine(g, max_seq_len=16)
    rb = orc.row_bytes(embd_type, D)
    emb = tensor_bytes(g, "token_embd.weight")
    for tok in (0, 64, 199, V - 1):
        eng.embed(tok)
        assert np.array_equal(eng.hidden(), orc.dequant_row(embd_type, emb[tok * rb:(tok + 1) * rb], D)), tok
    eng.kv_reset()
    ref = orc.OracleModel(g, kv_f16=True, max_seq=16, threads=THREADS)
    h, hr = eng.forward_single_streaming(42, 0), ref.forward(42, 0)
    assert np.abs(h - hr).max() <= 1e-3 * np.abs(hr).max()
    lg, am = eng.compute_logits()
    lr = ref.logits(hr)
    assert np.abs(lg - lr).max() <= 1e-3 * np.abs(lr).max() and am == orc.argmax(lr)
    eng.close()
