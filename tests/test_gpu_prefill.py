"""GPU parity of the tensor-core batched GEMM (rf_qgemm) and of the batched
prompt path against the CPU oracle (the reference's token-by-token executor).

Tolerance of the GEMM: max|y - y_ref| <= 2e-4 * max|y_ref| + 1e-6 per token, the
GEMV bar; the operands are split into bf16 hi + lo (three products), which keeps
the error near 2^-16 of the reference's f32 products.
"""
import os

import numpy as np
import pytest

from oracle import oracle as orc
from ramforge_b200 import QMatrix, synth
from ramforge_b200 import _lib

pytestmark = pytest.mark.gpu
THREADS = min(32, os.cpu_count() or 8)


def _weights(gtype, M, K, seed):
    return synth.quantize(gtype, synth.normal(seed, 100 + gtype, M * K, std=0.02).reshape(M, K))


def _qgemm(gtype, M, K, T, seed=1):
    import torch
    raw = _weights(gtype, M, K, seed)
    x = synth.normal(seed, 9, T * K, std=1.0).reshape(T, K)
    m = QMatrix(gtype, raw, M, K)
    dx = torch.from_numpy(x).cuda()
    dy = torch.full((T, M), float("nan"), device="cuda")
    m.gemm(dx.data_ptr(), dy.data_ptr(), T)
    torch.cuda.synchronize()
    y = dy.cpu().numpy()
    w = _lib.ctypes.c_uint32()
    _lib.check(_lib.lib().rf_qgemm_error_word(_lib.ctypes.byref(w)))
    assert w.value == 0
    m.close()
    return raw, x, y


@pytest.mark.parametrize("gtype", [synth.Q4_K, synth.Q8_0])
@pytest.mark.parametrize("M,K,T", [(64, 256, 1), (130, 512, 7), (384, 1024, 128), (300, 768, 129),
                                   (4096, 4096, 200)])
def test_qgemm_matches_reference_matvec_per_token(gtype, M, K, T):
    raw, x, y = _qgemm(gtype, M, K, T)
    assert not np.isnan(y).any()
    worst = 0.0
    for t in range(T):
        ref = orc.matvec(gtype, raw, K, M, x[t], threads=THREADS)
        err = np.abs(y[t] - ref).max() / (np.abs(ref).max() + 1e-30)
        worst = max(worst, err)
        assert np.abs(y[t] - ref).max() <= 2e-4 * np.abs(ref).max() + 1e-6, (gtype, M, K, T, t, err)
    print(f"qgemm {gtype} {M}x{K} T={T}: worst relative error {worst:.2e}")


def test_qgemm_refuses_unsupported_formats():
    import torch
    raw = _weights(synth.Q4_0, 64, 256, 2)
    m = QMatrix(synth.Q4_0, raw, 64, 256)
    dx = torch.zeros(4, 256, device="cuda")
    dy = torch.zeros(4, 64, device="cuda")
    rc = _lib.lib().rf_qgemm(m._h, dx.data_ptr(), dy.data_ptr(), 4, None)
    assert rc == _lib.RF_EUNSUPPORTED
    m.close()


# ---- engine-level batched prefill (rf_prefill) ----------------------------------------
# Bars: logits after the prompt within 1e-3 max relative error of the token-by-token
# oracle; layer 0's committed K/V entries within two f16 steps of the oracle's (both
# are f16 roundings of projections that differ only by the GEMM's ~2^-16 relative
# error); deeper layers' K/V, which inherit the differences of the layers before,
# within the engine's per-layer bar of tests/test_gpu_engine.py (2e-3 of
# max(1, max|K|)); greedy tokens after the prompt identical to the oracle's.

def _kv_close(got, want):
    tol = 2.0 ** -9 * np.maximum(np.abs(want), 0.01 * np.abs(want).max())
    return bool((np.abs(got - want) <= tol).all()), float(np.abs(got - want).max())


def _check_prefill(spec, n_prompt, n_new, max_seq):
    from ramforge_b200 import DecodeEngine
    g = synth.gguf_bytes(spec)
    prompt = np.random.default_rng(spec.seed).integers(0, spec.vocab_size, n_prompt).tolist()
    ref = orc.OracleModel(g, kv_f16=True, max_seq=max_seq, threads=os.cpu_count() or 8)
    want, want_logits, margins = ref.generate(prompt, n_new, want_logits=True)
    eng = DecodeEngine(g, max_seq_len=max_seq)
    eng.prefill(prompt)
    assert eng.kv_seq_len == n_prompt
    lg, am = eng.compute_logits()
    err = float(np.abs(lg - want_logits[0]).max() / np.abs(want_logits[0]).max())
    assert err <= 1e-3, err
    assert am == want[0]
    for layer in range(spec.n_layers):
        for which in (False, True):
            a, b = eng.kv_read(layer, which, 0, n_prompt), ref.kv_read(layer, which, 0, n_prompt)
            if layer == 0:
                ok, worst = _kv_close(a, b)
                assert ok, (layer, which, worst)
            else:
                assert np.abs(a - b).max() <= 2e-3 * max(1.0, np.abs(b).max()), (layer, which)
    ref.close()
    # greedy continuation: prefill of all but the last prompt token, then the decode loop
    eng.kv_reset()
    got = eng.generate(prompt, n_new, batched_prefill=True)
    assert got.tolist() == want.tolist(), (np.nonzero(got != want)[0][:3], float(margins.min()))
    eng.close()


@pytest.mark.parametrize("spec", [
    # Q4_K layers, Q8_0 embedding/output, head_dim 64, GQA 4
    synth.scaled(synth.LLAMA3_8B, name="pf-q4k", vocab_size=1000, n_embd=512, n_layers=3, n_ff=1024, n_heads=8,
                 n_kv_heads=2, seed=31, context_length=512),
    # Q8_0 everywhere, head_dim 32
    synth.scaled(synth.TINYLLAMA, name="pf-q8", vocab_size=777, n_embd=256, n_layers=2, n_ff=512, n_heads=8,
                 n_kv_heads=2, seed=32, context_length=512),
    # qwen2 Q/K/V biases and V in its own type (Q8_0 beside Q4_K Q/K): the second QKV GEMM
    synth.scaled(synth.LLAMA3_8B, name="pf-qwen2", vocab_size=600, n_embd=512, n_layers=2, n_ff=1536, n_heads=8,
                 n_kv_heads=4, seed=33, context_length=512, arch="qwen2", qkv_bias_std=0.02, v_type=synth.Q8_0),
])
def test_prefill_matches_token_by_token_oracle(spec):
    # 300 prompt tokens: a full 256-token chunk and a ragged one
    _check_prefill(spec, 300, 12, max_seq=384)


def test_prefill_llama3_8b_width_bench_prompt():
    """The benchmark's 512-token prompt at Llama-3-8B width (dim 4096, 32/8 heads,
    FFN 14336, vocab 128256, Q4_K layers, Q8_0 embedding/output, seed 3), two of its
    layers: KV cache and logits after the batched prefill against the token-by-token
    oracle, then 24 greedy tokens."""
    spec = synth.scaled(synth.LLAMA3_8B, name="pf-llama3-2l", n_layers=2)
    _check_prefill(spec, 512, 24, max_seq=600)


def test_prefill_refuses_what_it_does_not_cover():
    from ramforge_b200 import DecodeEngine, RfError
    spec = synth.scaled(synth.TINYLLAMA, name="pf-q40", vocab_size=300, n_embd=256, n_layers=2, n_ff=512, n_heads=4,
                        n_kv_heads=4, seed=34, context_length=64, layer_type=synth.Q4_0)
    eng = DecodeEngine(synth.gguf_bytes(spec), max_seq_len=64)
    with pytest.raises(RfError, match="UNSUPPORTED"):
        eng.prefill([1, 2, 3])
    assert eng.kv_seq_len == 0  # nothing changed
    eng.forward_single_streaming(1, 0)  # the token-by-token path still serves it
    assert eng.kv_seq_len == 1
    with pytest.raises(RfError, match="INVAL"):
        eng.prefill([spec.vocab_size])
    eng.close()


def test_prefill_long_prompt_streams_attention():
    # 1100 prompt tokens: the attention of the later chunks serves contexts past
    # 1024 positions, where the streaming kernel runs, with per-token history offsets
    spec = synth.scaled(synth.LLAMA3_8B, name="pf-long", vocab_size=500, n_embd=512, n_layers=2, n_ff=1024, n_heads=8,
                        n_kv_heads=2, seed=35, context_length=2048)
    _check_prefill(spec, 1100, 8, max_seq=1200)
