"""GPU parity of the decode engine against the CPU oracle (the reference's
executor restated), through the C ABI.

Bars: final logits within 1e-3 max relative error,
measured as max|l - l_ref| / max|l_ref| per step; greedy token sequences
identical; embedding rows bit-exact; KV entries within f16 rounding of the
oracle's (K/V come out of differently-ordered f32 sums before rounding).
"""
import os

import numpy as np
import pytest

from oracle import oracle as orc
from ramforge_b200 import DecodeEngine, RfError, _lib, synth
from tests import fixtures as fx

pytestmark = pytest.mark.gpu
THREADS = min(32, os.cpu_count() or 8)
LOGIT_RTOL = 1e-3

SMALL_Q4K = synth.scaled(synth.LLAMA3_8B, name="small-q4k", vocab_size=1000, n_embd=512, n_layers=3, n_ff=1024,
                         n_heads=8, n_kv_heads=2, seed=21, context_length=512)
SMALL_Q8 = synth.scaled(synth.TINYLLAMA, name="small-q8", vocab_size=777, n_embd=256, n_layers=2, n_ff=512,
                        n_heads=8, n_kv_heads=2, seed=22, context_length=256)
SMALL_Q40 = synth.scaled(synth.TINYLLAMA, name="small-q40", vocab_size=500, n_embd=256, n_layers=2, n_ff=640,
                         n_heads=4, n_kv_heads=4, seed=23, context_length=256, layer_type=synth.Q4_0,
                         embd_type=synth.Q4_0, out_type=-1)
# Q6_K everywhere: every GEMV epilogue, the embedding row and the LM head in Q6_K
SMALL_Q6K = synth.scaled(synth.LLAMA3_8B, name="small-q6k", vocab_size=700, n_embd=512, n_layers=2, n_ff=1536,
                         n_heads=8, n_kv_heads=2, seed=24, context_length=256, layer_type=synth.Q6_K,
                         embd_type=synth.Q6_K, out_type=synth.Q6_K)


@pytest.fixture(scope="module")
def models():
    return {s.name: synth.gguf_bytes(s) for s in (SMALL_Q4K, SMALL_Q8, SMALL_Q40, SMALL_Q6K)}


def rel_err(a, b):
    return float(np.abs(a - b).max() / max(np.abs(b).max(), 1e-30))


def check_stepwise(gguf, prompt, n_new, kv_f32=False, max_seq=256, engine_kw=None):
    """forward + logits per step through the ABI vs the oracle; returns tokens."""
    eng = DecodeEngine(gguf, max_seq_len=max_seq, kv_f32=kv_f32, **(engine_kw or {}))
    ref = orc.OracleModel(gguf, kv_f16=not kv_f32, max_seq=max_seq, threads=THREADS)
    toks, pos = [], 0
    seq = list(prompt)
    worst = 0.0
    for i in range(len(prompt) + n_new - 1):
        tok = seq[i]
        h = eng.forward_single_streaming(tok, pos)
        hr = ref.forward(tok, pos)
        assert rel_err(h, hr) < 1e-3, (i, rel_err(h, hr))
        pos += 1
        if i >= len(prompt) - 1:
            lg, am = eng.compute_logits()
            lr = ref.logits(hr)
            e = rel_err(lg, lr)
            worst = max(worst, e)
            assert e <= LOGIT_RTOL, (i, e)
            assert am == orc.argmax(lr), (i, am, orc.argmax(lr))
            assert am == int(np.argmax(lg))
            seq.append(am)
            toks.append(am)
    eng.close()
    return toks, worst


def test_gqa_fixture_matches_oracle_and_reference_forward():
    g = fx.gqa_gguf()
    eng = DecodeEngine(g, max_seq_len=8)
    assert eng.config["head_dim"] == 2 and eng.config["vocab_size"] == 16
    ref = orc.OracleModel(g, kv_f16=True, max_seq=8)
    w = fx.gqa_weights()
    kh, vh = [], []
    for tok, pos in [(3, 0), (7, 1), (11, 2)]:
        h = eng.forward_single_streaming(tok, pos)
        assert np.abs(h - ref.forward(tok, pos)).max() < 2e-4
        assert np.abs(h - fx.gqa_reference_forward(w, tok, pos, kh, vh)).max() < 2e-4  # inference.rs EPS
        lg, am = eng.compute_logits()
        assert np.abs(lg - ref.logits(h)).max() < 2e-4
    eng.close()


def test_kv_invariants_across_prompt_and_decode():  # inference.rs:2879-3003
    eng = DecodeEngine(fx.gqa_gguf(), max_seq_len=16)
    kvd = eng.config["n_kv_heads"] * eng.config["head_dim"]
    seq, pos = [1, 3, 5, 7], 0
    for _ in range(len(seq) + 3):
        assert eng.kv_seq_len == pos
        eng.forward_single_streaming(seq[pos], pos)
        assert eng.kv_seq_len == pos + 1
        for which in (False, True):
            assert eng.kv_read(0, which, 0, pos + 1).shape == (pos + 1, kvd)
        if pos >= len(seq) - 1:
            seq.append(eng.compute_logits()[1])
        pos += 1
    eng.close()


def test_gqa_fixture_greedy_generation():
    g = fx.gqa_gguf()
    ref = orc.OracleModel(g, kv_f16=True, max_seq=32).generate([1, 3], 12)[0]
    eng = DecodeEngine(g, max_seq_len=32)
    assert eng.generate([1, 3], 12).tolist() == ref.tolist()
    eng.kv_reset()
    assert eng.generate([1, 3], 12).tolist() == ref.tolist()  # deterministic (inference.rs:2567-2571)


# KV capacity 1024 makes the engine use the streaming attention kernel (the
# register-load kernel serves engines whose capacity is below 1024 positions)
@pytest.mark.parametrize("max_seq", [256, 1024])
@pytest.mark.parametrize("name", ["small-q4k", "small-q8", "small-q40", "small-q6k"])
def test_small_models_stepwise_parity(models, name, max_seq):
    g = models[name]
    rng = np.random.default_rng(5)
    prompt = rng.integers(0, orc.OracleModel(g, max_seq=4).config["vocab_size"], 6).tolist()
    toks, worst = check_stepwise(g, prompt, 10, max_seq=max_seq)
    assert len(toks) == 10


def test_kv_f32_mode_matches_reference_cache(models):
    g = models["small-q4k"]
    check_stepwise(g, [1, 2, 3], 6, kv_f32=True)


@pytest.mark.parametrize("max_seq", [128, 1024])
@pytest.mark.parametrize("graphs", [True, False])
def test_generate_matches_oracle_greedy(models, graphs, max_seq):
    g = models["small-q4k"]
    prompt = [5, 17, 99, 3]
    ref = orc.OracleModel(g, kv_f16=True, max_seq=max_seq, threads=THREADS)
    want, _, margins = ref.generate(prompt, 40)
    eng = DecodeEngine(g, max_seq_len=max_seq, disable_graphs=not graphs)
    got = eng.generate(prompt, 40)
    assert got.tolist() == want.tolist(), (got, want, margins)
    assert eng.kv_seq_len == len(prompt) + 40 - 1
    eng.close()


def test_decode_step_api_matches_generate(models):
    g = models["small-q8"]
    prompt = [3, 4, 5]
    eng = DecodeEngine(g, max_seq_len=64)
    ref = eng.generate(prompt, 12).tolist()
    eng.kv_reset()
    for t in prompt[:-1]:
        eng.forward_single_streaming(t, eng.kv_seq_len, want_hidden=False)
    tok, got = prompt[-1], []
    for _ in range(12):
        tok = eng.decode_step(tok)
        got.append(tok)
    assert got == ref
    eng.close()


def test_layer_level_api_matches_oracle(models):
    """embed -> execute_layer per layer -> commit, compared per layer (hidden) and KV."""
    g = models["small-q4k"]
    eng = DecodeEngine(g, max_seq_len=16)
    ref = orc.OracleModel(g, kv_f16=True, max_seq=16, threads=THREADS)
    L = eng.config["n_layers"]
    for pos, tok in enumerate([9, 8, 7]):
        ref.forward(tok, pos)
        ref_layers = ref.layer_hiddens()
        eng.embed(tok)
        emb = eng.hidden()
        rb = orc.row_bytes(orc.Q8_0, eng.config["n_embd"])
        assert np.array_equal(emb, orc.dequant_row(orc.Q8_0, _tensor_bytes(g, "token_embd.weight")[tok * rb:], eng.config["n_embd"]))
        for l in range(L):
            eng.execute_layer(l, pos)
            assert rel_err(eng.hidden(), ref_layers[l]) < 1e-3, (pos, l)
        eng.kv_commit()
        for l in range(L):
            for which in (False, True):
                a = eng.kv_read(l, which, 0, pos + 1)
                b = ref.kv_read(l, which, 0, pos + 1)
                assert np.abs(a - b).max() <= 2e-3 * max(1.0, np.abs(b).max()), (pos, l, which)
    eng.close()


@pytest.mark.parametrize("graphs", [True, False])
def test_q6_k_model_embedding_rows_and_greedy_generation(models, graphs):
    g = models["small-q6k"]
    eng = DecodeEngine(g, max_seq_len=64, disable_graphs=not graphs)
    d = eng.config["n_embd"]
    rb = orc.row_bytes(orc.Q6_K, d)
    emb = _tensor_bytes(g, "token_embd.weight")
    for tok in (0, 1, 345, eng.config["vocab_size"] - 1):
        eng.embed(tok)
        assert np.array_equal(eng.hidden(), orc.dequant_row(orc.Q6_K, emb[tok * rb:(tok + 1) * rb], d)), tok
    eng.kv_reset()
    prompt = [11, 402, 7, 650, 3]
    want, _, margins = orc.OracleModel(g, kv_f16=True, max_seq=64, threads=THREADS).generate(prompt, 24)
    got = eng.generate(prompt, 24)
    assert got.tolist() == want.tolist(), (got, want, margins)
    eng.close()


def _tensor_bytes(g, name):
    from tests.gguf_reader import tensor_bytes
    return tensor_bytes(g, name)


def test_layer_load_views_equals_gguf_load(models):
    from tests.gguf_reader import read_tensors
    g = models["small-q4k"]
    ts = read_tensors(g)
    a = DecodeEngine(g, max_seq_len=16)
    b = DecodeEngine(g, max_seq_len=16)
    for l in range(b.config["n_layers"]):
        b.release_layer(l)
        assert not b.layer_is_resident(l)
        views = {}
        for role in _lib.ROLE_NAMES:
            t = ts[f"blk.{l}.{role}.weight"]
            views[role] = (t["type"], t["dims"][0], t["dims"][1] if len(t["dims"]) > 1 else 1, t["data"])
        b.load_layer_views(l, views)
        assert b.layer_is_resident(l)
    ha = a.forward_single_streaming(4, 0)
    hb = b.forward_single_streaming(4, 0)
    assert np.array_equal(ha, hb)
    a.close()
    b.close()


def test_budget_accounting_and_release(models):
    g = models["small-q4k"]
    eng = DecodeEngine(g, max_seq_len=16)
    used = eng.budget_used
    assert used > 0 and eng.budget_available == eng.budget_total - used
    eng.release_layer(1)
    assert eng.budget_used < used
    with pytest.raises(RfError) as ei:
        eng.execute_layer(1, 0)
    assert ei.value.code == _lib.RF_ESTATE
    eng.load_layer(1)
    assert eng.budget_used == used
    with pytest.raises(RfError) as ei:
        eng.load_layer(1)
    assert ei.value.code == _lib.RF_ESTATE
    eng.close()


def test_budget_too_small_fails_cleanly(models):
    with pytest.raises(RfError) as ei:
        DecodeEngine(models["small-q4k"], max_seq_len=16, vram_budget_bytes=1 << 20)
    assert ei.value.code == _lib.RF_ENOMEM


def test_position_token_and_capacity_errors(models):
    g = models["small-q8"]
    eng = DecodeEngine(g, max_seq_len=3)
    with pytest.raises(RfError) as ei:
        eng.forward_single_streaming(1, 1)  # streaming_model.rs:921 position/history mismatch
    assert ei.value.code == _lib.RF_EINVAL
    with pytest.raises(RfError) as ei:
        eng.forward_single_streaming(10 ** 6, 0)
    assert ei.value.code == _lib.RF_EINVAL
    for p in range(3):
        eng.forward_single_streaming(1, p)
    with pytest.raises(RfError) as ei:
        eng.forward_single_streaming(1, 3)
    assert ei.value.code == _lib.RF_ESTATE  # KV cache full (kv_cache.rs:388)
    eng.close()


def test_residency_plan_streams_nonresident_layers(models):
    g = models["small-q4k"]
    a = DecodeEngine(g, max_seq_len=16)
    b = DecodeEngine(g, max_seq_len=16)
    b.set_residency_plan([True, False, True])
    assert not b.layer_is_resident(1)
    for pos, tok in enumerate([1, 2, 3, 4]):
        assert np.array_equal(a.forward_single_streaming(tok, pos), b.forward_single_streaming(tok, pos))
    st = b.residency_stats()
    assert st["cache_misses"] == 4 and st["layer_releases"] >= 5 and st["evictions"] == 1
    assert not b.layer_is_resident(1)
    a.close()
    b.close()


def test_tinyllama_config1_greedy_parity():
    """TinyLlama shape, Q8_0 everywhere: 32 seeded prompt tokens + 128 greedy tokens."""
    g = synth.gguf_bytes(synth.TINYLLAMA)
    prompt = np.random.default_rng(0).integers(0, 32000, 32).tolist()
    ref = orc.OracleModel(g, kv_f16=True, max_seq=256, threads=THREADS)
    want, want_logits, margins = ref.generate(prompt, 128, want_logits=True)
    eng = DecodeEngine(g, max_seq_len=256)
    got = eng.generate(prompt, 128)
    assert got.tolist() == want.tolist(), (np.nonzero(got != want)[0][:3], margins.min())
    # logits on a prefix of the run through the stepwise API
    eng.kv_reset()
    for p, t in enumerate(prompt):
        eng.forward_single_streaming(t, p, want_hidden=False)
    for i in range(8):
        lg, am = eng.compute_logits()
        assert rel_err(lg, want_logits[i]) <= LOGIT_RTOL
        assert am == want[i]
        eng.forward_single_streaming(int(want[i]), len(prompt) + i, want_hidden=False)
    eng.close()


def test_llama3_8b_config4_short_parity():
    """Llama-3-8B shape (Q4_K layers, Q8_0 embedding/output): 12 prompt + 8 greedy tokens."""
    g = synth.gguf_bytes(synth.LLAMA3_8B)
    prompt = np.random.default_rng(3).integers(0, 128256, 12).tolist()
    ref = orc.OracleModel(g, kv_f16=True, max_seq=64, threads=THREADS)
    want, want_logits, margins = ref.generate(prompt, 8, want_logits=True)
    eng = DecodeEngine(g, max_seq_len=64)
    got = eng.generate(prompt, 8)
    assert got.tolist() == want.tolist(), (got, want, margins)
    eng.kv_reset()
    for p, t in enumerate(prompt):
        eng.forward_single_streaming(t, p, want_hidden=False)
    lg, am = eng.compute_logits()
    assert rel_err(lg, want_logits[0]) <= LOGIT_RTOL and am == want[0]
    eng.close()


def test_llama3_8b_width_bench_context_parity():
    """The benchmark's decode context: Llama-3-8B width (dim 4096, 32/8 heads, FFN
    14336, vocab 128256, Q4_K layers, Q8_0 embedding/output, seed 3) with 4 of its
    layers, the benchmark's 512-token prompt, then 64 greedy tokens, out to context
    576.  Attention there runs ~9 context splits with the current position's K/V
    taken from the step, the path the timed decode uses.  Tokens from rf_generate
    (the decode graph) must equal the oracle's; logits of every generated step,
    through the stepwise API, within 1e-3."""
    spec = synth.scaled(synth.LLAMA3_8B, name="llama-3-8b-4l", n_layers=4)
    g = synth.gguf_bytes(spec)
    prompt = np.random.default_rng(3).integers(0, spec.vocab_size, 512).tolist()
    n_new = 64
    ref = orc.OracleModel(g, kv_f16=True, max_seq=600, threads=os.cpu_count() or 8)
    want, want_logits, margins = ref.generate(prompt, n_new, want_logits=True)
    ref.close()
    eng = DecodeEngine(g, max_seq_len=600)
    got = eng.generate(prompt, n_new)
    assert got.tolist() == want.tolist(), (np.nonzero(got != want)[0][:3], float(margins.min()))
    eng.kv_reset()
    for p, t in enumerate(prompt):
        eng.forward_single_streaming(t, p, want_hidden=False)
    worst = 0.0
    for i in range(n_new):
        lg, am = eng.compute_logits()
        e = rel_err(lg, want_logits[i])
        worst = max(worst, e)
        assert e <= LOGIT_RTOL, (i, e)
        assert am == want[i], (i, am, want[i])
        eng.forward_single_streaming(int(want[i]), len(prompt) + i, want_hidden=False)
    assert eng.kv_seq_len == len(prompt) + n_new
    eng.close()
