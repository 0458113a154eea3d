"""qwen2 Q/K/V biases and mixed-format layers on the engine, through the C ABI.

The biased fixture is the reference's own (inference.rs:1620-2077): one f32 layer
with Q/K/V biases, checked against the oracle and the restated reference forward
with the reference's bound (2e-4 on hidden state and logits).  Partial bias sets
and wrong bias shapes are refused at layer load with nothing charged
(streaming_model.rs:3256-3330).  The mixed model is laid out like a Q4_K_M file:
Q4_K Q/K/O/gate/up, Q6_K V, down and LM head, plus biases; V then runs as its own
matrix beside the [Q;K] one.  Bars as everywhere: greedy tokens identical to the
oracle, logits within 1e-3 relative, streamed layers bit-identical to resident.
"""
import os

import numpy as np
import pytest

from oracle import oracle as orc
from ramforge_b200 import DecodeEngine, RfError, _lib, synth
from tests import fixtures as fx
from tests.gguf_reader import read_tensors

pytestmark = pytest.mark.gpu
THREADS = min(32, os.cpu_count() or 8)

MIX = synth.scaled(synth.LLAMA3_8B, name="qwen2-mix", arch="qwen2", vocab_size=640, n_embd=512, n_layers=3,
                   n_ff=1024, n_heads=8, n_kv_heads=2, seed=25, context_length=256, v_type=synth.Q6_K,
                   down_type=synth.Q6_K, out_type=synth.Q6_K, qkv_bias_std=0.5)


@pytest.fixture(scope="module")
def mix():
    return synth.gguf_bytes(MIX)


def rel_err(a, b):
    return float(np.abs(a - b).max() / max(np.abs(b).max(), 1e-30))


def test_biased_fixture_matches_oracle_and_reference_forward():
    g = fx.qwen2_bias_gguf()
    eng = DecodeEngine(g, max_seq_len=8, kv_f32=True)
    ref = orc.OracleModel(g, kv_f16=False, max_seq=8)
    w = fx.qwen2_bias_weights()
    kh, vh = [], []
    for tok, pos in [(1, 0), (5, 1)]:
        h = eng.forward_single_streaming(tok, pos)
        ref_h = fx.qwen2_bias_reference_forward(w, tok, pos, kh, vh)
        assert np.abs(h - ref.forward(tok, pos)).max() < 2e-4
        assert np.abs(h - ref_h).max() < 2e-4, (pos, h, ref_h)
        lg, _ = eng.compute_logits()
        assert np.abs(lg - w["embd"].reshape(fx.QB_VOCAB, fx.QB_N_EMBD) @ ref_h).max() < 2e-4
    eng.close()
    want = orc.OracleModel(g, kv_f16=True, max_seq=16).generate([1, 3], 4)[0].tolist()
    eng = DecodeEngine(g, max_seq_len=16)
    assert eng.generate([1, 3], 4).tolist() == want
    eng.kv_reset()
    assert eng.generate([1, 3], 4).tolist() == want  # deterministic (inference.rs:2079-2087)
    eng.close()


@pytest.mark.parametrize("mode,match", [("only_q", "incomplete Q/K/V bias"), ("wrong_dim", "attn_q.bias shape")])
def test_bad_bias_sets_are_refused_without_leaking_charges(mode, match):
    bad = fx.qwen2_bias_gguf(mode)
    with pytest.raises(RfError, match=match):
        DecodeEngine(bad, max_seq_len=8)
    eng = DecodeEngine(fx.qwen2_bias_gguf(), max_seq_len=8)
    eng.release_layer(0)
    used = eng.budget_used
    ts = read_tensors(bad)
    views = {}
    for name in _lib.LAYER_VIEW_NAMES:
        key = f"blk.0.{name}" if name.endswith(".bias") else f"blk.0.{name}.weight"
        if key in ts:
            t = ts[key]
            views[name] = (t["type"], t["dims"][0], t["dims"][1] if len(t["dims"]) > 1 else 1, t["data"])
    with pytest.raises(RfError, match=match):
        eng.load_layer_views(0, views)
    assert eng.budget_used == used and not eng.layer_is_resident(0)
    eng.close()


def test_mixed_format_biased_model_stepwise_parity(mix):
    eng = DecodeEngine(mix, max_seq_len=64)
    ref = orc.OracleModel(mix, kv_f16=True, max_seq=64, threads=THREADS)
    seq = [7, 301, 55, 610, 2]
    for pos in range(len(seq) + 6 - 1):
        h = eng.forward_single_streaming(seq[pos], pos)
        hr = ref.forward(seq[pos], pos)
        assert rel_err(h, hr) < 1e-3, (pos, rel_err(h, hr))
        if pos >= 4:
            lg, am = eng.compute_logits()
            lr = ref.logits(hr)
            assert rel_err(lg, lr) <= 1e-3, (pos, rel_err(lg, lr))
            assert am == orc.argmax(lr)
            seq.append(am)
    eng.close()


@pytest.mark.parametrize("graphs", [True, False])
def test_mixed_format_biased_model_generation(mix, graphs):
    prompt = [11, 402, 7, 600, 3]
    want, _, margins = orc.OracleModel(mix, kv_f16=True, max_seq=64, threads=THREADS).generate(prompt, 24)
    eng = DecodeEngine(mix, max_seq_len=64, disable_graphs=not graphs)
    assert eng.generate(prompt, 24).tolist() == want.tolist(), margins
    eng.close()


def test_mixed_format_launch_count(mix):
    eng = DecodeEngine(mix, max_seq_len=16)
    L = MIX.n_layers
    assert eng.step_kernel_count == 6 * L + 4  # the V matrix is a sixth launch a layer
    eng.close()


def test_mixed_format_ring_is_bit_identical_to_resident(mix):
    a = DecodeEngine(mix, max_seq_len=32)
    b = DecodeEngine(mix, max_seq_len=32)
    b.set_residency_plan([True, False, False], ring_slots=2)
    for pos, tok in enumerate([5, 77, 301, 12]):
        assert np.array_equal(a.forward_single_streaming(tok, pos), b.forward_single_streaming(tok, pos)), pos
    assert b.residency_stats()["ring_copies"] == 4 * 2
    a.close()
    b.close()
