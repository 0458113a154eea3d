"""The persistent step kernel (one cooperative launch per token, grid barriers
between phases) against the CPU oracle and against the multi-kernel step.

Each model below has a shape the step kernel is instantiated for; the same
bars as the other engine tests apply: greedy tokens identical to the oracle's,
logits within 1e-3 max relative error, final hidden state within 1e-3.
"""
import ctypes
import os

import numpy as np
import pytest

from oracle import oracle as orc
from ramforge_b200 import DecodeEngine, _lib, synth

pytestmark = pytest.mark.gpu
THREADS = min(32, os.cpu_count() or 8)
LOGIT_RTOL = 1e-3

# (layer type, LM-head type, head_dim, query heads per KV head)
STEP_MODELS = {
    "q4k-q80-hd128-g4": synth.scaled(synth.LLAMA3_8B, name="step-q4k", vocab_size=1000, n_embd=1024, n_layers=3,
                                     n_ff=1024, n_heads=8, n_kv_heads=2, seed=31, context_length=512),
    "q4k-q4k-hd128-g8": synth.scaled(synth.LLAMA3_70B, name="step-q4k-g8", vocab_size=700, n_embd=1024, n_layers=2,
                                     n_ff=512, n_heads=8, n_kv_heads=1, seed=32, context_length=512),
    "q80-hd64-g8": synth.scaled(synth.TINYLLAMA, name="step-q8-64", vocab_size=500, n_embd=512, n_layers=2,
                                n_ff=768, n_heads=8, n_kv_heads=1, seed=33, context_length=256),
    "q80-hd128-g4": synth.scaled(synth.TINYLLAMA, name="step-q8-128", vocab_size=600, n_embd=512, n_layers=2,
                                 n_ff=512, n_heads=4, n_kv_heads=1, seed=34, context_length=256),
}


@pytest.fixture(scope="module")
def models():
    return {k: synth.gguf_bytes(s) for k, s in STEP_MODELS.items()}


def rel_err(a, b):
    return float(np.abs(a - b).max() / max(np.abs(b).max(), 1e-30))


@pytest.mark.parametrize("name", list(STEP_MODELS))
def test_step_kernel_is_used_and_can_be_turned_off(models, name):
    eng = DecodeEngine(models[name], max_seq_len=64)
    assert not eng.step_kernel_active  # opt-in
    eng.set_step_kernel(True)
    assert eng.step_kernel_active
    assert eng.step_kernel_count == 1
    eng.set_step_kernel(False)
    assert not eng.step_kernel_active
    assert eng.step_kernel_count == 5 * STEP_MODELS[name].n_layers + 4
    eng.close()


def test_step_kernel_not_used_for_uninstantiated_shapes():
    spec = synth.scaled(synth.TINYLLAMA, name="hd32", vocab_size=300, n_embd=256, n_layers=1, n_ff=512,
                        n_heads=8, n_kv_heads=2, seed=35)
    eng = DecodeEngine(synth.gguf_bytes(spec), max_seq_len=32)
    eng.set_step_kernel(True)
    assert not eng.step_kernel_active  # head_dim 32
    eng.close()
    g = synth.gguf_bytes(STEP_MODELS["q80-hd64-g8"])
    eng = DecodeEngine(g, max_seq_len=32, kv_f32=True)
    eng.set_step_kernel(True)
    assert not eng.step_kernel_active  # f32 KV cache
    eng.close()


@pytest.mark.parametrize("name", list(STEP_MODELS))
def test_step_kernel_generate_matches_oracle_and_multi_kernel_path(models, name):
    g = models[name]
    vocab = STEP_MODELS[name].vocab_size
    prompt = np.random.default_rng(7).integers(0, vocab, 9).tolist()
    want, _, margins = orc.OracleModel(g, kv_f16=True, max_seq=96, threads=THREADS).generate(prompt, 40)
    eng = DecodeEngine(g, max_seq_len=96)
    eng.set_step_kernel(True)
    assert eng.step_kernel_active
    got = eng.generate(prompt, 40)
    assert got.tolist() == want.tolist(), (np.nonzero(got != want)[0][:3], margins.min())
    eng.kv_reset()
    eng.set_step_kernel(False)
    assert eng.generate(prompt, 40).tolist() == want.tolist()
    eng.close()


@pytest.mark.parametrize("name", ["q4k-q80-hd128-g4", "q80-hd64-g8"])
def test_step_kernel_forward_hidden_and_logits(models, name):
    """Forward steps through the step kernel (final RMSNorm into final_hidden), then
    the LM head on that state, against the oracle at every position."""
    g = models[name]
    vocab = STEP_MODELS[name].vocab_size
    eng = DecodeEngine(g, max_seq_len=64)
    eng.set_step_kernel(True)
    ref = orc.OracleModel(g, kv_f16=True, max_seq=64, threads=THREADS)
    toks = np.random.default_rng(8).integers(0, vocab, 12).tolist()
    for pos, t in enumerate(toks):
        h = eng.forward_single_streaming(t, pos)
        hr = ref.forward(t, pos)
        assert rel_err(h, hr) < 1e-3, (pos, rel_err(h, hr))
        lg, am = eng.compute_logits()
        lr = ref.logits(hr)
        assert rel_err(lg, lr) <= LOGIT_RTOL
        assert am == orc.argmax(lr)
    eng.close()


def test_step_kernel_long_context_attention_splits(models):
    """The history grows through several split counts (about 64 positions per
    split), so partial merges of 2..3 splits run inside the step kernel."""
    g = models["q80-hd128-g4"]
    prompt = np.random.default_rng(9).integers(0, 600, 150).tolist()
    want = orc.OracleModel(g, kv_f16=True, max_seq=256, threads=THREADS).generate(prompt, 20)[0]
    eng = DecodeEngine(g, max_seq_len=256)
    eng.set_step_kernel(True)
    assert eng.generate(prompt, 20).tolist() == want.tolist()
    eng.close()


def test_barrier_wait_is_bounded_and_reported():
    L = _lib.lib()
    err = ctypes.c_uint32(7)
    _lib.check(L.rf_selftest_barrier(0, 0, ctypes.byref(err)))
    assert err.value == 0  # every CTA arrived: no wait gave up
    _lib.check(L.rf_selftest_barrier(0, 1, ctypes.byref(err)))
    assert err.value == 1  # one expected arrival never came: the wait gave up and said so
    _lib.check(L.rf_selftest_barrier(0, 0, ctypes.byref(err)))
    assert err.value == 0  # the device is still usable
