"""The out-of-core ring: layers the residency plan leaves out are streamed each
step from pinned host images into a few device slots (cudaMemcpyAsync on a side
stream, event-ordered against the layers' kernels).

The streamed layers run the same kernels on the same packed bytes as resident
ones, so hidden states and tokens must be bit-identical to an all-resident
engine; against the CPU oracle the usual bars hold (greedy tokens identical,
logits within 1e-3).
"""
import os

import numpy as np
import pytest

from oracle import oracle as orc
from ramforge_b200 import DecodeEngine, RfError, synth

pytestmark = pytest.mark.gpu
THREADS = min(32, os.cpu_count() or 8)

RING_MODEL = synth.scaled(synth.LLAMA3_8B, name="ring-q4k", vocab_size=900, n_embd=512, n_layers=6, n_ff=1024,
                          n_heads=8, n_kv_heads=2, seed=41, context_length=256)


@pytest.fixture(scope="module")
def gguf():
    return synth.gguf_bytes(RING_MODEL)


@pytest.mark.parametrize("slots,mask", [(2, [True, False, False, True, False, False]),
                                        (1, [False] * 6),
                                        (3, [False, True, False, False, False, True])])
def test_ring_steps_are_bit_identical_to_resident(gguf, slots, mask):
    a = DecodeEngine(gguf, max_seq_len=32)
    b = DecodeEngine(gguf, max_seq_len=32)
    b.set_residency_plan(mask, ring_slots=slots)
    streamed = mask.count(False)
    for pos, tok in enumerate([5, 77, 301, 12, 640]):
        ha = a.forward_single_streaming(tok, pos)
        hb = b.forward_single_streaming(tok, pos)
        assert np.array_equal(ha, hb), pos
        for i, r in enumerate(mask):
            assert b.layer_is_resident(i) == r
    st = b.residency_stats()
    assert st["ring_copies"] == 5 * streamed
    assert st["cache_misses"] == 5 * streamed
    assert st["host_image_bytes"] > 0
    a.close()
    b.close()


def test_ring_generate_matches_oracle_and_resident(gguf):
    prompt = np.random.default_rng(5).integers(0, RING_MODEL.vocab_size, 7).tolist()
    want, _, margins = orc.OracleModel(gguf, kv_f16=True, max_seq=64, threads=THREADS).generate(prompt, 24)
    eng = DecodeEngine(gguf, max_seq_len=64)
    eng.set_residency_plan([False, False, True, False, False, False], ring_slots=2)
    got = eng.generate(prompt, 24)
    assert got.tolist() == want.tolist(), (np.nonzero(got != want)[0][:3], margins.min())
    assert eng.residency_stats()["ring_copies"] == 5 * (len(prompt) + 24 - 1)
    eng.close()


def test_ring_slots_are_charged_to_the_budget(gguf):
    eng = DecodeEngine(gguf, max_seq_len=16)
    used0 = eng.budget_used
    eng.set_residency_plan([True] * 3 + [False] * 3, ring_slots=2)
    used1 = eng.budget_used  # three layers released
    eng.forward_single_streaming(3, 0)
    used2 = eng.budget_used  # two ring slots allocated on first use
    assert used1 < used0 and used2 > used1
    slot = (used2 - used1) // 2
    assert slot >= (used0 - used1) // 3  # a slot holds a whole layer image
    eng.close()


def test_ring_plan_over_budget_fails_cleanly(gguf):
    eng = DecodeEngine(gguf, max_seq_len=16)
    with pytest.raises(RfError):
        eng.set_residency_plan([False] * 6, ring_slots=4, vram_weight_budget_bytes=1 << 20)
    # the engine is unchanged and still steps
    h = eng.forward_single_streaming(7, 0)
    assert np.isfinite(h).all()
    eng.close()


@pytest.mark.parametrize("slots", [2, 0])
def test_file_engine_reads_streamed_layers_through_coalesced_ranges(gguf, tmp_path, slots):
    """An engine created from a path reads each streamed layer's tensors with the
    coalesced read plan (layer_read.rs:50) into pinned staging: through the ring
    (slots 2: once, into the layer's pinned image) or load -> compute -> release
    (slots 0: every step).  Steps stay bit-identical to an all-resident engine."""
    path = tmp_path / "ring.gguf"
    path.write_bytes(np.asarray(gguf).tobytes())
    a = DecodeEngine(gguf, max_seq_len=32)
    b = DecodeEngine(str(path), max_seq_len=32)
    mask = [True, False, True, False, False, True]
    b.set_residency_plan(mask, ring_slots=slots)
    steps = [5, 77, 301]
    for pos, tok in enumerate(steps):
        assert np.array_equal(a.forward_single_streaming(tok, pos), b.forward_single_streaming(tok, pos)), pos
    st = b.residency_stats()
    reads_per_pass = 3 if slots else 3 * len(steps)
    assert st["file_reads"] >= reads_per_pass  # at least one read per streamed layer and pass
    assert st["file_read_bytes"] > 0 and st["file_gap_bytes"] < st["file_read_bytes"] // 100
    a.close()
    b.close()


def _layer_bytes(gguf):
    eng = DecodeEngine(gguf, max_seq_len=16)
    used_all = eng.budget_used
    eng.set_residency_plan([False] * RING_MODEL.n_layers)
    per_layer = (used_all - eng.budget_used) // RING_MODEL.n_layers
    eng.close()
    return per_layer


def test_planner_maps_a_weight_budget_onto_a_resident_prefix(gguf):
    per = _layer_bytes(gguf)
    a = DecodeEngine(gguf, max_seq_len=32)
    b = DecodeEngine(gguf, max_seq_len=32)
    assert b.plan_residency(0) == [True] * 6  # no budget: everything resident
    mask = b.plan_residency(int(per * 4.5), ring_slots=2)  # two slots + two layers fit
    assert mask == [True, True, False, False, False, False]
    for pos, tok in enumerate([5, 77, 301]):
        assert np.array_equal(a.forward_single_streaming(tok, pos), b.forward_single_streaming(tok, pos)), pos
    assert b.residency_stats()["ring_copies"] == 3 * 4
    with pytest.raises(RfError, match="NOMEM"):
        b.plan_residency(int(per * 1.5), ring_slots=2)  # the slots alone exceed the budget
    a.close()
    b.close()


@pytest.mark.parametrize("cached_layers", [2.5, 6.5])
def test_layer_cache_keeps_streamed_layers_least_recently_used_first(gguf, cached_layers):
    per = _layer_bytes(gguf)
    a = DecodeEngine(gguf, max_seq_len=32)
    b = DecodeEngine(gguf, max_seq_len=32)
    b.set_residency_plan([False] * 6, ring_slots=0)  # load -> compute -> release
    b.set_layer_cache(int(per * cached_layers))
    st0 = b.residency_stats()  # the plan's own releases count as evictions too
    for pos, tok in enumerate([5, 77, 301, 9]):
        assert np.array_equal(a.forward_single_streaming(tok, pos), b.forward_single_streaming(tok, pos)), pos
    st = {k: v - st0[k] for k, v in b.residency_stats().items()}
    if cached_layers > 6:  # every layer stays after the first step: later steps hit
        assert st["cache_misses"] == 6 and st["evictions"] == 0
        assert all(b.layer_is_resident(i) for i in range(6))
    else:  # a cyclic pass over six layers through a two-layer LRU misses every time
        assert st["cache_misses"] == 4 * 6 and st["evictions"] == 4 * 6 - 2
        assert sum(b.layer_is_resident(i) for i in range(6)) == 2
    a.close()
    b.close()


def test_persistent_tensors_over_a_quarter_of_the_budget_stay_in_host_memory():
    """should_keep_resident (persistent.rs:468) under an explicit VRAM budget: a
    token_embd/output larger than a quarter of it is held in mapped pinned host
    memory and read over the host link by the same kernels; tokens are the ones an
    unconstrained engine produces, and less device memory is charged."""
    spec = synth.scaled(synth.LLAMA3_8B, name="host-lm", vocab_size=16000, n_embd=256, n_layers=2, n_ff=512,
                        n_heads=4, n_kv_heads=2, seed=43, context_length=64)
    g = synth.gguf_bytes(spec)
    a = DecodeEngine(g, max_seq_len=32)
    lm = 16000 * 256 * 34 // 32  # Q8_0 bytes of each of token_embd and output
    budget = a.budget_used - 2 * lm + (1 << 20)
    assert lm > budget // 4
    b = DecodeEngine(g, max_seq_len=32, vram_budget_bytes=budget)
    st = b.residency_stats()
    assert st["host_mapped_bytes"] >= 2 * lm
    assert b.budget_used < a.budget_used - lm
    prompt = [3, 1000, 15000, 7]
    assert b.generate(prompt, 16).tolist() == a.generate(prompt, 16).tolist()
    a.close()
    b.close()


def test_plan_loads_the_resident_layers_of_an_engine_created_with_a_ring(gguf):
    # an engine created with ring_slots > 0 uploads no layer; the plan loads the
    # layers it keeps, and only the others stream
    per = _layer_bytes(gguf)
    a = DecodeEngine(gguf, max_seq_len=32)
    b = DecodeEngine(gguf, max_seq_len=32, ring_slots=2)
    assert not any(b.layer_is_resident(i) for i in range(6))
    mask = b.plan_residency(int(per * 5.5), ring_slots=2)
    assert mask == [True, True, True, False, False, False]
    assert [b.layer_is_resident(i) for i in range(6)] == mask
    for pos, tok in enumerate([5, 77, 301]):
        assert np.array_equal(a.forward_single_streaming(tok, pos), b.forward_single_streaming(tok, pos)), pos
    assert b.residency_stats()["ring_copies"] == 3 * 3
    a.close()
    b.close()
