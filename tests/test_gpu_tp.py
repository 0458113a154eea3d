"""Tensor parallelism on several GPUs (skipped where the box has fewer): one
process per GPU, the row-parallel sums over NVLink peer memory (and, at two
ranks, NCCL all-reduce for comparison).  Every rank must produce the oracle's
greedy tokens.
"""
import multiprocessing as mp
import os

import numpy as np
import pytest

from oracle import oracle as orc
from ramforge_b200 import synth

pytestmark = pytest.mark.gpu
THREADS = min(32, os.cpu_count() or 8)

# 8 KV heads of head_dim 128 and 4096 FFN rows: shards of up to 8 ranks fall on
# Q4_K super-block boundaries.
TP_MODEL = synth.scaled(synth.LLAMA3_8B, name="tp-q4k", vocab_size=1024, n_embd=2048, n_layers=2, n_ff=4096,
                        n_heads=16, n_kv_heads=8, seed=51, context_length=128)
# A Q4_K_M-like qwen2 layout: Q6_K V (its own matrix), down and LM head, Q/K/V biases
# sharded with their heads.
TP_MIX = synth.scaled(TP_MODEL, name="tp-qwen2-mix", arch="qwen2", seed=52, v_type=synth.Q6_K, down_type=synth.Q6_K,
                      out_type=synth.Q6_K, qkv_bias_std=0.5)


def _gpu_count():
    try:
        import torch
        return torch.cuda.device_count()
    except Exception:
        return 0


def _rank(rank, world, path, nid, prompt, n_new, peer_sum, q):
    try:
        os.environ["RF_PEER_SUM"] = "1" if peer_sum else "0"
        from ramforge_b200 import DecodeEngine
        eng = DecodeEngine(path, device=rank, max_seq_len=64, tp_rank=rank, tp_size=world, nccl_id=nid)
        toks = eng.generate(prompt, n_new).tolist()
        q.put((rank, toks, eng.tp_peer_sum, None))
        eng.close()
    except Exception as ex:  # reported to the test
        q.put((rank, None, None, repr(ex)))


def _model(tmp_path_factory, spec):
    g = synth.gguf_bytes(spec)
    path = str(tmp_path_factory.mktemp("tp") / f"{spec.name}.gguf")
    g.tofile(path)
    prompt = np.random.default_rng(6).integers(0, spec.vocab_size, 7).tolist()
    want = orc.OracleModel(g, kv_f16=True, max_seq=64, threads=THREADS).generate(prompt, 16)[0].tolist()
    return path, prompt, want


@pytest.fixture(scope="module")
def model(tmp_path_factory):
    return _model(tmp_path_factory, TP_MODEL)


@pytest.fixture(scope="module")
def mixed_model(tmp_path_factory):
    return _model(tmp_path_factory, TP_MIX)


@pytest.mark.parametrize("world,peer_sum", [(2, True), (2, False), (4, True), (8, True)])
def test_tp_greedy_matches_oracle(model, world, peer_sum):
    _run_tp(model, world, peer_sum)


@pytest.mark.parametrize("world", [2, 4])
def test_tp_mixed_format_biased_model_matches_oracle(mixed_model, world):
    _run_tp(mixed_model, world, True)


def _run_tp(model, world, peer_sum):
    if _gpu_count() < world:
        pytest.skip(f"needs {world} GPUs")
    path, prompt, want = model
    from ramforge_b200 import tp_unique_id
    nid = tp_unique_id()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    ps = [ctx.Process(target=_rank, args=(r, world, path, nid, prompt, 16, peer_sum, q)) for r in range(world)]
    for p in ps:
        p.start()
    res = {}
    for _ in ps:
        r, toks, active, err = q.get(timeout=300)
        res[r] = (toks, active, err)
    for p in ps:
        p.join(timeout=60)
    for r in range(world):
        toks, active, err = res[r]
        assert err is None, err
        assert toks == want, (r, toks, want)
        assert active == peer_sum
