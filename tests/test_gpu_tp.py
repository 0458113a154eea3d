"""Tensor parallelism on two GPUs (skipped with fewer): two ranks, one process
per GPU, the row-parallel sums over NVLink peer memory (and, for comparison,
NCCL all-reduce).  Both ranks must produce the oracle's greedy tokens.
"""
import multiprocessing as mp
import os

import numpy as np
import pytest

from oracle import oracle as orc
from ramforge_b200 import synth

pytestmark = pytest.mark.gpu
THREADS = min(32, os.cpu_count() or 8)

TP_MODEL = synth.scaled(synth.LLAMA3_8B, name="tp-q4k", vocab_size=1024, n_embd=1024, n_layers=3, n_ff=1536,
                        n_heads=8, n_kv_heads=2, seed=51, context_length=128)


def _gpu_count():
    try:
        import torch
        return torch.cuda.device_count()
    except Exception:
        return 0


def _rank(rank, path, nid, prompt, n_new, peer_sum, q):
    try:
        os.environ["RF_PEER_SUM"] = "1" if peer_sum else "0"
        from ramforge_b200 import DecodeEngine
        eng = DecodeEngine(path, device=rank, max_seq_len=64, tp_rank=rank, tp_size=2, nccl_id=nid)
        toks = eng.generate(prompt, n_new).tolist()
        q.put((rank, toks, eng.tp_peer_sum, None))
        eng.close()
    except Exception as ex:  # reported to the test
        q.put((rank, None, None, repr(ex)))


@pytest.mark.skipif(_gpu_count() < 2, reason="needs two GPUs")
@pytest.mark.parametrize("peer_sum", [True, False])
def test_tp2_greedy_matches_oracle(tmp_path, peer_sum):
    g = synth.gguf_bytes(TP_MODEL)
    path = str(tmp_path / "tp.gguf")
    g.tofile(path)
    prompt = np.random.default_rng(6).integers(0, TP_MODEL.vocab_size, 7).tolist()
    want = orc.OracleModel(g, kv_f16=True, max_seq=64, threads=THREADS).generate(prompt, 16)[0].tolist()
    from ramforge_b200 import tp_unique_id
    nid = tp_unique_id()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    ps = [ctx.Process(target=_rank, args=(r, path, nid, prompt, 16, peer_sum, q)) for r in range(2)]
    for p in ps:
        p.start()
    res = {}
    for _ in ps:
        r, toks, active, err = q.get(timeout=300)
        res[r] = (toks, active, err)
    for p in ps:
        p.join(timeout=60)
    for r in (0, 1):
        toks, active, err = res[r]
        assert err is None, err
        assert toks == want, (r, toks, want)
        assert active == peer_sum
