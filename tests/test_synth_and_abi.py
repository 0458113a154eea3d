"""CPU tests: synthetic GGUF generator, encoders, the C ABI surface and the
engine's host-side logic (GGUF config parsing, tensor-parallel shard plan)."""
import ctypes
import os
import re
import struct

import numpy as np
import pytest

from oracle import oracle as orc
from ramforge_b200 import _lib, synth
from tests import fixtures as fx
from tests.gguf_writer import STR, U32, U64, F32, write_gguf

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))

SMALL = synth.scaled(synth.LLAMA3_8B, name="small-q4k", vocab_size=512, n_embd=512, n_layers=2, n_ff=1024,
                     n_heads=8, n_kv_heads=4, seed=11)


# ---- generator / encoders ---------------------------------------------------------
def test_generator_is_deterministic_and_seeded():
    a = synth.gguf_bytes(SMALL)
    b = synth.gguf_bytes(SMALL)
    c = synth.gguf_bytes(synth.scaled(SMALL, seed=12))
    assert np.array_equal(a, b)
    assert not np.array_equal(a, c)
    assert a.size == c.size


def test_generated_gguf_parses_in_oracle_and_engine():
    g = synth.gguf_bytes(SMALL)
    m = orc.OracleModel(g, max_seq=8)
    cfg = m.config
    assert (cfg["n_embd"], cfg["n_layers"], cfg["n_ff"], cfg["n_heads"], cfg["n_kv_heads"], cfg["head_dim"]) == \
        (512, 2, 1024, 8, 4, 64)
    assert cfg["rope_theta"] == 500000.0 and abs(cfg["rms_eps"] - 1e-5) < 1e-12
    c = _lib.ModelConfig()
    _lib.check(_lib.lib().rf_gguf_read_config(g.ctypes.data, g.size, ctypes.byref(c)))
    assert c.as_dict() == cfg


@pytest.mark.parametrize("gtype,tol", [(synth.Q8_0, 0.6 / 127), (synth.Q4_0, 0.6 / 7), (synth.Q4_K, 0.12),
                                      (synth.Q6_K, 0.6 / 31)])
def test_encoders_round_trip_through_reference_decoder(gtype, tol):
    x = synth.normal(1, 7, 64 * 512, std=1.0).reshape(64, 512)
    raw = synth.quantize(gtype, x)
    assert raw.size == 64 * synth.row_bytes(gtype, 512)
    rb = synth.row_bytes(gtype, 512)
    for r in range(64):
        d = orc.dequant_row(gtype, raw[r * rb:(r + 1) * rb], 512)
        amax = np.abs(x[r]).max()
        assert np.abs(d - x[r]).max() <= tol * amax * (2.0 if gtype == synth.Q4_K else 1.0)


def test_normal_generator_statistics():
    z = synth.normal(0, 1, 1 << 20, std=0.02)
    assert abs(z.mean()) < 2e-4 and abs(z.std() - 0.02) < 2e-4
    assert np.array_equal(synth.normal(0, 1, 100, std=0.02, start=50), z[50:150])


# ---- C ABI surface ------------------------------------------------------------------
def _header_functions():
    src = open(os.path.join(ROOT, "include", "rfcuda.h")).read()
    src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
    return sorted(set(re.findall(r"\b(rf_[a-z0-9_]+)\s*\(", src)))


def test_library_exports_every_declared_symbol():
    declared = _header_functions()
    assert sorted(_lib.EXPORTS) == declared
    L = ctypes.CDLL(_lib.LIB_PATH)
    for name in declared:
        assert hasattr(L, name), name


def _header_defines(prefix):
    hdr = open(os.path.join(ROOT, "include", "rfcuda.h")).read()
    return {m.group(1): int(m.group(2)) for m in re.finditer(r"#define (%s\w+) \(?(-?\d+)\)?" % prefix, hdr)}


def test_type_and_role_ids_agree_across_header_bindings_and_oracle():
    types = _header_defines("RF_TYPE_")
    assert set(types) == {"RF_TYPE_" + n for n in ("F32", "F16", "Q4_0", "Q5_0", "Q8_0", "Q2_K", "Q3_K", "Q4_K",
                                                    "Q5_K", "Q6_K", "Q8_K")}
    for name, v in types.items():
        short = name[len("RF_TYPE_"):]
        assert getattr(_lib, "TYPE_" + short) == v, name
        assert getattr(orc, short) == v, name
        if hasattr(synth, short):
            assert getattr(synth, short) == v, name
    roles = _header_defines("RF_ROLE_")
    for i, n in enumerate(_lib.LAYER_VIEW_NAMES):
        assert roles["RF_ROLE_" + n.replace(".", "_").upper()] == i, n
    assert (roles["RF_ROLE_TOKEN_EMBD"], roles["RF_ROLE_OUTPUT_NORM"], roles["RF_ROLE_OUTPUT"]) == (
        _lib.ROLE_TOKEN_EMBD, _lib.ROLE_OUTPUT_NORM, _lib.ROLE_OUTPUT)


def test_abi_version_matches_header():
    src = open(os.path.join(ROOT, "include", "rfcuda.h")).read()
    v = int(re.search(r"#define RF_ABI_VERSION (\d+)", src).group(1))
    assert _lib.lib().rf_abi_version() == v


def test_product_library_does_not_link_the_oracle():
    data = open(_lib.LIB_PATH, "rb").read()
    assert b"orc_" not in data and b"liboracle" not in data


# ---- host logic: GGUF config (model.rs:40-161) ---------------------------------------------
def _cfg(meta):
    g = write_gguf(meta, [])
    c = _lib.ModelConfig()
    rc = _lib.lib().rf_gguf_read_config(g, len(g), ctypes.byref(c))
    return rc, c


def test_config_defaults_and_fallback_keys():
    rc, c = _cfg([("general.architecture", STR, "qwen2"), ("llama.vocab_size", U32, 100),
                  ("qwen2.context_length", U64, 64), ("qwen2.embedding_length", U32, 64),
                  ("qwen2.block_count", U32, 2), ("qwen2.intermediate_size", U32, 128),
                  ("qwen2.attention.head_count", U32, 4)])
    assert rc == 0
    assert c.vocab_size == 100 and c.n_ff == 128 and c.n_kv_heads == 4 and c.head_dim == 16
    assert abs(c.rms_eps - 1e-5) < 1e-12 and c.rope_theta == 10000.0


def test_config_rejects_unsupported_arch_and_missing_keys():
    rc, _ = _cfg([("general.architecture", STR, "bert")])
    assert rc == _lib.RF_EFORMAT and b"unsupported execution architecture" in _lib.lib().rf_last_error()
    rc, _ = _cfg([("general.architecture", STR, "llama"), ("llama.vocab_size", U32, 10)])
    assert rc == _lib.RF_EFORMAT and b"context_length" in _lib.lib().rf_last_error()


def test_gguf_parser_rejects_bad_images():
    for bad in [b"GGUX" + bytes(20), b"GGUF" + struct.pack("<I", 4) + bytes(16), b"GGUF" + struct.pack("<I", 3)]:
        c = _lib.ModelConfig()
        assert _lib.lib().rf_gguf_read_config(bad, len(bad), ctypes.byref(c)) == _lib.RF_EFORMAT


def test_gguf_alignment_override_is_honoured():
    meta = [("general.architecture", STR, "llama"), ("general.alignment", U32, 64)]
    g = write_gguf(meta, [("t", [4], 0, np.ones(4, np.float32).tobytes())], alignment=64)
    c = _lib.ModelConfig()
    assert _lib.lib().rf_gguf_read_config(g, len(g), ctypes.byref(c)) == _lib.RF_EFORMAT  # arch ok, keys missing


def test_gqa_fixture_config():
    g = fx.gqa_gguf()
    c = _lib.ModelConfig()
    _lib.check(_lib.lib().rf_gguf_read_config(g, len(g), ctypes.byref(c)))
    assert (c.n_heads, c.n_kv_heads, c.head_dim, c.vocab_size) == (4, 2, 2, 16)


# ---- host logic: tensor-parallel shard plan ----------------------------------------------
def shard(cfg: dict, tp, rank, gtype=synth.Q4_K):
    c = _lib.ModelConfig(**{k: cfg[k] for k, _ in _lib.ModelConfig._fields_})
    s = _lib.TpShard()
    rc = _lib.lib().rf_tp_shard_plan(ctypes.byref(c), tp, rank, gtype, ctypes.byref(s))
    return rc, {f: getattr(s, f) for f, _ in s._fields_}


def _spec_cfg(spec):
    return dict(vocab_size=spec.vocab_size, context_length=spec.context_length, n_embd=spec.n_embd,
                n_layers=spec.n_layers, n_ff=spec.n_ff, n_heads=spec.n_heads, n_kv_heads=spec.n_kv_heads,
                head_dim=spec.head_dim, rms_eps=spec.rms_eps, rope_theta=spec.rope_theta)


@pytest.mark.parametrize("tp", [1, 2, 4, 8])
def test_llama3_8b_shards_cover_everything_once(tp):
    cfg = _spec_cfg(synth.LLAMA3_8B)
    kv, ff, voc = [], [], []
    for r in range(tp):
        rc, s = shard(cfg, tp, r)
        assert rc == 0
        assert s["q_heads"] == s["kv_heads"] * 4 and s["q_head_offset"] == s["kv_head_offset"] * 4
        assert (s["q_heads"] * 128) % 256 == 0 and s["ff_rows"] % 256 == 0
        kv += range(s["kv_head_offset"], s["kv_head_offset"] + s["kv_heads"])
        ff += range(s["ff_offset"], s["ff_offset"] + s["ff_rows"])
        voc += range(s["vocab_offset"], s["vocab_offset"] + s["vocab_rows"])
    assert kv == list(range(8)) and ff == list(range(14336)) and voc == list(range(128256))


def test_shard_plan_rejects_uneven_or_block_cutting_splits():
    cfg = _spec_cfg(synth.TINYLLAMA)  # 4 KV heads
    assert shard(cfg, 8, 0)[0] == _lib.RF_EINVAL
    cfg = _spec_cfg(synth.scaled(synth.LLAMA3_8B, n_ff=14336 + 256 * 2))
    assert shard(cfg, 8, 0)[0] == _lib.RF_EINVAL  # FFN rows not divisible by 8
    # 1 head of 128 columns per rank: cuts a 256-element Q4_K super-block, fine for Q8_0
    cfg = _spec_cfg(synth.scaled(synth.LLAMA3_8B, n_embd=1024, n_heads=8, n_kv_heads=8))
    assert shard(cfg, 8, 0, synth.Q4_K)[0] == _lib.RF_EINVAL
    assert shard(cfg, 8, 0, synth.Q8_0)[0] == 0
    # every 256-element K-quant has Q4_K's constraint; the 32-element formats have Q8_0's
    for t in (synth.Q2_K, synth.Q3_K, synth.Q5_K, synth.Q6_K, synth.Q8_K):
        assert shard(cfg, 8, 0, t)[0] == _lib.RF_EINVAL, t
        assert shard(cfg, 4, 0, t)[0] == 0, t
    assert shard(cfg, 8, 0, synth.Q5_0)[0] == 0


def test_engine_creation_fails_cleanly_without_gpu():
    try:
        import torch
        if torch.cuda.is_available():
            pytest.skip("a GPU is present")
    except Exception:
        pass
    g = fx.gqa_gguf()
    h = ctypes.c_void_p()
    rc = _lib.lib().rf_engine_create_from_gguf(g, len(g), None, ctypes.byref(h))
    assert rc == _lib.RF_ECUDA and not h.value
