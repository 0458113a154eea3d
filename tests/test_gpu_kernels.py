"""GPU parity of the standalone kernels against the CPU oracle.

Tolerances: quantized matvec max|y - y_ref| <= 2e-4 * max|y_ref| (f32
reassociation only: the engine sums per sub-block and across lanes, the
reference sums sequentially); attention max|o - o_ref| <= 1e-4 * max|o_ref| + 1e-6;
embedding rows and per-element dequantisation are bit-exact.
"""
import os

import numpy as np
import pytest

from oracle import oracle as orc
from ramforge_b200 import QMatrix, decode_attention, synth
from tests import fixtures as fx

pytestmark = pytest.mark.gpu
THREADS = min(32, os.cpu_count() or 8)


def torch_mod():
    import torch
    return torch


Q5_K, Q3_K, Q2_K = orc.Q5_K, orc.Q3_K, orc.Q2_K  # no synthetic encoders: random blocks (tests/fixtures.py)
RANDOM_BLOCK_TYPES = (Q5_K, Q3_K, Q2_K)


def _weights(gtype, M, K, seed=1):
    if gtype in RANDOM_BLOCK_TYPES:
        return fx.random_blocks(gtype, M, K, seed)
    w = synth.normal(seed, 100 + gtype, M * K, std=0.02).reshape(M, K)
    return synth.quantize(gtype, w)


def _run_qmv(gtype, M, K, batch=1, seed=1, raw=None):
    torch = torch_mod()
    raw = _weights(gtype, M, K, seed) if raw is None else raw
    x = synth.normal(seed, 7, batch * K, std=1.0).reshape(batch, K)
    m = QMatrix(gtype, raw, M, K)
    dx = torch.from_numpy(x).cuda()
    dy = torch.empty(batch, M, device="cuda")
    m.matvec(dx.data_ptr(), dy.data_ptr(), batch)
    torch.cuda.synchronize()
    y = dy.cpu().numpy()
    for b in range(batch):
        ref = orc.matvec(gtype, raw, K, M, x[b], threads=THREADS)
        err = np.abs(y[b] - ref).max()
        assert err <= 2e-4 * np.abs(ref).max() + 1e-6, (gtype, M, K, b, err, np.abs(ref).max())
    m.close()


@pytest.mark.parametrize("gtype", [synth.Q8_0, synth.Q4_0, synth.Q4_K, synth.Q6_K, Q5_K, Q3_K, Q2_K, synth.F16,
                                   synth.F32])
@pytest.mark.parametrize("M,K", [(1, 256), (7, 512), (33, 768), (130, 2304), (257, 4096)])
def test_qmatvec_small_shapes(gtype, M, K):
    _run_qmv(gtype, M, K)


@pytest.mark.parametrize("gtype,M,K", [(synth.Q8_0, 5, 32), (synth.Q4_0, 3, 32), (synth.Q4_0, 2, 96),
                                       (synth.Q8_0, 9, 160), (synth.F32, 3, 8), (synth.F32, 2, 12)])
def test_qmatvec_ragged_rows_padded_to_units(gtype, M, K):
    _run_qmv(gtype, M, K)


@pytest.mark.parametrize("gtype", [synth.Q8_0, synth.Q4_0, synth.Q4_K, synth.Q6_K, Q5_K, Q3_K, Q2_K])
@pytest.mark.parametrize("M,K", [(4096, 4096), (14336, 4096), (4096, 14336), (128256, 4096)])
def test_qmatvec_config2_shapes(gtype, M, K):
    _run_qmv(gtype, M, K)


@pytest.mark.parametrize("gtype", [synth.Q8_0, synth.Q4_0, synth.Q4_K, synth.Q6_K, Q5_K, Q3_K, Q2_K])
@pytest.mark.parametrize("batch", [4, 8])
def test_qmatvec_batched(gtype, batch):
    _run_qmv(gtype, 1024, 4096, batch=batch)


def test_qmatvec_subnormal_scales_follow_reference_decode():
    # A Q8_0 block whose f16 scale is subnormal: the reference decodes it at half
    # its IEEE value (quant.rs:40-65); the GPU must agree.
    raw = bytearray(_weights(synth.Q8_0, 4, 64))
    for r in range(4):
        raw[r * 68:r * 68 + 2] = (0x0155 + r).to_bytes(2, "little")
    _run_qmv(synth.Q8_0, 4, 64, raw=np.frombuffer(bytes(raw), np.uint8))


def test_qmatvec_q6_k_subnormal_super_scale_follows_reference_decode():
    # Q6_K's f16 d sits at bytes 208-209 of each 210-byte block; rows 1 and 3 get
    # a subnormal one.
    raw = bytearray(_weights(synth.Q6_K, 4, 512))
    for r in (1, 3):
        for b in range(2):
            o = (r * 2 + b) * 210 + 208
            raw[o:o + 2] = (0x0123 + b).to_bytes(2, "little")
    _run_qmv(synth.Q6_K, 4, 512, raw=np.frombuffer(bytes(raw), np.uint8))


def test_qmatvec_q5_k_subnormal_scales_follow_reference_decode():
    # Q5_K's f16 d and dmin sit at bytes 0-3 of each 176-byte block; rows 1 and 2
    # get a subnormal dmin, row 3 a subnormal d.
    raw = bytearray(_weights(Q5_K, 4, 512))
    for r, o in ((1, 2), (2, 2), (3, 0)):
        for b in range(2):
            p = (r * 2 + b) * 176 + o
            raw[p:p + 2] = (0x0155 + b).to_bytes(2, "little")
    _run_qmv(Q5_K, 4, 512, raw=np.frombuffer(bytes(raw), np.uint8))


@pytest.mark.parametrize("gtype,size,offs", [(Q3_K, 110, (108,)), (Q2_K, 84, (80, 82))])
def test_qmatvec_low_bit_k_quants_subnormal_scales_follow_reference_decode(gtype, size, offs):
    # each row gets a subnormal f16 d (Q3_K) or d and dmin (Q2_K) in one of its blocks
    raw = bytearray(_weights(gtype, 4, 512))
    for r in range(4):
        for o in offs:
            p = (2 * r + r % 2) * size + o
            raw[p:p + 2] = (0x0101 + r).to_bytes(2, "little")
    _run_qmv(gtype, 4, 512, raw=np.frombuffer(bytes(raw), np.uint8))


@pytest.mark.parametrize("gtype", [synth.Q8_0, synth.Q4_0, synth.Q4_K, synth.Q6_K, Q5_K, Q3_K, Q2_K, synth.F16])
def test_device_packing_equals_host_packing(gtype):
    # rf_matrix_create packs device-resident GGUF bytes with the pack kernel and
    # host bytes on the CPU; both must give the same packed matrix, so the same
    # products bit for bit.
    torch = torch_mod()
    M, K = 193, 1024
    raw = _weights(gtype, M, K, seed=4)
    x = torch.from_numpy(synth.normal(4, 7, K, std=1.0)).cuda()
    draw = torch.from_numpy(np.ascontiguousarray(raw)).cuda()
    a = QMatrix(gtype, raw, M, K)
    b = QMatrix(gtype, None, M, K, on_device_ptr=draw.data_ptr(), nbytes=raw.size)
    assert a.device_bytes == b.device_bytes
    ya = torch.empty(M, device="cuda")
    yb = torch.empty(M, device="cuda")
    a.matvec(x.data_ptr(), ya.data_ptr())
    b.matvec(x.data_ptr(), yb.data_ptr())
    torch.cuda.synchronize()
    assert torch.equal(ya, yb)
    a.close()
    b.close()


def _qmv_once(gtype, raw, M, K, x):
    torch = torch_mod()
    m = QMatrix(gtype, np.frombuffer(bytes(raw), np.uint8), M, K)
    dx = torch.from_numpy(np.ascontiguousarray(x, np.float32)).cuda()
    dy = torch.empty(M, device="cuda")
    m.matvec(dx.data_ptr(), dy.data_ptr())
    torch.cuda.synchronize()
    m.close()
    return dy.cpu().numpy()


def test_qmatvec_nonsquare_layout_anchors():
    # the ggml [in, out] anchors of tensor.rs:1161-1306 through rf_qmatvec
    import struct
    f32 = np.array([1, 2, 3, 4, 5, 6], np.float32).tobytes()
    assert _qmv_once(synth.F32, f32, 3, 2, [10, 20]).tolist() == [50.0, 110.0, 170.0]
    assert _qmv_once(synth.F32, f32, 2, 3, [1, 0, -1]).tolist() == [-2.0, -2.0]
    f16 = struct.pack("<4H", 0x3C00, 0x4000, 0x4200, 0x4400)
    assert np.allclose(_qmv_once(synth.F16, f16, 2, 2, [1, 1]), [3.0, 7.0], atol=1e-3)
    blk = lambda fill: struct.pack("<H", 0x3C00) + bytes([fill] * 16)
    q40 = b"".join(blk(fill) * 2 for fill in (0x11, 0x23, 0xF8))
    assert np.allclose(_qmv_once(synth.Q4_0, q40, 3, 64, [1.0] * 32 + [2.0] * 32), [-672.0, -528.0, 336.0], atol=1e-3)
    q4k = b"".join(struct.pack("<HH", 0x3C00, 0) + bytes([1] * 12) + bytes([fill] * 128) for fill in (0x11, 0x22))
    assert np.allclose(_qmv_once(synth.Q4_K, q4k, 2, 256, [1.0] * 256), [256.0, 512.0], atol=1e-3)


def test_qmatvec_q4_0_lcg_rows_at_qwen2_5_q_shape():
    # the pseudorandom Q4_0 matrix of streaming_model.rs:3332-3411 against the oracle
    from tests.test_oracle_golden import lcg_q4_0_rows
    n = 1536
    raw = lcg_q4_0_rows(n, n)
    x = (np.sin(np.arange(n, dtype=np.float32) * np.float32(0.0137) - np.float32(0.5)) * np.float32(0.7)).astype(
        np.float32)
    _run_qmv(synth.Q4_0, n, n, raw=np.frombuffer(raw, np.uint8))
    ref = orc.matvec(orc.Q4_0, raw, n, n, x, reference=True)
    assert np.abs(_qmv_once(synth.Q4_0, raw, n, n, x) - ref).max() < 1e-2


@pytest.mark.parametrize("ctx", [1, 5, 512, 2048, 8192, 32768])
@pytest.mark.parametrize("batch", [1, 8])
def test_decode_attention_config3(ctx, batch):
    torch = torch_mod()
    H, KV, hd = 32, 8, 128
    q = synth.normal(2, 1, batch * H * hd).reshape(batch, H, hd)
    k = synth.normal(2, 2, batch * KV * ctx * hd).reshape(batch, KV, ctx, hd).astype(np.float16)
    v = synth.normal(2, 3, batch * KV * ctx * hd).reshape(batch, KV, ctx, hd).astype(np.float16)
    dq = torch.from_numpy(q).cuda()
    dk = torch.from_numpy(k.view(np.uint16)).cuda()
    dv = torch.from_numpy(v.view(np.uint16)).cuda()
    do = torch.empty(batch, H, hd, device="cuda")
    decode_attention(dq.data_ptr(), dk.data_ptr(), dv.data_ptr(), ctx, H, KV, hd, batch, do.data_ptr())
    torch.cuda.synchronize()
    out = do.cpu().numpy()
    del dq, dk, dv, do

    def check(b):
        # reference layout [pos][kv_head][hd]: history = first ctx-1 positions, current = last
        kk = np.ascontiguousarray(k[b].astype(np.float32).transpose(1, 0, 2))
        vv = np.ascontiguousarray(v[b].astype(np.float32).transpose(1, 0, 2))
        ref = orc.attention(q[b], kk[:-1], vv[:-1], kk[-1], vv[-1], ctx - 1, H, KV, hd)
        err = np.abs(out[b].reshape(-1) - ref).max()
        return err, 1e-4 * np.abs(ref).max() + 1e-6

    # the oracle call releases the GIL: sequences are checked in parallel
    from concurrent.futures import ThreadPoolExecutor
    with ThreadPoolExecutor(max_workers=min(batch, os.cpu_count() or 1)) as ex:
        for b, (err, tol) in enumerate(ex.map(check, range(batch))):
            assert err <= tol, (ctx, b, err)


@pytest.mark.parametrize("H,KV,hd", [(8, 8, 128), (16, 8, 128), (32, 4, 128), (64, 8, 128), (4, 4, 64),
                                     (8, 4, 64), (32, 8, 64), (16, 2, 64), (2, 2, 32), (4, 2, 32), (8, 2, 32),
                                     (16, 2, 32)])
@pytest.mark.parametrize("ctx,batch", [(1024, 1), (1025, 2), (1039, 1), (1087, 3), (2065, 2), (4099, 1)])
def test_decode_attention_streamed_kernel_shapes(H, KV, hd, ctx, batch):
    """Every instance of the streaming kernel (GQA group 1/2/4/8, head_dim
    32/64/128; it serves contexts from 1024 positions) at contexts whose splits
    end inside a tile or on a tile edge, against an fp32 torch restatement of
    attention_reference."""
    torch = torch_mod()
    g = torch.Generator(device="cuda").manual_seed(H * 1000 + KV * 10 + hd + ctx)
    q = torch.randn(batch, H, hd, device="cuda", generator=g)
    k = torch.randn(batch, KV, ctx, hd, device="cuda", generator=g).half()
    v = torch.randn(batch, KV, ctx, hd, device="cuda", generator=g).half()
    o = torch.full((batch, H, hd), float("nan"), device="cuda")
    decode_attention(q.data_ptr(), k.data_ptr(), v.data_ptr(), ctx, H, KV, hd, batch, o.data_ptr())
    G = H // KV
    s = (q.view(batch, KV, G, hd) @ k.float().transpose(-1, -2)) / hd ** 0.5
    ref = (torch.softmax(s, -1) @ v.float()).view(batch, H, hd)
    torch.cuda.synchronize()
    tol = 1e-4 * ref.abs().max().item() + 1e-6
    assert (o - ref).abs().max().item() <= tol


def test_decode_attention_unaligned_cache_takes_register_path():
    """A cache that starts 8 bytes past a 16-byte boundary cannot be bulk-copied;
    the register-load kernel serves it with the same results."""
    torch = torch_mod()
    H, KV, hd, ctx = 32, 8, 128, 700
    g = torch.Generator(device="cuda").manual_seed(7)
    q = torch.randn(1, H, hd, device="cuda", generator=g)
    kbuf = torch.randn(KV * ctx * hd + 4, device="cuda", generator=g).half()
    vbuf = torch.randn(KV * ctx * hd + 4, device="cuda", generator=g).half()
    k, v = kbuf[4:].view(1, KV, ctx, hd), vbuf[4:].view(1, KV, ctx, hd)
    assert k.data_ptr() % 16 == 8
    o = torch.empty(1, H, hd, device="cuda")
    decode_attention(q.data_ptr(), k.data_ptr(), v.data_ptr(), ctx, H, KV, hd, 1, o.data_ptr())
    s = (q.view(1, KV, H // KV, hd) @ k.float().transpose(-1, -2)) / hd ** 0.5
    ref = (torch.softmax(s, -1) @ v.float()).view(1, H, hd)
    torch.cuda.synchronize()
    assert (o - ref).abs().max().item() <= 1e-4 * ref.abs().max().item() + 1e-6


def test_decode_attention_repeated_calls_reuse_workspace():
    torch = torch_mod()
    H, KV, hd, ctx = 32, 8, 128, 3000
    q = torch.randn(1, H, hd, device="cuda")
    k = torch.randn(1, KV, ctx, hd, device="cuda").half()
    v = torch.randn(1, KV, ctx, hd, device="cuda").half()
    outs = []
    for _ in range(3):
        o = torch.empty(1, H, hd, device="cuda")
        decode_attention(q.data_ptr(), k.data_ptr(), v.data_ptr(), ctx, H, KV, hd, 1, o.data_ptr())
        outs.append(o)
    torch.cuda.synchronize()
    assert torch.equal(outs[0], outs[1]) and torch.equal(outs[1], outs[2])
    ref = torch.softmax((q.view(1, KV, 4, hd) @ k.float().transpose(-1, -2)) / hd ** 0.5, -1) @ v.float()
    assert torch.allclose(outs[0], ref.view(1, H, hd), atol=1e-4, rtol=1e-4)


def test_bounded_peer_sum_wait_gives_up_and_reports():
    """The tensor-parallel peer sum's wait is bounded: a rank whose flag never
    comes makes it give up after about a second, set the error bit and return,
    and the device stays usable (a matvec right after it is correct)."""
    from ramforge_b200 import selftest_wait
    assert selftest_wait(0) == 1
    _run_qmv(synth.Q4_K, 512, 1024)
