"""Pins the CPU oracle (oracle/) to the reference's own known-answer tests.

Each case restates a #[test] of NeonMC23/RAMforge with its literal inputs,
expected outputs and tolerance (file:line given per test).  The oracle is the
parity checker for the GPU engine, so these run first and on CPU.
"""
import struct

import numpy as np
import pytest

from oracle import oracle as orc
from tests import fixtures as fx


def q4_0_block(scale: int, quants) -> bytes:
    return struct.pack("<H", scale) + bytes(quants)


def q5_0_block(scale: int, qh: int, quants) -> bytes:
    return struct.pack("<H", scale) + struct.pack("<I", qh) + bytes(quants)


def q8_0_block(scale: int, quants) -> bytes:
    return struct.pack("<H", scale) + bytes((q & 0xFF) for q in quants)


# ---- f16 ------------------------------------------------------------------------
def test_f16_to_f32_follows_reference_decode():
    # quant.rs:40-65 (and tensor.rs:1017-1041): normal halves, zeros, inf are IEEE-exact;
    # a subnormal half decodes to half its IEEE value (exponent 127-15-e, one short).
    for bits in [0x0000, 0x8000, 0x3C00, 0x3800, 0xBC00, 0x4000, 0x0400, 0x7BFF, 0x7C00, 0xFC00, 0x1234]:
        assert orc.f16_to_f32(bits) == float(np.frombuffer(struct.pack("<H", bits), np.float16)[0])
    for bits in [0x0001, 0x0002, 0x0155, 0x03FF, 0x8001, 0x83FF]:
        ieee = float(np.frombuffer(struct.pack("<H", bits), np.float16)[0])
        assert orc.f16_to_f32(bits) == ieee / 2


def test_f32_to_f16_matches_ieee_rne():
    rng = np.random.default_rng(7)
    vals = np.concatenate([rng.normal(0, 1, 2000), rng.normal(0, 1e-5, 500), rng.normal(0, 3e4, 500),
                           [65504.0, 65519.0, 65520.0, 6.0e-8, 2.98e-8, 0.0, -0.0]]).astype(np.float32)
    for v in vals:
        want = int(np.array([v], np.float32).astype(np.float16).view(np.uint16)[0])
        assert orc.f32_to_f16(float(v)) == want, v


# ---- quant.rs block decoders ----------------------------------------------------
def test_q5_0_decode_high_bits():  # quant.rs:1570-1585
    q = [0] * 16
    q[1] = 0xFF
    d = orc.dequant_row(orc.Q5_0, q5_0_block(0x3C00, 0x0003_0003, q), 32)
    assert (d[0], d[1], d[2], d[16], d[17], d[18]) == (0.0, 15.0, -16.0, 0.0, 15.0, -16.0)


def test_q5_0_decode_matches_native_reference_vector():  # quant.rs:1587-1606
    qs = [3, 10, 17, 24, 31, 38, 45, 52, 59, 66, 73, 80, 87, 94, 101, 108]
    d = orc.dequant_row(orc.Q5_0, q5_0_block(0x3800, 0x9E37_79B9, qs), 32)
    want = [1.5, -3.0, -7.5, 4.0, 7.5, 3.0, -1.5, 2.0, 5.5, -7.0, -3.5, 0.0, 3.5, 7.0, 2.5, -2.0, 0.0, 0.0, 0.5,
            -7.5, 0.5, 1.0, -7.0, -6.5, -6.5, 2.0, 2.0, 2.5, 2.5, -5.5, -5.0, 3.0]
    assert d.tolist() == want


def test_q5_0_row_decode_and_matvec():  # quant.rs:1608-1624
    raw = q5_0_block(0x3C00, 0, [0] * 16) + q5_0_block(0x3800, 0, [0] * 16)
    d = orc.dequant_row(orc.Q5_0, raw, 64)
    assert d[0] == -16.0 and d[32] == -8.0
    y = orc.matvec(orc.Q5_0, raw, 32, 2, np.ones(32, np.float32))
    assert y.tolist() == [-512.0, -256.0]


def test_q4_0_decode():  # quant.rs:1660-1683
    assert np.allclose(orc.dequant_row(orc.Q4_0, q4_0_block(0x3C00, [0x88] * 16), 32), 0.0, atol=1e-5)
    assert np.allclose(orc.dequant_row(orc.Q4_0, q4_0_block(0x3C00, [0x00] * 16), 32), -8.0, atol=1e-5)


def test_q4_0_row_decode_edge_nibbles():  # quant.rs:1685-1707
    quants = [0xF0, 0x08, 0x87, 0x7F, 0x00, 0xFF, 0x18, 0xE9, 0x26, 0xD3, 0x45, 0xBC, 0x6A, 0x95, 0x70, 0x8F]
    a = orc.dequant_row(orc.Q4_0, q4_0_block(0x3800, quants), 32)
    assert (a[0], a[16], a[1], a[17]) == (-4.0, 3.5, 0.0, -4.0)
    assert (a < 0).any() and (a > 0).any()
    assert (orc.dequant_row(orc.Q4_0, q4_0_block(0x3C00, [0x88] * 16), 32) == 0.0).all()


def test_q4_0_row_decode_multiple_rows_and_blocks():  # quant.rs:1709-1726
    row0 = q4_0_block(0x3C00, [0x00] * 16) + q4_0_block(0x3800, [0xFF] * 16)
    row1 = q4_0_block(0x4000, [0x18] * 16) + q4_0_block(0xBC00, [0xF0] * 16)
    o = orc.dequant_row(orc.Q4_0, row0, 64)
    assert (o[:32] == -8.0).all() and (o[32:] == 3.5).all()
    o = orc.dequant_row(orc.Q4_0, row1, 64)
    assert (o[:16] == 0.0).all() and (o[16:32] == -14.0).all() and (o[32:48] == 8.0).all() and (o[48:] == -7.0).all()


def test_q4_0_row_decode_validation():  # quant.rs:1728-1740
    with pytest.raises(orc.OracleError, match="row truncated"):
        orc.dequant_row(orc.Q4_0, bytes(17), 32)
    with pytest.raises(orc.OracleError, match="not divisible"):
        orc.dequant_row(orc.Q4_0, q4_0_block(0x3C00, [0x88] * 16), 31)


def test_q8_0_decode():  # quant.rs:1742-1754
    assert np.allclose(orc.dequant_row(orc.Q8_0, q8_0_block(0x3C00, [1] * 32), 32), 1.0, atol=1e-5)


def test_q8_0_row_direct_decode():  # quant.rs:1756-1781
    quants = [-128, 127, -64, 64, -17, 17, -8, 8, -1, 0, 1, 2, -2, 31, -31, 63, -63, 126, -127, 5, -5, 12, -12, 42,
              -42, 99, -99, 3, -3, 7, -7, 16]
    a = orc.dequant_row(orc.Q8_0, q8_0_block(0x3800, quants), 32)
    assert a[0] == -64.0 and a[1] == 63.5
    assert np.array_equal(a, np.array(quants, np.float32) * np.float32(0.5))
    assert (orc.dequant_row(orc.Q8_0, q8_0_block(0x3C00, [0] * 32), 32) == 0.0).all()


def test_q8_0_row_direct_decode_multiple_rows():  # quant.rs:1783-1797
    for row, want in [(q8_0_block(0x3C00, [-3] * 32) + q8_0_block(0x3800, [7] * 32), [-3.0] * 32 + [3.5] * 32),
                      (q8_0_block(0xBC00, [-8] * 32) + q8_0_block(0x4000, [5] * 32), [8.0] * 32 + [10.0] * 32)]:
        assert orc.dequant_row(orc.Q8_0, row, 64).tolist() == want


def test_q4_k_decode_all_ones():  # quant.rs:1818-1833
    raw = struct.pack("<HH", 0x3C00, 0x0000) + bytes([1] * 12) + bytes([0x11] * 128)
    assert np.allclose(orc.dequant_row(orc.Q4_K, raw, 256), 1.0, atol=1e-5)


def test_q6_k_decode_runs():  # quant.rs:1852-1866
    raw = bytes([0x11] * 128) + bytes(64) + bytes([1] * 16) + struct.pack("<H", 0x3C00)
    assert orc.dequant_row(orc.Q6_K, raw, 256).shape == (256,)


# ---- the other K-quants (quant.rs:257-612) ---------------------------------------
def test_k_quant_block_sizes():  # quant.rs:1626-1649
    for t, n in ((orc.Q2_K, 84), (orc.Q3_K, 110), (orc.Q5_K, 176), (orc.Q6_K, 210), (orc.Q8_K, 292)):
        assert orc.row_bytes(t, 256) == n


def test_q5_k_decode_all_ones():  # quant.rs:1826-1841
    raw = struct.pack("<HH", 0x3C00, 0x0000) + bytes([1] * 12) + bytes(32) + bytes([0x11] * 128)
    assert np.allclose(orc.dequant_row(orc.Q5_K, raw, 256), 1.0, atol=1e-5)


def test_q8_k_decode_all_ones():  # quant.rs:1888-1900
    raw = struct.pack("<f", 1.0) + bytes([1] * 256) + bytes(32)
    assert np.allclose(orc.dequant_row(orc.Q8_K, raw, 256), 1.0, atol=1e-5)


def test_q2_k_and_q3_k_decode_run():  # quant.rs:1859-1886
    q2 = bytes([0x11] * 16) + bytes([0x11] * 64) + struct.pack("<HH", 0x3C00, 0x0000)
    q3 = bytes([0x11] * 32) + bytes([0x11] * 64) + bytes([1] * 12) + struct.pack("<H", 0x3C00)
    assert np.isfinite(orc.dequant_row(orc.Q2_K, q2, 256)).all()
    assert np.isfinite(orc.dequant_row(orc.Q3_K, q3, 256)).all()


def _f16(b, o):
    return np.frombuffer(bytes(b[o:o + 2]), np.float16)[0].astype(np.float32)


def _py_dequant(t, b):
    """A second, independent transcription of BlockQ{2,3,5,8}K::dequantize
    (quant.rs:303-343, 443-474, 506-574, 605-609), in float32 numpy scalars."""
    f = np.float32
    out = np.zeros(256, np.float32)
    if t == orc.Q8_K:
        d = np.frombuffer(bytes(b[0:4]), np.float32)[0]
        return (d * np.frombuffer(bytes(b[4:260]), np.int8).astype(np.float32)).astype(np.float32)
    if t == orc.Q5_K:
        d, dmin, sc, qh, qs = _f16(b, 0), _f16(b, 2), b[4:16], b[16:48], b[48:176]

        def sm(j):
            if j < 4:
                return sc[j] & 63, sc[j + 4] & 63
            return (sc[j + 4] & 0xF) | ((sc[j - 4] >> 6) << 4), (sc[j + 4] >> 4) | ((sc[j] >> 6) << 4)
        y = 0
        for g in range(4):
            (s0, m0), (s1, m1) = sm(2 * g), sm(2 * g + 1)
            u1, u2 = 1 << (2 * g), 2 << (2 * g)
            for l in range(32):
                hb = qh[32 * g // 4 + l // 8]
                out[y + l] = f(d * f(s0)) * f((qs[32 * g + l] & 0xF) + (16 if hb & u1 else 0)) - f(dmin * f(m0))
                out[y + 32 + l] = f(d * f(s1)) * f((qs[32 * g + l] >> 4) + (16 if hb & u2 else 0)) - f(dmin * f(m1))
            y += 64
        return out
    if t == orc.Q2_K:
        sc, qs, d, dmin = b[0:16], b[16:80], _f16(b, 80), _f16(b, 82)
        y, i = 0, 0
        for n in range(2):
            for shift in (0, 2, 4, 6):
                for h in range(2):
                    dl, ml = f(d * f(sc[i] & 0xF)), f(dmin * f(sc[i] >> 4))
                    i += 1
                    for l in range(16):
                        out[y + l] = dl * f((qs[32 * n + 16 * h + l] >> shift) & 3) - ml
                    y += 16
        return out
    hm, qs, sb, d = b[0:32], b[32:96], b[96:108], _f16(b, 108)  # Q3_K
    a = [int.from_bytes(bytes(sb[4 * i:4 * i + 4]), "little") for i in range(3)]
    k1, k2 = 0x03030303, 0x0F0F0F0F
    aux = [(a[0] & k2) | (((a[2] >> 0) & k1) << 4), (a[1] & k2) | (((a[2] >> 2) & k1) << 4),
           ((a[0] >> 4) & k2) | (((a[2] >> 4) & k1) << 4), ((a[1] >> 4) & k2) | (((a[2] >> 6) & k1) << 4)]
    s8 = np.frombuffer(b"".join(v.to_bytes(4, "little") for v in aux), np.int8)
    y, m = 0, 1
    for n in range(2):
        for j, shift in enumerate((0, 2, 4, 6)):
            for h in range(2):
                dl = f(d * f(int(s8[j + 4 * h]) - 32))
                for l in range(16):
                    q = ((qs[32 * n + 16 * h + l] >> shift) & 3) - (0 if hm[16 * h + l] & m else 4)
                    out[y + l] = dl * f(q)
                y += 16
            m <<= 1
    return out


@pytest.mark.parametrize("gtype,size,dpos", [(orc.Q5_K, 176, (0, 2)), (orc.Q2_K, 84, (80, 82)),
                                            (orc.Q3_K, 110, (108,)), (orc.Q8_K, 292, ())])
def test_k_quant_decoders_match_an_independent_transcription(gtype, size, dpos):
    rng = np.random.default_rng(gtype)
    for _ in range(8):
        b = bytearray(rng.integers(0, 256, size, dtype=np.uint8).tobytes())
        for o in dpos:  # finite, normal f16 super-scales
            b[o:o + 2] = int(rng.integers(0x2000, 0x3C00)).to_bytes(2, "little")
        if gtype == orc.Q8_K:
            b[0:4] = struct.pack("<f", float(rng.uniform(0.001, 0.1)))
        assert np.array_equal(orc.dequant_row(gtype, bytes(b), 256), _py_dequant(gtype, b))


def test_truncated_block_rejection():  # quant.rs:1911-1921
    for t in (orc.Q4_0, orc.Q8_0, orc.Q4_K, orc.Q6_K, orc.Q2_K, orc.Q3_K, orc.Q5_K, orc.Q8_K):
        with pytest.raises(orc.OracleError):
            orc.dequant_row(t, bytes(5), {orc.Q4_0: 32, orc.Q8_0: 32}.get(t, 256))


# ---- quantized matvecs ----------------------------------------------------------
def test_quantized_matvec_q4_0():  # quant.rs:1923-1948
    row = q4_0_block(0x3C00, [0x99] * 16)
    y = orc.matvec(orc.Q4_0, row + row, 32, 2, np.ones(32, np.float32))
    assert abs(y[0] - 32.0) < 1e-3
    yref = orc.matvec(orc.Q4_0, row + row, 32, 2, np.ones(32, np.float32), reference=True)
    assert abs(y[0] - yref[0]) < 1e-3


def _diag_q4_0_row(blocks):  # quant.rs:1950-1978
    scales = [0x3C00, 0x3800, 0x3A00, 0x4000, 0xBC00, 0x3400, 0x3E00, 0xB800]
    out = b""
    for b in range(blocks):
        q = [(((j * 5 + b * 3 + 1) & 0x0F) | (((j * 7 + b * 11 + 9) & 0x0F) << 4)) for j in range(16)]
        out += q4_0_block(scales[b % len(scales)], q)
    return out


def _diag_input(pattern, n):  # quant.rs:1980-2001
    if pattern == "constant":
        return np.full(n, 1.25, np.float32)
    if pattern == "ramp":
        return (np.arange(n, dtype=np.float32) * np.float32(0.125) - np.float32(2.0)).astype(np.float32)
    if pattern == "alternating":
        return np.where(np.arange(n) % 2 == 0, 1.5, -0.75).astype(np.float32)
    state, out = 0x12345678, []
    for _ in range(n):
        state = (state * 1664525 + 1013904223) & 0xFFFFFFFF
        out.append(np.float32(np.float32(state >> 8) / np.float32(16777215.0)) * np.float32(2.0) - np.float32(1.0))
    return np.array(out, np.float32)


@pytest.mark.parametrize("blocks", [4, 48])
@pytest.mark.parametrize("pattern", ["constant", "ramp", "alternating", "pseudo_random"])
def test_q4_0_fused_row_dot_matches_dequantize_reference(blocks, pattern):  # quant.rs:2003-2044
    row = _diag_q4_0_row(blocks)
    x = _diag_input(pattern, blocks * 32)
    ref = orc.matvec(orc.Q4_0, row, blocks * 32, 1, x, reference=True)[0]
    fused = orc.matvec(orc.Q4_0, row, blocks * 32, 1, x)[0]
    scale = max(abs(ref), abs(fused), 1.0)
    assert abs(fused - ref) <= 1e-5 + 1e-6 * scale


def test_quantized_matvec_q8_0():  # quant.rs:2046-2059
    row = q8_0_block(0x3C00, [1] * 32)
    y = orc.matvec(orc.Q8_0, row + row, 32, 2, np.full(32, 2.0, np.float32))
    assert abs(y[0] - 64.0) < 1e-3


def test_quantized_matvec_q4_k():  # quant.rs:2061-2086
    row = struct.pack("<HH", 0x3C00, 0) + bytes([1] * 12) + bytes([0x11] * 128)
    y = orc.matvec(orc.Q4_K, row + row, 256, 2, np.ones(256, np.float32))
    assert abs(y[0] - 256.0) < 1e-3
    yref = orc.matvec(orc.Q4_K, row + row, 256, 2, np.ones(256, np.float32), reference=True)
    assert abs(y[0] - yref[0]) < 1e-3


def test_q4_0_row_range_local_indexing():  # quant.rs:2170-2186 (row-slice of the same rows)
    raw = b"".join(struct.pack("<H", 0x3C00) + bytes([(0x88 + r) & 0xFF] * 16) for r in range(3))
    x = np.ones(32, np.float32)
    full = orc.matvec(orc.Q4_0, raw, 32, 3, x)
    local = orc.matvec(orc.Q4_0, raw[2 * 18:], 32, 1, x)
    assert local[0] == full[2]
    threaded = orc.matvec(orc.Q4_0, raw, 32, 3, x, threads=3)
    assert np.array_equal(threaded, full)


# ---- compute.rs ------------------------------------------------------------------
def test_f32_matvec_explicit_shape():  # compute.rs:565-578
    w = np.array([1, 2, 3, 4, 5, 6], np.float32)
    assert orc.matvec(orc.F32, w.tobytes(), 3, 2, np.ones(3, np.float32)).tolist() == [6.0, 15.0]


def test_row_range_relative_to_local_output():  # compute.rs:580-594
    w = np.array([1, 2, 3, 4, 5, 6], np.float32)
    assert orc.matvec(orc.F32, w[4:].tobytes(), 2, 1, np.ones(2, np.float32)).tolist() == [11.0]


def test_rms_norm_reference():  # compute.rs:596-602
    y = orc.rmsnorm([3.0, 4.0], [1.0, 1.0], 0.0)
    assert abs(y[0] - 0.84852814) < 1e-6 and abs(y[1] - 1.1313709) < 1e-6


def test_swiglu_reference():  # compute.rs:604-611
    y = orc.swiglu(np.array([-1.0, 0.0, 2.0], np.float32), np.array([2.0, 3.0, 4.0], np.float32))
    assert abs(y[0] - (-1.0 / (1.0 + np.exp(1.0)) * 2.0)) < 1e-6
    assert y[1] == 0.0
    assert abs(y[2] - (2.0 / (1.0 + np.exp(-2.0)) * 4.0)) < 1e-6


def test_rope_position_zero_identity():  # compute.rs:613-620
    q, k = orc.rope([1.0, 2.0, 3.0, 4.0], [1.0, 2.0, 3.0, 4.0], 0, 4, 1, 1, 10000.0)
    assert q.tolist() == [1.0, 2.0, 3.0, 4.0] and k.tolist() == q.tolist()


def test_rope_half_split_rotation():  # compute.rs:622-630
    q, k = orc.rope([1.0, 0.0], [1.0, 0.0], 1, 2, 1, 1, 10000.0)
    assert abs(q[0] - np.cos(1.0)) < 1e-6 and abs(q[1] - np.sin(1.0)) < 1e-6
    assert q.tolist() == k.tolist()


def test_gqa_attention_maps_query_heads():  # compute.rs:632-645
    out = orc.attention([1.0, 0.0, 0.0, 1.0], [], [], [1.0, 0.0], [2.0, 3.0], 0, 2, 1, 2)
    assert out.tolist() == [2.0, 3.0, 2.0, 3.0]


def test_quantized_reference_matches_q4_0_and_q6_k_fused_rows():  # compute.rs:647-697
    raw = bytearray(3 * 18)
    for r in range(3):
        raw[r * 18:r * 18 + 2] = struct.pack("<H", 0x3C00)
        raw[r * 18 + 2:(r + 1) * 18] = bytes([(0x11 + r) & 0xFF] * 16)
    x = np.arange(32, dtype=np.float32) * np.float32(0.03125)
    a = orc.matvec(orc.Q4_0, bytes(raw), 32, 3, x, reference=True)
    b = orc.matvec(orc.Q4_0, bytes(raw), 32, 3, x)
    assert np.all(np.abs(a - b) < 1e-3)
    raw6 = bytearray(2 * 210)
    for r in range(2):
        o = r * 210
        raw6[o:o + 128] = bytes(((i + r) & 0xFF) for i in range(128))
        raw6[o + 128:o + 192] = bytes(((i * 3) & 0xFF) for i in range(64))
        raw6[o + 192:o + 208] = bytes([1] * 16)
        raw6[o + 208:o + 210] = struct.pack("<H", 0x3C00)
    x6 = np.sin(np.arange(256, dtype=np.float32) * np.float32(0.0078125)).astype(np.float32)
    a = orc.matvec(orc.Q6_K, bytes(raw6), 256, 2, x6, reference=True)
    b = orc.matvec(orc.Q6_K, bytes(raw6), 256, 2, x6)
    assert np.all(np.abs(a - b) < 1e-3)


@pytest.mark.parametrize("gtype,qk,block", [
    (orc.Q4_0, 32, struct.pack("<H", 0x3C00) + bytes([0x11] * 16)),
    (orc.Q8_0, 32, struct.pack("<H", 0x3C00) + bytes([0x11] * 32)),
    (orc.Q4_K, 256, struct.pack("<HH", 0x3C00, 0) + bytes([0x11] * 140)),
    (orc.Q6_K, 256, bytes([0x11] * 208) + struct.pack("<H", 0x3C00)),
])
def test_quantized_reference_covers_every_format(gtype, qk, block):  # compute.rs:699-767
    x = np.cos(np.arange(qk, dtype=np.float32) * np.float32(0.013)).astype(np.float32)
    a = orc.matvec(gtype, block * 2, qk, 2, x, reference=True)
    b = orc.matvec(gtype, block * 2, qk, 2, x)
    assert np.all(np.abs(a - b) <= 1e-2 + 1e-5 * np.maximum(np.abs(a), np.abs(b)))


# ---- ggml [in, out] layout anchors (tensor.rs:1161-1306) -------------------------
def test_matvec_nonsquare_layout_anchors():
    f32 = np.array([1, 2, 3, 4, 5, 6], np.float32).tobytes()
    assert orc.matvec(orc.F32, f32, 2, 3, np.array([10, 20], np.float32)).tolist() == [50.0, 110.0, 170.0]
    assert orc.matvec(orc.F32, f32, 3, 2, np.array([1, 0, -1], np.float32)).tolist() == [-2.0, -2.0]
    f16 = struct.pack("<4H", 0x3C00, 0x4000, 0x4200, 0x4400)  # 1, 2, 3, 4
    assert np.allclose(orc.matvec(orc.F16, f16, 2, 2, np.ones(2, np.float32)), [3.0, 7.0], atol=1e-3)
    with pytest.raises(orc.OracleError, match="arity mismatch"):  # x of 3 for a 2-input matrix
        orc.matvec(orc.F32, f32, 2, 3, np.ones(3, np.float32))
    q40 = b"".join(q4_0_block(0x3C00, [fill] * 16) * 2 for fill in (0x11, 0x23, 0xF8))
    x = np.array([1.0] * 32 + [2.0] * 32, np.float32)
    y = orc.matvec(orc.Q4_0, q40, 64, 3, x)
    assert np.allclose(y, [-672.0, -528.0, 336.0], atol=1e-3)
    assert np.allclose(y, orc.matvec(orc.Q4_0, q40, 64, 3, x, reference=True), atol=1e-3)
    q4k = b"".join(struct.pack("<HH", 0x3C00, 0) + bytes([1] * 12) + bytes([fill] * 128) for fill in (0x11, 0x22))
    assert np.allclose(orc.matvec(orc.Q4_K, q4k, 256, 2, np.ones(256, np.float32)), [256.0, 512.0], atol=1e-3)


def lcg_q4_0_rows(in_dim, out_dim, seed=0xC0FFEE):
    """The pseudorandom Q4_0 rows of streaming_model.rs:3344-3362: a u32 LCG (1664525,
    1013904223) per row, d = f16 of 0.05 + 0.45 * (s >> 8) / 2^24, nibbles from s."""
    M = 0xFFFFFFFF
    step = lambda v: (v * 1664525 + 1013904223) & M
    out = bytearray()
    for _ in range(out_dim):
        s, seed = seed, step(seed)
        for _ in range(in_dim // 32):
            s = step(s)
            d = np.float32(0.05) + np.float32((s >> 8) / float(1 << 24)) * np.float32(0.45)
            out += np.float16(d).tobytes()
            for _ in range(16):
                s = step(s)
                out.append((s & 0x0F) | (((s >> 4) & 0x0F) << 4))
    return bytes(out)


def test_q4_0_parallel_matvec_matches_scalar_at_qwen2_5_q_shape():  # streaming_model.rs:3332-3411
    n = 1536
    raw = lcg_q4_0_rows(n, n)
    x = (np.sin(np.arange(n, dtype=np.float32) * np.float32(0.0137) - np.float32(0.5)) * np.float32(0.7)).astype(
        np.float32)
    ref = orc.matvec(orc.Q4_0, raw, n, n, x, reference=True)
    got = orc.matvec(orc.Q4_0, raw, n, n, x, threads=4)
    assert np.abs(got - ref).max() < 1e-2


def test_kv_invariants_across_prompt_and_decode():  # inference.rs:2879-3003
    m = orc.OracleModel(fx.gqa_gguf(), kv_f16=False, max_seq=16)
    kvd = fx.GQA_N_KV_HEADS * fx.GQA_HEAD_DIM
    seq, pos = [1, 3, 5, 7], 0
    for step in range(len(seq) + 3):
        assert m.kv_len == pos
        h = m.forward(seq[pos], pos)
        assert m.kv_len == pos + 1
        for which in (False, True):
            assert m.kv_read(0, which, 0, pos + 1).size == (pos + 1) * kvd
        if pos >= len(seq) - 1:
            seq.append(orc.argmax(m.logits(h)))
        pos += 1


def test_greedy_argmax_first_max_wins():  # sampling.rs:45-56
    assert orc.argmax([1.0, 3.0, 3.0, 2.0]) == 1
    assert orc.argmax([5.0]) == 0
    assert orc.argmax([-1.0, -1.0]) == 0


# ---- executor: the GQA forward fixture (inference.rs:2479-2571, EPS 2e-4) -------
def test_gqa_forward_matches_scalar_reference():
    m = orc.OracleModel(fx.gqa_gguf(), kv_f16=False, max_seq=4)
    assert (m.config["n_heads"], m.config["n_kv_heads"], m.config["head_dim"]) == (4, 2, 2)
    w = fx.gqa_weights()
    kh, vh = [], []
    EPS = 2e-4
    for tok, pos in [(3, 0), (7, 1), (11, 2)]:
        hidden = m.forward(tok, pos)
        logits = m.logits(hidden)
        ref_h = fx.gqa_reference_forward(w, tok, pos, kh, vh)
        assert np.all(np.abs(hidden - ref_h) < EPS), (pos, hidden, ref_h)
        ref_logits = w["embd"].reshape(fx.GQA_VOCAB, fx.GQA_N_EMBD) @ ref_h
        assert np.all(np.abs(logits - ref_logits) < EPS)
        assert m.kv_len == pos + 1
        assert m.kv_read(0, False, 0, pos + 1).size == (pos + 1) * fx.GQA_N_KV_HEADS * fx.GQA_HEAD_DIM


# ---- qwen2 Q/K/V biases (inference.rs:1995-2077, streaming_model.rs:3256-3330) ----
def test_qwen2_biased_forward_matches_reference():
    m = orc.OracleModel(fx.qwen2_bias_gguf(), kv_f16=False, max_seq=4)
    assert (m.config["n_heads"], m.config["n_kv_heads"], m.config["head_dim"]) == (2, 2, 4)
    w = fx.qwen2_bias_weights()
    kh, vh = [], []
    EPS = 2e-4
    for tok, pos in [(1, 0), (5, 1)]:  # no history, then history + biases + RoPE at pos 1
        hidden = m.forward(tok, pos)
        ref_h = fx.qwen2_bias_reference_forward(w, tok, pos, kh, vh)
        assert np.all(np.abs(hidden - ref_h) < EPS), (pos, hidden, ref_h)
        ref_logits = w["embd"].reshape(fx.QB_VOCAB, fx.QB_N_EMBD) @ ref_h
        assert np.all(np.abs(m.logits(hidden) - ref_logits) < EPS)
    # the biases change the result: the fixture without them is measurably different
    nb = {k: v for k, v in w.items() if not k.startswith("bias_")}
    assert np.abs(fx.qwen2_bias_reference_forward(nb, 1, 0, [], []) -
                  fx.qwen2_bias_reference_forward(w, 1, 0, [], [])).max() > 10 * EPS
    g = fx.qwen2_bias_gguf()
    t1 = orc.OracleModel(g, kv_f16=False, max_seq=16).generate([1, 3], 4)[0]
    t2 = orc.OracleModel(g, kv_f16=False, max_seq=16).generate([1, 3], 4)[0]
    assert len(t1) == 4 and t1.tolist() == t2.tolist()


def test_qwen2_partial_bias_set_rejected():
    m = orc.OracleModel(fx.qwen2_bias_gguf("only_q"), kv_f16=False, max_seq=4)
    with pytest.raises(orc.OracleError, match="incomplete Q/K/V bias"):
        m.forward(1, 0)


def test_qwen2_bias_shape_mismatch_rejected():
    m = orc.OracleModel(fx.qwen2_bias_gguf("wrong_dim"), kv_f16=False, max_seq=4)
    with pytest.raises(orc.OracleError, match="attn_q.bias.*shape"):
        m.forward(1, 0)


def test_gqa_greedy_generation_is_deterministic():  # inference.rs:2567-2571
    g = fx.gqa_gguf()
    t1 = orc.OracleModel(g, kv_f16=False, max_seq=16).generate([1, 3], 5)[0]
    t2 = orc.OracleModel(g, kv_f16=False, max_seq=16).generate([1, 3], 5)[0]
    assert len(t1) == 5 and t1.tolist() == t2.tolist()


def test_forward_position_must_match_history():  # streaming_model.rs:921-928
    m = orc.OracleModel(fx.gqa_gguf(), kv_f16=False, max_seq=4)
    with pytest.raises(orc.OracleError, match="position"):
        m.forward(3, 1)
    m.forward(3, 0)
    with pytest.raises(orc.OracleError, match="position"):
        m.forward(3, 0)


def test_kv_f16_mode_rounds_history_only():
    g = fx.gqa_gguf()
    a = orc.OracleModel(g, kv_f16=False, max_seq=8)
    b = orc.OracleModel(g, kv_f16=True, max_seq=8)
    ha = a.forward(3, 0)
    hb = b.forward(3, 0)
    assert np.array_equal(ha, hb)  # position 0 attends only to the current (f32) K/V
    ka, kb = a.kv_read(0, False, 0, 1), b.kv_read(0, False, 0, 1)
    assert np.array_equal(kb, ka.astype(np.float16).astype(np.float32))
