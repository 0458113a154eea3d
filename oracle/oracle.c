/*
 * oracle.c - CPU restatement of RAMforge's legacy decode hot path.
 *
 * TEST INFRASTRUCTURE ONLY (the parity checker, never the product).  See
 * oracle.h for who may load it.  Compile with -O2 -ffp-contract=off and no
 * -ffast-math: every float expression below is evaluated left to right with
 * one IEEE rounding per operation, as the Rust reference does (Rust never
 * contracts a*b+c into an FMA).
 *
 * Reference paths cited as crates/<crate>/src/<file>:<line>.
 */
#define _GNU_SOURCE
#include "oracle.h"

#include <math.h>
#include <pthread.h>
#include <stdarg.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

static __thread char g_err[512];
static void set_err(const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_err, sizeof g_err, fmt, ap);
  va_end(ap);
}
const char* orc_last_error(void) { return g_err; }

/* ---------------------------------------------------------------------
 * f16 <-> f32
 * ------------------------------------------------------------------- */

/* Half -> single exactly as the reference does it (ramforge-core/src/quant.rs:40-65,
 * identical copy at tensor.rs:1017-1041).  Normal numbers, zeros, inf and NaN are
 * IEEE-exact; a subnormal is normalised by shifting, but the exponent it gets is
 * 127-15-e where IEEE needs 127-15-e+1, so every subnormal half decodes to half
 * its IEEE value.  Restated as is: block scales and F16 tensors go through it. */
float orc_f16_to_f32(uint16_t bits) {
  uint32_t sign = (bits >> 15) & 1u, exp = (bits >> 10) & 0x1Fu, frac = bits & 0x3FFu, out;
  if (exp == 0) {
    if (frac == 0) {
      out = sign << 31;
    } else {
      uint32_t e = 0, f = frac;
      while ((f & 0x400u) == 0) { f <<= 1; e++; }
      f &= 0x3FFu;
      out = (sign << 31) | ((127u - 15u - e) << 23) | (f << 13);
    }
  } else if (exp == 0x1F) {
    out = (sign << 31) | (0xFFu << 23) | (frac << 13);
  } else {
    out = (sign << 31) | ((exp + 127u - 15u) << 23) | (frac << 13);
  }
  float r;
  memcpy(&r, &out, 4);
  return r;
}

/* Round-to-nearest-even single -> half.  The reference has no f16 KV cache
 * (its cache is f32, ramforge-runtime/src/kv_cache.rs:28-29); this is the
 * build's kv_f16 mode, matching the GPU cache's __float2half_rn. */
uint16_t orc_f32_to_f16(float f) {
  uint32_t x;
  memcpy(&x, &f, 4);
  uint32_t sign = (x >> 16) & 0x8000u;
  uint32_t ax = x & 0x7FFFFFFFu;
  if (ax >= 0x7F800000u) /* inf / nan */
    return (uint16_t)(sign | 0x7C00u | (ax > 0x7F800000u ? 0x200u | ((ax >> 13) & 0x3FFu) : 0));
  if (ax >= 0x477FF000u) return (uint16_t)(sign | 0x7C00u); /* rounds to inf */
  if (ax < 0x38800000u) {                                   /* subnormal half or zero */
    if (ax < 0x33000000u) return (uint16_t)sign;            /* < 2^-25: rounds to 0 */
    uint32_t e = ax >> 23, m = (ax & 0x7FFFFFu) | 0x800000u;
    uint32_t shift = 126u - e; /* 14 + (112 - e) + ... : value = m * 2^(e-150) */
    /* half subnormal unit = 2^-24 ; m*2^(e-150) / 2^-24 = m >> (126 - e) */
    uint32_t q = m >> shift, rem = m & ((1u << shift) - 1u), half = 1u << (shift - 1u);
    if (rem > half || (rem == half && (q & 1u))) q++;
    return (uint16_t)(sign | q);
  }
  uint32_t e = (ax >> 23) - 112u, m = ax & 0x7FFFFFu;
  uint32_t q = (e << 10) | (m >> 13), rem = m & 0x1FFFu;
  if (rem > 0x1000u || (rem == 0x1000u && (q & 1u))) q++;
  return (uint16_t)(sign | q);
}

/* IEEE half -> single, for the build's kv_f16 cache mode only (the GPU cache uses
 * __float2half_rn / __half2float; the reference has no f16 cache). */
static float ieee_f16_to_f32(uint16_t h) {
  uint32_t sign = (uint32_t)(h & 0x8000u) << 16, e = (h >> 10) & 0x1Fu, m = h & 0x3FFu, o;
  if (e == 0) {
    if (m == 0) o = sign;
    else {
      int s = 0;
      while (!(m & 0x400u)) { m <<= 1; s++; }
      o = sign | ((uint32_t)(113 - s) << 23) | ((m & 0x3FFu) << 13);
    }
  } else if (e == 31) o = sign | 0x7F800000u | (m << 13);
  else o = sign | ((e + 112u) << 23) | (m << 13);
  float r;
  memcpy(&r, &o, 4);
  return r;
}

static float rd_f16(const uint8_t* p) { return orc_f16_to_f32((uint16_t)(p[0] | (p[1] << 8))); }

/* ---------------------------------------------------------------------
 * block layouts (ramforge-core/src/quant.rs:5-13, :24-37)
 * ------------------------------------------------------------------- */
static int type_block(int type, size_t* qk, size_t* bsz) {
  switch (type) {
    case ORC_F32: *qk = 1; *bsz = 4; return 1;
    case ORC_F16: *qk = 1; *bsz = 2; return 1;
    case ORC_Q4_0: *qk = 32; *bsz = 18; return 1;
    case ORC_Q5_0: *qk = 32; *bsz = 22; return 1;
    case ORC_Q8_0: *qk = 32; *bsz = 34; return 1;
    case ORC_Q2_K: *qk = 256; *bsz = 84; return 1;
    case ORC_Q3_K: *qk = 256; *bsz = 110; return 1;
    case ORC_Q4_K: *qk = 256; *bsz = 144; return 1;
    case ORC_Q5_K: *qk = 256; *bsz = 176; return 1;
    case ORC_Q6_K: *qk = 256; *bsz = 210; return 1;
    case ORC_Q8_K: *qk = 256; *bsz = 292; return 1;
    default: return 0;
  }
}

size_t orc_row_bytes(int type, size_t n) {
  size_t qk, bsz;
  if (!type_block(type, &qk, &bsz) || n % qk) return 0;
  return n / qk * bsz;
}

/* BlockQ4_0::dequantize (quant.rs:104-112): out[j] = (q_lo-8)*d, out[16+j] = (q_hi-8)*d. */
static void dq_q4_0(const uint8_t* b, float* out) {
  float d = rd_f16(b);
  for (int j = 0; j < 16; j++) {
    uint8_t byte = b[2 + j];
    int q0 = (int)(byte & 0x0F) - 8, q1 = (int)(byte >> 4) - 8;
    out[j] = (float)q0 * d;
    out[16 + j] = (float)q1 * d;
  }
}

/* BlockQ5_0::dequantize (quant.rs:139-151). */
static void dq_q5_0(const uint8_t* b, float* out) {
  float d = rd_f16(b);
  uint32_t qh = (uint32_t)b[2] | ((uint32_t)b[3] << 8) | ((uint32_t)b[4] << 16) | ((uint32_t)b[5] << 24);
  const uint8_t* qs = b + 6;
  for (int j = 0; j < 16; j++) {
    uint8_t xh0 = (uint8_t)(((qh >> j) << 4) & 0x10);
    uint8_t xh1 = (uint8_t)((qh >> (j + 12)) & 0x10);
    int q0 = (int)((qs[j] & 0x0F) | xh0) - 16;
    int q1 = (int)((qs[j] >> 4) | xh1) - 16;
    out[j] = (float)q0 * d;
    out[16 + j] = (float)q1 * d;
  }
}

/* BlockQ8_0::dequantize (quant.rs:176-180): out[i] = q*d. */
static void dq_q8_0(const uint8_t* b, float* out) {
  float d = rd_f16(b);
  for (int i = 0; i < 32; i++) out[i] = (float)(int8_t)b[2 + i] * d;
}

/* BlockQ4K::get_scale_min (quant.rs:216-226). */
static void q4k_scale_min(const uint8_t* s, int j, uint8_t* sc, uint8_t* m) {
  if (j < 4) {
    *sc = s[j] & 63;
    *m = s[j + 4] & 63;
  } else {
    *sc = (uint8_t)((s[j + 4] & 0xF) | ((s[j - 4] >> 6) << 4));
    *m = (uint8_t)((s[j + 4] >> 4) | ((s[j] >> 6) << 4));
  }
}

/* BlockQ4K::dequantize (quant.rs:228-254): per 64 elements, d1 = d*sc, min1 = dmin*m,
 * value = d1*q - min1 (mul then sub, two roundings). */
static void dq_q4_k(const uint8_t* b, float* out) {
  float d = rd_f16(b), dmin = rd_f16(b + 2);
  const uint8_t* s = b + 4;
  const uint8_t* qs = b + 16;
  int y = 0, is = 0, qo = 0;
  for (int g = 0; g < 4; g++) {
    uint8_t sc0, m0, sc1, m1;
    q4k_scale_min(s, is, &sc0, &m0);
    q4k_scale_min(s, is + 1, &sc1, &m1);
    float d1 = d * (float)sc0, min1 = dmin * (float)m0;
    float d2 = d * (float)sc1, min2 = dmin * (float)m1;
    for (int l = 0; l < 32; l++) out[y + l] = d1 * (float)(qs[qo + l] & 0x0F) - min1;
    y += 32;
    for (int l = 0; l < 32; l++) out[y + l] = d2 * (float)(qs[qo + l] >> 4) - min2;
    y += 32;
    qo += 32;
    is += 2;
  }
}

/* BlockQ5K::dequantize (quant.rs:303-343): per 64 elements d1 = d*sc, min1 = dmin*m
 * (get_scale_min as Q4_K's, :288-299), value = d1*(q + 16*high) - min1.  The high
 * bit of element l of group g is bit 2g (low nibbles) or 2g+1 (high nibbles) of
 * qh[8g + l/8], the reference's own indexing. */
static void dq_q5_k(const uint8_t* b, float* out) {
  float d = rd_f16(b), dmin = rd_f16(b + 2);
  const uint8_t* s = b + 4;
  const uint8_t* qh = b + 16;
  const uint8_t* qs = b + 48;
  int y = 0, is = 0, qo = 0;
  uint8_t u1 = 1, u2 = 2;
  for (int g = 0; g < 4; g++) {
    uint8_t sc0, m0, sc1, m1;
    q4k_scale_min(s, is, &sc0, &m0);
    q4k_scale_min(s, is + 1, &sc1, &m1);
    float d1 = d * (float)sc0, min1 = dmin * (float)m0;
    float d2 = d * (float)sc1, min2 = dmin * (float)m1;
    for (int l = 0; l < 32; l++) {
      int q = (qs[qo + l] & 0xF) + ((qh[qo / 4 + l / 8] & u1) ? 16 : 0);
      out[y + l] = d1 * (float)q - min1;
    }
    y += 32;
    for (int l = 0; l < 32; l++) {
      int q = (qs[qo + l] >> 4) + ((qh[qo / 4 + l / 8] & u2) ? 16 : 0);
      out[y + l] = d2 * (float)q - min2;
    }
    y += 32;
    qo += 32;
    is += 2;
    u1 = (uint8_t)(u1 << 2);
    u2 = (uint8_t)(u2 << 2);
  }
}

/* BlockQ2K::dequantize (quant.rs:443-474): 16 scale bytes (low nibble scale, high
 * nibble min), value = (d*sc)*q - dmin*m for 2-bit q. */
static void dq_q2_k(const uint8_t* b, float* out) {
  const uint8_t* sc = b;
  const uint8_t* qs = b + 16;
  float d = rd_f16(b + 80), dmin = rd_f16(b + 82);
  int y = 0, is = 0, qo = 0;
  for (int n = 0; n < 2; n++) {
    int shift = 0;
    for (int j = 0; j < 4; j++) {
      for (int half = 0; half < 2; half++) {
        uint8_t v = sc[is++];
        float dl = d * (float)(v & 0xF), ml = dmin * (float)(v >> 4);
        for (int l = 0; l < 16; l++) out[y + l] = dl * (float)((qs[qo + 16 * half + l] >> shift) & 3) - ml;
        y += 16;
      }
      shift += 2;
    }
    qo += 32;
  }
}

/* BlockQ3K::dequantize (quant.rs:506-574): the 12 scale bytes unpack to 16 six-bit
 * scales (minus 32); q = 2 low bits - (hmask bit clear ? 4 : 0); value (d*sc)*q.
 * As in the reference, both 128-element halves use scales 0-7 (j and j+4). */
static void dq_q3_k(const uint8_t* b, float* out) {
  const uint8_t* hm = b;
  const uint8_t* qs = b + 32;
  const uint8_t* sb = b + 96;
  float d = rd_f16(b + 108);
  uint32_t aux[4];
  for (int i = 0; i < 3; i++) aux[i] = (uint32_t)sb[4 * i] | ((uint32_t)sb[4 * i + 1] << 8) |
                                       ((uint32_t)sb[4 * i + 2] << 16) | ((uint32_t)sb[4 * i + 3] << 24);
  const uint32_t k1 = 0x03030303u, k2 = 0x0F0F0F0Fu, tmp = aux[2], a0 = aux[0], a1 = aux[1];
  aux[2] = ((a0 >> 4) & k2) | (((tmp >> 4) & k1) << 4);
  aux[3] = ((a1 >> 4) & k2) | (((tmp >> 6) & k1) << 4);
  aux[0] = (a0 & k2) | (((tmp >> 0) & k1) << 4);
  aux[1] = (a1 & k2) | (((tmp >> 2) & k1) << 4);
  int8_t s8[16];
  for (int i = 0; i < 16; i++) s8[i] = (int8_t)(uint8_t)(aux[i / 4] >> (8 * (i % 4)));
  int y = 0, qo = 0;
  uint8_t m = 1;
  for (int n = 0; n < 2; n++) {
    int shift = 0;
    for (int j = 0; j < 4; j++) {
      for (int half = 0; half < 2; half++) {
        float dl = d * (float)((int)s8[j + 4 * half] - 32);
        for (int l = 0; l < 16; l++) {
          int q = (qs[qo + 16 * half + l] >> shift) & 3;
          q -= (hm[16 * half + l] & m) ? 0 : 4;
          out[y + l] = dl * (float)q;
        }
        y += 16;
      }
      shift += 2;
      m = (uint8_t)(m << 1);
    }
    qo += 32;
  }
}

/* BlockQ8K::dequantize (quant.rs:605-609): f32 d, value d*q. */
static void dq_q8_k(const uint8_t* b, float* out) {
  float d;
  memcpy(&d, b, 4);
  for (int i = 0; i < 256; i++) out[i] = d * (float)(int8_t)b[4 + i];
}

/* BlockQ6K::dequantize (quant.rs:376-406): value = (d*sc)*q. */
static void dq_q6_k(const uint8_t* b, float* out) {
  const uint8_t* ql = b;
  const uint8_t* qh = b + 128;
  const int8_t* sc = (const int8_t*)(b + 192);
  float d = rd_f16(b + 208);
  int y = 0, qlo = 0, qho = 0, so = 0;
  for (int h = 0; h < 2; h++) {
    for (int l = 0; l < 32; l++) {
      int is = l / 16;
      int q1 = (int)(int8_t)((ql[qlo + l] & 0xF) | ((qh[qho + l] & 3) << 4)) - 32;
      int q2 = (int)(int8_t)((ql[qlo + 32 + l] & 0xF) | (((qh[qho + l] >> 2) & 3) << 4)) - 32;
      int q3 = (int)(int8_t)((ql[qlo + l] >> 4) | (((qh[qho + l] >> 4) & 3) << 4)) - 32;
      int q4 = (int)(int8_t)((ql[qlo + 32 + l] >> 4) | (((qh[qho + l] >> 6) & 3) << 4)) - 32;
      out[y + l] = d * (float)sc[so + is] * (float)q1;
      out[y + l + 32] = d * (float)sc[so + is + 2] * (float)q2;
      out[y + l + 64] = d * (float)sc[so + is + 4] * (float)q3;
      out[y + l + 96] = d * (float)sc[so + is + 6] * (float)q4;
    }
    y += 128;
    qlo += 64;
    qho += 32;
    so += 8;
  }
}

/* dequantize_row_* (quant.rs:615-868) and the F32/F16 TensorData views
 * (tensor.rs:460-562, F16 rows converted by f16_to_f32). */
int orc_dequant_row(int type, const uint8_t* bytes, size_t nbytes, size_t n, float* out) {
  size_t qk, bsz;
  if (!type_block(type, &qk, &bsz)) { set_err("unsupported type %d", type); return -1; }
  if (n % qk) { set_err("row size %zu not divisible by block size %zu", n, qk); return -1; }
  size_t nb = n / qk;
  if (nbytes < nb * bsz) { set_err("row truncated: expected %zu bytes, got %zu", nb * bsz, nbytes); return -1; }
  for (size_t i = 0; i < nb; i++) {
    const uint8_t* b = bytes + i * bsz;
    float* o = out + i * qk;
    switch (type) {
      case ORC_F32: memcpy(o, b, 4); break;
      case ORC_F16: o[0] = rd_f16(b); break;
      case ORC_Q4_0: dq_q4_0(b, o); break;
      case ORC_Q5_0: dq_q5_0(b, o); break;
      case ORC_Q8_0: dq_q8_0(b, o); break;
      case ORC_Q4_K: dq_q4_k(b, o); break;
      case ORC_Q6_K: dq_q6_k(b, o); break;
      case ORC_Q2_K: dq_q2_k(b, o); break;
      case ORC_Q3_K: dq_q3_k(b, o); break;
      case ORC_Q5_K: dq_q5_k(b, o); break;
      case ORC_Q8_K: dq_q8_k(b, o); break;
    }
  }
  return 0;
}

/* ---------------------------------------------------------------------
 * per-row dot products in the runtime kernel order
 * ------------------------------------------------------------------- */

/* q4_0_row_dot (quant.rs:875-895): sum += (q_lo*d)*x[j]; sum += (q_hi*d)*x[16+j]. */
static float row_dot_q4_0(const uint8_t* row, size_t nb, const float* x) {
  float sum = 0.0f;
  for (size_t b = 0; b < nb; b++) {
    const uint8_t* p = row + b * 18;
    float d = rd_f16(p);
    const float* xb = x + b * 32;
    for (int j = 0; j < 16; j++) {
      uint8_t byte = p[2 + j];
      int q0 = (int)(byte & 0x0F) - 8, q1 = (int)(byte >> 4) - 8;
      sum += (float)q0 * d * xb[j];
      sum += (float)q1 * d * xb[16 + j];
    }
  }
  return sum;
}

/* matvec_q8_0 inner loop (quant.rs:1014-1025): decode block, sum += deq[j]*x[j]. */
static float row_dot_q8_0(const uint8_t* row, size_t nb, const float* x) {
  float sum = 0.0f, deq[32];
  for (size_t b = 0; b < nb; b++) {
    dq_q8_0(row + b * 34, deq);
    const float* xb = x + b * 32;
    for (int j = 0; j < 32; j++) sum += deq[j] * xb[j];
  }
  return sum;
}

/* matvec_q4_k inner loop (quant.rs:1121-1134): decode superblock, sequential dot. */
static float row_dot_q4_k(const uint8_t* row, size_t nb, const float* x) {
  float sum = 0.0f, deq[256];
  for (size_t b = 0; b < nb; b++) {
    dq_q4_k(row + b * 144, deq);
    const float* xb = x + b * 256;
    for (int j = 0; j < 256; j++) sum += deq[j] * xb[j];
  }
  return sum;
}

/* q6_k_row_dot (quant.rs:1194-1252): sum += ((sc*d)*q)*x in dequantize order. */
static float row_dot_q6_k(const uint8_t* row, size_t nb, const float* x) {
  float sum = 0.0f;
  for (size_t b = 0; b < nb; b++) {
    const uint8_t* ql = row + b * 210;
    const uint8_t* qh = ql + 128;
    const int8_t* sc = (const int8_t*)(ql + 192);
    float d = rd_f16(ql + 208);
    const float* xb = x + b * 256;
    int xo = 0, qlo = 0, qho = 0, so = 0;
    for (int h = 0; h < 2; h++) {
      for (int l = 0; l < 32; l++) {
        int is = l / 16;
        uint8_t qhb = qh[qho + l], lo = ql[qlo + l], hi = ql[qlo + 32 + l];
        float s1 = (float)sc[so + is] * d, s2 = (float)sc[so + is + 2] * d;
        float s3 = (float)sc[so + is + 4] * d, s4 = (float)sc[so + is + 6] * d;
        int q1 = (int)(int8_t)((lo & 0x0F) | ((qhb & 0x03) << 4)) - 32;
        int q2 = (int)(int8_t)((hi & 0x0F) | (((qhb >> 2) & 0x03) << 4)) - 32;
        int q3 = (int)(int8_t)((lo >> 4) | (((qhb >> 4) & 0x03) << 4)) - 32;
        int q4 = (int)(int8_t)((hi >> 4) | (((qhb >> 6) & 0x03) << 4)) - 32;
        sum += s1 * (float)q1 * xb[xo + l];
        sum += s2 * (float)q2 * xb[xo + l + 32];
        sum += s3 * (float)q3 * xb[xo + l + 64];
        sum += s4 * (float)q4 * xb[xo + l + 96];
      }
      xo += 128;
      qlo += 64;
      qho += 32;
      so += 8;
    }
  }
  return sum;
}

/* Generic decode-then-dot (quantized_matvec_reference, compute.rs:185-229;
 * also the F32 reference matvec, compute.rs:105-120, and F16 tensors which
 * the reference stores as f32 after load). */
static float row_dot_decoded(int type, const uint8_t* row, size_t rb, size_t in, const float* x,
                             float* scratch) {
  orc_dequant_row(type, row, rb, in, scratch);
  float sum = 0.0f;
  for (size_t i = 0; i < in; i++) sum += scratch[i] * x[i];
  return sum;
}

typedef struct {
  int type;
  const uint8_t* w;
  size_t rb, in, r0, r1;
  const float* x;
  float* y;
  int use_reference;
} mv_job;

static void* mv_worker(void* arg) {
  mv_job* j = (mv_job*)arg;
  float* scratch = NULL;
  /* matvec_q5_0/_q5_k/_q2_k/_q3_k/_q8_k (quant.rs:1050-1490) decode each block then
   * sum deq[j]*x[j] in order: the generic decode-then-dot */
  int decoded = j->use_reference || j->type == ORC_F32 || j->type == ORC_F16 || j->type == ORC_Q5_0 ||
                j->type == ORC_Q2_K || j->type == ORC_Q3_K || j->type == ORC_Q5_K || j->type == ORC_Q8_K;
  if (decoded) scratch = (float*)malloc(sizeof(float) * (j->in ? j->in : 1));
  for (size_t r = j->r0; r < j->r1; r++) {
    const uint8_t* row = j->w + r * j->rb;
    float v;
    if (decoded) {
      v = row_dot_decoded(j->type, row, j->rb, j->in, j->x, scratch);
    } else {
      switch (j->type) {
        case ORC_Q4_0: v = row_dot_q4_0(row, j->in / 32, j->x); break;
        case ORC_Q8_0: v = row_dot_q8_0(row, j->in / 32, j->x); break;
        case ORC_Q4_K: v = row_dot_q4_k(row, j->in / 256, j->x); break;
        default: v = row_dot_q6_k(row, j->in / 256, j->x); break;
      }
    }
    j->y[r] = v;
  }
  free(scratch);
  return NULL;
}

static int matvec_impl(int type, const uint8_t* w, size_t wbytes, size_t in, size_t out,
                       const float* x, float* y, int threads, int use_reference) {
  size_t rb = orc_row_bytes(type, in);
  if (rb == 0) { set_err("type %d: in_dim %zu not a block multiple (or unsupported)", type, in); return -1; }
  if (wbytes < rb * out) { set_err("weight truncated: expected %zu bytes, got %zu", rb * out, wbytes); return -1; }
  if (threads < 1) threads = 1;
  if ((size_t)threads > out) threads = out ? (int)out : 1;
  mv_job jobs[256];
  pthread_t tids[256];
  if (threads > 256) threads = 256;
  /* make_row_chunks (compute_dispatch.rs:75-88): contiguous ranges, at most one row of imbalance. */
  size_t base = out / threads, extra = out % threads, cur = 0;
  for (int t = 0; t < threads; t++) {
    size_t cnt = base + ((size_t)t < extra ? 1 : 0);
    jobs[t] = (mv_job){type, w, rb, in, cur, cur + cnt, x, y, use_reference};
    cur += cnt;
  }
  if (threads == 1) {
    mv_worker(&jobs[0]);
    return 0;
  }
  for (int t = 1; t < threads; t++) pthread_create(&tids[t], NULL, mv_worker, &jobs[t]);
  mv_worker(&jobs[0]);
  for (int t = 1; t < threads; t++) pthread_join(tids[t], NULL);
  return 0;
}

int orc_matvec(int type, const uint8_t* w, size_t wbytes, size_t in, size_t out, const float* x,
               float* y, int threads) {
  return matvec_impl(type, w, wbytes, in, out, x, y, threads, 0);
}

int orc_matvec_reference(int type, const uint8_t* w, size_t wbytes, size_t in, size_t out,
                         const float* x, float* y) {
  return matvec_impl(type, w, wbytes, in, out, x, y, 1, 1);
}

/* ---------------------------------------------------------------------
 * numeric core (ramforge-core/src/compute.rs)
 * ------------------------------------------------------------------- */

/* rms_norm_reference (compute.rs:291-319): rms = sqrt(sum(x^2)/n + eps); y = x / rms * w. */
int orc_rmsnorm(const float* x, const float* w, float eps, size_t n, float* y) {
  if (n == 0) { set_err("RMSNorm shape mismatch"); return -1; }
  if (!isfinite(eps) || eps < 0.0f) { set_err("RMSNorm epsilon must be finite and non-negative"); return -1; }
  float ss = 0.0f;
  for (size_t i = 0; i < n; i++) ss += x[i] * x[i];
  float rms = sqrtf(ss / (float)n + eps);
  for (size_t i = 0; i < n; i++) y[i] = x[i] / rms * w[i];
  return 0;
}

/* silu_reference (compute.rs:337-350): v / (1 + exp(-v)). */
void orc_silu(const float* x, float* y, size_t n) {
  for (size_t i = 0; i < n; i++) {
    float v = x[i];
    y[i] = v / (1.0f + expf(-v));
  }
}

/* swiglu_reference (compute.rs:354-361) == silu then mul_reference (compute.rs:328-335),
 * which is what the executor runs (model_executor.rs:229-230). */
void orc_swiglu(const float* g, const float* u, float* y, size_t n) {
  for (size_t i = 0; i < n; i++) {
    float v = g[i];
    float s = v / (1.0f + expf(-v));
    y[i] = s * u[i];
  }
}

/* softmax_reference (compute.rs:363-384): max via f32::max fold from -inf,
 * exp(v - max), sequential sum, divide. */
int orc_softmax(float* v, size_t n) {
  if (n == 0) { set_err("softmax requires a non-empty vector"); return -1; }
  float mx = -INFINITY;
  for (size_t i = 0; i < n; i++) mx = fmaxf(mx, v[i]);
  float sum = 0.0f;
  for (size_t i = 0; i < n; i++) {
    v[i] = expf(v[i] - mx);
    sum += v[i];
  }
  if (!isfinite(sum) || sum == 0.0f) { set_err("softmax normalization is not finite"); return -1; }
  for (size_t i = 0; i < n; i++) v[i] /= sum;
  return 0;
}

/* rope_head (compute.rs:440-456): half-split pairs (i, i+hd/2);
 * angle = theta^(-2i/hd) * pos evaluated in f32; first*cos - second*sin. */
static void rope_head(float* v, size_t hd, size_t pos, float theta) {
  size_t half = hd / 2;
  for (size_t i = 0; i < half; i++) {
    float e = -2.0f * (float)i / (float)hd;
    float angle = powf(theta, e) * (float)pos;
    float c = cosf(angle), s = sinf(angle);
    float a = v[i], b = v[i + half];
    v[i] = a * c - b * s;
    v[i + half] = a * s + b * c;
  }
}

/* rope_reference (compute.rs:389-438). */
int orc_rope(float* q, float* k, size_t pos, size_t hd, size_t nh, size_t nkv, float theta) {
  if (hd == 0 || hd % 2) { set_err("RoPE head dimension must be non-zero and even"); return -1; }
  if (nh == 0 || nkv == 0) { set_err("RoPE requires non-zero query and KV head counts"); return -1; }
  if (!isfinite(theta) || theta <= 0.0f) { set_err("RoPE frequency base must be finite and positive"); return -1; }
  for (size_t h = 0; h < nh; h++) rope_head(q + h * hd, hd, pos, theta);
  for (size_t h = 0; h < nkv; h++) rope_head(k + h * hd, hd, pos, theta);
  return 0;
}

/* attention_reference (compute.rs:461-547): kv_head = h*KV/H; score = dot/sqrt(hd);
 * softmax over hist+1 positions (the last is the current K/V); out += p*v. */
int orc_attention(const float* q, const float* kh, const float* vh, const float* kc,
                  const float* vc, size_t hist, size_t nh, size_t nkv, size_t hd, float* out) {
  if (nh == 0 || nkv == 0 || hd == 0) { set_err("attention requires non-zero dims"); return -1; }
  if (nh % nkv) { set_err("GQA requires query_heads %zu divisible by kv_heads %zu", nh, nkv); return -1; }
  size_t kvw = nkv * hd, total = hist + 1;
  float* scores = (float*)malloc(sizeof(float) * total);
  if (!scores) { set_err("failed to reserve attention scores"); return -1; }
  memset(out, 0, sizeof(float) * nh * hd);
  float sq = sqrtf((float)hd);
  for (size_t h = 0; h < nh; h++) {
    size_t kvh = h * nkv / nh;
    const float* qh = q + h * hd;
    for (size_t p = 0; p < total; p++) {
      const float* kall = p < hist ? kh + p * kvw : kc;
      const float* k = kall + kvh * hd;
      float dot = 0.0f;
      for (size_t i = 0; i < hd; i++) dot += qh[i] * k[i];
      scores[p] = dot / sq;
    }
    if (orc_softmax(scores, total)) { free(scores); return -1; }
    float* oh = out + h * hd;
    for (size_t p = 0; p < total; p++) {
      const float* vall = p < hist ? vh + p * kvw : vc;
      const float* v = vall + kvh * hd;
      for (size_t i = 0; i < hd; i++) oh[i] += scores[p] * v[i];
    }
  }
  free(scores);
  return 0;
}

/* Sampler::sample_checked greedy branch (ramforge-runtime/src/sampling.rs:45-56):
 * strict '>' so the lowest index wins ties; empty -> 0. */
uint32_t orc_argmax(const float* logits, size_t n) {
  if (n == 0) return 0;
  size_t best = 0;
  float bv = logits[0];
  for (size_t i = 1; i < n; i++)
    if (logits[i] > bv) { bv = logits[i]; best = i; }
  return (uint32_t)best;
}

/* ---------------------------------------------------------------------
 * GGUF (ramforge-core/src/gguf.rs:196-330) and LlamaConfig
 * (ramforge-runtime/src/model.rs:40-161)
 * ------------------------------------------------------------------- */
typedef struct {
  char* name;
  uint32_t ndims;
  uint64_t dims[8];
  uint32_t type;
  uint64_t offset;      /* relative to the aligned data start */
  const uint8_t* data;  /* resolved pointer */
  uint64_t nbytes;
} orc_tensor;

typedef struct {
  char* key;
  uint32_t vtype;
  uint64_t u;  /* integer payload (as_u64 semantics) */
  int has_u;
  double f;    /* float payload */
  int has_f;
  char* str;
  uint64_t arr_len;
} orc_kv;

typedef struct {
  const uint8_t* p;
  size_t len, pos;
  int err;
} rdr;

static int rd(rdr* r, void* dst, size_t n) {
  if (r->pos + n > r->len) { r->err = 1; return -1; }
  if (dst) memcpy(dst, r->p + r->pos, n);
  r->pos += n;
  return 0;
}
static uint64_t rd_u64(rdr* r) { uint64_t v = 0; rd(r, &v, 8); return v; }
static uint32_t rd_u32(rdr* r) { uint32_t v = 0; rd(r, &v, 4); return v; }
static char* rd_str(rdr* r) {
  uint64_t n = rd_u64(r);
  if (r->err || n > 10u * 1024u * 1024u || r->pos + n > r->len) { r->err = 1; return NULL; }
  char* s = (char*)malloc(n + 1);
  memcpy(s, r->p + r->pos, n);
  s[n] = 0;
  r->pos += n;
  return s;
}

/* Reads one scalar of GGUF value type `t` into kv (gguf.rs:130-151; as_u64 at types.rs:86-98). */
static void rd_scalar(rdr* r, uint32_t t, orc_kv* kv) {
  uint8_t b1 = 0; uint16_t b2 = 0; uint32_t b4 = 0; uint64_t b8 = 0;
  switch (t) {
    case 0: rd(r, &b1, 1); kv->u = b1; kv->has_u = 1; break;
    case 1: rd(r, &b1, 1); kv->u = (uint64_t)(int64_t)(int8_t)b1; kv->has_u = 1; break;
    case 2: rd(r, &b2, 2); kv->u = b2; kv->has_u = 1; break;
    case 3: rd(r, &b2, 2); kv->u = (uint64_t)(int64_t)(int16_t)b2; kv->has_u = 1; break;
    case 4: rd(r, &b4, 4); kv->u = b4; kv->has_u = 1; kv->f = (double)b4; kv->has_f = 1; break;
    case 5: rd(r, &b4, 4); kv->u = (uint64_t)(int64_t)(int32_t)b4; kv->has_u = 1; kv->f = (double)(int32_t)b4; kv->has_f = 1; break;
    case 6: { float f; rd(r, &f, 4); kv->f = f; kv->has_f = 1; break; }
    case 7: rd(r, &b1, 1); break;
    case 8: free(rd_str(r)); break;
    case 10: rd(r, &b8, 8); kv->u = b8; kv->has_u = 1; kv->f = (double)b8; kv->has_f = 1; break;
    case 11: rd(r, &b8, 8); kv->u = b8; kv->has_u = 1; kv->f = (double)(int64_t)b8; kv->has_f = 1; break;
    case 12: { double d; rd(r, &d, 8); kv->f = d; kv->has_f = 1; break; }
    default: r->err = 1;
  }
}

struct orc_model {
  orc_config cfg;
  int kv_f16, threads;
  uint32_t max_seq, seq_len;
  size_t n_kv;
  orc_kv* kvs;
  size_t n_t;
  orc_tensor* ts;
  /* per layer tensor pointers */
  orc_tensor** L; /* [n_layers][9] */
  orc_tensor *embd, *onorm, *out;
  float* kcache; /* [layers][max_seq][kv_dim] */
  float* vcache;
  float* layer_hidden; /* [layers][n_embd] of the last forward */
};

static const orc_kv* find_kv(const orc_model* m, const char* key) {
  for (size_t i = 0; i < m->n_kv; i++)
    if (strcmp(m->kvs[i].key, key) == 0) return &m->kvs[i];
  return NULL;
}
static orc_tensor* find_t(orc_model* m, const char* name) {
  for (size_t i = 0; i < m->n_t; i++)
    if (strcmp(m->ts[i].name, name) == 0) return &m->ts[i];
  return NULL;
}

/* get_u64_arch (model.rs:54-77): {arch}., llama., qwen2., general. */
static int get_u64_arch(const orc_model* m, const char* arch, const char* sfx, uint64_t* v) {
  const char* pre[4] = {arch, "llama", "qwen2", "general"};
  char key[256];
  for (int i = 0; i < 4; i++) {
    snprintf(key, sizeof key, "%s.%s", pre[i], sfx);
    const orc_kv* kv = find_kv(m, key);
    if (kv && kv->has_u) { *v = kv->u; return 1; }
  }
  return 0;
}
/* get_f32_arch (model.rs:79-98). */
static int get_f32_arch(const orc_model* m, const char* arch, const char* sfx, float* v) {
  const char* pre[4] = {arch, "llama", "qwen2", "general"};
  char key[256];
  for (int i = 0; i < 4; i++) {
    snprintf(key, sizeof key, "%s.%s", pre[i], sfx);
    const orc_kv* kv = find_kv(m, key);
    if (kv && kv->has_f) { *v = (float)kv->f; return 1; }
  }
  return 0;
}

void orc_model_close(orc_model* m) {
  if (!m) return;
  for (size_t i = 0; i < m->n_kv; i++) { free(m->kvs[i].key); free(m->kvs[i].str); }
  for (size_t i = 0; i < m->n_t; i++) free(m->ts[i].name);
  free(m->kvs); free(m->ts); free(m->L);
  free(m->kcache); free(m->vcache); free(m->layer_hidden);
  free(m);
}

static const char* LAYER_NAMES[9] = {"attn_norm", "attn_q", "attn_k", "attn_v", "attn_output",
                                     "ffn_norm", "ffn_gate", "ffn_up", "ffn_down"};

orc_model* orc_model_open(const uint8_t* data, size_t len, int kv_f16, uint32_t max_seq, int threads) {
  orc_model* m = (orc_model*)calloc(1, sizeof *m);
  rdr r = {data, len, 0, 0};
  char magic[4];
  if (rd(&r, magic, 4) || memcmp(magic, "GGUF", 4)) { set_err("invalid GGUF magic"); goto fail; }
  uint32_t version = rd_u32(&r);
  if (version < 1 || version > 3) { set_err("unsupported GGUF version %u", version); goto fail; }
  m->n_t = rd_u64(&r);
  m->n_kv = rd_u64(&r);
  if (r.err || m->n_t > 10000000u || m->n_kv > 100000u) { set_err("bad GGUF counts"); goto fail; }
  m->kvs = (orc_kv*)calloc(m->n_kv ? m->n_kv : 1, sizeof(orc_kv));
  for (size_t i = 0; i < m->n_kv; i++) {
    orc_kv* kv = &m->kvs[i];
    kv->key = rd_str(&r);
    kv->vtype = rd_u32(&r);
    if (r.err) { set_err("truncated GGUF metadata"); goto fail; }
    if (kv->vtype == 9) { /* read_array_value (gguf.rs:153-194) */
      uint32_t at = rd_u32(&r);
      uint64_t n = rd_u64(&r);
      if (at == 9 || n > 10000000u) { set_err("bad GGUF array"); goto fail; }
      kv->arr_len = n;
      for (uint64_t j = 0; j < n && !r.err; j++) { orc_kv tmp = {0}; rd_scalar(&r, at, &tmp); }
    } else if (kv->vtype == 8) {
      kv->str = rd_str(&r);
    } else {
      rd_scalar(&r, kv->vtype, kv);
    }
    if (r.err) { set_err("truncated/invalid GGUF metadata value"); goto fail; }
  }
  uint64_t align = 32; /* DEFAULT_ALIGNMENT (gguf.rs:11); general.alignment override (gguf.rs:251-255) */
  const orc_kv* akv = find_kv(m, "general.alignment");
  if (akv && akv->has_u) align = akv->u;
  m->ts = (orc_tensor*)calloc(m->n_t ? m->n_t : 1, sizeof(orc_tensor));
  for (size_t i = 0; i < m->n_t; i++) {
    orc_tensor* t = &m->ts[i];
    t->name = rd_str(&r);
    t->ndims = rd_u32(&r);
    if (r.err || t->ndims > 8) { set_err("bad tensor info"); goto fail; }
    for (uint32_t d = 0; d < t->ndims; d++) t->dims[d] = rd_u64(&r);
    t->type = rd_u32(&r);
    t->offset = rd_u64(&r);
    if (r.err) { set_err("truncated tensor info"); goto fail; }
  }
  uint64_t ds = r.pos;
  if (align && ds % align) ds += align - ds % align; /* align_offset (model.rs:197-207) */
  for (size_t i = 0; i < m->n_t; i++) {
    orc_tensor* t = &m->ts[i];
    uint64_t ne = 1;
    for (uint32_t d = 0; d < t->ndims; d++) ne *= t->dims[d];
    size_t qk, bsz;
    if (!type_block((int)t->type, &qk, &bsz)) { t->nbytes = 0; t->data = NULL; continue; }
    t->nbytes = (ne + qk - 1) / qk * bsz;
    if (ds + t->offset + t->nbytes > len) { set_err("tensor %s out of file bounds", t->name); goto fail; }
    t->data = data + ds + t->offset;
  }
  /* LlamaConfig::from_gguf (model.rs:40-161) */
  const orc_kv* archkv = find_kv(m, "general.architecture");
  const char* arch = archkv && archkv->str ? archkv->str : "unknown";
  if (strcmp(arch, "llama") && strcmp(arch, "qwen2")) { set_err("unsupported execution architecture %s", arch); goto fail; }
  uint64_t v;
  orc_config* c = &m->cfg;
  if (get_u64_arch(m, arch, "vocab_size", &v)) c->vocab_size = (uint32_t)v;
  else {
    const orc_kv* tok = find_kv(m, "tokenizer.ggml.tokens");
    if (!tok) { set_err("missing vocab_size"); goto fail; }
    c->vocab_size = (uint32_t)tok->arr_len;
  }
  if (!get_u64_arch(m, arch, "context_length", &v)) { set_err("missing context_length"); goto fail; }
  c->context_length = (uint32_t)v;
  if (!get_u64_arch(m, arch, "embedding_length", &v)) { set_err("missing embedding_length"); goto fail; }
  c->n_embd = (uint32_t)v;
  if (!get_u64_arch(m, arch, "block_count", &v)) { set_err("missing block_count"); goto fail; }
  c->n_layers = (uint32_t)v;
  if (!get_u64_arch(m, arch, "feed_forward_length", &v) && !get_u64_arch(m, arch, "intermediate_size", &v)) {
    set_err("missing feed_forward_length"); goto fail;
  }
  c->n_ff = (uint32_t)v;
  if (!get_u64_arch(m, arch, "attention.head_count", &v)) { set_err("missing head_count"); goto fail; }
  c->n_heads = (uint32_t)v;
  c->n_kv_heads = get_u64_arch(m, arch, "attention.head_count_kv", &v) ? (uint32_t)v : c->n_heads;
  if (!get_f32_arch(m, arch, "attention.layer_norm_rms_epsilon", &c->rms_eps) &&
      !get_f32_arch(m, arch, "attention.layer_norm_epsilon", &c->rms_eps))
    c->rms_eps = 1e-5f;
  if (!get_f32_arch(m, arch, "rope.freq_base", &c->rope_theta)) c->rope_theta = 10000.0f;
  c->head_dim = c->n_embd / c->n_heads; /* model.rs:148 */
  /* validate_required_tensors (model.rs:168-200) */
  m->embd = find_t(m, "token_embd.weight");
  m->onorm = find_t(m, "output_norm.weight");
  m->out = find_t(m, "output.weight"); /* tied embedding when absent (streaming_model.rs:1353) */
  if (!m->embd || !m->onorm) { set_err("missing token_embd/output_norm"); goto fail; }
  m->L = (orc_tensor**)calloc((size_t)c->n_layers * 9, sizeof(orc_tensor*));
  for (uint32_t l = 0; l < c->n_layers; l++)
    for (int j = 0; j < 9; j++) {
      char name[128];
      snprintf(name, sizeof name, "blk.%u.%s.weight", l, LAYER_NAMES[j]);
      m->L[l * 9 + j] = find_t(m, name);
      if (!m->L[l * 9 + j] || !m->L[l * 9 + j]->data) { set_err("missing tensor '%s'", name); goto fail; }
    }
  m->kv_f16 = kv_f16;
  m->threads = threads < 1 ? 1 : threads;
  m->max_seq = max_seq ? max_seq : c->context_length;
  size_t kvd = (size_t)c->n_kv_heads * c->head_dim;
  m->kcache = (float*)calloc((size_t)c->n_layers * m->max_seq * kvd, sizeof(float));
  m->vcache = (float*)calloc((size_t)c->n_layers * m->max_seq * kvd, sizeof(float));
  m->layer_hidden = (float*)calloc((size_t)c->n_layers * c->n_embd, sizeof(float));
  if (!m->kcache || !m->vcache || !m->layer_hidden) { set_err("KV cache allocation failed"); goto fail; }
  return m;
fail:
  orc_model_close(m);
  return NULL;
}

int orc_model_config(const orc_model* m, orc_config* cfg) { *cfg = m->cfg; return 0; }
uint32_t orc_kv_len(const orc_model* m) { return m->seq_len; }
void orc_kv_reset(orc_model* m) { m->seq_len = 0; }

/* Timing support for the CPU baseline, not a reference function: set the history
 * length to n and fill positions [0, n) of every layer with seeded values in
 * [-1, 1) (f16-exact when the cache is f16), so a layer step can be timed at the
 * context a long decode reaches without running n forwards first.  Attention
 * cost depends on the length only, not on the values. */
int orc_kv_fill_synthetic(orc_model* m, uint32_t n, uint32_t seed) {
  if (n > m->max_seq) { set_err("KV fill beyond max_seq"); return -1; }
  size_t kvd = (size_t)m->cfg.n_kv_heads * m->cfg.head_dim;
  uint64_t st = 0x9E3779B97F4A7C15ull * (seed + 1);
  for (uint32_t l = 0; l < m->cfg.n_layers; l++)
    for (int w = 0; w < 2; w++) {
      float* base = (w ? m->vcache : m->kcache) + (size_t)l * m->max_seq * kvd;
      for (size_t i = 0; i < (size_t)n * kvd; i++) {
        st ^= st << 13; st ^= st >> 7; st ^= st << 17;
        base[i] = (float)((int)(st >> 40 & 0x7FF) - 1024) / 1024.0f;
      }
    }
  m->seq_len = n;
  return 0;
}

int orc_kv_read(const orc_model* m, uint32_t layer, int which_v, uint32_t start, uint32_t end, float* out) {
  if (layer >= m->cfg.n_layers || start > end || end > m->seq_len) { set_err("KV read out of range"); return -1; }
  size_t kvd = (size_t)m->cfg.n_kv_heads * m->cfg.head_dim;
  const float* base = (which_v ? m->vcache : m->kcache) + (size_t)layer * m->max_seq * kvd;
  memcpy(out, base + (size_t)start * kvd, sizeof(float) * (end - start) * kvd);
  return 0;
}

int orc_last_layer_hiddens(const orc_model* m, float* out) {
  memcpy(out, m->layer_hidden, sizeof(float) * m->cfg.n_layers * m->cfg.n_embd);
  return 0;
}

/* Matrix tensors are ggml [in, out] (ne0 = in); rows of `in` elements. */
static int mv_tensor(orc_model* m, const orc_tensor* t, const float* x, size_t in, size_t out, float* y) {
  if (t->ndims != 2 || t->dims[0] != in || t->dims[1] != out) {
    set_err("matvec arity mismatch for %s", t->name);
    return -1;
  }
  /* compute_dispatch.rs:72,114-210: Q4_0/Q6_K row-parallel when out >= 128; the rest
   * single-threaded.  Thread count never changes a row's arithmetic. */
  return orc_matvec((int)t->type, t->data, t->nbytes, in, out, x, y, m->threads);
}

static int f32_view(const orc_tensor* t, size_t n, float* out) {
  return orc_dequant_row((int)t->type, t->data, t->nbytes, n, out);
}

/* validate_qkv_bias (ramforge-runtime/src/streaming_model.rs:1654-1696): layer l's
 * qwen2 Q/K/V biases (load_layer's map, :829-831), all three or none, each 1-D of
 * the projection's output size.  B[0..2] = NULL when the layer has none. */
static int layer_biases(orc_model* m, uint32_t l, size_t qd, size_t kvd, const orc_tensor* B[3]) {
  static const char* nm[3] = {"attn_q", "attn_k", "attn_v"};
  int count = 0;
  for (int i = 0; i < 3; i++) {
    char name[128];
    snprintf(name, sizeof name, "blk.%u.%s.bias", l, nm[i]);
    B[i] = find_t(m, name);
    if (B[i] && !B[i]->data) B[i] = NULL;
    count += B[i] != NULL;
  }
  if (count == 0) return 0;
  if (count != 3) {
    set_err("layer %u has an incomplete Q/K/V bias set (q.bias: %s, k.bias: %s, v.bias: %s); refusing to run "
            "inference with partial biases", l, B[0] ? "true" : "false", B[1] ? "true" : "false",
            B[2] ? "true" : "false");
    return -1;
  }
  const size_t want[3] = {qd, kvd, kvd};
  for (int i = 0; i < 3; i++)
    if (B[i]->ndims != 1 || B[i]->dims[0] != want[i]) {
      set_err("invalid blk.%u.%s.bias shape: expected 1D [%zu]", l, nm[i], want[i]);
      return -1;
    }
  return 0;
}

/* ModelExecutor::execute_layer (ramforge-runtime/src/model_executor.rs:102-236). */
static int execute_layer(orc_model* m, uint32_t l, uint32_t pos, float* hidden, float* k_tmp, float* v_tmp) {
  const orc_config* c = &m->cfg;
  size_t d = c->n_embd, hd = c->head_dim, qd = (size_t)c->n_heads * hd, kvd = (size_t)c->n_kv_heads * hd, ff = c->n_ff;
  orc_tensor** T = m->L + (size_t)l * 9;
  int rc = -1;
  float *tmp = malloc(4 * d), *norm = malloc(4 * d), *q = malloc(4 * qd), *att = malloc(4 * qd),
        *proj = malloc(4 * d), *g = malloc(4 * ff), *u = malloc(4 * ff), *act = malloc(4 * ff),
        *gs = malloc(4 * ff);
  float* kh = NULL;
  float* vh = NULL;
  if (f32_view(T[0], d, norm)) goto out;
  if (orc_rmsnorm(hidden, norm, c->rms_eps, d, tmp)) goto out;          /* :155 */
  if (mv_tensor(m, T[1], tmp, d, qd, q)) goto out;                     /* :157 */
  if (mv_tensor(m, T[2], tmp, d, kvd, k_tmp)) goto out;                /* :158 */
  if (mv_tensor(m, T[3], tmp, d, kvd, v_tmp)) goto out;                /* :159 */
  { /* :161-194 biases after the projections, before RoPE and the KV insert */
    const orc_tensor* B[3];
    if (layer_biases(m, l, qd, kvd, B)) goto out;
    if (B[0]) {
      float* b = malloc(4 * qd);
      int bad = f32_view(B[0], qd, b);
      for (size_t i = 0; !bad && i < qd; i++) q[i] += b[i];
      bad = bad || f32_view(B[1], kvd, b);
      for (size_t i = 0; !bad && i < kvd; i++) k_tmp[i] += b[i];
      bad = bad || f32_view(B[2], kvd, b);
      for (size_t i = 0; !bad && i < kvd; i++) v_tmp[i] += b[i];
      free(b);
      if (bad) goto out;
    }
  }
  if (orc_rope(q, k_tmp, pos, hd, c->n_heads, c->n_kv_heads, c->rope_theta)) goto out; /* :196 */
  /* :205-211 attention over kv[0, hist) + current K/V */
  kh = m->kcache + (size_t)l * m->max_seq * kvd;
  vh = m->vcache + (size_t)l * m->max_seq * kvd;
  if (orc_attention(q, kh, vh, k_tmp, v_tmp, m->seq_len, c->n_heads, c->n_kv_heads, hd, att)) goto out;
  if (mv_tensor(m, T[4], att, qd, d, proj)) goto out;                  /* :213 */
  for (size_t i = 0; i < d; i++) tmp[i] = hidden[i] + proj[i];          /* :214 add */
  memcpy(hidden, tmp, 4 * d);
  if (f32_view(T[5], d, norm)) goto out;
  if (orc_rmsnorm(hidden, norm, c->rms_eps, d, tmp)) goto out;          /* :225 */
  if (mv_tensor(m, T[6], tmp, d, ff, g)) goto out;                     /* :227 */
  if (mv_tensor(m, T[7], tmp, d, ff, u)) goto out;                     /* :228 */
  orc_silu(g, gs, ff);                                                 /* :229 */
  for (size_t i = 0; i < ff; i++) act[i] = gs[i] * u[i];               /* :230 */
  if (mv_tensor(m, T[8], act, ff, d, proj)) goto out;                  /* :231 */
  for (size_t i = 0; i < d; i++) tmp[i] = hidden[i] + proj[i];          /* :232 */
  memcpy(hidden, tmp, 4 * d);
  rc = 0;
out:
  free(tmp); free(norm); free(q); free(att); free(proj); free(g); free(u); free(act); free(gs);
  return rc;
}

/* forward_single_streaming (ramforge-runtime/src/streaming_model.rs:909-1305):
 * embed row, every layer, then commit every layer's K/V (:1291-1295),
 * seq_len += 1, then output RMSNorm into final_hidden (:1301). */
int orc_forward(orc_model* m, uint32_t token, uint32_t pos, float* final_hidden) {
  const orc_config* c = &m->cfg;
  if (pos != m->seq_len) { set_err("KV position/history mismatch: position %u, history %u", pos, m->seq_len); return -1; }
  if (m->seq_len >= m->max_seq) { set_err("KV cache full"); return -1; }
  if (token >= c->vocab_size) { set_err("token_id %u out of bounds", token); return -1; }
  size_t d = c->n_embd, kvd = (size_t)c->n_kv_heads * c->head_dim;
  size_t rb = orc_row_bytes((int)m->embd->type, d);
  float* hidden = malloc(4 * d);
  float* ks = malloc(4 * kvd * c->n_layers);
  float* vs = malloc(4 * kvd * c->n_layers);
  float* norm = malloc(4 * d);
  int rc = -1;
  /* get_embedding (tensor.rs:701-760): decode row `token`. */
  if (orc_dequant_row((int)m->embd->type, m->embd->data + (size_t)token * rb, rb, d, hidden)) goto out;
  for (uint32_t l = 0; l < c->n_layers; l++) {
    if (execute_layer(m, l, pos, hidden, ks + l * kvd, vs + l * kvd)) goto out;
    memcpy(m->layer_hidden + (size_t)l * d, hidden, 4 * d);
  }
  for (uint32_t l = 0; l < c->n_layers; l++) { /* KvCache::append (kv_cache.rs:381-412) */
    float* kd = m->kcache + ((size_t)l * m->max_seq + m->seq_len) * kvd;
    float* vd = m->vcache + ((size_t)l * m->max_seq + m->seq_len) * kvd;
    for (size_t i = 0; i < kvd; i++) {
      float kv = ks[l * kvd + i], vv = vs[l * kvd + i];
      if (m->kv_f16) { kv = ieee_f16_to_f32(orc_f32_to_f16(kv)); vv = ieee_f16_to_f32(orc_f32_to_f16(vv)); }
      kd[i] = kv;
      vd[i] = vv;
    }
  }
  m->seq_len++; /* increment_seq_len (kv_cache.rs:415) */
  if (final_hidden) {
    if (f32_view(m->onorm, d, norm)) goto out;
    if (orc_rmsnorm(hidden, norm, c->rms_eps, d, final_hidden)) goto out;
  }
  rc = 0;
out:
  free(hidden); free(ks); free(vs); free(norm);
  return rc;
}

/* One layer of a token forward on a caller-owned hidden vector, reading history
 * [0, pos) without committing: a bounded CPU-baseline sample (1/n_layers of a token). */
int orc_layer_step(orc_model* m, uint32_t layer, uint32_t pos, float* hidden) {
  if (layer >= m->cfg.n_layers || pos > m->seq_len) { set_err("bad layer step"); return -1; }
  size_t kvd = (size_t)m->cfg.n_kv_heads * m->cfg.head_dim;
  float* ks = malloc(4 * kvd);
  float* vs = malloc(4 * kvd);
  uint32_t saved = m->seq_len;
  m->seq_len = pos;
  int rc = execute_layer(m, layer, pos, hidden, ks, vs);
  m->seq_len = saved;
  free(ks);
  free(vs);
  return rc;
}

/* Output-projection rows [r0, r1) of compute_logits (a slice of the LM head). */
int orc_logits_rows(orc_model* m, const float* final_hidden, uint32_t r0, uint32_t r1, float* out) {
  const orc_tensor* w = m->out ? m->out : m->embd;
  if (r0 > r1 || r1 > m->cfg.vocab_size) { set_err("bad logits row range"); return -1; }
  size_t rb = orc_row_bytes((int)w->type, m->cfg.n_embd);
  return orc_matvec((int)w->type, w->data + (size_t)r0 * rb, (size_t)(r1 - r0) * rb, m->cfg.n_embd, r1 - r0,
                    final_hidden, out, m->threads);
}

/* compute_logits (streaming_model.rs:1334-1371): output.weight or the tied token_embd. */
int orc_logits(orc_model* m, const float* final_hidden, float* logits) {
  const orc_tensor* w = m->out ? m->out : m->embd;
  return mv_tensor(m, w, final_hidden, m->cfg.n_embd, m->cfg.vocab_size, logits);
}

/* generate_impl (ramforge-runtime/src/inference.rs:445-759), greedy:
 * prompt token by token (:578-592), then logits -> argmax -> forward (:595-712). */
int orc_generate(orc_model* m, const uint32_t* prompt, uint32_t n_prompt, uint32_t n_new,
                 uint32_t* out_tokens, float* out_logits, float* out_margin) {
  const orc_config* c = &m->cfg;
  if (n_prompt == 0) { set_err("empty prompt"); return -1; }
  float* fh = malloc(4 * (size_t)c->n_embd);
  float* lg = malloc(4 * (size_t)c->vocab_size);
  int rc = -1;
  uint32_t pos = m->seq_len;
  for (uint32_t i = 0; i < n_prompt; i++)
    if (orc_forward(m, prompt[i], pos++, fh)) goto out;
  for (uint32_t t = 0; t < n_new; t++) {
    if (orc_logits(m, fh, lg)) goto out;
    uint32_t tok = orc_argmax(lg, c->vocab_size);
    out_tokens[t] = tok;
    if (out_logits) memcpy(out_logits + (size_t)t * c->vocab_size, lg, 4 * (size_t)c->vocab_size);
    if (out_margin) {
      float b1 = lg[tok], b2 = -INFINITY;
      for (uint32_t i = 0; i < c->vocab_size; i++)
        if (i != tok && lg[i] > b2) b2 = lg[i];
      out_margin[t] = b1 - b2;
    }
    if (t + 1 < n_new && orc_forward(m, tok, pos++, fh)) goto out;
  }
  rc = 0;
out:
  free(fh); free(lg);
  return rc;
}
