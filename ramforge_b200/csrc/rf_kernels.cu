// rf_kernels.cu - sm_100a kernels of the decode engine.
//
// Batch-1 decode is HBM-bound: every weight byte is read once per token and
// used for exactly one multiply-add per element, so none of these kernels uses
// tensor cores.  The GEMV streams packed weights with 256-bit non-allocating
// loads (one 32-byte unit per lane per row), keeps the activation vector in
// shared memory (swizzled so the 32 lanes of a warp, which read 32 different
// units, hit 32 different bank groups), and fuses the op that precedes it
// (RMSNorm) and the ops that follow it (RoPE + KV append, SwiGLU, residual add,
// greedy argmax) so activations never make an extra round trip through HBM.
// Reference arithmetic (crates/ramforge-core/src/compute.rs, quant.rs) is kept
// where it is cheap: exact per-element dequantisation for the embedding row,
// division-based RMSNorm, dot/sqrt(hd) scores, v/(1+exp(-v)) SiLU and RoPE from
// a host-built cos/sin table evaluated with the same libm as the reference.
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <algorithm>

#include "rf_kernels.cuh"

namespace rf {

// ---------------------------------------------------------------------------
// small device helpers
// ---------------------------------------------------------------------------
__device__ __forceinline__ void griddep_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void griddep_launch() { asm volatile("griddepcontrol.launch_dependents;" :::); }

// One 256-bit streaming load of weights (read once per token: no L1 allocation).
__device__ __forceinline__ void ldg256(const uint8_t* p, uint32_t (&w)[8]) {
  asm volatile("ld.global.nc.L1::no_allocate.v8.b32 {%0,%1,%2,%3,%4,%5,%6,%7}, [%8];"
               : "=r"(w[0]), "=r"(w[1]), "=r"(w[2]), "=r"(w[3]), "=r"(w[4]), "=r"(w[5]), "=r"(w[6]), "=r"(w[7])
               : "l"(p));
}

// f16 -> f32 as the reference decodes block scales and F16 tensors
// (quant.rs:40-65, tensor.rs:1017-1041): IEEE for normal numbers, but a
// subnormal half comes out at half its IEEE value (the normalising loop's
// exponent is one short).  The engine reproduces that for bit-parity.
__device__ __forceinline__ float h2f(uint32_t bits16) {
  const float f = __half2float(__ushort_as_half((unsigned short)bits16));
  return (bits16 & 0x7C00u) ? f : f * 0.5f;
}

// exact float of a 4-bit field (v >> sh) & 15, minus `bias` (0 or 8)
template <int BIAS>
__device__ __forceinline__ float nib(uint32_t v, int sh) {
  return __uint_as_float(((v >> sh) & 0xFu) | 0x4B000000u) - (8388608.0f + (float)BIAS);
}
// exact float of the signed byte (v >> sh) & 255
__device__ __forceinline__ float sbyte_f(uint32_t v, int sh) {
  return __uint_as_float((((v >> sh) & 0xFFu) ^ 0x80u) | 0x4B000000u) - 8388736.0f;
}

// Swizzled shared-memory position of element e: units of EPU elements, 16-byte
// chunks rotated by the unit index so lanes reading consecutive units at the
// same chunk index land in different bank groups.
template <int EPU>
__device__ __forceinline__ int swz(int e) {
  constexpr int CPU = EPU / 4;
  int u = e / EPU, o = e % EPU;
  return u * EPU + ((((o >> 2) + u) & (CPU - 1)) << 2) + (o & 3);
}
template <int EPU>
__device__ __forceinline__ float4 ldx(const float* sx, int u, int c) {
  constexpr int CPU = EPU / 4;
  return *reinterpret_cast<const float4*>(sx + u * EPU + (((c + u) & (CPU - 1)) << 2));
}

constexpr int GEMV_THREADS = 256;
constexpr int GEMV_WARPS = GEMV_THREADS / 32;

// Block-wide sum of squares; blockDim must be GEMV_THREADS so every kernel that
// normalises the same vector produces bit-identical results.
__device__ float block_sumsq(const float* __restrict__ x, int n, float* sred) {
  float s = 0.f;
  for (int i = threadIdx.x; i < n; i += GEMV_THREADS) {
    float v = x[i];
    s = fmaf(v, v, s);
  }
#pragma unroll
  for (int o = 16; o; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
  if ((threadIdx.x & 31) == 0) sred[threadIdx.x >> 5] = s;
  __syncthreads();
  if (threadIdx.x == 0) {
    float t = 0.f;
    for (int w = 0; w < GEMV_WARPS; w++) t += sred[w];
    sred[32] = t;
  }
  __syncthreads();
  float r = sred[32];
  __syncthreads();
  return r;
}

// RMSNorm value of element i given the block sum of squares:
// rms = sqrt(sum/n + eps); y = x / rms * w   (compute.rs:312-317)
__device__ __forceinline__ float rms_of(float ss, int n, float eps) { return sqrtf(ss / (float)n + eps); }

// ---------------------------------------------------------------------------
// per-unit dot products: 32 bytes of each of R rows against the unit's EPU
// activations, accumulated into acc[R].
//
// Quant fields are never shifted down or converted.  A 4- or 8-bit field masked
// in place inside a 32-bit word, bits [off, off+n) with off + n <= 24, is read
// as an f32 whose value is exactly q * 2^(off-149) (a subnormal, or a normal
// number with exponent field 1 - the bit pattern and the value are linear in
// that range).  Shared memory holds x pre-multiplied by 2^(85-off) for the field
// position each element is decoded from, so every product is exactly
// q * x * 2^-64 and one packed fma.rn.f32x2 accumulates two elements; the 2^64 is
// folded into the block scale.  Per 8 quants of Q4: 1 shift, 8 masks, 4 FFMA2.
// ---------------------------------------------------------------------------
constexpr float kTwo64 = 18446744073709551616.0f;  // 2^64

// Field offset (bit position inside its 32-bit word, after the one 8-bit shift
// that brings byte 3's fields below bit 24) of the element at unit-relative
// index l; EPU-specific layouts below.
template <int FMT>
__device__ __forceinline__ int field_off(int l);
template <>
__device__ __forceinline__ int field_off<T_Q4_K>(int l) {  // byte l%32 of the unit; high nibble for l >= 32
  const int b = l & 3;
  return (b < 3 ? 8 * b : 16) + (l >= 32 ? 4 : 0);
}
template <>
__device__ __forceinline__ int field_off<T_Q4_0>(int l) {  // block byte (l%32)%16; high nibble for (l%32) >= 16
  const int b = l & 3;
  return (b < 3 ? 8 * b : 16) + ((l & 31) >= 16 ? 4 : 0);
}
template <>
__device__ __forceinline__ int field_off<T_Q8_0>(int l) {  // byte l of the block
  const int b = l & 3;
  return b < 3 ? 8 * b : 16;
}
template <>
__device__ __forceinline__ int field_off<T_F16>(int) { return 85; }  // scale 1: weights are real floats
template <>
__device__ __forceinline__ int field_off<T_F32>(int) { return 85; }

// 2^(85 - off): exact power-of-two pre-scale of x for a field at bit `off`
// (85 - off >= 65 for quant fields; 0 for float weights).
__device__ __forceinline__ float prescale(int off) { return __int_as_float((127 + 149 - 64 - off) << 23); }

__device__ __forceinline__ float as_f(uint32_t bits) { return __uint_as_float(bits); }

// Scale words come from global memory (read-only path) or from a shared-memory stage.
template <bool SMEM, class T>
__device__ __forceinline__ T ld_scale(const T* p) {
  if constexpr (SMEM) return *p;
  else return __ldg(p);
}

template <int FMT>
struct UnitDot;

// Q4_K super-block header fields of sub-block pair i = u%4 (get_scale_min,
// quant.rs:216-226, for j = 2i and 2i+1): d*sc and dmin*m of both sub-blocks,
// with d*sc carrying the 2^64 of the scaled products.  Branch-free: lanes of a
// warp decode different i.
template <bool SMEM>
__device__ __forceinline__ void q4k_scales(const uint8_t* sc_row, int u, float& d1, float& mn1, float& d2,
                                           float& mn2) {
  const uint4 h = ld_scale<SMEM>(reinterpret_cast<const uint4*>(sc_row + (size_t)(u >> 2) * 16));
  const float d = h2f(h.x & 0xFFFFu) * kTwo64, dmin = h2f(h.x >> 16);
  const int i = u & 3;
  const int sh = (i & 1) * 16;
  const uint32_t y = (h.y >> sh) & 0xFFFFu;  // s[2i'], s[2i'+1]      (i' = i & 1)
  const uint32_t z = (h.z >> sh) & 0xFFFFu;  // s[2i'+4], s[2i'+5]
  const uint32_t w = (h.w >> sh) & 0xFFFFu;  // s[2i'+8], s[2i'+9]
  // j < 4: sc = s[j] & 63, m = s[j+4] & 63; j >= 4: low 4 bits from s[j+4], high 2 from s[j-4] / s[j]
  const uint32_t sc_lo = y & 0x3F3Fu, m_lo = z & 0x3F3Fu;
  const uint32_t sc_hi = (w & 0x0F0Fu) | ((y >> 2) & 0x3030u);
  const uint32_t m_hi = ((w >> 4) & 0x0F0Fu) | ((z >> 2) & 0x3030u);
  const uint32_t sc = i >= 2 ? sc_hi : sc_lo, m = i >= 2 ? m_hi : m_lo;
  d1 = d * (float)(sc & 0xFFu);
  d2 = d * (float)(sc >> 8);
  mn1 = dmin * (float)(m & 0xFFu);
  mn2 = dmin * (float)(m >> 8);
}

template <>
struct UnitDot<T_Q4_K> {
  static constexpr int EPU = 64;
  static constexpr bool NEED_XS = true;
  // Unit u = sub-block pair i = u%4 of super-block u/4: byte l holds element l
  // (low nibble, sub-block 2i) and element 32+l (high nibble, sub-block 2i+1).
  // value = d*sc*q - dmin*m (quant.rs:235-248), summed as
  // (d*sc) * sum(q*x) - (dmin*m) * sum(x).
  template <int R, class XA, bool SMEM = false>
  __device__ __forceinline__ static void accum(const uint32_t (&w)[R][8], XA xa, const uint8_t* const (&srow)[R],
                                               int u, float xs_lo, float xs_hi, float (&acc)[R]) {
    float2 lo[R], hi[R];
#pragma unroll
    for (int r = 0; r < R; r++) lo[r] = hi[r] = make_float2(0.f, 0.f);
#pragma unroll
    for (int k = 0; k < 8; k++) {
      const float4 a = xa(k), b = xa(8 + k);
#pragma unroll
      for (int r = 0; r < R; r++) {
        const uint32_t v = w[r][k], t = v >> 8;
        lo[r] = __ffma2_rn(make_float2(as_f(v & 0xFu), as_f(v & 0xF00u)), make_float2(a.x, a.y), lo[r]);
        lo[r] = __ffma2_rn(make_float2(as_f(v & 0xF0000u), as_f(t & 0xF0000u)), make_float2(a.z, a.w), lo[r]);
        hi[r] = __ffma2_rn(make_float2(as_f(v & 0xF0u), as_f(v & 0xF000u)), make_float2(b.x, b.y), hi[r]);
        hi[r] = __ffma2_rn(make_float2(as_f(v & 0xF00000u), as_f(t & 0xF00000u)), make_float2(b.z, b.w), hi[r]);
      }
    }
#pragma unroll
    for (int r = 0; r < R; r++) {
      float d1, mn1, d2, mn2;
      q4k_scales<SMEM>(srow[r], u, d1, mn1, d2, mn2);
      acc[r] += d1 * (lo[r].x + lo[r].y) - mn1 * xs_lo + (d2 * (hi[r].x + hi[r].y) - mn2 * xs_hi);
    }
  }
};

template <>
struct UnitDot<T_Q4_0> {
  static constexpr int EPU = 64;
  static constexpr bool NEED_XS = true;
  // Unit u = blocks 2u, 2u+1: block byte j holds element j (low) and 16+j (high);
  // value (q-8)*d (quant.rs:104-112), summed as d * (sum(q*x) - 8*sum(x)).
  template <int R, class XA, bool SMEM = false>
  __device__ __forceinline__ static void accum(const uint32_t (&w)[R][8], XA xa, const uint8_t* const (&srow)[R],
                                               int u, float xs0, float xs1, float (&acc)[R]) {
    float2 s0[R], s1[R];
#pragma unroll
    for (int r = 0; r < R; r++) s0[r] = s1[r] = make_float2(0.f, 0.f);
#pragma unroll
    for (int k = 0; k < 4; k++) {
      const float4 a = xa(k), b = xa(4 + k), c = xa(8 + k), e = xa(12 + k);
#pragma unroll
      for (int r = 0; r < R; r++) {
        const uint32_t v0 = w[r][k], t0 = v0 >> 8, v1 = w[r][4 + k], t1 = v1 >> 8;
        s0[r] = __ffma2_rn(make_float2(as_f(v0 & 0xFu), as_f(v0 & 0xF00u)), make_float2(a.x, a.y), s0[r]);
        s0[r] = __ffma2_rn(make_float2(as_f(v0 & 0xF0000u), as_f(t0 & 0xF0000u)), make_float2(a.z, a.w), s0[r]);
        s0[r] = __ffma2_rn(make_float2(as_f(v0 & 0xF0u), as_f(v0 & 0xF000u)), make_float2(b.x, b.y), s0[r]);
        s0[r] = __ffma2_rn(make_float2(as_f(v0 & 0xF00000u), as_f(t0 & 0xF00000u)), make_float2(b.z, b.w), s0[r]);
        s1[r] = __ffma2_rn(make_float2(as_f(v1 & 0xFu), as_f(v1 & 0xF00u)), make_float2(c.x, c.y), s1[r]);
        s1[r] = __ffma2_rn(make_float2(as_f(v1 & 0xF0000u), as_f(t1 & 0xF0000u)), make_float2(c.z, c.w), s1[r]);
        s1[r] = __ffma2_rn(make_float2(as_f(v1 & 0xF0u), as_f(v1 & 0xF000u)), make_float2(e.x, e.y), s1[r]);
        s1[r] = __ffma2_rn(make_float2(as_f(v1 & 0xF00000u), as_f(t1 & 0xF00000u)), make_float2(e.z, e.w), s1[r]);
      }
    }
#pragma unroll
    for (int r = 0; r < R; r++) {
      const uint32_t dd = ld_scale<SMEM>(reinterpret_cast<const uint32_t*>(srow[r]) + u);
      const float d0 = h2f(dd & 0xFFFFu), d1 = h2f(dd >> 16);
      acc[r] += d0 * ((s0[r].x + s0[r].y) * kTwo64 - 8.f * xs0) + d1 * ((s1[r].x + s1[r].y) * kTwo64 - 8.f * xs1);
    }
  }
};

template <>
struct UnitDot<T_Q8_0> {
  static constexpr int EPU = 32;
  static constexpr bool NEED_XS = true;
  // Unit u = block u: 32 signed bytes, value q*d (quant.rs:176-180).  Bytes are
  // biased to q+128 (xor 0x80) and summed as d * (sum((q+128)*x) - 128*sum(x)).
  template <int R, class XA, bool SMEM = false>
  __device__ __forceinline__ static void accum(const uint32_t (&w)[R][8], XA xa, const uint8_t* const (&srow)[R],
                                               int u, float xs, float, float (&acc)[R]) {
    float2 s[R];
#pragma unroll
    for (int r = 0; r < R; r++) s[r] = make_float2(0.f, 0.f);
#pragma unroll
    for (int k = 0; k < 8; k++) {
      const float4 a = xa(k);
#pragma unroll
      for (int r = 0; r < R; r++) {
        const uint32_t v = w[r][k] ^ 0x80808080u, t = v >> 8;
        s[r] = __ffma2_rn(make_float2(as_f(v & 0xFFu), as_f(v & 0xFF00u)), make_float2(a.x, a.y), s[r]);
        s[r] = __ffma2_rn(make_float2(as_f(v & 0xFF0000u), as_f(t & 0xFF0000u)), make_float2(a.z, a.w), s[r]);
      }
    }
#pragma unroll
    for (int r = 0; r < R; r++) {
      const float d = h2f(ld_scale<SMEM>(reinterpret_cast<const unsigned short*>(srow[r]) + u));
      acc[r] += d * ((s[r].x + s[r].y) * kTwo64 - 128.f * xs);
    }
  }
};

template <>
struct UnitDot<T_F16> {
  static constexpr int EPU = 16;
  static constexpr bool NEED_XS = false;
  template <int R, class XA, bool SMEM = false>
  __device__ __forceinline__ static void accum(const uint32_t (&w)[R][8], XA xa, const uint8_t* const (&)[R], int,
                                               float, float, float (&acc)[R]) {
#pragma unroll
    for (int k = 0; k < 4; k++) {
      const float4 a = xa(k);
#pragma unroll
      for (int r = 0; r < R; r++) {
        float s = acc[r];
        s = fmaf(h2f(w[r][2 * k] & 0xFFFFu), a.x, s);
        s = fmaf(h2f(w[r][2 * k] >> 16), a.y, s);
        s = fmaf(h2f(w[r][2 * k + 1] & 0xFFFFu), a.z, s);
        acc[r] = fmaf(h2f(w[r][2 * k + 1] >> 16), a.w, s);
      }
    }
  }
};

template <>
struct UnitDot<T_F32> {
  static constexpr int EPU = 8;
  static constexpr bool NEED_XS = false;
  template <int R, class XA, bool SMEM = false>
  __device__ __forceinline__ static void accum(const uint32_t (&w)[R][8], XA xa, const uint8_t* const (&)[R], int,
                                               float, float, float (&acc)[R]) {
#pragma unroll
    for (int k = 0; k < 2; k++) {
      const float4 a = xa(k);
#pragma unroll
      for (int r = 0; r < R; r++) {
        float s = acc[r];
        s = fmaf(__uint_as_float(w[r][4 * k]), a.x, s);
        s = fmaf(__uint_as_float(w[r][4 * k + 1]), a.y, s);
        s = fmaf(__uint_as_float(w[r][4 * k + 2]), a.z, s);
        acc[r] = fmaf(__uint_as_float(w[r][4 * k + 3]), a.w, s);
      }
    }
  }
};

// Stage the activation vector into shared memory: optional RMSNorm
// (rms_norm_reference, compute.rs:291-319), the per-field pre-scale of the
// weight format, the unit swizzle, and (formats with a min/bias term) the
// unscaled sum of every 32 consecutive elements.
template <int FMT>
__device__ void stage_x(const float* __restrict__ x, const float* __restrict__ nw, float eps, int K, int Kp,
                        float* sx, float* sxs, float* sred) {
  using D = UnitDot<FMT>;
  constexpr int EPU = D::EPU;
  float rms = 1.f;
  if (nw) rms = rms_of(block_sumsq(x, K, sred), K, eps);
  // warp w stages 32-element chunks w, w+8, ...: coalesced loads, and the chunk
  // sums come from one shuffle reduction
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  for (int c = warp; c * 32 < Kp; c += GEMV_WARPS) {
    const int e = c * 32 + lane;
    float v = 0.f;
    if (e < K) {
      const float xv = x[e];
      v = nw ? xv / rms * nw[e] : xv;
    }
    if (e < Kp) sx[swz<EPU>(e)] = v * prescale(field_off<FMT>(e % EPU));
    if (D::NEED_XS) {
      float s = v;
#pragma unroll
      for (int o = 16; o; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
      if (lane == 0) sxs[c] = s;
    }
  }
  __syncthreads();
}

// ---------------------------------------------------------------------------
// epilogues (called by lane 0 of a warp with the R finished row sums)
// ---------------------------------------------------------------------------
struct EpiStore {
  float* y;
  __device__ void operator()(int row0, const float* v, int n) {
    for (int i = 0; i < n; i++) y[row0 + i] = v[i];
  }
  __device__ void finish() {}
  __device__ void flush() {}
};

struct EpiResidual {
  const float* res;
  float* out;
  __device__ void operator()(int row0, const float* v, int n) {
    for (int i = 0; i < n; i++) out[row0 + i] = res ? res[row0 + i] + v[i] : v[i];
  }
  __device__ void finish() {}
  __device__ void flush() {}
};

struct EpiRope {
  RopeQKVArgs a;
  // Rows come in pairs: Q and K rows are packed (i, i+hd/2) per head so that the
  // half-split rotation (compute.rs:440-456) happens in registers; V rows are in
  // natural order.
  __device__ void operator()(int row0, const float* v, int n) {
    const int pos = *a.d_pos;
    const uint32_t half = a.head_dim / 2;
    for (int t = 0; t < n; t += 2) {
      const uint32_t p = (uint32_t)row0 + t;
      if (p < a.q_rows + a.kv_rows) {
        if (t + 1 >= n) break;
        const bool isq = p < a.q_rows;
        const uint32_t j = (isq ? p : p - a.q_rows) / 2;
        const uint32_t h = j / half, i = j % half;
        const float2 cs = a.rope_cs[(size_t)pos * half + i];
        const float x0 = v[t], x1 = v[t + 1];
        // first*cos - second*sin ; first*sin + second*cos, one rounding per op
        const float o0 = __fsub_rn(__fmul_rn(x0, cs.x), __fmul_rn(x1, cs.y));
        const float o1 = __fadd_rn(__fmul_rn(x0, cs.y), __fmul_rn(x1, cs.x));
        const uint32_t e0 = h * a.head_dim + i, e1 = e0 + half;
        if (isq) {
          a.q_out[e0] = o0;
          a.q_out[e1] = o1;
        } else {
          a.k_cur[e0] = o0;
          a.k_cur[e1] = o1;
          const size_t c0 = ((size_t)h * a.max_seq + pos) * a.head_dim + i;
          if (a.kv_f32) {
            ((float*)a.kcache)[c0] = o0;
            ((float*)a.kcache)[c0 + half] = o1;
          } else {
            ((__half*)a.kcache)[c0] = __float2half_rn(o0);
            ((__half*)a.kcache)[c0 + half] = __float2half_rn(o1);
          }
        }
      } else {
        for (int s = 0; s < 2 && t + s < n; s++) {
          const uint32_t o = p + s - a.q_rows - a.kv_rows;
          const uint32_t h = o / a.head_dim, dd = o % a.head_dim;
          a.v_cur[o] = v[t + s];
          const size_t c = ((size_t)h * a.max_seq + pos) * a.head_dim + dd;
          if (a.kv_f32) ((float*)a.vcache)[c] = v[t + s];
          else ((__half*)a.vcache)[c] = __float2half_rn(v[t + s]);
        }
      }
    }
  }
  __device__ void finish() {}
  __device__ void flush() {}
};

struct EpiSwiGLU {
  float* act;
  // rows (2j, 2j+1) = (gate_j, up_j); silu(g) = g/(1+exp(-g)) then * up
  // (compute.rs:337-350, model_executor.rs:229-230)
  __device__ void operator()(int row0, const float* v, int n) {
    for (int t = 0; t + 1 < n; t += 2) {
      const float g = v[t], u = v[t + 1];
      const float s = g / (1.0f + expf(-g));
      act[(row0 + t) >> 1] = __fmul_rn(s, u);
    }
  }
  __device__ void finish() {}
  __device__ void flush() {}
};

// Order-preserving 64-bit key: high word = float bits mapped to unsigned order,
// low word = ~row so that equal values prefer the lower row (the reference's
// strict '>' scan keeps the first maximum, sampling.rs:48-53).
__device__ __forceinline__ unsigned long long argmax_key(float v, uint32_t row) {
  uint32_t b = __float_as_uint(v);
  b = (b & 0x80000000u) ? ~b : (b | 0x80000000u);
  return ((unsigned long long)b << 32) | (unsigned long long)(~row);
}

struct EpiArgmax {
  float* logits;
  unsigned long long* key;
  uint32_t row_offset;
  unsigned long long best;
  __device__ void operator()(int row0, const float* v, int n) {
    for (int i = 0; i < n; i++) {
      if (logits) logits[row0 + i] = v[i];
      const unsigned long long k = argmax_key(v[i], row_offset + row0 + i);
      best = k > best ? k : best;
    }
  }
  // barrier-free end of kernel: every thread that saw rows merges its own best
  __device__ void flush() {
    if (best) atomicMax(key, best);
  }
  __device__ void finish() {
    __shared__ unsigned long long sb[GEMV_WARPS];
    if ((threadIdx.x & 31) == 0) sb[threadIdx.x >> 5] = best;
    __syncthreads();
    if (threadIdx.x == 0) {
      unsigned long long m = 0;
      for (int w = 0; w < GEMV_WARPS; w++) m = sb[w] > m ? sb[w] : m;
      if (m) atomicMax(key, m);
    }
  }
};

// ---------------------------------------------------------------------------
// the GEMV kernel
// ---------------------------------------------------------------------------
// Each warp owns groups of R consecutive packed rows; its lanes stride over the
// 32-byte units of those rows (unit u by lane u % 32), so one warp-wide load
// instruction reads 1 KB of contiguous weights per row.  A lane keeps R x CH
// units (256 bytes) in flight: HBM needs tens of KB outstanding per SM to reach
// its bandwidth, and the grid is two 8-warp CTAs per SM.  The first chunk of a
// warp's first group is loaded before waiting on the previous kernel (weights
// never depend on it), and the next group's first chunk is loaded before the
// current group's reduction.  x lives in shared memory.
template <int FMT, int R, class Epi>
__global__ void __launch_bounds__(GEMV_THREADS, 2) gemv_kernel(PackedMat W, const float* __restrict__ x,
                                                               const float* __restrict__ nw, float eps, Epi epi) {
  using D = UnitDot<FMT>;
  constexpr int EPU = D::EPU;
  constexpr int CH = 8 / R;  // units per row in flight per lane
  extern __shared__ __align__(16) float smem[];
  float* sx = smem;
  float* sxs = smem + W.Kp;
  float* sred = sxs + W.Kp / 32;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int n_groups = (int)((W.M + R - 1) / R);
  const int units = (int)W.units;
  const int nch = (units + 32 * CH - 1) / (32 * CH);
  const int gstride = gridDim.x * GEMV_WARPS;
  int g = blockIdx.x * GEMV_WARPS + warp;

  uint32_t w[CH][R][8];
  auto load = [&](int grp, int c) {
#pragma unroll
    for (int r = 0; r < R; r++) {
      const uint8_t* q = W.qs + (size_t)min((uint32_t)(grp * R + r), W.M - 1) * W.qs_stride;
#pragma unroll
      for (int j = 0; j < CH; j++) {
        const int u = (c * CH + j) * 32 + lane;
        if (u < units) ldg256(q + (size_t)u * 32, w[j][r]);
      }
    }
  };
  if (g < n_groups) load(g, 0);
  griddep_wait();
  stage_x<FMT>(x, nw, eps, (int)W.K, (int)W.Kp, sx, sxs, sred);
  griddep_launch();

  for (; g < n_groups; g += gstride) {
    float acc[R];
    const uint8_t* srow[R];
#pragma unroll
    for (int r = 0; r < R; r++) {
      acc[r] = 0.f;
      srow[r] = W.sc + (size_t)min((uint32_t)(g * R + r), W.M - 1) * W.sc_stride;
    }
    for (int c = 0; c < nch; c++) {
      if (c > 0) load(g, c);
#pragma unroll
      for (int j = 0; j < CH; j++) {
        const int u = (c * CH + j) * 32 + lane;
        if (u < units) {
          auto xa = [&](int k) { return ldx<EPU>(sx, u, k); };
          const float xs_lo = D::NEED_XS ? sxs[u * (EPU / 32)] : 0.f;
          const float xs_hi = (D::NEED_XS && EPU == 64) ? sxs[2 * u + 1] : 0.f;
          D::template accum<R>(w[j], xa, srow, u, xs_lo, xs_hi, acc);
        }
      }
    }
    if (g + gstride < n_groups) load(g + gstride, 0);
#pragma unroll
    for (int r = 0; r < R; r++) {
#pragma unroll
      for (int o = 16; o; o >>= 1) acc[r] += __shfl_xor_sync(0xffffffffu, acc[r], o);
    }
    if (lane == 0) epi(g * R, acc, min(R, (int)W.M - g * R));
  }
  epi.finish();
}

// ---------------------------------------------------------------------------
// the TMA-pipelined GEMV (quantized formats)
// ---------------------------------------------------------------------------
// One persistent CTA per SM (two when shared memory allows).  Warp 8 is the
// producer: its lane 0 streams 64-row x 16-unit weight tiles, with their scale
// headers, into a ring of shared-memory stages through 2D TMA loads (no cluster
// multicast) that complete on per-stage mbarriers.  Warps 0-7 consume: thread t
// handles rows 4*(t/16) .. +3 of the tile and unit t%16 of the chunk, so every x
// chunk read from shared memory serves four rows.  Bytes in flight per SM are
// the ring (tens of KB), independent of registers, and scale headers arrive with
// their weights instead of as dependent loads.  The first stages are requested
// before waiting on the previous kernel (weights never depend on it).
//
// Every mbarrier wait is bounded (kWaitLimitCycles); on expiry the thread sets
// g_rf_error and returns, and the producer first waits, again bounded, for the
// copies it has in flight.  No wait depends on another CTA or another GPU.
constexpr int TMA_TR = 64;    // rows per tile
constexpr int TMA_NU = 16;    // 32-byte units per row per chunk
constexpr int TMA_CONSUMERS = 256;
constexpr int TMA_THREADS = TMA_CONSUMERS + 32;
constexpr long long kWaitLimitCycles = 4000000000LL;  // about 2 s at 1.9 GHz

__device__ unsigned g_rf_error;  // nonzero after a bounded wait gave up

__device__ __forceinline__ uint32_t smem_u32(const void* p) { return (uint32_t)__cvta_generic_to_shared(p); }
__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}
__device__ __forceinline__ void mbar_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes) : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}
// Bounded wait for phase `parity` of `bar`; false when the limit expired.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity) {
  if (mbar_try_wait(bar, parity)) return true;
  const long long t0 = clock64();
  while (!mbar_try_wait(bar, parity))
    if (clock64() - t0 > kWaitLimitCycles) return false;
  return true;
}
__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* tm, int x, int y, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::"r"(
          smem_u32(dst)),
      "l"(tm), "r"(x), "r"(y), "r"(smem_u32(bar))
      : "memory");
}

// Block-wide sum of squares over NT threads (every thread of the block).
template <int NT>
__device__ float block_sumsq_nt(const float* __restrict__ x, int n, float* sred) {
  float s = 0.f;
  for (int i = threadIdx.x; i < n; i += NT) {
    const float v = x[i];
    s = fmaf(v, v, s);
  }
#pragma unroll
  for (int o = 16; o; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
  if ((threadIdx.x & 31) == 0) sred[threadIdx.x >> 5] = s;
  __syncthreads();
  if (threadIdx.x == 0) {
    float t = 0.f;
    for (int w = 0; w < NT / 32; w++) t += sred[w];
    sred[32] = t;
  }
  __syncthreads();
  const float r = sred[32];
  __syncthreads();
  return r;
}

// stage_x for NT threads over Kc >= Kp elements (zero beyond K).
template <int FMT, int NT>
__device__ void stage_x_nt(const float* __restrict__ x, const float* __restrict__ nw, float eps, int K, int Kc,
                           float* sx, float* sxs, float* sred) {
  using D = UnitDot<FMT>;
  constexpr int EPU = D::EPU;
  float rms = 1.f;
  if (nw) rms = rms_of(block_sumsq_nt<NT>(x, K, sred), K, eps);
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  for (int c = warp; c * 32 < Kc; c += NT / 32) {
    const int e = c * 32 + lane;
    float v = 0.f;
    if (e < K) {
      const float xv = x[e];
      v = nw ? xv / rms * nw[e] : xv;
    }
    sx[swz<EPU>(e)] = v * prescale(field_off<FMT>(e % EPU));
    if (D::NEED_XS) {
      float s = v;
#pragma unroll
      for (int o = 16; o; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
      if (lane == 0) sxs[c] = s;
    }
  }
  __syncthreads();
}

template <int FMT, class Epi>
__global__ void __launch_bounds__(TMA_THREADS, 1)
    gemv_tma_kernel(const __grid_constant__ CUtensorMap tm_qs, const __grid_constant__ CUtensorMap tm_sc, PackedMat W,
                    const float* __restrict__ x, const float* __restrict__ nw, float eps, int nstages,
                    uint32_t sc_chunk_bytes, Epi epi) {
  using D = UnitDot<FMT>;
  constexpr int EPU = D::EPU;
  extern __shared__ __align__(128) uint8_t smem_raw[];
  const int tid = threadIdx.x, lane = tid & 31;
  const uint32_t qs_tile = TMA_TR * TMA_NU * 32;
  const uint32_t sc_tile = TMA_TR * sc_chunk_bytes;
  const uint32_t stage_bytes = (qs_tile + sc_tile + 127) & ~127u;
  uint64_t* full = reinterpret_cast<uint64_t*>(smem_raw);
  uint64_t* empty = full + nstages;
  uint8_t* stages = smem_raw + 128;
  const int units = (int)W.units;
  const int nch = (units + TMA_NU - 1) / TMA_NU;
  const int Kc = nch * TMA_NU * EPU;
  float* sx = reinterpret_cast<float*>(stages + (size_t)nstages * stage_bytes);
  float* sxs = sx + Kc;
  float* sred = sxs + Kc / 32;
  const int ntiles = (int)((W.M + TMA_TR - 1) / TMA_TR);
  const int my_tiles = (int)blockIdx.x < ntiles ? (ntiles - 1 - (int)blockIdx.x) / (int)gridDim.x + 1 : 0;
  const int total = my_tiles * nch;
  const bool producer = tid == TMA_CONSUMERS;

  if (producer) {
    for (int i = 0; i < nstages; i++) {
      mbar_init(&full[i], 1);
      mbar_init(&empty[i], TMA_CONSUMERS / 32);
    }
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  __syncthreads();
  auto issue = [&](int k) {
    const int slot = k % nstages;
    const int t = (int)blockIdx.x + (k / nch) * (int)gridDim.x, c = k % nch;
    uint8_t* st = stages + (size_t)slot * stage_bytes;
    mbar_expect_tx(&full[slot], qs_tile + sc_tile);
    tma_load_2d(st, &tm_qs, c * TMA_NU * 8, t * TMA_TR, &full[slot]);
    tma_load_2d(st + qs_tile, &tm_sc, c * (int)(sc_chunk_bytes / 4), t * TMA_TR, &full[slot]);
  };
  if (producer)
    for (int k = 0; k < min(nstages, total); k++) issue(k);
  griddep_wait();
  stage_x_nt<FMT, TMA_THREADS>(x, nw, eps, (int)W.K, Kc, sx, sxs, sred);
  griddep_launch();

  if (tid >= TMA_CONSUMERS) {  // producer warp
    if (lane == 0) {
      for (int k = nstages; k < total; k++) {
        const int slot = k % nstages;
        if (!mbar_wait(&empty[slot], ((k / nstages) - 1) & 1)) {
          atomicExch(&g_rf_error, 1u);
          for (int j = max(0, k - nstages); j < k; j++)  // let the copies in flight land
            if (!mbar_wait(&full[j % nstages], (j / nstages) & 1)) break;
          return;
        }
        issue(k);
      }
    }
    return;
  }
  const int g = tid >> 4, s = tid & 15;
  int k = 0;
  for (int ti = 0; ti < my_tiles; ti++) {
    const int t = (int)blockIdx.x + ti * (int)gridDim.x;
    float acc[4] = {0.f, 0.f, 0.f, 0.f};
    for (int c = 0; c < nch; c++, k++) {
      const int slot = k % nstages;
      if (!mbar_wait(&full[slot], (k / nstages) & 1)) {
        atomicExch(&g_rf_error, 2u);
        return;
      }
      const uint8_t* st = stages + (size_t)slot * stage_bytes;
      const int u = c * TMA_NU + s;
      if (u < units) {
        uint32_t w[4][8];
        const uint8_t* srow[4];
#pragma unroll
        for (int r = 0; r < 4; r++) {
          const uint4* p = reinterpret_cast<const uint4*>(st + (size_t)(4 * g + r) * (TMA_NU * 32) + s * 32);
          const uint4 a = p[0], b = p[1];
          w[r][0] = a.x; w[r][1] = a.y; w[r][2] = a.z; w[r][3] = a.w;
          w[r][4] = b.x; w[r][5] = b.y; w[r][6] = b.z; w[r][7] = b.w;
          srow[r] = st + qs_tile + (size_t)(4 * g + r) * sc_chunk_bytes;
        }
        auto xa = [&](int kk) { return ldx<EPU>(sx, u, kk); };
        const float xs_lo = D::NEED_XS ? sxs[u * (EPU / 32)] : 0.f;
        const float xs_hi = (D::NEED_XS && EPU == 64) ? sxs[2 * u + 1] : 0.f;
        D::template accum<4, decltype(xa), true>(w, xa, srow, s, xs_lo, xs_hi, acc);
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&empty[slot]);
    }
#pragma unroll
    for (int r = 0; r < 4; r++) {
#pragma unroll
      for (int o = 8; o; o >>= 1) acc[r] += __shfl_xor_sync(0xffffffffu, acc[r], o);
    }
    const int row0 = t * TMA_TR + 4 * g;
    if (s == 0 && row0 < (int)W.M) epi(row0, acc, min(4, (int)W.M - row0));
  }
  epi.flush();
}

// Batched variant for the standalone op: x[b][K] read through L1, R = 1.
template <int FMT, int B>
__global__ void __launch_bounds__(GEMV_THREADS) gemv_batched_kernel(PackedMat W, const float* __restrict__ x,
                                                                    float* __restrict__ y) {
  using D = UnitDot<FMT>;
  constexpr int EPU = D::EPU;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int units = (int)W.units;
  for (int row = blockIdx.x * GEMV_WARPS + warp; row < (int)W.M; row += gridDim.x * GEMV_WARPS) {
    float acc[B];
#pragma unroll
    for (int b = 0; b < B; b++) acc[b] = 0.f;
    const uint8_t* q = W.qs + (size_t)row * W.qs_stride;
    const uint8_t* s = W.sc + (size_t)row * W.sc_stride;
    const uint8_t* const srow[1] = {s};
    for (int u = lane; u < units; u += 32) {
      uint32_t w[1][8];
      ldg256(q + (size_t)u * 32, w[0]);
#pragma unroll
      for (int b = 0; b < B; b++) {
        const float* xb = x + (size_t)b * W.Kp + (size_t)u * EPU;
        auto xa = [&](int c) {
          const float4 f = __ldg(reinterpret_cast<const float4*>(xb) + c);
          return make_float4(f.x * prescale(field_off<FMT>(4 * c)), f.y * prescale(field_off<FMT>(4 * c + 1)),
                             f.z * prescale(field_off<FMT>(4 * c + 2)), f.w * prescale(field_off<FMT>(4 * c + 3)));
        };
        float xs_lo = 0.f, xs_hi = 0.f;
        if (D::NEED_XS) {
#pragma unroll 8
          for (int l = 0; l < 32; l++) xs_lo += xb[l];
          if (EPU == 64) {
#pragma unroll 8
            for (int l = 0; l < 32; l++) xs_hi += xb[32 + l];
          }
        }
        float a1[1] = {acc[b]};
        D::template accum<1>(w, xa, srow, u, xs_lo, xs_hi, a1);
        acc[b] = a1[0];
      }
    }
#pragma unroll
    for (int b = 0; b < B; b++) {
#pragma unroll
      for (int o = 16; o; o >>= 1) acc[b] += __shfl_xor_sync(0xffffffffu, acc[b], o);
      if (lane == 0) y[(size_t)b * W.M + row] = acc[b];
    }
  }
}

// ---------------------------------------------------------------------------
// launch plumbing
// ---------------------------------------------------------------------------
static int g_num_sms = 0;
static int num_sms() {
  if (!g_num_sms) {
    int dev = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&g_num_sms, cudaDevAttrMultiProcessorCount, dev);
    if (g_num_sms <= 0) g_num_sms = 148;
  }
  return g_num_sms;
}

template <typename... KArgs, typename... Args>
static cudaError_t launch_k(const Launch& L, void (*k)(KArgs...), dim3 grid, dim3 block, size_t smem,
                            Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = L.stream;
  cudaLaunchAttribute attr[1];
  if (L.pdl) {
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
  }
  return cudaLaunchKernelEx(&cfg, k, std::forward<Args>(args)...);
}

static size_t gemv_smem(const PackedMat& W) { return ((size_t)W.Kp + W.Kp / 32 + 40) * sizeof(float); }

template <int FMT, int R, class Epi>
static cudaError_t run_gemv_t(const Launch& L, const PackedMat& W, const float* x, const float* nw, float eps,
                              Epi epi) {
  auto k = gemv_kernel<FMT, R, Epi>;
  const size_t smem = gemv_smem(W);
  if (smem > 48 * 1024) {
    cudaError_t e = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return e;
  }
  const int groups = (int)((W.M + R - 1) / R);
  int blocks = (groups + GEMV_WARPS - 1) / GEMV_WARPS;
  const int per_sm = smem <= 110 * 1024 ? 2 : 1;  // persistent: 2 CTAs (16 warps) per SM
  blocks = std::max(1, std::min(blocks, num_sms() * per_sm));
  return launch_k(L, k, dim3(blocks), dim3(GEMV_THREADS), smem, W, x, nw, eps, epi);
}

template <int R, class Epi>
static cudaError_t run_gemv_r(const Launch& L, const PackedMat& W, const float* x, const float* nw, float eps,
                              Epi epi) {
  switch (W.type) {
    case T_Q4_K: return run_gemv_t<T_Q4_K, R>(L, W, x, nw, eps, epi);
    case T_Q4_0: return run_gemv_t<T_Q4_0, R>(L, W, x, nw, eps, epi);
    case T_Q8_0: return run_gemv_t<T_Q8_0, R>(L, W, x, nw, eps, epi);
    case T_F16: return run_gemv_t<T_F16, R>(L, W, x, nw, eps, epi);
    case T_F32: return run_gemv_t<T_F32, R>(L, W, x, nw, eps, epi);
    default: return cudaErrorInvalidValue;
  }
}

constexpr size_t kMaxSmem = 227 * 1024;

template <int FMT, class Epi>
static cudaError_t run_gemv_tma_t(const Launch& L, const PackedMat& W, const GemvMaps& m, const float* x,
                                  const float* nw, float eps, Epi epi) {
  constexpr int EPU = UnitDot<FMT>::EPU;
  auto k = gemv_tma_kernel<FMT, Epi>;
  const int nch = (int)((W.units + TMA_NU - 1) / TMA_NU);
  const size_t Kc = (size_t)nch * TMA_NU * EPU;
  const size_t x_bytes = (Kc + Kc / 32 + 40) * sizeof(float);
  const size_t stage_bytes = ((size_t)TMA_TR * TMA_NU * 32 + (size_t)TMA_TR * m.sc_chunk_bytes + 127) & ~(size_t)127;
  if (128 + 2 * stage_bytes + x_bytes > kMaxSmem) return cudaErrorInvalidValue;
  const int nstages = (int)std::min<size_t>(6, (kMaxSmem - 128 - x_bytes) / stage_bytes);
  const size_t smem = 128 + (size_t)nstages * stage_bytes + x_bytes;
  cudaError_t e = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) return e;
  const int ntiles = (int)((W.M + TMA_TR - 1) / TMA_TR);
  const int blocks = std::max(1, std::min(ntiles, num_sms()));
  return launch_k(L, k, dim3(blocks), dim3(TMA_THREADS), smem, m.qs, m.sc, W, x, nw, eps, nstages,
                  m.sc_chunk_bytes, epi);
}

// Rows per warp group of the register-streaming GEMV: 4 when a row has at most
// 64 units (every lane then holds 2 units of each of 4 rows), else 2 (4 units of
// each of 2 rows).  Both are even, which the RoPE and SwiGLU row pairs need.
template <class Epi>
static cudaError_t run_gemv(const Launch& L, const PackedMat& W, const GemvMaps* maps, const float* x,
                            const float* nw, float eps, Epi epi) {
  if (maps && maps->ok) {
    cudaError_t e = cudaErrorInvalidValue;
    switch (W.type) {
      case T_Q4_K: e = run_gemv_tma_t<T_Q4_K>(L, W, *maps, x, nw, eps, epi); break;
      case T_Q4_0: e = run_gemv_tma_t<T_Q4_0>(L, W, *maps, x, nw, eps, epi); break;
      case T_Q8_0: e = run_gemv_tma_t<T_Q8_0>(L, W, *maps, x, nw, eps, epi); break;
    }
    if (e != cudaErrorInvalidValue) return e;  // too large for shared memory: fall through
  }
  if (W.units <= 64) return run_gemv_r<4>(L, W, x, nw, eps, epi);
  return run_gemv_r<2>(L, W, x, nw, eps, epi);
}

cudaError_t gemv_store(const Launch& L, const PackedMat& W, const GemvMaps* maps, const float* x, const float* nw,
                       float eps, float* y) {
  return run_gemv(L, W, maps, x, nw, eps, EpiStore{y});
}
cudaError_t gemv_residual(const Launch& L, const PackedMat& W, const GemvMaps* maps, const float* x, const float* res,
                          float* out) {
  return run_gemv(L, W, maps, x, nullptr, 0.f, EpiResidual{res, out});
}
cudaError_t gemv_qkv_rope(const Launch& L, const PackedMat& W, const GemvMaps* maps, const float* x,
                          const float* nw, float eps, const RopeQKVArgs& a) {
  return run_gemv(L, W, maps, x, nw, eps, EpiRope{a});
}
cudaError_t gemv_swiglu(const Launch& L, const PackedMat& W, const GemvMaps* maps, const float* x, const float* nw,
                        float eps, float* act) {
  return run_gemv(L, W, maps, x, nw, eps, EpiSwiGLU{act});
}
cudaError_t gemv_argmax(const Launch& L, const PackedMat& W, const GemvMaps* maps, const float* x, const float* nw,
                        float eps, float* logits, unsigned long long* key, uint32_t row_offset) {
  return run_gemv(L, W, maps, x, nw, eps, EpiArgmax{logits, key, row_offset, 0ull});
}

// ---- TMA descriptors ----------------------------------------------------------
typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);
static EncodeTiledFn encode_tiled() {
  static EncodeTiledFn fn = nullptr;
  static bool tried = false;
  if (!tried) {
    tried = true;
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = (EncodeTiledFn)p;
  }
  return fn;
}

// 2D map over rows of `row_bytes` (uint32 elements), box = box_words x TMA_TR rows.
static bool encode_rows(CUtensorMap* tm, void* base, uint64_t row_bytes, uint64_t stride, uint32_t rows,
                        uint32_t box_words) {
  EncodeTiledFn fn = encode_tiled();
  if (!fn || row_bytes % 4 || stride % 16 || ((uintptr_t)base & 15) || box_words == 0 || box_words > 256)
    return false;
  const cuuint64_t dims[2] = {row_bytes / 4, rows};
  const cuuint64_t strides[1] = {stride};
  const cuuint32_t box[2] = {box_words, (cuuint32_t)TMA_TR};
  const cuuint32_t estr[2] = {1, 1};
  return fn(tm, CU_TENSOR_MAP_DATA_TYPE_UINT32, 2, base, dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
            CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

bool make_gemv_maps(const PackedMat& W, GemvMaps* out) {
  out->ok = false;
  uint32_t sc_chunk = 0;
  switch (W.type) {
    case T_Q4_K: sc_chunk = TMA_NU / 4 * 16; break;  // one 16-byte header per 4 units
    case T_Q4_0: sc_chunk = TMA_NU * 4; break;       // two f16 scales per unit
    case T_Q8_0: sc_chunk = TMA_NU * 2; break;       // one f16 scale per unit
    default: return false;
  }
  if (!encode_rows(&out->qs, W.qs, W.qs_stride, W.qs_stride, W.M, TMA_NU * 8)) return false;
  if (!encode_rows(&out->sc, W.sc, W.sc_stride, W.sc_stride, W.M, sc_chunk / 4)) return false;
  out->sc_chunk_bytes = sc_chunk;
  out->ok = true;
  return true;
}

template <int FMT>
static cudaError_t run_batched_t(cudaStream_t s, const PackedMat& W, const float* x, int batch, float* y) {
  int blocks = std::max(1, std::min((int)((W.M + GEMV_WARPS - 1) / GEMV_WARPS), num_sms() * 8));
  switch (batch) {
    case 1: gemv_batched_kernel<FMT, 1><<<blocks, GEMV_THREADS, 0, s>>>(W, x, y); break;
    case 2: gemv_batched_kernel<FMT, 2><<<blocks, GEMV_THREADS, 0, s>>>(W, x, y); break;
    case 3: gemv_batched_kernel<FMT, 3><<<blocks, GEMV_THREADS, 0, s>>>(W, x, y); break;
    case 4: gemv_batched_kernel<FMT, 4><<<blocks, GEMV_THREADS, 0, s>>>(W, x, y); break;
    case 5: gemv_batched_kernel<FMT, 5><<<blocks, GEMV_THREADS, 0, s>>>(W, x, y); break;
    case 6: gemv_batched_kernel<FMT, 6><<<blocks, GEMV_THREADS, 0, s>>>(W, x, y); break;
    case 7: gemv_batched_kernel<FMT, 7><<<blocks, GEMV_THREADS, 0, s>>>(W, x, y); break;
    case 8: gemv_batched_kernel<FMT, 8><<<blocks, GEMV_THREADS, 0, s>>>(W, x, y); break;
    default: return cudaErrorInvalidValue;
  }
  return cudaGetLastError();
}

cudaError_t gemv_batched(cudaStream_t s, const PackedMat& W, const float* x, int batch, float* y) {
  switch (W.type) {
    case T_Q4_K: return run_batched_t<T_Q4_K>(s, W, x, batch, y);
    case T_Q4_0: return run_batched_t<T_Q4_0>(s, W, x, batch, y);
    case T_Q8_0: return run_batched_t<T_Q8_0>(s, W, x, batch, y);
    case T_F16: return run_batched_t<T_F16>(s, W, x, batch, y);
    case T_F32: return run_batched_t<T_F32>(s, W, x, batch, y);
    default: return cudaErrorInvalidValue;
  }
}

bool packed_geometry(int type, uint32_t M, uint32_t K, PackedMat* p) {
  if (!block_elems(type) || K == 0 || M == 0 || K % block_elems(type)) return false;
  p->type = type;
  p->M = M;
  p->K = K;
  p->Kp = padded_k(type, K);
  switch (type) {
    case T_F32: p->qs_stride = (uint64_t)p->Kp * 4; p->sc_stride = 0; break;
    case T_F16: p->qs_stride = (uint64_t)p->Kp * 2; p->sc_stride = 0; break;
    case T_Q8_0: p->qs_stride = p->Kp; p->sc_stride = (uint64_t)p->Kp / 32 * 2; break;
    case T_Q4_0: p->qs_stride = p->Kp / 2; p->sc_stride = (uint64_t)p->Kp / 32 * 2; break;
    case T_Q4_K: p->qs_stride = p->Kp / 2; p->sc_stride = (uint64_t)p->Kp / 256 * 16; break;
  }
  p->units = (uint32_t)(p->qs_stride / 32);
  p->qs = p->sc = nullptr;
  return true;
}

// ---------------------------------------------------------------------------
// packing: GGUF rows -> PackedMat (pure byte shuffle)
// ---------------------------------------------------------------------------
__global__ void pack_kernel(const uint8_t* __restrict__ src, const int* __restrict__ src_row_of, PackedMat d,
                            uint32_t nblk, uint32_t bsz, uint64_t src_row_bytes) {
  const uint64_t total = (uint64_t)d.M * nblk;
  for (uint64_t t = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x; t < total;
       t += (uint64_t)gridDim.x * blockDim.x) {
    const uint32_t r = (uint32_t)(t / nblk), b = (uint32_t)(t % nblk);
    const uint32_t sr = src_row_of ? (uint32_t)src_row_of[r] : r;
    const uint8_t* s = src + sr * src_row_bytes + (uint64_t)b * bsz;
    uint8_t* q = d.qs + (uint64_t)r * d.qs_stride;
    uint8_t* c = d.sc + (uint64_t)r * d.sc_stride;
    switch (d.type) {
      case T_F32:
      case T_F16:
        for (uint32_t i = 0; i < bsz; i++) q[(uint64_t)b * bsz + i] = s[i];
        break;
      case T_Q8_0:
        c[2 * b] = s[0]; c[2 * b + 1] = s[1];
        for (int i = 0; i < 32; i++) q[(uint64_t)b * 32 + i] = s[2 + i];
        break;
      case T_Q4_0:
        c[2 * b] = s[0]; c[2 * b + 1] = s[1];
        for (int i = 0; i < 16; i++) q[(uint64_t)b * 16 + i] = s[2 + i];
        break;
      case T_Q4_K:
        for (int i = 0; i < 16; i++) c[(uint64_t)b * 16 + i] = s[i];
        for (int i = 0; i < 128; i++) q[(uint64_t)b * 128 + i] = s[16 + i];
        break;
    }
  }
}

cudaError_t launch_pack(const uint8_t* gguf, const int* src_row_of, PackedMat dst, cudaStream_t s) {
  const uint32_t nblk = dst.K / block_elems(dst.type), bsz = block_bytes(dst.type);
  const uint64_t row_bytes = (uint64_t)nblk * bsz;
  cudaError_t e = cudaMemsetAsync(dst.qs, 0, dst.qs_stride * dst.M, s);
  if (e == cudaSuccess && dst.sc_stride) e = cudaMemsetAsync(dst.sc, 0, dst.sc_stride * dst.M, s);
  if (e != cudaSuccess) return e;
  const uint64_t total = (uint64_t)dst.M * nblk;
  const int blocks = (int)std::min<uint64_t>((total + 255) / 256, 65535ull * 8);
  pack_kernel<<<blocks, 256, 0, s>>>(gguf, src_row_of, dst, nblk, bsz, row_bytes);
  return cudaGetLastError();
}

// ---------------------------------------------------------------------------
// element-exact dequantisation (embedding rows, parity dumps)
// ---------------------------------------------------------------------------
__device__ float dequant_elem(const PackedMat& W, uint32_t row, uint32_t e) {
  const uint8_t* q = W.qs + (uint64_t)row * W.qs_stride;
  const uint8_t* c = W.sc + (uint64_t)row * W.sc_stride;
  switch (W.type) {
    case T_F32: return reinterpret_cast<const float*>(q)[e];
    case T_F16: return h2f(reinterpret_cast<const unsigned short*>(q)[e]);
    case T_Q8_0: {  // q*d (quant.rs:176-180)
      const float d = h2f(c[2 * (e / 32)] | (c[2 * (e / 32) + 1] << 8));
      return __fmul_rn((float)(int8_t)q[e], d);
    }
    case T_Q4_0: {  // (q-8)*d (quant.rs:104-112)
      const uint32_t b = e / 32, j = e % 32;
      const uint8_t byte = q[b * 16 + (j & 15)];
      const int v = (j < 16 ? (byte & 0xF) : (byte >> 4)) - 8;
      const float d = h2f(c[2 * b] | (c[2 * b + 1] << 8));
      return __fmul_rn((float)v, d);
    }
    case T_Q4_K: {  // d1*q - min1 (quant.rs:228-254)
      const uint32_t sb = e / 256, r = e % 256, gi = r / 64, t = r % 64;
      const uint8_t byte = q[sb * 128 + gi * 32 + (t & 31)];
      const uint32_t nq = t < 32 ? (byte & 0xF) : (byte >> 4);
      const uint8_t* h = c + sb * 16;
      const float d = h2f(h[0] | (h[1] << 8)), dmin = h2f(h[2] | (h[3] << 8));
      const uint8_t* s = h + 4;
      const int j = (int)(2 * gi + (t >= 32));
      uint32_t sc, m;
      if (j < 4) {
        sc = s[j] & 63;
        m = s[j + 4] & 63;
      } else {
        sc = (s[j + 4] & 0xF) | ((s[j - 4] >> 6) << 4);
        m = (s[j + 4] >> 4) | ((s[j] >> 6) << 4);
      }
      const float d1 = __fmul_rn(d, (float)sc), mn = __fmul_rn(dmin, (float)m);
      return __fsub_rn(__fmul_rn(d1, (float)nq), mn);
    }
  }
  return 0.f;
}

__global__ void embed_kernel(PackedMat E, const uint32_t* __restrict__ d_token, float* __restrict__ hidden,
                             unsigned long long* key) {
  griddep_wait();
  const uint32_t tok = min(*d_token, E.M - 1);
  for (uint32_t e = threadIdx.x; e < E.K; e += blockDim.x) hidden[e] = dequant_elem(E, tok, e);
  if (key && threadIdx.x == 0) *key = 0ull;
  griddep_launch();
}

cudaError_t launch_embed(const Launch& L, const PackedMat& E, const uint32_t* d_token, float* hidden,
                         unsigned long long* key) {
  return launch_k(L, embed_kernel, dim3(1), dim3(512), 0, E, d_token, hidden, key);
}

__global__ void dequant_rows_kernel(PackedMat W, uint32_t r0, uint32_t n, float* out) {
  const uint64_t total = (uint64_t)n * W.K;
  for (uint64_t t = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x; t < total; t += (uint64_t)gridDim.x * blockDim.x)
    out[t] = dequant_elem(W, r0 + (uint32_t)(t / W.K), (uint32_t)(t % W.K));
}
cudaError_t launch_dequant_rows(const PackedMat& W, uint32_t r0, uint32_t n, float* out, cudaStream_t s) {
  const uint64_t total = (uint64_t)n * W.K;
  dequant_rows_kernel<<<(int)std::min<uint64_t>((total + 255) / 256, 4096), 256, 0, s>>>(W, r0, n, out);
  return cudaGetLastError();
}

__global__ void __launch_bounds__(GEMV_THREADS) rmsnorm_kernel(const float* __restrict__ x,
                                                               const float* __restrict__ w, float eps, uint32_t n,
                                                               float* __restrict__ y) {
  __shared__ float sred[40];
  griddep_wait();
  const float rms = rms_of(block_sumsq(x, (int)n, sred), (int)n, eps);
  for (uint32_t i = threadIdx.x; i < n; i += GEMV_THREADS) y[i] = x[i] / rms * w[i];
  griddep_launch();
}
cudaError_t launch_rmsnorm(const Launch& L, const float* x, const float* w, float eps, uint32_t n, float* y) {
  return launch_k(L, rmsnorm_kernel, dim3(1), dim3(GEMV_THREADS), 0, x, w, eps, n, y);
}

__global__ void finalize_kernel(const unsigned long long* key, uint32_t* d_token, int* d_pos, uint32_t* hist,
                                int hist_len) {
  griddep_wait();
  if (threadIdx.x == 0) {
    const uint32_t tok = ~(uint32_t)(*key & 0xFFFFFFFFull);
    const int p = *d_pos;
    *d_token = tok;
    if (hist && p >= 0 && p < hist_len) hist[p] = tok;
    *d_pos = p + 1;
  }
  griddep_launch();
}
cudaError_t launch_finalize(const Launch& L, const unsigned long long* key, uint32_t* d_token, int* d_pos,
                            uint32_t* hist, int hist_len) {
  return launch_k(L, finalize_kernel, dim3(1), dim3(32), 0, key, d_token, d_pos, hist, hist_len);
}

__global__ void kv_gather_kernel(const void* cache, int kv_f32, uint32_t kvh, uint32_t max_seq, uint32_t hd,
                                 uint32_t start, uint32_t end, float* out) {
  const uint64_t total = (uint64_t)(end - start) * kvh * hd;
  for (uint64_t t = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x; t < total; t += (uint64_t)gridDim.x * blockDim.x) {
    const uint32_t d = (uint32_t)(t % hd), h = (uint32_t)((t / hd) % kvh), p = start + (uint32_t)(t / hd / kvh);
    const uint64_t c = ((uint64_t)h * max_seq + p) * hd + d;
    out[t] = kv_f32 ? ((const float*)cache)[c] : __half2float(((const __half*)cache)[c]);
  }
}
cudaError_t launch_kv_gather(const void* cache, int kv_f32, uint32_t kvh, uint32_t max_seq, uint32_t hd,
                             uint32_t start, uint32_t end, float* out, cudaStream_t s) {
  if (end <= start) return cudaSuccess;
  const uint64_t total = (uint64_t)(end - start) * kvh * hd;
  kv_gather_kernel<<<(int)std::min<uint64_t>((total + 255) / 256, 4096), 256, 0, s>>>(cache, kv_f32, kvh, max_seq,
                                                                                      hd, start, end, out);
  return cudaGetLastError();
}

// ---------------------------------------------------------------------------
// decode attention: split-K over context, GQA group per CTA
// ---------------------------------------------------------------------------
// attention_reference (compute.rs:461-547) for one query token: query head h
// reads KV head h*KV/H (contiguous groups of G = H/KV heads), so one CTA loads
// each K/V row once for its G heads.  A CTA covers a chunk of about 32+
// positions; each warp takes ATT_UNROLL consecutive positions at a time and
// issues all their row loads before using any (lane i holds dims
// [i*DPL, i*DPL+DPL) of every row), so a CTA's pass over K and over V each cost
// one memory round trip.  The last CTA of a head to finish merges the chunk
// partials (max-rescaled sums); nothing waits on another CTA.
constexpr int ATT_THREADS = 128;
constexpr int ATT_WARPS = ATT_THREADS / 32;
constexpr int ATT_MAX_CHUNK = 512;
constexpr int ATT_MIN_CHUNK = 32;
constexpr int ATT_UNROLL = 8;
constexpr int ATT_MERGE_SPLITS = 64;  // merges of up to this many splits take the parallel path

__host__ __device__ inline int attn_nsplit(int ctx, int max_splits) {
  int s = (ctx + ATT_MIN_CHUNK - 1) / ATT_MIN_CHUNK;
  s = s < 1 ? 1 : s;
  return s < max_splits ? s : max_splits;
}

size_t attn_part_floats(int batch, int n_kv_heads, int max_splits, int G, int hd) {
  return (size_t)batch * n_kv_heads * max_splits * G * (hd + 2);
}

// DPL consecutive elements of one K/V row into f32 registers (zero past hd).
template <int DPL>
__device__ __forceinline__ void load_row(const __half* p, int d0, int hd, float (&v)[DPL]) {
  if (DPL == 4 && d0 + 4 <= hd) {
    const uint2 r = __ldg(reinterpret_cast<const uint2*>(p + d0));
    const float2 a = __half22float2(*reinterpret_cast<const __half2*>(&r.x));
    const float2 b = __half22float2(*reinterpret_cast<const __half2*>(&r.y));
    v[0] = a.x; v[1] = a.y; v[2 % DPL] = b.x; v[3 % DPL] = b.y;
  } else if (DPL == 2 && d0 + 2 <= hd) {
    const float2 a = __half22float2(__ldg(reinterpret_cast<const __half2*>(p + d0)));
    v[0] = a.x; v[1 % DPL] = a.y;
  } else {
#pragma unroll
    for (int i = 0; i < DPL; i++) v[i] = d0 + i < hd ? __half2float(p[d0 + i]) : 0.f;
  }
}
template <int DPL>
__device__ __forceinline__ void load_row(const float* p, int d0, int hd, float (&v)[DPL]) {
#pragma unroll
  for (int i = 0; i < DPL; i++) v[i] = d0 + i < hd ? p[d0 + i] : 0.f;
}

template <int DPL, int G, typename KT>
__global__ void __launch_bounds__(ATT_THREADS) attn_kernel(AttnArgs a) {
  __shared__ float ssc[G][ATT_MAX_CHUNK];
  __shared__ float sred[ATT_WARPS][G][DPL * 32];
  __shared__ float sm[G], sl[G];
  __shared__ float s_w[ATT_MERGE_SPLITS][G];
  __shared__ int s_last;
  const int kvh = blockIdx.x, split = blockIdx.y, b = blockIdx.z;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int hd = a.head_dim;
  griddep_wait();
  const int nhist = a.d_nhist ? *a.d_nhist : a.nhist;
  const bool has_cur = a.k_cur != nullptr;
  const int ctx = nhist + (has_cur ? 1 : 0);
  const int nsplit = attn_nsplit(ctx, a.max_splits);
  if (split >= nsplit || ctx <= 0) {
    griddep_launch();
    return;
  }
  const int chunk = (ctx + nsplit - 1) / nsplit;
  const int h0 = kvh * G;
  if (chunk > ATT_MAX_CHUNK) {  // host sizes max_splits >= ctx/ATT_MAX_CHUNK; never index past ssc
    if (split == 0)
      for (int t = threadIdx.x; t < G * hd; t += ATT_THREADS)
        a.out[((size_t)b * a.n_heads + h0) * hd + t] = __int_as_float(0x7fc00000);
    griddep_launch();
    return;
  }
  const int p0 = split * chunk, p1 = min(ctx, p0 + chunk);
  const int d0 = lane * DPL;
  const float* qb = a.q + ((size_t)b * a.n_heads + h0) * hd;
  float qr[G][DPL];
#pragma unroll
  for (int h = 0; h < G; h++)
#pragma unroll
    for (int i = 0; i < DPL; i++) qr[h][i] = d0 + i < hd ? qb[(size_t)h * hd + d0 + i] : 0.f;
  const KT* kb = reinterpret_cast<const KT*>(a.kc) + (size_t)b * a.batch_stride + (size_t)kvh * a.head_stride;
  const KT* vb = reinterpret_cast<const KT*>(a.vc) + (size_t)b * a.batch_stride + (size_t)kvh * a.head_stride;
  const float* kcur = has_cur ? a.k_cur + (size_t)kvh * hd : nullptr;
  const float* vcur = has_cur ? a.v_cur + (size_t)kvh * hd : nullptr;
  const float div = sqrtf((float)hd);  // score = dot / sqrt(hd)  (compute.rs:530)

  // pass 1: scores
  for (int p = p0 + warp * ATT_UNROLL; p < p1; p += ATT_WARPS * ATT_UNROLL) {
    float k[ATT_UNROLL][DPL];
#pragma unroll
    for (int t = 0; t < ATT_UNROLL; t++) {
      const int pp = p + t;
      if (pp < min(p1, nhist)) load_row<DPL>(kb + (size_t)pp * hd, d0, hd, k[t]);
      else if (pp < p1) load_row<DPL>(kcur, d0, hd, k[t]);
      else {
#pragma unroll
        for (int i = 0; i < DPL; i++) k[t][i] = 0.f;
      }
    }
#pragma unroll
    for (int t = 0; t < ATT_UNROLL; t++) {
#pragma unroll
      for (int h = 0; h < G; h++) {
        float s = 0.f;
#pragma unroll
        for (int i = 0; i < DPL; i++) s = fmaf(qr[h][i], k[t][i], s);
#pragma unroll
        for (int o = 16; o; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
        if (lane == 0 && p + t < p1) ssc[h][p + t - p0] = s / div;
      }
    }
  }
  __syncthreads();
  // per-head max and exp-sum over the chunk (softmax_reference, compute.rs:363-384)
  const int n = p1 - p0;
  for (int h = warp; h < G; h += ATT_WARPS) {
    float m = -INFINITY;
    for (int i = lane; i < n; i += 32) m = fmaxf(m, ssc[h][i]);
#pragma unroll
    for (int o = 16; o; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    float l = 0.f;
    for (int i = lane; i < n; i += 32) {
      const float e = expf(ssc[h][i] - m);
      ssc[h][i] = e;
      l += e;
    }
#pragma unroll
    for (int o = 16; o; o >>= 1) l += __shfl_xor_sync(0xffffffffu, l, o);
    if (lane == 0) {
      sm[h] = m;
      sl[h] = l;
    }
  }
  __syncthreads();
  // pass 2: sum_p e_p * v_p
  float acc[G][DPL];
#pragma unroll
  for (int h = 0; h < G; h++)
#pragma unroll
    for (int i = 0; i < DPL; i++) acc[h][i] = 0.f;
  for (int p = p0 + warp * ATT_UNROLL; p < p1; p += ATT_WARPS * ATT_UNROLL) {
    float v[ATT_UNROLL][DPL];
#pragma unroll
    for (int t = 0; t < ATT_UNROLL; t++) {
      const int pp = p + t;
      if (pp < min(p1, nhist)) load_row<DPL>(vb + (size_t)pp * hd, d0, hd, v[t]);
      else if (pp < p1) load_row<DPL>(vcur, d0, hd, v[t]);
      else {
#pragma unroll
        for (int i = 0; i < DPL; i++) v[t][i] = 0.f;
      }
    }
#pragma unroll
    for (int t = 0; t < ATT_UNROLL; t++) {
      if (p + t < p1) {
#pragma unroll
        for (int h = 0; h < G; h++) {
          const float e = ssc[h][p + t - p0];
#pragma unroll
          for (int i = 0; i < DPL; i++) acc[h][i] = fmaf(e, v[t][i], acc[h][i]);
        }
      }
    }
  }
#pragma unroll
  for (int h = 0; h < G; h++)
#pragma unroll
    for (int i = 0; i < DPL; i++) sred[warp][h][d0 + i] = acc[h][i];
  __syncthreads();
  float* out_b = a.out + ((size_t)b * a.n_heads + h0) * hd;
  if (nsplit == 1) {
    for (int t = threadIdx.x; t < G * hd; t += ATT_THREADS) {
      const int h = t / hd, d = t % hd;
      float s = 0.f;
      for (int w = 0; w < ATT_WARPS; w++) s += sred[w][h][d];
      out_b[(size_t)h * hd + d] = s / sl[h];
    }
    griddep_launch();
    return;
  }
  // write this chunk's partial: [G][hd] sums then (m, l) per head
  const size_t slot = ((size_t)b * a.n_kv_heads + kvh) * a.max_splits;
  float* part = a.part + (slot + split) * (size_t)G * (hd + 2);
  for (int t = threadIdx.x; t < G * hd; t += ATT_THREADS) {
    const int h = t / hd, d = t % hd;
    float s = 0.f;
    for (int w = 0; w < ATT_WARPS; w++) s += sred[w][h][d];
    part[(size_t)h * (hd + 2) + d] = s;
  }
  if (threadIdx.x < G) {
    part[(size_t)threadIdx.x * (hd + 2) + hd] = sm[threadIdx.x];
    part[(size_t)threadIdx.x * (hd + 2) + hd + 1] = sl[threadIdx.x];
  }
  __threadfence();
  __syncthreads();
  if (threadIdx.x == 0) {
    const unsigned prev = atomicAdd(&a.counters[(size_t)b * a.n_kv_heads + kvh], 1u);
    s_last = prev == (unsigned)(nsplit - 1);
  }
  __syncthreads();
  if (!s_last) {
    griddep_launch();
    return;
  }
  __threadfence();
  const float* pall = a.part + slot * (size_t)G * (hd + 2);
  if (nsplit <= ATT_MERGE_SPLITS) {
    // one warp per head: split weights exp(m_s - M) / sum_s exp(m_s - M) l_s in one load round
    for (int h = warp; h < G; h += ATT_WARPS) {
      float ms[ATT_MERGE_SPLITS / 32], ls[ATT_MERGE_SPLITS / 32];
      float M = -INFINITY;
#pragma unroll
      for (int j = 0; j < ATT_MERGE_SPLITS / 32; j++) {
        const int sp = lane + 32 * j;
        const float* ps = pall + ((size_t)sp * G + h) * (hd + 2);
        ms[j] = sp < nsplit ? __ldcg(ps + hd) : -INFINITY;
        ls[j] = sp < nsplit ? __ldcg(ps + hd + 1) : 0.f;
        M = fmaxf(M, ms[j]);
      }
#pragma unroll
      for (int o = 16; o; o >>= 1) M = fmaxf(M, __shfl_xor_sync(0xffffffffu, M, o));
      float L = 0.f;
#pragma unroll
      for (int j = 0; j < ATT_MERGE_SPLITS / 32; j++) {
        ms[j] = lane + 32 * j < nsplit ? expf(ms[j] - M) : 0.f;
        L = fmaf(ms[j], ls[j], L);
      }
#pragma unroll
      for (int o = 16; o; o >>= 1) L += __shfl_xor_sync(0xffffffffu, L, o);
#pragma unroll
      for (int j = 0; j < ATT_MERGE_SPLITS / 32; j++) s_w[lane + 32 * j][h] = ms[j] / L;
    }
    __syncthreads();
    // every output element: sum_s w_s * O_s, eight independent loads at a time
    for (int t = threadIdx.x; t < G * hd; t += ATT_THREADS) {
      const int h = t / hd, d = t % hd;
      float O = 0.f;
      for (int s0 = 0; s0 < nsplit; s0 += 8) {
        float v[8];
#pragma unroll
        for (int j = 0; j < 8; j++)
          v[j] = s0 + j < nsplit ? __ldcg(pall + ((size_t)(s0 + j) * G + h) * (hd + 2) + d) : 0.f;
#pragma unroll
        for (int j = 0; j < 8; j++)
          if (s0 + j < nsplit) O = fmaf(s_w[s0 + j][h], v[j], O);
      }
      out_b[(size_t)h * hd + d] = O;
    }
  } else {
    for (int t = threadIdx.x; t < G * hd; t += ATT_THREADS) {
      const int h = t / hd, d = t % hd;
      float M = -INFINITY;
      for (int s = 0; s < nsplit; s++) M = fmaxf(M, __ldcg(pall + ((size_t)s * G + h) * (hd + 2) + hd));
      float L = 0.f, O = 0.f;
      for (int s = 0; s < nsplit; s++) {
        const float* ps = pall + ((size_t)s * G + h) * (hd + 2);
        const float sc = expf(__ldcg(ps + hd) - M);
        L = fmaf(sc, __ldcg(ps + hd + 1), L);
        O = fmaf(sc, __ldcg(ps + d), O);
      }
      out_b[(size_t)h * hd + d] = O / L;
    }
  }
  if (threadIdx.x == 0) a.counters[(size_t)b * a.n_kv_heads + kvh] = 0u;
  griddep_launch();
}

template <int DPL, int G>
static cudaError_t attn_dispatch_kt(const Launch& L, const AttnArgs& a) {
  dim3 grid(a.n_kv_heads, a.max_splits, a.batch);
  if (a.kv_f32) return launch_k(L, attn_kernel<DPL, G, float>, grid, dim3(ATT_THREADS), 0, a);
  return launch_k(L, attn_kernel<DPL, G, __half>, grid, dim3(ATT_THREADS), 0, a);
}
template <int DPL>
static cudaError_t attn_dispatch_g(const Launch& L, const AttnArgs& a, int G) {
  switch (G) {
    case 1: return attn_dispatch_kt<DPL, 1>(L, a);
    case 2: return attn_dispatch_kt<DPL, 2>(L, a);
    case 4: return attn_dispatch_kt<DPL, 4>(L, a);
    case 8: return attn_dispatch_kt<DPL, 8>(L, a);
    default: return cudaErrorInvalidValue;
  }
}

cudaError_t launch_attention(const Launch& L, const AttnArgs& a) {
  if (a.n_kv_heads <= 0 || a.n_heads % a.n_kv_heads) return cudaErrorInvalidValue;
  const int G = a.n_heads / a.n_kv_heads;
  if (a.head_dim <= 32) return attn_dispatch_g<1>(L, a, G);
  if (a.head_dim <= 64) return attn_dispatch_g<2>(L, a, G);
  if (a.head_dim <= 128) return attn_dispatch_g<4>(L, a, G);
  return cudaErrorInvalidValue;
}

}  // namespace rf
