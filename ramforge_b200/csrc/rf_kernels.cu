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

template <int EPU>
__device__ void stage_x(const float* __restrict__ x, const float* __restrict__ nw, float eps, int K, int Kp,
                        float* sx, float* sxs, float* sred, bool need_xs) {
  float rms = 1.f;
  if (nw) rms = rms_of(block_sumsq(x, K, sred), K, eps);
  // warp w stages 32-element chunks w, w+8, ...: coalesced loads, and the chunk
  // sums sum(x) that the Q4_K min term needs come from one shuffle reduction
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  for (int c = warp; c * 32 < Kp; c += GEMV_WARPS) {
    const int e = c * 32 + lane;
    float v = 0.f;
    if (e < K) {
      const float xv = x[e];
      v = nw ? xv / rms * nw[e] : xv;
    }
    if (e < Kp) sx[swz<EPU>(e)] = v;
    if (need_xs) {
      float s = v;
#pragma unroll
      for (int o = 16; o; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
      if (lane == 0) sxs[c] = s;
    }
  }
  __syncthreads();
}

// ---------------------------------------------------------------------------
// per-unit dot products: 32 bytes of each of R rows against the unit's EPU
// activations, accumulated into acc[R].  x is read one 16-byte chunk at a time
// and reused across the rows, so only a few activations are live at once.
// ---------------------------------------------------------------------------
// XA(c) returns the float4 of unit-relative elements [4c, 4c+4).
template <int FMT>
struct UnitDot;

// Q4_K super-block header fields of sub-block pair i = u%4 (get_scale_min,
// quant.rs:216-226, for j = 2i and 2i+1): d*sc and dmin*m for both sub-blocks.
__device__ __forceinline__ void q4k_scales(const uint8_t* sc_row, int u, float& d1, float& mn1, float& d2,
                                           float& mn2) {
  const uint4 h = __ldg(reinterpret_cast<const uint4*>(sc_row + (size_t)(u >> 2) * 16));
  const float d = h2f(h.x & 0xFFFFu), dmin = h2f(h.x >> 16);
  const int i = u & 3;
  uint32_t sc0, m0, sc1, m1;
  if (i < 2) {
    const uint32_t a = h.y >> (16 * i), b = h.z >> (16 * i);  // s[2i], s[2i+1] / s[2i+4], s[2i+5]
    sc0 = a & 63u;
    sc1 = (a >> 8) & 63u;
    m0 = b & 63u;
    m1 = (b >> 8) & 63u;
  } else {
    const int k = i - 2;  // j = 4+2k, 5+2k: low 4 bits in s[8+2k], s[9+2k]; high 2 bits in s[2k..], s[4+2k..]
    const uint32_t lo = h.w >> (16 * k), hs = h.y >> (16 * k), hm = h.z >> (16 * k);
    sc0 = (lo & 0xFu) | (((hs >> 6) & 3u) << 4);
    sc1 = ((lo >> 8) & 0xFu) | (((hs >> 14) & 3u) << 4);
    m0 = ((lo >> 4) & 0xFu) | (((hm >> 6) & 3u) << 4);
    m1 = ((lo >> 12) & 0xFu) | (((hm >> 14) & 3u) << 4);
  }
  d1 = d * (float)sc0;
  mn1 = dmin * (float)m0;
  d2 = d * (float)sc1;
  mn2 = dmin * (float)m1;
}

template <>
struct UnitDot<T_Q4_K> {
  static constexpr int EPU = 64;
  static constexpr bool NEED_XS = true;
  // Unit u = sub-block pair i = u%4 of super-block u/4: byte l holds element l
  // (low nibble, sub-block 2i) and element 32+l (high nibble, sub-block 2i+1).
  // value = d*sc*q - dmin*m (quant.rs:235-248), summed as
  // (d*sc) * sum(q*x) - (dmin*m) * sum(x).
  template <int R, class XA>
  __device__ __forceinline__ static void accum(const uint32_t (&w)[R][8], XA xa, const uint8_t* const (&srow)[R],
                                               int u, float xs_lo, float xs_hi, float (&acc)[R]) {
    float lo[R], hi[R];
#pragma unroll
    for (int r = 0; r < R; r++) lo[r] = hi[r] = 0.f;
#pragma unroll
    for (int k = 0; k < 8; k++) {
      const float4 a = xa(k), b = xa(8 + k);
#pragma unroll
      for (int r = 0; r < R; r++) {
        const uint32_t v = w[r][k];
        lo[r] = fmaf(nib<0>(v, 0), a.x, lo[r]);
        hi[r] = fmaf(nib<0>(v, 4), b.x, hi[r]);
        lo[r] = fmaf(nib<0>(v, 8), a.y, lo[r]);
        hi[r] = fmaf(nib<0>(v, 12), b.y, hi[r]);
        lo[r] = fmaf(nib<0>(v, 16), a.z, lo[r]);
        hi[r] = fmaf(nib<0>(v, 20), b.z, hi[r]);
        lo[r] = fmaf(nib<0>(v, 24), a.w, lo[r]);
        hi[r] = fmaf(nib<0>(v, 28), b.w, hi[r]);
      }
    }
#pragma unroll
    for (int r = 0; r < R; r++) {
      float d1, mn1, d2, mn2;
      q4k_scales(srow[r], u, d1, mn1, d2, mn2);
      acc[r] += d1 * lo[r] - mn1 * xs_lo + (d2 * hi[r] - mn2 * xs_hi);
    }
  }
};

template <>
struct UnitDot<T_Q4_0> {
  static constexpr int EPU = 64;
  static constexpr bool NEED_XS = false;
  // Unit u = blocks 2u, 2u+1: block byte j holds element j (low) and 16+j (high);
  // value (q-8)*d (quant.rs:104-112).
  template <int R, class XA>
  __device__ __forceinline__ static void accum(const uint32_t (&w)[R][8], XA xa, const uint8_t* const (&srow)[R],
                                               int u, float, float, float (&acc)[R]) {
    float s0[R], s1[R];
#pragma unroll
    for (int r = 0; r < R; r++) s0[r] = s1[r] = 0.f;
#pragma unroll
    for (int k = 0; k < 4; k++) {
      const float4 a = xa(k), b = xa(4 + k), c = xa(8 + k), e = xa(12 + k);
#pragma unroll
      for (int r = 0; r < R; r++) {
        const uint32_t v0 = w[r][k], v1 = w[r][4 + k];
        s0[r] = fmaf(nib<8>(v0, 0), a.x, s0[r]);
        s0[r] = fmaf(nib<8>(v0, 8), a.y, s0[r]);
        s0[r] = fmaf(nib<8>(v0, 16), a.z, s0[r]);
        s0[r] = fmaf(nib<8>(v0, 24), a.w, s0[r]);
        s0[r] = fmaf(nib<8>(v0, 4), b.x, s0[r]);
        s0[r] = fmaf(nib<8>(v0, 12), b.y, s0[r]);
        s0[r] = fmaf(nib<8>(v0, 20), b.z, s0[r]);
        s0[r] = fmaf(nib<8>(v0, 28), b.w, s0[r]);
        s1[r] = fmaf(nib<8>(v1, 0), c.x, s1[r]);
        s1[r] = fmaf(nib<8>(v1, 8), c.y, s1[r]);
        s1[r] = fmaf(nib<8>(v1, 16), c.z, s1[r]);
        s1[r] = fmaf(nib<8>(v1, 24), c.w, s1[r]);
        s1[r] = fmaf(nib<8>(v1, 4), e.x, s1[r]);
        s1[r] = fmaf(nib<8>(v1, 12), e.y, s1[r]);
        s1[r] = fmaf(nib<8>(v1, 20), e.z, s1[r]);
        s1[r] = fmaf(nib<8>(v1, 28), e.w, s1[r]);
      }
    }
#pragma unroll
    for (int r = 0; r < R; r++) {
      const uint32_t dd = __ldg(reinterpret_cast<const uint32_t*>(srow[r]) + u);
      acc[r] += h2f(dd & 0xFFFFu) * s0[r] + h2f(dd >> 16) * s1[r];
    }
  }
};

template <>
struct UnitDot<T_Q8_0> {
  static constexpr int EPU = 32;
  static constexpr bool NEED_XS = false;
  // Unit u = block u: 32 signed bytes, value q*d (quant.rs:176-180).
  template <int R, class XA>
  __device__ __forceinline__ static void accum(const uint32_t (&w)[R][8], XA xa, const uint8_t* const (&srow)[R],
                                               int u, float, float, float (&acc)[R]) {
    float s0[R], s1[R];
#pragma unroll
    for (int r = 0; r < R; r++) s0[r] = s1[r] = 0.f;
#pragma unroll
    for (int k = 0; k < 8; k++) {
      const float4 a = xa(k);
#pragma unroll
      for (int r = 0; r < R; r++) {
        const uint32_t v = w[r][k];
        s0[r] = fmaf(sbyte_f(v, 0), a.x, s0[r]);
        s1[r] = fmaf(sbyte_f(v, 8), a.y, s1[r]);
        s0[r] = fmaf(sbyte_f(v, 16), a.z, s0[r]);
        s1[r] = fmaf(sbyte_f(v, 24), a.w, s1[r]);
      }
    }
#pragma unroll
    for (int r = 0; r < R; r++)
      acc[r] += h2f(__ldg(reinterpret_cast<const unsigned short*>(srow[r]) + u)) * (s0[r] + s1[r]);
  }
};

template <>
struct UnitDot<T_F16> {
  static constexpr int EPU = 16;
  static constexpr bool NEED_XS = false;
  template <int R, class XA>
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
  template <int R, class XA>
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

// ---------------------------------------------------------------------------
// epilogues (called by lane 0 of a warp with the R finished row sums)
// ---------------------------------------------------------------------------
struct EpiStore {
  float* y;
  __device__ void operator()(int row0, const float* v, int n) {
    for (int i = 0; i < n; i++) y[row0 + i] = v[i];
  }
  __device__ void finish() {}
};

struct EpiResidual {
  const float* res;
  float* out;
  __device__ void operator()(int row0, const float* v, int n) {
    for (int i = 0; i < n; i++) out[row0 + i] = res ? res[row0 + i] + v[i] : v[i];
  }
  __device__ void finish() {}
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
  stage_x<EPU>(x, nw, eps, (int)W.K, (int)W.Kp, sx, sxs, sred, D::NEED_XS);
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
          const float xs_lo = D::NEED_XS ? sxs[2 * u] : 0.f;
          const float xs_hi = D::NEED_XS ? sxs[2 * u + 1] : 0.f;
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
        auto xa = [&](int c) { return __ldg(reinterpret_cast<const float4*>(xb) + c); };
        float xs_lo = 0.f, xs_hi = 0.f;
        if (D::NEED_XS) {
#pragma unroll 8
          for (int l = 0; l < 32; l++) { xs_lo += xb[l]; xs_hi += xb[32 + l]; }
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

// Rows per warp group: 4 when a row has at most 64 units (every lane then holds
// 2 units of each of 4 rows), else 2 (4 units of each of 2 rows).  Both are even,
// which the RoPE and SwiGLU row pairs need.
template <class Epi>
static cudaError_t run_gemv(const Launch& L, const PackedMat& W, const float* x, const float* nw, float eps,
                            Epi epi) {
  if (W.units <= 64) return run_gemv_r<4>(L, W, x, nw, eps, epi);
  return run_gemv_r<2>(L, W, x, nw, eps, epi);
}

cudaError_t gemv_store(const Launch& L, const PackedMat& W, const float* x, const float* nw, float eps, float* y) {
  return run_gemv(L, W, x, nw, eps, EpiStore{y});
}
cudaError_t gemv_residual(const Launch& L, const PackedMat& W, const float* x, const float* res, float* out) {
  return run_gemv(L, W, x, nullptr, 0.f, EpiResidual{res, out});
}
cudaError_t gemv_qkv_rope(const Launch& L, const PackedMat& W, const float* x, const float* nw, float eps,
                          const RopeQKVArgs& a) {
  return run_gemv(L, W, x, nw, eps, EpiRope{a});
}
cudaError_t gemv_swiglu(const Launch& L, const PackedMat& W, const float* x, const float* nw, float eps,
                        float* act) {
  return run_gemv(L, W, x, nw, eps, EpiSwiGLU{act});
}
cudaError_t gemv_argmax(const Launch& L, const PackedMat& W, const float* x, const float* nw, float eps,
                        float* logits, unsigned long long* key, uint32_t row_offset) {
  return run_gemv(L, W, x, nw, eps, EpiArgmax{logits, key, row_offset, 0ull});
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
