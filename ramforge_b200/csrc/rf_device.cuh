// rf_device.cuh - device helpers and launch plumbing shared by the kernel
// translation units (rf_kernels.cu, rf_gemv.cu).
#pragma once
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <utility>

#include "rf_kernels.cuh"

namespace rf {

__device__ __forceinline__ void griddep_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void griddep_launch() { asm volatile("griddepcontrol.launch_dependents;" :::); }

// Flags of the tensor-parallel sums (written and read across GPUs).
__device__ __forceinline__ void st_release_sys(unsigned* p, unsigned v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ unsigned ld_acquire_sys(const unsigned* p) {
  unsigned v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
// Wait until *f == e: 4096 polls, then 64 ns sleeps between polls, about a second
// in all; false when it gave up.
__device__ __forceinline__ bool wait_flag_sys(const unsigned* f, unsigned e) {
  constexpr unsigned kSpinFast = 1u << 12, kSpinLimit = 1u << 24;
  unsigned it = 0;
  while (ld_acquire_sys(f) != e) {
    if (++it > kSpinLimit) return false;
    if (it > kSpinFast) __nanosleep(64);
  }
  return true;
}

// Arrival on a (possibly peer) counter, after this thread's (and, through a
// preceding barrier, its CTA's) stores.
__device__ __forceinline__ void red_release_sys_add(unsigned* p, unsigned v) {
  asm volatile("red.release.sys.global.add.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
// Wait until the counter *f has reached `want` (it only grows between resets;
// compared modulo 2^32), bounded like wait_flag_sys.
__device__ __forceinline__ bool wait_count_sys(const unsigned* f, unsigned want) {
  constexpr unsigned kSpinFast = 1u << 12, kSpinLimit = 1u << 24;
  unsigned it = 0;
  while ((int)(ld_acquire_sys(f) - want) < 0) {
    if (++it > kSpinLimit) return false;
    if (it > kSpinFast) __nanosleep(64);
  }
  return true;
}

// Streaming loads of weights (read once per token: no L1 allocation).
__device__ __forceinline__ void ldg256(const uint8_t* p, uint32_t (&w)[8]) {
  asm volatile("ld.global.nc.L1::no_allocate.v8.b32 {%0,%1,%2,%3,%4,%5,%6,%7}, [%8];"
               : "=r"(w[0]), "=r"(w[1]), "=r"(w[2]), "=r"(w[3]), "=r"(w[4]), "=r"(w[5]), "=r"(w[6]), "=r"(w[7])
               : "l"(p));
}
__device__ __forceinline__ void ldg128(const uint8_t* p, uint32_t (&w)[4]) {
  asm volatile("ld.global.nc.L1::no_allocate.v4.b32 {%0,%1,%2,%3}, [%4];"
               : "=r"(w[0]), "=r"(w[1]), "=r"(w[2]), "=r"(w[3])
               : "l"(p));
}
__device__ __forceinline__ void ldg64(const uint8_t* p, uint32_t (&w)[2]) {
  asm volatile("ld.global.nc.L1::no_allocate.v2.b32 {%0,%1}, [%2];" : "=r"(w[0]), "=r"(w[1]) : "l"(p));
}
// The same loads under a predicate (no branch): registers keep their values when
// `on` is false, and nothing is read.
__device__ __forceinline__ void ldg256_if(bool on, const uint8_t* p, uint32_t (&w)[8]) {
  asm volatile(
      "{ .reg .pred q; setp.ne.u32 q, %9, 0;\n"
      "@q ld.global.nc.L1::no_allocate.v8.b32 {%0,%1,%2,%3,%4,%5,%6,%7}, [%8]; }"
      : "+r"(w[0]), "+r"(w[1]), "+r"(w[2]), "+r"(w[3]), "+r"(w[4]), "+r"(w[5]), "+r"(w[6]), "+r"(w[7])
      : "l"(p), "r"((uint32_t)on));
}
__device__ __forceinline__ void ldg128_if(bool on, const uint8_t* p, uint32_t (&w)[4]) {
  asm volatile(
      "{ .reg .pred q; setp.ne.u32 q, %5, 0;\n"
      "@q ld.global.nc.L1::no_allocate.v4.b32 {%0,%1,%2,%3}, [%4]; }"
      : "+r"(w[0]), "+r"(w[1]), "+r"(w[2]), "+r"(w[3])
      : "l"(p), "r"((uint32_t)on));
}
__device__ __forceinline__ void ldg64_if(bool on, const uint8_t* p, uint32_t (&w)[2]) {
  asm volatile(
      "{ .reg .pred q; setp.ne.u32 q, %3, 0;\n"
      "@q ld.global.nc.L1::no_allocate.v2.b32 {%0,%1}, [%2]; }"
      : "+r"(w[0]), "+r"(w[1])
      : "l"(p), "r"((uint32_t)on));
}

// f16 -> f32 as the reference decodes block scales and F16 tensors
// (quant.rs:40-65, tensor.rs:1017-1041): IEEE for normal numbers, but a
// subnormal half comes out at half its IEEE value (the normalising loop's
// exponent is one short).  The engine reproduces that for bit-parity.
__device__ __forceinline__ float h2f(uint32_t bits16) {
  const float f = __half2float(__ushort_as_half((unsigned short)bits16));
  return (bits16 & 0x7C00u) ? f : f * 0.5f;
}

// Element e of packed row `row`, dequantised exactly as the reference does it
// (embedding rows, parity dumps).
__device__ __forceinline__ float dequant_elem(const PackedMat& W, uint32_t row, uint32_t e) {
  const uint8_t* q = W.qs;
  const uint8_t* c = W.sc;
  switch (W.type) {
    case T_F32: return reinterpret_cast<const float*>(q + (uint64_t)row * W.qs_stride)[e];
    case T_F16: return h2f(reinterpret_cast<const unsigned short*>(q + (uint64_t)row * W.qs_stride)[e]);
    case T_Q8_0: {  // q*d (quant.rs:176-180)
      const uint8_t* sp = c + sc_byte_off(W, row, 2ull * (e / 32));
      const float d = h2f(sp[0] | (sp[1] << 8));
      return __fmul_rn((float)(int8_t)q[qs_byte_off(W, row, e)], d);
    }
    case T_Q4_0: {  // (q-8)*d (quant.rs:104-112)
      const uint32_t b = e / 32, j = e % 32;
      const uint8_t byte = q[qs_byte_off(W, row, (uint64_t)b * 16 + (j & 15))];
      const int v = (j < 16 ? (byte & 0xF) : (byte >> 4)) - 8;
      const uint8_t* sp = c + sc_byte_off(W, row, 2ull * b);
      const float d = h2f(sp[0] | (sp[1] << 8));
      return __fmul_rn((float)v, d);
    }
    case T_Q4_K: {  // d1*q - min1 (quant.rs:228-254)
      const uint32_t sb = e / 256, r = e % 256, gi = r / 64, t = r % 64;
      const uint8_t byte = q[qs_byte_off(W, row, (uint64_t)sb * 128 + gi * 32 + (t & 31))];
      const uint32_t nq = t < 32 ? (byte & 0xF) : (byte >> 4);
      const uint8_t* h = c + sc_byte_off(W, row, (uint64_t)sb * 16);
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
    case T_Q3_K:
    case T_Q2_K: {  // Q3_K (d*sc)*(u-4) (quant.rs:506-574), Q2_K (d*sc)*u - dmin*m (:443-474)
      const uint32_t ch = e / 256, G = (e % 256) / 16, t = e % 16;
      const uint8_t byte = q[qs_byte_off(W, row, (uint64_t)ch * QT_CHUNK_BYTES + 32 * (G / 4) + 8 * (G % 4) + t % 8)];
      const uint32_t u = t < 8 ? (byte & 15u) : (uint32_t)(byte >> 4);
      const uint64_t hb = (uint64_t)ch * NG_HDR_BYTES;
      const uint8_t sbyte = c[sc_byte_off(W, row, hb + G)];
      const uint8_t* dp = c + sc_byte_off(W, row, hb + 16);
      const float d = h2f(dp[0] | (dp[1] << 8));
      if (W.type == T_Q3_K) return __fmul_rn(__fmul_rn(d, (float)(int8_t)sbyte), (float)((int)u - 4));
      const float dmin = h2f(dp[2] | (dp[3] << 8));
      return __fsub_rn(__fmul_rn(__fmul_rn(d, (float)(sbyte & 15)), (float)u), __fmul_rn(dmin, (float)(sbyte >> 4)));
    }
    case T_Q5_K:
    case T_Q6_K: {  // Q6_K (d*sc)*q (quant.rs:376-406), Q5_K (d*sc)*u - dmin*m (:303-343); words as
                    // six_bit_words packs them
      const uint32_t ch = e / 128, j = (e % 128) / 16, t = e % 16;
      const uint64_t wb = (uint64_t)ch * Q6_CHUNK_BYTES + 12 * j;
      auto word = [&](uint32_t k) {
        const uint8_t* p = q + qs_byte_off(W, row, wb + 4 * k);
        return (uint32_t)p[0] | ((uint32_t)p[1] << 8) | ((uint32_t)p[2] << 16) | ((uint32_t)p[3] << 24);
      };
      const uint32_t src = t < 12 ? word(t / 4) : (word(0) >> 24) | ((word(1) >> 24) << 8) | ((word(2) >> 24) << 16);
      const uint32_t u = (src >> (6 * (t % 4))) & 63u;
      const uint64_t hb = (uint64_t)ch * Q6_HDR_BYTES;
      if (W.type == T_Q5_K) {
        const uint32_t sb = (e % 128) / 32;
        const float sc = (float)c[sc_byte_off(W, row, hb + sb)], m = (float)c[sc_byte_off(W, row, hb + 4 + sb)];
        const uint8_t* dp = c + sc_byte_off(W, row, hb + 8);
        const float d = h2f(dp[0] | (dp[1] << 8)), dmin = h2f(dp[2] | (dp[3] << 8));
        return __fsub_rn(__fmul_rn(__fmul_rn(d, sc), (float)u), __fmul_rn(dmin, m));
      }
      const int v = (int)u - 32;
      const float sc = (float)(int8_t)c[sc_byte_off(W, row, hb + j)];
      const uint8_t* dp = c + sc_byte_off(W, row, hb + 8);
      const float d = h2f(dp[0] | (dp[1] << 8));
      return __fmul_rn(__fmul_rn(d, sc), (float)v);
    }
  }
  return 0.f;
}

constexpr int GEMV_THREADS = 256;
constexpr int GEMV_WARPS = GEMV_THREADS / 32;

// Block-wide sum of squares of x[0..n).  Threads 0..255 accumulate elements
// i, i+256, ... and warps 0..7 are summed in order, whatever the block size
// (NT >= 256, a multiple of 32), so every kernel that normalises the same vector
// produces bit-identical results.  sred holds at least 33 floats.
template <int NT>
__device__ __forceinline__ float block_sumsq_n(const float* __restrict__ x, int n, float* sred) {
  static_assert(NT >= GEMV_THREADS && NT % 32 == 0, "block too small");
  float s = 0.f;
  if (threadIdx.x < GEMV_THREADS)
    for (int i = threadIdx.x; i < n; i += GEMV_THREADS) {
      const float v = x[i];
      s = fmaf(v, v, s);
    }
#pragma unroll
  for (int o = 16; o; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
  if ((threadIdx.x & 31) == 0 && threadIdx.x < GEMV_THREADS) sred[threadIdx.x >> 5] = s;
  __syncthreads();
  if (threadIdx.x == 0) {
    float t = 0.f;
    for (int w = 0; w < GEMV_WARPS; w++) t += sred[w];
    sred[32] = t;
  }
  __syncthreads();
  const float r = sred[32];
  __syncthreads();
  return r;
}
__device__ __forceinline__ float block_sumsq(const float* __restrict__ x, int n, float* sred) {
  return block_sumsq_n<GEMV_THREADS>(x, n, sred);
}

// Block-wide sum of squares of x[0..n) (n a multiple of 4, x 16-byte aligned).
// x is read through L2, so it may have been written earlier by the same kernel.
// Thread t takes float4s t, t+NT, ... in order, then warps and warp partials are
// summed in a fixed order.  Up to four loads per thread are in flight at once.
template <int NT>
__device__ __forceinline__ float block_sumsq_v4(const float* __restrict__ x, int n, float* sred) {
  const float4* x4 = reinterpret_cast<const float4*>(x);
  const int nq = n / 4;
  float s = 0.f;
  for (int q0 = threadIdx.x; q0 < nq; q0 += 4 * NT) {
    float4 v[4];
#pragma unroll
    for (int u = 0; u < 4; u++) v[u] = q0 + u * NT < nq ? __ldcg(x4 + q0 + u * NT) : make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
    for (int u = 0; u < 4; u++) {
      s = fmaf(v[u].x, v[u].x, s);
      s = fmaf(v[u].y, v[u].y, s);
      s = fmaf(v[u].z, v[u].z, s);
      s = fmaf(v[u].w, v[u].w, s);
    }
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

// RMSNorm scale given the sum of squares: rms = sqrt(sum/n + eps), and the
// normalised element is x / rms * w   (compute.rs:312-317).
__device__ __forceinline__ float rms_of(float ss, int n, float eps) { return sqrtf(ss / (float)n + eps); }

inline int num_sms() {
  static int n = 0;
  if (!n) {
    int dev = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
    if (n <= 0) n = 148;
  }
  return n;
}

template <typename... KArgs, typename... Args>
inline cudaError_t launch_k(const Launch& L, void (*k)(KArgs...), dim3 grid, dim3 block, size_t smem,
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

}  // namespace rf
