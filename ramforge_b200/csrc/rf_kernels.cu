// rf_kernels.cu - sm_100a kernels of the decode engine other than the GEMV
// (rf_gemv.cu): weight packing, embedding lookup, RMSNorm, the decode-step
// bookkeeping kernels, KV reads and split-K GQA decode attention.
//
// Batch-1 decode attention is HBM-bound (each K/V byte is used for one
// multiply-add per query head of its group), so it uses no tensor cores.
// Reference arithmetic (crates/ramforge-core/src/compute.rs, quant.rs) is kept
// where it is cheap: exact per-element dequantisation for the embedding row,
// division-based RMSNorm, dot/sqrt(hd) scores and RoPE from a host-built
// cos/sin table evaluated with the same libm as the reference.
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <algorithm>

#include "rf_device.cuh"

namespace rf {

bool packed_geometry(int type, uint32_t M, uint32_t K, PackedMat* p) {
  if (!block_elems(type) || K == 0 || M == 0 || K % block_elems(type)) return false;
  p->type = type;
  p->M = M;
  p->K = K;
  p->Kp = padded_k(type, K);
  p->Mp = M;
  p->nk = 0;
  p->sbytes = 0;
  switch (type) {
    case T_F32: p->qs_stride = (uint64_t)p->Kp * 4; p->sc_stride = 0; break;
    case T_F16: p->qs_stride = (uint64_t)p->Kp * 2; p->sc_stride = 0; break;
    case T_Q8_0: p->qs_stride = p->Kp; break;
    case T_Q4_0:
    case T_Q4_K: p->qs_stride = p->Kp / 2; break;
  }
  if (is_tiled(type)) {
    p->Mp = (M + QT_ROWS - 1) / QT_ROWS * QT_ROWS;
    p->nk = p->Kp / (uint32_t)chunk_elems(type);
    p->sbytes = (uint32_t)chunk_scale_bytes(type);
    p->sc_stride = (uint64_t)p->nk * p->sbytes;
  }
  p->units = (uint32_t)(p->qs_stride / 32);
  p->qs = p->sc = nullptr;
  p->sub_scales = 0;
  return true;
}

// A block scale that the reference decodes differently from IEEE (h2f).
__host__ __device__ inline bool subnormal_half(uint32_t lo, uint32_t hi) {
  const uint32_t h = lo | (hi << 8);
  return (h & 0x7C00u) == 0 && (h & 0x03FFu) != 0;
}

bool has_subnormal_scales(const PackedMat& W, const uint8_t* sc) {
  if (!is_tiled(W.type)) return false;
  const uint64_t n = packed_sc_bytes(W);
  // f16 scales: Q8_0/Q4_0 every pair of bytes; Q4_K the first two pairs (d, dmin)
  // of each 16-byte header
  const uint64_t step = W.type == T_Q4_K ? 16 : 2, per = W.type == T_Q4_K ? 2 : 1;
  for (uint64_t o = 0; o < n; o += step)
    for (uint64_t k = 0; k < per; k++)
      if (subnormal_half(sc[o + 2 * k], sc[o + 2 * k + 1])) return true;
  return false;
}

// ---------------------------------------------------------------------------
// packing: GGUF rows -> PackedMat (pure byte shuffle)
// ---------------------------------------------------------------------------
__global__ void pack_kernel(const uint8_t* __restrict__ src, const int* __restrict__ src_row_of, PackedMat d,
                            uint32_t nblk, uint32_t bsz, uint64_t src_row_bytes, unsigned* flags) {
  const uint64_t total = (uint64_t)d.M * nblk;
  for (uint64_t t = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x; t < total;
       t += (uint64_t)gridDim.x * blockDim.x) {
    const uint32_t r = (uint32_t)(t / nblk), b = (uint32_t)(t % nblk);
    const uint32_t sr = src_row_of ? (uint32_t)src_row_of[r] : r;
    const uint8_t* s = src + sr * src_row_bytes + (uint64_t)b * bsz;
    bool sub = false;
    switch (d.type) {
      case T_F32:
      case T_F16: {
        uint8_t* q = d.qs + (uint64_t)r * d.qs_stride;
        for (uint32_t i = 0; i < bsz; i++) q[(uint64_t)b * bsz + i] = s[i];
        break;
      }
      case T_Q8_0: {
        uint8_t* c = d.sc + sc_byte_off(d, r, 2ull * b);
        c[0] = s[0]; c[1] = s[1];
        sub = subnormal_half(s[0], s[1]);
        uint8_t* q = d.qs + qs_byte_off(d, r, 32ull * b);
        for (int i = 0; i < 32; i++) q[i] = s[2 + i];
        break;
      }
      case T_Q4_0: {
        uint8_t* c = d.sc + sc_byte_off(d, r, 2ull * b);
        c[0] = s[0]; c[1] = s[1];
        sub = subnormal_half(s[0], s[1]);
        uint8_t* q = d.qs + qs_byte_off(d, r, 16ull * b);
        for (int i = 0; i < 16; i++) q[i] = s[2 + i];
        break;
      }
      case T_Q4_K: {
        uint8_t* c = d.sc + sc_byte_off(d, r, 16ull * b);
        for (int i = 0; i < 16; i++) c[i] = s[i];
        sub = subnormal_half(s[0], s[1]) || subnormal_half(s[2], s[3]);
        for (int p = 0; p < 4; p++) {
          uint8_t* q = d.qs + qs_byte_off(d, r, 128ull * b + 32 * p);
          for (int i = 0; i < 32; i++) q[i] = s[16 + 32 * p + i];
        }
        break;
      }
    }
    if (sub && flags) atomicOr(flags, 1u);
  }
}

cudaError_t launch_pack(const uint8_t* gguf, const int* src_row_of, PackedMat dst, unsigned* flags, cudaStream_t s) {
  const uint32_t nblk = dst.K / block_elems(dst.type), bsz = block_bytes(dst.type);
  const uint64_t row_bytes = (uint64_t)nblk * bsz;
  cudaError_t e = cudaMemsetAsync(dst.qs, 0, packed_qs_bytes(dst), s);
  if (e == cudaSuccess && dst.sc_stride) e = cudaMemsetAsync(dst.sc, 0, packed_sc_bytes(dst), s);
  if (e == cudaSuccess && flags) e = cudaMemsetAsync(flags, 0, sizeof(unsigned), s);
  if (e != cudaSuccess) return e;
  const uint64_t total = (uint64_t)dst.M * nblk;
  const int blocks = (int)std::min<uint64_t>((total + 255) / 256, 65535ull * 8);
  pack_kernel<<<blocks, 256, 0, s>>>(gguf, src_row_of, dst, nblk, bsz, row_bytes, flags);
  return cudaGetLastError();
}

// ---------------------------------------------------------------------------
// element-exact dequantisation (embedding rows, parity dumps)
// ---------------------------------------------------------------------------
__device__ float dequant_elem(const PackedMat& W, uint32_t row, uint32_t e) {
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
