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

#include "rf_attn.cuh"
#include "rf_attn_stream.cuh"
#include "rf_device.cuh"

namespace rf {

bool packed_geometry(int type, uint32_t M, uint32_t K, PackedMat* p) {
  if (expands_to_f32(type)) return false;  // stored as F32 (expand_rows_f32)
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
    case T_Q4_K:
    case T_Q3_K:
    case T_Q2_K: p->qs_stride = p->Kp / 2; break;
    case T_Q5_K:
    case T_Q6_K: p->qs_stride = (uint64_t)p->Kp / 128 * Q6_CHUNK_BYTES; break;
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
  if (six_bit_fields(W.type) || nibble_group_fields(W.type)) {
    // f16 d in the first two bytes of the 4-byte header plane (and Q5_K's or Q2_K's dmin after it)
    const bool two = W.type == T_Q5_K || W.type == T_Q2_K;
    for (uint32_t r = 0; r < W.Mp; r++)
      for (uint32_t c = 0; c < W.nk; c++) {
        const uint64_t o = sc_byte_off(W, r, (uint64_t)c * W.sbytes + (W.sbytes - 4));
        if (subnormal_half(sc[o], sc[o + 1])) return true;
        if (two && subnormal_half(sc[o + 2], sc[o + 3])) return true;
      }
    return false;
  }
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
      case T_Q6_K: {
        six_bit_pack_block(d, d.qs, d.sc, r, b, s);
        sub = subnormal_half(s[208], s[209]);
        break;
      }
      case T_Q5_K: {
        six_bit_pack_block(d, d.qs, d.sc, r, b, s);
        sub = subnormal_half(s[0], s[1]) || subnormal_half(s[2], s[3]);
        break;
      }
      case T_Q3_K: {
        nibble_group_pack_block(d, d.qs, d.sc, r, b, s);
        sub = subnormal_half(s[108], s[109]);
        break;
      }
      case T_Q2_K: {
        nibble_group_pack_block(d, d.qs, d.sc, r, b, s);
        sub = subnormal_half(s[80], s[81]) || subnormal_half(s[82], s[83]);
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
// embedding rows, parity dumps (dequant_elem, rf_device.cuh)
// ---------------------------------------------------------------------------
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

__global__ void embed_rows_kernel(PackedMat E, const uint32_t* __restrict__ tokens, float* __restrict__ x) {
  const uint32_t tok = min(tokens[blockIdx.x], E.M - 1);
  float* row = x + (size_t)blockIdx.x * E.K;
  for (uint32_t e = threadIdx.x; e < E.K; e += blockDim.x) row[e] = dequant_elem(E, tok, e);
}
cudaError_t launch_embed_rows(const Launch& L, const PackedMat& E, const uint32_t* tokens, uint32_t T, float* x) {
  if (T == 0) return cudaSuccess;
  return launch_k(L, embed_rows_kernel, dim3(T), dim3(256), 0, E, tokens, x);
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
// decode attention: split-K over context, GQA group per CTA (rf_attn.cuh)
// ---------------------------------------------------------------------------
size_t attn_part_floats(int batch, int n_kv_heads, int max_splits, int G, int hd) {
  return (size_t)batch * n_kv_heads * max_splits * G * (hd + 2);
}

// One unit per CTA: grid (KV heads, max_splits, batch).
template <int DPL, int G, typename KT>
__global__ void __launch_bounds__(ATT_THREADS) attn_kernel(AttnArgs a) {
  __shared__ __align__(16) float gsm[attn_group_floats<DPL, G>()];
  griddep_wait();
  attn_unit<DPL, G, KT>(a, blockIdx.x, blockIdx.y, blockIdx.z, gsm, 0);
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

// The streaming kernel (f16 cache, head_dim 32/64/128): as many splits as fill
// the CTAs that fit on the GPU at once (occupancy of this instance x SMs).
template <int G, int HD>
static cudaError_t attn_stream_launch(const Launch& L, const AttnArgs& a) {
  auto k = attn_stream_kernel<G, HD>;
  constexpr size_t smem = as_smem_bytes<G, HD>();
  cudaError_t e = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) return e;
  static int per_sm = 0;
  if (!per_sm) {
    int nb = 0;
    e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&nb, k, AS_THREADS, smem);
    if (e != cudaSuccess) return e;
    per_sm = nb > 0 ? nb : 1;
  }
  const int slots = per_sm * num_sms();
  const int units = a.n_kv_heads * a.batch;
  const int gy = std::max(1, std::min(a.max_splits, slots / std::max(1, units)));
  return launch_k(L, k, dim3(a.n_kv_heads, gy, a.batch), dim3(AS_THREADS), smem, a, slots);
}
template <int HD>
static cudaError_t attn_stream_g(const Launch& L, const AttnArgs& a, int G) {
  switch (G) {
    case 1: return attn_stream_launch<1, HD>(L, a);
    case 2: return attn_stream_launch<2, HD>(L, a);
    case 4: return attn_stream_launch<4, HD>(L, a);
    case 8: return attn_stream_launch<8, HD>(L, a);
    default: return cudaErrorInvalidValue;
  }
}

cudaError_t launch_attention(const Launch& L, const AttnArgs& a) {
  if (a.n_kv_heads <= 0 || a.n_heads % a.n_kv_heads) return cudaErrorInvalidValue;
  const int G = a.n_heads / a.n_kv_heads;
  // bulk copies need 16-byte aligned rows: an f16 cache whose base and strides are
  // multiples of 16 bytes
  const bool aligned = ((uintptr_t)a.kc % 16 == 0) && ((uintptr_t)a.vc % 16 == 0) && (a.head_stride * 2) % 16 == 0 &&
                       (a.batch_stride * 2) % 16 == 0;
  // Streaming pays from about a thousand positions: below that the unit is one
  // latency-bound pass either way, and inside the decode step the register kernel
  // measured faster (ctx ~530: 418 vs 411 tokens/s), while at 32768 positions the
  // streaming kernel takes half the time.  The engine's hint is its KV capacity
  // (the graph serves every context up to it); a standalone call's is its context.
  const int ctx_hint =
      a.d_nhist ? a.max_ctx : a.nhist + (a.batch - 1) * a.nhist_step + (a.k_cur ? 1 : 0);
  if (ctx_hint >= kAttnStreamMinCtx && !a.kv_f32 && aligned && (G == 1 || G == 2 || G == 4 || G == 8)) {
    if (a.head_dim == 128) return attn_stream_g<128>(L, a, G);
    if (a.head_dim == 64) return attn_stream_g<64>(L, a, G);
    if (a.head_dim == 32) return attn_stream_g<32>(L, a, G);
  }
  if (a.head_dim <= 32) return attn_dispatch_g<1>(L, a, G);
  if (a.head_dim <= 64) return attn_dispatch_g<2>(L, a, G);
  if (a.head_dim <= 128) return attn_dispatch_g<4>(L, a, G);
  return cudaErrorInvalidValue;
}

}  // namespace rf
