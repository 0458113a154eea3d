// rf_gemv.cu - standalone GEMV kernels and launchers of the decode engine
// (quantized matrices: the routine of rf_gemv.cuh over one kernel launch;
// F32/F16 matrices: a plain row-major kernel).
#include <algorithm>
#include <type_traits>

#include "rf_gemv.cuh"

namespace rf {

template <int FMT, bool QUIRK, class Epi, int NW>
__global__ void __launch_bounds__(NW * 32, QG_WARPS / NW)
    qgemv_kernel(PackedMat W, const float* __restrict__ x, const float* __restrict__ nw, float eps,
                 float* __restrict__ part, unsigned* __restrict__ cnt, Epi epi) {
  extern __shared__ __align__(16) float qsm[];
  qgemv_body<FMT, QUIRK, NW>(W, x, nw, eps, part, cnt, epi, qsm, [] { griddep_wait(); });
  epi.flush();
}
// The same with x pulled from a tensor-parallel sum (PeerLink::pull_site).
template <int FMT, bool QUIRK, class Epi, int NW>
__global__ void __launch_bounds__(NW * 32, QG_WARPS / NW)
    qgemv_pull_kernel(PackedMat W, const float* __restrict__ nw, float eps, float* __restrict__ part,
                      unsigned* __restrict__ cnt, Epi epi, PeerLink pl) {
  extern __shared__ __align__(16) float qsm[];
  qgemv_body<FMT, QUIRK, NW, true>(W, nullptr, nw, eps, part, cnt, epi, qsm, [] { griddep_wait(); }, &pl);
  epi.flush();
}
// Epilogues that follow a rank sum and may pull it (the normed products).
template <class Epi>
constexpr bool qgemv_can_pull() {
  return std::is_same<Epi, EpiRope>::value || std::is_same<Epi, EpiSwiGLU>::value;
}

// Warps per CTA: the QKV, W_o and down products run as two 8-warp CTAs per SM
// (the same warps a SM, half the warps behind each CTA barrier, and an SM frees
// half its slots for the next kernel as soon as one CTA ends), which measured
// faster in the single-GPU decode step; gate/up and the LM head measured faster
// as one 16-warp CTA per SM, and so did every product of a tensor-parallel step
// (Launch::wide), whose sums over ranks follow W_o and down.
template <class Epi>
constexpr bool qgemv_split_ctas() {
  return !(std::is_same<Epi, EpiSwiGLU>::value || std::is_same<Epi, EpiArgmax>::value);
}

constexpr size_t kMaxSmem = 227 * 1024;

// Whether a product runs as one 16-warp CTA per 64-row tile (run_qgemv_w).
template <class Epi>
static bool qgemv_tile_ctas(const PackedMat& W) {
  return std::is_same<Epi, EpiRope>::value && (W.Mp / QT_ROWS) * 2 >= (uint32_t)num_sms();
}

template <int FMT, class Epi, int NW>
static cudaError_t run_qgemv_w(const Launch& L, const PackedMat& W, const GemvScratch& ws, const float* x,
                               const float* nw, float eps, Epi epi, const PeerLink& pl) {
  int grid = num_sms() * (QG_WARPS / NW);
  // QKV + RoPE: one 16-warp CTA per 64-row tile when the tiles fill at least half the
  // SMs, so no tile is split across CTAs (no cross-CTA merge) and every CTA's RoPE
  // inputs are prefetched; measured +4 % on the single-GPU step (the other
  // products lost: W_o on 64 SMs no gain, W_down on 64 SMs 16.8 -> 23.9 us)
  const uint32_t ntiles = W.Mp / QT_ROWS;
  if (qgemv_tile_ctas<Epi>(W) && NW == QG_WARPS)
    grid = std::min<int>(grid, (int)ntiles);
  const size_t smem = qgemv_smem_bytes(W, grid, NW);
  if (smem > kMaxSmem) return cudaErrorInvalidValue;
  if (ws.part_floats < (uint64_t)W.Mp * W.nk * QT_PIECES || ws.n_cnt < W.Mp / QT_ROWS) return cudaErrorInvalidValue;
  if constexpr (qgemv_can_pull<Epi>()) {
    if (pl.pull_site >= 0) {
      auto k = W.sub_scales ? qgemv_pull_kernel<FMT, true, Epi, NW> : qgemv_pull_kernel<FMT, false, Epi, NW>;
      cudaError_t e = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
      if (e != cudaSuccess) return e;
      return launch_k(L, k, dim3(grid), dim3(NW * 32), smem, W, nw, eps, ws.part, ws.cnt, epi, pl);
    }
  }
  if (pl.pull_site >= 0) return cudaErrorInvalidValue;
  auto k = W.sub_scales ? qgemv_kernel<FMT, true, Epi, NW> : qgemv_kernel<FMT, false, Epi, NW>;
  cudaError_t e = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) return e;
  return launch_k(L, k, dim3(grid), dim3(NW * 32), smem, W, x, nw, eps, ws.part, ws.cnt, epi);
}

template <int FMT, class Epi>
static cudaError_t run_qgemv_t(const Launch& L, const PackedMat& W, const GemvScratch& ws, const float* x,
                               const float* nw, float eps, Epi epi, const PeerLink& pl) {
  if constexpr (qgemv_split_ctas<Epi>())
    if (!L.wide && !qgemv_tile_ctas<Epi>(W)) return run_qgemv_w<FMT, Epi, QG_WARPS / 2>(L, W, ws, x, nw, eps, epi, pl);
  return run_qgemv_w<FMT, Epi, QG_WARPS>(L, W, ws, x, nw, eps, epi, pl);
}

int gemv_ctas(const Launch& L, const PackedMat&, bool residual_epilogue) {
  const int nw = residual_epilogue && !L.wide ? QG_WARPS / 2 : QG_WARPS;
  return num_sms() * (QG_WARPS / nw);
}

void gemv_scratch_need(const PackedMat& W, uint64_t* part_floats, uint32_t* n_cnt) {
  if (is_tiled(W.type)) {
    *part_floats = (uint64_t)W.Mp * W.nk * QT_PIECES;
    *n_cnt = W.Mp / QT_ROWS;
  } else {
    *part_floats = 0;
    *n_cnt = 0;
  }
}

// ---------------------------------------------------------------------------
// F32 / F16 matrices (row-major): one warp per row, lanes over 16-byte pieces
// of the row, x read through L1.  These carry no quantization and no hot path
// of the benchmark models; they exist for GGUF files that store a matrix
// unquantized.
// ---------------------------------------------------------------------------
template <int FMT, class Epi>
__global__ void __launch_bounds__(GEMV_THREADS) fgemv_kernel(PackedMat W, const float* __restrict__ x,
                                                             const float* __restrict__ nw, float eps, Epi epi) {
  __shared__ float sred[40];
  griddep_wait();
  float rms = 1.f;
  if (nw) rms = rms_of(block_sumsq(x, (int)W.K, sred), (int)W.K, eps);
  griddep_launch();
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int rows = (int)W.M;
  // rows in pairs so pair epilogues see both values
  for (int r0 = 2 * (blockIdx.x * GEMV_WARPS + warp); r0 < rows; r0 += 2 * gridDim.x * GEMV_WARPS) {
    float acc[2] = {0.f, 0.f};
#pragma unroll
    for (int rr = 0; rr < 2; rr++) {
      const int r = min(r0 + rr, rows - 1);
      const uint8_t* q = W.qs + (size_t)r * W.qs_stride;
      float a = 0.f;
      for (uint32_t e = lane * 4; e < W.K; e += 128) {
        float wv[4];
        if (FMT == T_F32) {
          const float4 t = *reinterpret_cast<const float4*>(q + (size_t)e * 4);
          wv[0] = t.x; wv[1] = t.y; wv[2] = t.z; wv[3] = t.w;
        } else {
          const uint2 t = *reinterpret_cast<const uint2*>(q + (size_t)e * 2);
          wv[0] = h2f(t.x & 0xFFFFu); wv[1] = h2f(t.x >> 16); wv[2] = h2f(t.y & 0xFFFFu); wv[3] = h2f(t.y >> 16);
        }
#pragma unroll
        for (int k = 0; k < 4; k++) {
          const uint32_t ek = e + k;
          if (ek < W.K) {
            const float xv = nw ? x[ek] / rms * nw[ek] : x[ek];
            a = fmaf(wv[k], xv, a);
          }
        }
      }
#pragma unroll
      for (int o = 16; o; o >>= 1) a += __shfl_xor_sync(0xffffffffu, a, o);
      acc[rr] = a;
    }
    if (lane == 0) epi(r0, acc, min(2, rows - r0));
  }
  epi.flush();
}

template <int FMT, class Epi>
static cudaError_t run_fgemv_t(const Launch& L, const PackedMat& W, const float* x, const float* nw, float eps,
                               Epi epi) {
  const int pairs = (int)((W.M + 1) / 2);
  const int blocks = std::max(1, std::min((pairs + GEMV_WARPS - 1) / GEMV_WARPS, num_sms() * 4));
  return launch_k(L, fgemv_kernel<FMT, Epi>, dim3(blocks), dim3(GEMV_THREADS), 0, W, x, nw, eps, epi);
}

// `pl`: a peer sum this GEMV pulls x from or pushes its rows into (quantized
// matrices only; pulling needs the RMSNorm pass, which visits all of x).
template <class Epi>
static cudaError_t run_gemv(const Launch& L, const PackedMat& W, const GemvScratch* ws, const float* x,
                            const float* nw, float eps, Epi epi, const PeerLink& pl = PeerLink{}) {
  if (is_tiled(W.type) && !ws) return cudaErrorInvalidValue;
  if ((pl.pull_site >= 0 || pl.push_site >= 0) && !is_tiled(W.type)) return cudaErrorInvalidValue;
  if (pl.pull_site >= 0 && (!nw || !pl.hidden || W.K % 4 || W.K > (uint32_t)pl.P.n_max)) return cudaErrorInvalidValue;
  if (pl.push_site >= 0 && W.M > (uint32_t)pl.P.n_max) return cudaErrorInvalidValue;
  switch (W.type) {
    case T_Q4_K: return run_qgemv_t<T_Q4_K>(L, W, *ws, x, nw, eps, epi, pl);
    case T_Q4_0: return run_qgemv_t<T_Q4_0>(L, W, *ws, x, nw, eps, epi, pl);
    case T_Q8_0: return run_qgemv_t<T_Q8_0>(L, W, *ws, x, nw, eps, epi, pl);
    case T_Q6_K: return run_qgemv_t<T_Q6_K>(L, W, *ws, x, nw, eps, epi, pl);
    case T_Q5_K: return run_qgemv_t<T_Q5_K>(L, W, *ws, x, nw, eps, epi, pl);
    case T_Q3_K: return run_qgemv_t<T_Q3_K>(L, W, *ws, x, nw, eps, epi, pl);
    case T_Q2_K: return run_qgemv_t<T_Q2_K>(L, W, *ws, x, nw, eps, epi, pl);
    case T_F16: return run_fgemv_t<T_F16>(L, W, x, nw, eps, epi);
    case T_F32: return run_fgemv_t<T_F32>(L, W, x, nw, eps, epi);
    default: return cudaErrorInvalidValue;
  }
}

cudaError_t gemv_store(const Launch& L, const PackedMat& W, const GemvScratch* ws, const float* x, const float* nw,
                       float eps, float* y) {
  return run_gemv(L, W, ws, x, nw, eps, EpiStore{y});
}
cudaError_t gemv_residual(const Launch& L, const PackedMat& W, const GemvScratch* ws, const float* x,
                          const float* res, float* out) {
  return run_gemv(L, W, ws, x, nullptr, 0.f, EpiResidual{res, out});
}
cudaError_t gemv_qkv_rope(const Launch& L, const PackedMat& W, const GemvScratch* ws, const float* x,
                          const float* nw, float eps, const RopeQKVArgs& a, const PeerLink* pull) {
  return run_gemv(L, W, ws, x, nw, eps, EpiRope{a, -1}, pull ? *pull : PeerLink{});
}
cudaError_t gemv_swiglu(const Launch& L, const PackedMat& W, const GemvScratch* ws, const float* x, const float* nw,
                        float eps, float* act, const PeerLink* pull) {
  return run_gemv(L, W, ws, x, nw, eps, EpiSwiGLU{act}, pull ? *pull : PeerLink{});
}
cudaError_t gemv_peer_push(const Launch& L, const PackedMat& W, const GemvScratch* ws, const float* x,
                           const float* res, const PeerLink& pl) {
  if (pl.push_site < 0) return cudaErrorInvalidValue;
  return run_gemv(L, W, ws, x, nullptr, 0.f, EpiPeerPush{res, pl}, pl);
}
cudaError_t gemv_argmax(const Launch& L, const PackedMat& W, const GemvScratch* ws, const float* x, const float* nw,
                        float eps, float* logits, unsigned long long* key, uint32_t row_offset) {
  return run_gemv(L, W, ws, x, nw, eps, EpiArgmax{logits, key, row_offset, 0ull});
}

cudaError_t gemv_batched(cudaStream_t s, const PackedMat& W, const GemvScratch* ws, const float* x, int batch,
                         float* y) {
  // One pass per vector: batch-1 is what the engine runs; the standalone op
  // keeps the batched entry point for benchmark configuration 2.
  for (int b = 0; b < batch; b++) {
    cudaError_t e = run_gemv(Launch{s, false}, W, ws, x + (size_t)b * W.K, nullptr, 0.f, EpiStore{y + (size_t)b * W.M});
    if (e != cudaSuccess) return e;
  }
  return cudaSuccess;
}

}  // namespace rf
