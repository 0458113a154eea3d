// rf_step.cu - the whole decode step as one persistent kernel.
//
// A token step of the executor (model_executor.rs:147-233 per layer, then
// compute_logits + greedy sampling, streaming_model.rs:1334, sampling.rs:40) is
// a chain of ~160 dependent operations, each of which streams one weight matrix
// or one layer's KV history.  Launched as separate kernels, every link pays a
// launch ramp, a tail where SMs drain, and a serial first-load latency.  Here one
// CTA per SM (all co-resident: cooperative launch) runs every phase of the step
// in order, with a grid-wide barrier between dependent phases.  A GEMV phase
// loads its first weights before waiting at its barrier (weights never depend on
// the previous phase), so the barrier and the previous phase's tail overlap the
// HBM latency.  Split-K merges inside a phase need no barrier (the last arrival
// finishes a tile or an attention head).
//
// Barriers count arrivals in one global word; each CTA waits, bounded by
// kBarrierSpin cycles, for the count of its barrier generation.  On expiry it
// sets err bit 0 and every later barrier stops waiting, so the kernel always
// ends; the host reports the step as failed.
#include <algorithm>

#include "rf_attn.cuh"
#include "rf_gemv.cuh"

namespace rf {

constexpr long long kBarrierSpin = 2000000000LL;  // about 1 s at 1.9 GHz
constexpr int STEP_GROUPS = QG_THREADS / ATT_THREADS;  // attention groups per CTA

__device__ __forceinline__ unsigned ld_acquire(const unsigned* p) {
  unsigned v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

__device__ __forceinline__ unsigned long long global_ns() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// With `stamps`, CTA 0 records the time each barrier completes (entry k for
// barrier k; entry 0 is the kernel start, written by the caller).
__device__ __forceinline__ void grid_barrier(unsigned* bar, unsigned* err, unsigned& target,
                                             unsigned long long* stamps = nullptr) {
  __syncthreads();
  target += gridDim.x;
  if (threadIdx.x == 0) {
    __threadfence();
    atomicAdd(bar, 1u);
    if (ld_acquire(bar) < target && !(ld_acquire(err) & 1u)) {
      const long long t0 = clock64();
      while (ld_acquire(bar) < target) {
        if (clock64() - t0 > kBarrierSpin) {
          atomicOr(err, 1u);
          break;
        }
      }
    }
    __threadfence();
    if (stamps && blockIdx.x == 0) stamps[target / gridDim.x] = global_ns();
  }
  __syncthreads();
}

// Epilogue of the four layer GEMVs, chosen per phase (one inlined GEMV body
// serves all four, which keeps the kernel's register allocation close to the
// standalone GEMV's).
struct EpiLayer {
  static constexpr bool kPre = false;
  int kind;                 // 0: RoPE + K/V append, 1: residual add into out, 2: SwiGLU into out
  const RopeQKVArgs* rope;  // kind 0
  float* out;
  __device__ void pre_begin() {}
  __device__ float pre_load(uint32_t) { return 0.f; }
  __device__ void operator()(int row0, const float* v, int n, const float* = nullptr) {
    if (kind == 0) {
      rope_store(*rope, row0, v, n);
    } else if (kind == 1) {  // out = out + W.x  (model_executor.rs:213-215, 231-233)
      for (int i = 0; i < n; i++) out[row0 + i] = __ldcg(out + row0 + i) + v[i];
    } else {
      EpiSwiGLU{out}(row0, v, n);
    }
  }
  __device__ void flush() {}
};

template <int DPL, int G>
__device__ __forceinline__ void attention_phase(const AttnArgs& aa, const StepArgs& a, float* sm) {
  const int nsplit = attn_nsplit(__ldcg(a.d_pos) + 1, a.max_splits);
  const int units = (int)a.n_kv_heads * nsplit;
  const int gid = threadIdx.x / ATT_THREADS;
  float* gsm = sm + gid * attn_group_floats<DPL, G>();
  // unit u runs on CTA u % grid first, so units spread over all SMs before any
  // SM takes a second one
  for (int u = gid * gridDim.x + blockIdx.x; u < units; u += gridDim.x * STEP_GROUPS)
    attn_unit<DPL, G, __half, 8>(aa, u / nsplit, u % nsplit, 0, gsm, gid);  // 128 registers a thread
}

template <int FL, int FO, int DPL, int G>
__global__ void __launch_bounds__(QG_THREADS, 1) step_kernel(const __grid_constant__ StepArgs a) {
  extern __shared__ __align__(16) float sm[];
  unsigned target = 0;
  auto sync = [&] { grid_barrier(a.bar, a.err, target, a.stamps); };
  const uint32_t gtid = blockIdx.x * QG_THREADS + threadIdx.x, nthreads = gridDim.x * QG_THREADS;
  if (a.stamps && gtid == 0) a.stamps[0] = global_ns();

  // embedding row of the step's token (get_embedding, tensor.rs:706-714)
  {
    const uint32_t tok = min(__ldcg(a.d_token), a.embd.M - 1);
    for (uint32_t e = gtid; e < a.n_embd; e += nthreads) a.hidden[e] = dequant_elem(a.embd, tok, e);
    if (gtid == 0 && a.decode) *a.key = 0ull;
  }
  // phase p of the layers: layer p/5, step p%5 =
  //   0 RMSNorm(attn_norm) -> [Q;K;V] -> RoPE, K/V append   1 attention
  //   2 Wo + residual   3 RMSNorm(ffn_norm) -> [gate_j; up_j] -> SwiGLU   4 down + residual
#pragma unroll 1
  for (int p = 0; p < 5 * a.n_layers; p++) {
    const int l = p / 5, k = p % 5;
    const StepLayer& L = a.layers[l];
    if (k == 1) {
      sync();
      attention_phase<DPL, G>(L.attn, a, sm);
      continue;
    }
    const PackedMat& W = k == 0 ? L.qkv : k == 2 ? L.wo : k == 3 ? L.gateup : L.down;
    const float* x = k == 0 || k == 3 ? a.hidden : k == 2 ? a.att : a.act;
    const float* nw = k == 0 ? L.attn_norm : k == 3 ? L.ffn_norm : nullptr;
    EpiLayer ep{k == 0 ? 0 : k == 3 ? 2 : 1, &L.rope, k == 3 ? a.act : a.hidden};
    qgemv_body<FL, false>(W, x, nw, a.eps, a.gws.part, a.gws.cnt, ep, sm, sync);
  }
  if (a.decode) {
    // RMSNorm(output_norm) -> LM head -> greedy argmax key, then advance
    EpiArgmax ea{a.logits, a.key, a.vocab_off, 0ull};
    qgemv_body<FO, false>(a.lm, a.hidden, a.out_norm, a.eps, a.gws.part, a.gws.cnt, ea, sm, sync);
    ea.flush();
    sync();
    if (gtid == 0) {
      const unsigned long long k = __ldcg(a.key);
      const uint32_t tok = ~(uint32_t)(k & 0xFFFFFFFFull);
      const int p = __ldcg(a.d_pos);
      *a.d_token = tok;
      if (a.hist && p >= 0 && p < a.hist_len) a.hist[p] = tok;
      *a.d_pos = p + 1;
    }
  } else {
    sync();
    if (blockIdx.x == 0) {  // final_hidden = RMSNorm(hidden) (rms_norm_reference, compute.rs:291-319)
      float* sred = sm;
      const float rms = rms_of(block_sumsq_v4<QG_THREADS>(a.hidden, (int)a.n_embd, sred), (int)a.n_embd, a.eps);
      for (uint32_t e = threadIdx.x; e < a.n_embd; e += QG_THREADS)
        a.final_hidden[e] = __ldcg(a.hidden + e) / rms * a.out_norm[e];
    }
  }
}

// Check of the barrier's bounded wait: one barrier whose target also counts
// `phantom` arrivals that never come.  With phantom > 0 every CTA gives up after
// kBarrierSpin cycles, sets err bit 0 and returns.
__global__ void barrier_selftest_kernel(unsigned* bar, unsigned* err, unsigned phantom) {
  unsigned target = phantom;
  grid_barrier(bar, err, target);
}

cudaError_t barrier_selftest(unsigned phantom, unsigned* err_out) {
  unsigned* w = nullptr;
  cudaError_t e = cudaMalloc(&w, 2 * sizeof(unsigned));
  if (e != cudaSuccess) return e;
  e = cudaMemset(w, 0, 2 * sizeof(unsigned));
  if (e == cudaSuccess) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(num_sms());
    cfg.blockDim = dim3(32);
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeCooperative;
    attr[0].val.cooperative = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    e = cudaLaunchKernelEx(&cfg, barrier_selftest_kernel, w, w + 1, phantom);
  }
  if (e == cudaSuccess) e = cudaDeviceSynchronize();
  if (e == cudaSuccess) e = cudaMemcpy(err_out, w + 1, sizeof(unsigned), cudaMemcpyDeviceToHost);
  cudaFree(w);
  return e;
}

namespace {
using StepKernel = void (*)(StepArgs);

// Instances: the benchmark models (Llama-3-8B: Q4_K layers, Q8_0 LM head, head_dim
// 128, 4 query heads per KV head; Llama-3-70B: Q4_K everywhere, 8 per KV head;
// TinyLlama: Q8_0, head_dim 64, 8 per KV head) and the Q8_0 / head_dim 128 / 4
// per KV head shape of the small test models.
StepKernel pick(int fl, int fo, int dpl, int g) {
  if (fl == T_Q4_K && fo == T_Q8_0 && dpl == 4 && g == 4) return step_kernel<T_Q4_K, T_Q8_0, 4, 4>;
  if (fl == T_Q4_K && fo == T_Q4_K && dpl == 4 && g == 8) return step_kernel<T_Q4_K, T_Q4_K, 4, 8>;
  if (fl == T_Q8_0 && fo == T_Q8_0 && dpl == 2 && g == 8) return step_kernel<T_Q8_0, T_Q8_0, 2, 8>;
  if (fl == T_Q8_0 && fo == T_Q8_0 && dpl == 4 && g == 4) return step_kernel<T_Q8_0, T_Q8_0, 4, 4>;
  return nullptr;
}

int dpl_of(uint32_t hd) { return hd == 128 ? 4 : hd == 64 ? 2 : 0; }

StepKernel kernel_for(const StepArgs& a, const StepLayer& l0) {
  const int fl = l0.qkv.type;
  if (l0.wo.type != fl || l0.gateup.type != fl || l0.down.type != fl) return nullptr;
  if (l0.qkv.sub_scales || l0.wo.sub_scales || l0.gateup.sub_scales || l0.down.sub_scales || a.lm.sub_scales)
    return nullptr;
  if (a.n_kv_heads == 0 || a.n_heads % a.n_kv_heads) return nullptr;
  return pick(fl, a.lm.type, dpl_of(a.head_dim), (int)(a.n_heads / a.n_kv_heads));
}
}  // namespace

size_t step_kernel_smem(const StepArgs& a, const StepLayer& l0) {
  const StepKernel k = kernel_for(a, l0);
  if (!k) return 0;
  const int grid = num_sms();
  size_t s = std::max({qgemv_smem_bytes(l0.qkv, grid), qgemv_smem_bytes(l0.wo, grid),
                       qgemv_smem_bytes(l0.gateup, grid), qgemv_smem_bytes(l0.down, grid),
                       qgemv_smem_bytes(a.lm, grid), (size_t)(QG_THREADS / 32 + 1) * 4 * sizeof(float)});
  const int G = (int)(a.n_heads / a.n_kv_heads);
  const size_t att = (size_t)STEP_GROUPS * sizeof(float) *
                     (dpl_of(a.head_dim) == 4 ? (G == 4 ? attn_group_floats<4, 4>() : attn_group_floats<4, 8>())
                                              : (G == 4 ? attn_group_floats<2, 4>() : attn_group_floats<2, 8>()));
  s = std::max(s, att);
  if (s > 227 * 1024) return 0;
  if (cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)s) != cudaSuccess) return 0;
  int per_sm = 0;
  if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, k, QG_THREADS, s) != cudaSuccess || per_sm < 1) return 0;
  return s;
}

cudaError_t launch_step_kernel(cudaStream_t s, const StepArgs& a, const StepLayer& l0, size_t smem) {
  const StepKernel k = kernel_for(a, l0);
  if (!k || !smem) return cudaErrorInvalidValue;
  cudaError_t e = cudaMemsetAsync(a.bar, 0, sizeof(unsigned), s);
  if (e != cudaSuccess) return e;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(num_sms());
  cfg.blockDim = dim3(QG_THREADS);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeCooperative;
  attr[0].val.cooperative = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, k, a);
}

}  // namespace rf
