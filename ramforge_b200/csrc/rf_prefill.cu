// rf_prefill.cu - batched prompt processing on the tensor cores (tcgen05).
//
// The reference forwards a prompt one token at a time (inference.rs:578-592), so
// every layer's weights are streamed once per prompt token.  Here a prompt of T
// tokens goes through each layer as four GEMMs (Q/K/V, W_o, gate/up, down) whose
// B operand is the T tokens' activations, on the 5th-generation tensor cores:
//
//  * A CTA owns 128 weight rows (two 64-row tiles of the packed layout) and
//    PG_N tokens; its f32 accumulator D[128 x PG_N] lives in tensor memory.
//  * K advances 64 elements a step.  All 8 warps dequantize the step's weights
//    (Q4_K or Q8_0, the reference's exact f32 value) into shared memory in the
//    K-major canonical layout, each value split into bf16 hi + lo; the step's
//    activations, split the same way by prefill_split_kernel and stored tiled,
//    arrive by one cp.async.bulk on an mbarrier.
//  * One thread issues, per 16-element substep, hi*hi + hi*lo + lo*hi into D
//    (tcgen05.mma kind::f16), then tcgen05.commit frees the stage: a 3-stage
//    ring, so the dequantization of later steps overlaps the MMAs.
//  * The split keeps about 16 significant bits of each operand (relative error
//    near 2^-16 per product against the f32 reference), enough for the greedy
//    tokens after a prompt to match the token-by-token reference.
//  * Epilogue: tcgen05.ld of D, one row per thread, 32 tokens per load; the
//    epilogue functor gets (row, token, value, value of the row's pair partner).
// Every mbarrier wait is bounded (about a second); on expiry the kernel records
// bit 0 of its error word, waits (bounded) for its own copies and MMAs, frees
// its tensor memory and returns.
#include <cuda_bf16.h>

#include "rf_attn.cuh"
#include "rf_gemv.cuh"
#include "rf_tc.cuh"

namespace rf {

constexpr int PG_M = 128;     // weight rows per CTA
constexpr int PG_N = 128;     // tokens per CTA (tensor-memory columns)
constexpr int PG_KS = 64;     // K elements per step
constexpr int PG_STAGES = 3;  // shared-memory ring depth
constexpr int PG_THREADS = 256;
constexpr uint32_t PG_A_BYTES = PG_M * PG_KS * 2;     // one of A hi / A lo (bf16)
constexpr uint32_t PG_B_BYTES = PG_N * PG_KS * 2;     // one of B hi / B lo
constexpr uint32_t PG_STAGE_BYTES = 2 * PG_A_BYTES + 2 * PG_B_BYTES;

// Element offset of (row or token r, k) inside one canonical K-major operand
// block of `rows` rows and PG_KS columns: 8-element K chunks are the slowest
// index, then rows, then the 8 elements (one 16-byte core-matrix row).
__host__ __device__ inline uint32_t pg_canon(uint32_t rows, uint32_t r, uint32_t k) {
  return (k / 8) * rows * 8 + r * 8 + k % 8;
}

// ---------------------------------------------------------------------------
// Activations -> tiled bf16 hi/lo.  X is [T][K] f32 (row stride ldx); with nw
// each token row is RMS-normalised first, x / rms * w with rms = sqrt(sum/K +
// eps) (rms_norm_reference, compute.rs:312-317).  Xt holds, for token block nb
// and K step ks, the 2 * PG_B_BYTES block [hi | lo] at ((nb * nks) + ks) blocks
// (nks = Kp / 64, Kp the matrix's padded row length); tokens >= T and elements
// >= K are zero.  One CTA per token row of the padded token count.
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(256) prefill_split_kernel(const float* __restrict__ X, uint32_t ldx, uint32_t T,
                                                            uint32_t K, uint32_t Kp, const float* __restrict__ nw,
                                                            float eps, __nv_bfloat16* __restrict__ Xt) {
  __shared__ float sred[40];
  const uint32_t t = blockIdx.x, nb = t / PG_N, n = t % PG_N, nks = Kp / PG_KS;
  const float* x = X + (size_t)t * ldx;
  const bool live = t < T;
  griddep_wait();
  float rms = 1.f;
  if (nw && live) rms = rms_of(block_sumsq(x, (int)K, sred), (int)K, eps);
  for (uint32_t k = threadIdx.x; k < Kp; k += blockDim.x) {  // elements K..Kp-1 (row padding) are 0
    float v = 0.f;
    if (live && k < K) v = nw ? x[k] / rms * nw[k] : x[k];
    const __nv_bfloat16 hi = __float2bfloat16_rn(v);
    const __nv_bfloat16 lo = __float2bfloat16_rn(v - __bfloat162float(hi));
    const uint32_t ks = k / PG_KS, kk = k % PG_KS;
    __nv_bfloat16* blk = Xt + ((size_t)nb * nks + ks) * (2 * PG_N * PG_KS);
    const uint32_t o = pg_canon(PG_N, n, kk);
    blk[o] = hi;
    blk[PG_N * PG_KS + o] = lo;
  }
}

// ---------------------------------------------------------------------------
// Weights of one K step -> shared memory, in two parts so that the next step's
// loads are in flight while this step is converted.  Thread t handles half a
// row's step: row r = t / 2 of the CTA's 128, 32 of the step's 64 elements.
// pg_load fetches the raw words (quant bytes and scales), pg_dequant_step
// applies the reference's decode (Q4_K: (d*sc)*q - dmin*m, quant.rs:228-254;
// Q8_0: q*d, quant.rs:176-180) and stores hi and lo into the canonical A blocks.
// ---------------------------------------------------------------------------
struct PgRaw {
  uint4 q0, q1;  // Q4_K: q0 = 16 quant bytes, q1 = the row's 16-byte header; Q8_0: the 32 quant bytes
  uint32_t d;    // Q8_0: the block's f16 scale bits
};

template <int FMT>
__device__ __forceinline__ PgRaw pg_load(const PackedMat& W, uint32_t m0, uint32_t ks) {
  const uint32_t r = threadIdx.x >> 1, h = threadIdx.x & 1;
  const uint32_t row = m0 + r;  // rows past W.Mp (the last 64-row tile) are zero rows
  const uint32_t tile = row / QT_ROWS, lr = row % QT_ROWS;
  PgRaw raw{};
  if (row >= W.Mp) return raw;
  if constexpr (FMT == T_Q4_K) {
    // step ks = chunk ks/4, piece c = ks%4: bytes 32c.. of the super-block; byte l
    // holds element 64c + l (low nibble) and 64c + 32 + l (high nibble)
    const uint32_t kc = ks / 4, c = ks % 4;
    const uint64_t item = (uint64_t)tile * W.nk + kc;
    raw.q0 = *reinterpret_cast<const uint4*>(W.qs + (item * 4 + c) * (QT_ROWS * 32) + lr * 32 + 16 * h);
    raw.q1 = *reinterpret_cast<const uint4*>(W.sc + (item * QT_ROWS + lr) * 16);
  } else {  // Q8_0: step ks = pieces 2(ks%2), 2(ks%2)+1 of chunk ks/2 (one 32-element block each)
    const uint32_t kc = ks / 2, blk = 2 * (ks % 2) + h;
    const uint64_t item = (uint64_t)tile * W.nk + kc;
    const uint8_t* qp = W.qs + (item * 4 + blk) * (QT_ROWS * 32) + lr * 32;
    raw.q0 = *reinterpret_cast<const uint4*>(qp);
    raw.q1 = *reinterpret_cast<const uint4*>(qp + 16);
    raw.d = *reinterpret_cast<const uint16_t*>(W.sc + (item * QT_ROWS + lr) * 8 + 2 * blk);
  }
  return raw;
}

// Scale and min j (0..7) of a Q4_K row header held in registers (hw.y, hw.z, hw.w
// = the 12 packed scale bytes): the fields k4_scale_min reads, taken by shifts so
// that the header never leaves registers.
__device__ __forceinline__ void k4_scale_min_w(const uint4& hw, uint32_t j, uint32_t* sc, uint32_t* m) {
  const uint32_t sh = 8 * (j & 3u);
  const uint32_t by = (hw.y >> sh) & 0xFFu, bz = (hw.z >> sh) & 0xFFu, bw = (hw.w >> sh) & 0xFFu;
  if (j < 4) {
    *sc = by & 63u;
    *m = bz & 63u;
  } else {
    *sc = (bw & 0xFu) | ((by >> 6) << 4);
    *m = (bw >> 4) | ((bz >> 6) << 4);
  }
}

template <int FMT>
__device__ __forceinline__ void pg_dequant_step(const PackedMat& W, uint32_t m0, uint32_t ks, const PgRaw& raw,
                                                __nv_bfloat16* a_hi, __nv_bfloat16* a_lo) {
  const uint32_t r = threadIdx.x >> 1, h = threadIdx.x & 1;
  const uint32_t row = m0 + r;
  float v[32];  // elements this thread produces, at step offsets kidx[]
  uint32_t kidx[32];
  if (row >= W.Mp) {  // past the last 64-row tile: zero rows
#pragma unroll
    for (int i = 0; i < 32; i++) {
      v[i] = 0.f;
      kidx[i] = 32 * h + i;
    }
  } else if constexpr (FMT == T_Q4_K) {
    const uint32_t c = ks % 4;
    const float d = h2f(raw.q1.x & 0xFFFFu), dmin = h2f(raw.q1.x >> 16);
    uint32_t sc0, m0v, sc1, m1v;
    k4_scale_min_w(raw.q1, 2 * c, &sc0, &m0v);
    k4_scale_min_w(raw.q1, 2 * c + 1, &sc1, &m1v);
    const float d0 = __fmul_rn(d, (float)sc0), mn0 = __fmul_rn(dmin, (float)m0v);
    const float d1 = __fmul_rn(d, (float)sc1), mn1 = __fmul_rn(dmin, (float)m1v);
    const uint32_t w[4] = {raw.q0.x, raw.q0.y, raw.q0.z, raw.q0.w};
#pragma unroll
    for (int i = 0; i < 16; i++) {
      const uint32_t byte = (w[i / 4] >> (8 * (i % 4))) & 0xFFu;
      v[i] = __fsub_rn(__fmul_rn(d0, (float)(byte & 15u)), mn0);
      kidx[i] = 16 * h + i;
      v[16 + i] = __fsub_rn(__fmul_rn(d1, (float)(byte >> 4)), mn1);
      kidx[16 + i] = 32 + 16 * h + i;
    }
  } else {  // Q8_0
    const float d = h2f(raw.d);
    const uint32_t w[8] = {raw.q0.x, raw.q0.y, raw.q0.z, raw.q0.w, raw.q1.x, raw.q1.y, raw.q1.z, raw.q1.w};
#pragma unroll
    for (int i = 0; i < 32; i++) {
      const int8_t qv = (int8_t)((w[i / 4] >> (8 * (i % 4))) & 0xFFu);
      v[i] = __fmul_rn((float)qv, d);
      kidx[i] = 32 * h + i;
    }
  }
#pragma unroll
  for (int g = 0; g < 4; g++) {  // four 8-element runs, one 16-byte store each for hi and lo
    __align__(16) __nv_bfloat16 hi[8], lo[8];
#pragma unroll
    for (int i = 0; i < 8; i++) {
      hi[i] = __float2bfloat16_rn(v[8 * g + i]);
      lo[i] = __float2bfloat16_rn(v[8 * g + i] - __bfloat162float(hi[i]));
    }
    const uint32_t o = pg_canon(PG_M, r, kidx[8 * g]);
    *reinterpret_cast<uint4*>(a_hi + o) = *reinterpret_cast<const uint4*>(hi);
    *reinterpret_cast<uint4*>(a_lo + o) = *reinterpret_cast<const uint4*>(lo);
  }
}

// ---------------------------------------------------------------------------
// The GEMM: D[row][t] = sum_k W[row][k] * X[t][k] for the CTA's 128 rows (m0 =
// blockIdx.x * 128) and PG_N tokens (block blockIdx.y), K = W.Kp, or half of K
// when gridDim.z == 2 (CTA z takes the steps [z*nks/2, (z+1)*nks/2); the pair
// meets through kpart / kcnt, below).  Xt is the tiled hi/lo activation buffer
// of prefill_split_kernel for K = W.Kp.
// Shared memory: PG_STAGES x [A hi | A lo | B hi | B lo], then the barriers, the
// tensor-memory address and the K-split pair's last-arrival flag.
// ---------------------------------------------------------------------------
constexpr size_t PG_SMEM = (size_t)PG_STAGES * PG_STAGE_BYTES + 128;

template <int FMT, class Epi>
__global__ void __launch_bounds__(PG_THREADS, 1)
    prefill_gemm_kernel(PackedMat W, const __nv_bfloat16* __restrict__ Xt, uint32_t T, unsigned* err, Epi epi,
                        float* __restrict__ kpart, unsigned* __restrict__ kcnt) {
  extern __shared__ __align__(1024) uint8_t psm[];
  uint64_t* bars = reinterpret_cast<uint64_t*>(psm + (size_t)PG_STAGES * PG_STAGE_BYTES);  // x_full[S], mma_done[S]
  uint32_t* tslot = reinterpret_cast<uint32_t*>(bars + 2 * PG_STAGES);
  int* s_last = reinterpret_cast<int*>(tslot + 1);
  const uint32_t tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const uint32_t m0 = blockIdx.x * PG_M, nb = blockIdx.y;
  // K split over gridDim.z CTAs (1 or 2): this CTA's steps [kb, ke) of the Kp / 64
  const uint32_t nks_all = W.Kp / PG_KS, kz = blockIdx.z, nz = gridDim.z;
  const uint32_t kb = (uint32_t)((uint64_t)nks_all * kz / nz), ke = (uint32_t)((uint64_t)nks_all * (kz + 1) / nz);
  const uint32_t nks = ke - kb;
  auto stage = [&](uint32_t s) { return psm + (size_t)s * PG_STAGE_BYTES; };
  auto x_full = [&](uint32_t s) { return tc_smem_u32(bars + s); };
  auto mma_done = [&](uint32_t s) { return tc_smem_u32(bars + PG_STAGES + s); };

  if (warp == 0) tc_tmem_alloc(tc_smem_u32(tslot), PG_N);
  if (tid == 0) {
    for (int s = 0; s < PG_STAGES; s++) {
      tc_mbar_init(x_full(s), 1);
      tc_mbar_init(mma_done(s), 1);
    }
    tc_fence_barrier_init();
  }
  tc_fence_before_sync();
  __syncthreads();
  tc_fence_after_sync();
  const uint32_t tmem = *tslot;
  // the first step's weight words (no earlier kernel writes weights), then the
  // wait: the activations this kernel reads were written by the previous kernel
  PgRaw nxt = nks > 0 ? pg_load<FMT>(W, m0, kb) : PgRaw{};
  griddep_wait();

  constexpr uint32_t idesc = tc_idesc_bf16_f32(PG_M, PG_N);
  uint32_t n_x[PG_STAGES] = {0, 0, 0}, n_m[PG_STAGES] = {0, 0, 0};  // copies / commits issued (thread 0)
  bool bad = false;
  for (uint32_t ks = 0; ks < nks; ks++) {
    const uint32_t s = ks % PG_STAGES, use = ks / PG_STAGES;
    uint8_t* st = stage(s);
    // the stage is free once the MMAs of step ks - PG_STAGES have completed
    if (use > 0 && !bad && !tc_mbar_wait(mma_done(s), (use - 1) & 1)) bad = true;
    if (__syncthreads_or(bad)) {
      bad = true;
      break;
    }
    if (tid == 0) {
      tc_bulk_g2s(tc_smem_u32(st + 2 * PG_A_BYTES), Xt + ((size_t)nb * nks_all + kb + ks) * (2 * PG_N * PG_KS),
                  2 * PG_B_BYTES, x_full(s));
      n_x[s]++;
    }
    // this step's weight words arrived during the previous step; request the next
    // step's before converting these
    const PgRaw cur = nxt;
    if (ks + 1 < nks) nxt = pg_load<FMT>(W, m0, kb + ks + 1);
    pg_dequant_step<FMT>(W, m0, kb + ks, cur, reinterpret_cast<__nv_bfloat16*>(st),
                         reinterpret_cast<__nv_bfloat16*>(st + PG_A_BYTES));
    tc_fence_proxy_async();  // this thread's A stores, before the MMAs read them
    __syncthreads();
    if (tid == 0) {
      if (!tc_mbar_wait(x_full(s), use & 1)) {
        bad = true;
      } else {
        tc_fence_after_sync();
        const uint32_t a_hi = tc_smem_u32(st), a_lo = a_hi + PG_A_BYTES;
        const uint32_t b_hi = a_hi + 2 * PG_A_BYTES, b_lo = b_hi + PG_B_BYTES;
#pragma unroll
        for (uint32_t kk = 0; kk < PG_KS; kk += 16) {
          // K-major no-swizzle operands: 8-element K chunks PG_M*16 (A) or
          // PG_N*16 (B) bytes apart, 8-row groups 128 bytes apart
          const uint32_t ao = (kk / 8) * PG_M * 16, bo = (kk / 8) * PG_N * 16;
          const uint64_t ah = tc_smem_desc(a_hi + ao, PG_M * 16, 128), al = tc_smem_desc(a_lo + ao, PG_M * 16, 128);
          const uint64_t bh = tc_smem_desc(b_hi + bo, PG_N * 16, 128), bl = tc_smem_desc(b_lo + bo, PG_N * 16, 128);
          tc_mma_bf16(tmem, ah, bh, idesc, ks > 0 || kk > 0);
          tc_mma_bf16(tmem, ah, bl, idesc, true);
          tc_mma_bf16(tmem, al, bh, idesc, true);
        }
        tc_commit(mma_done(s));
        n_m[s]++;
      }
    }
  }
  // every MMA done (they complete in order: the last commit covers them all)
  if (!bad && nks > 0) {
    const uint32_t L = nks - 1;
    if (!tc_mbar_wait(mma_done(L % PG_STAGES), (L / PG_STAGES) & 1)) bad = true;
  }
  bad = __syncthreads_or(bad);
  if (bad) {
    // record, then let every copy and MMA this CTA issued land before the shared
    // and tensor memory they target are released
    if (tid == 0) {
      if (err) atomicOr(err, 1u);
      for (int s = 0; s < PG_STAGES; s++) {
        if (n_x[s]) tc_mbar_wait(x_full(s), (n_x[s] - 1) & 1);
        if (n_m[s]) tc_mbar_wait(mma_done(s), (n_m[s] - 1) & 1);
      }
    }
  }
  // warp w holds lanes 32*(w%4).. of D (rows) and tokens 64*(w/4).. of it
  const uint32_t q = warp % 4, half = warp / 4;
  const uint32_t row = m0 + 32 * q + lane;
  float v[2][32];
  if (!bad) {
    tc_fence_after_sync();
#pragma unroll
    for (int part = 0; part < 2; part++) tc_ld_32cols(tmem + ((32 * q) << 16) + 64 * half + 32 * part, v[part]);
  }
  bool emit = !bad;
  if (nz > 1) {
    // K split: each CTA publishes its [128 x PG_N] partial; the last of the pair to
    // arrive adds the other's (two terms, so the sum does not depend on which
    // arrives last) and runs the epilogue.  The barrier orders every thread's
    // stores before thread 0's arrival, whose release is cumulative; its acquire,
    // then the barrier, orders the other partial before the loads.
    const uint32_t tile = nb * gridDim.x + blockIdx.x;
    float* mine = kpart + ((size_t)tile * 2 + kz) * (PG_M * PG_N);
    const float* other = kpart + ((size_t)tile * 2 + (1 - kz)) * (PG_M * PG_N);
    if (!bad) {
#pragma unroll
      for (int part = 0; part < 2; part++)
#pragma unroll
        for (int j = 0; j < 32; j++) __stcg(mine + (size_t)(64 * half + 32 * part + j) * PG_M + 32 * q + lane, v[part][j]);
    }
    __syncthreads();
    if (tid == 0) {
      unsigned old;
      asm volatile("atom.acq_rel.gpu.global.add.u32 %0, [%1], 1;" : "=r"(old) : "l"(kcnt + tile) : "memory");
      *s_last = old == nz - 1;
      if (old == nz - 1) kcnt[tile] = 0u;
    }
    __syncthreads();
    emit = emit && *s_last;
    if (emit) {
#pragma unroll
      for (int part = 0; part < 2; part++)
#pragma unroll
        for (int j = 0; j < 32; j++)
          v[part][j] += __ldcg(other + (size_t)(64 * half + 32 * part + j) * PG_M + 32 * q + lane);
    }
  }
  if (emit) {
#pragma unroll
    for (int part = 0; part < 2; part++) {
      const uint32_t c0 = 64 * half + 32 * part;
#pragma unroll
      for (int j = 0; j < 32; j++) {
        const float vp = __shfl_xor_sync(0xffffffffu, v[part][j], 1);
        const uint32_t t = nb * PG_N + c0 + j;
        if (t < T && row < W.M) epi(row, t, v[part][j], vp);
      }
    }
  }
  tc_fence_before_sync();
  __syncthreads();
  if (warp == 0) {
    tc_fence_after_sync();
    tc_tmem_dealloc(tmem, PG_N);
  }
  griddep_launch();
}

// ---- epilogues (row, token, value, value of row ^ 1) ------------------------------
struct PgEpiStore {  // y[t][row]
  float* y;
  uint32_t ldy;
  __device__ void operator()(uint32_t row, uint32_t t, float v, float) const { y[(size_t)t * ldy + row] = v; }
};

// Q/K/V of token t at position pos0 + t (the decode step's rope_store, so the
// same bias, rotation and f16 rounding): the even row of a Q/K pair rotates both
// values (its partner's arrives as vp), V rows are stored one by one; Q and the
// step's K/V rows go to [t][rows] buffers, K/V also into the cache.
struct PgEpiRope {
  RopeQKVArgs a;       // q_out/k_cur/v_cur: token 0's rows
  uint32_t pos0;
  uint32_t q_stride, kv_stride;  // floats per token of q_out and of k_cur/v_cur
  __device__ void operator()(uint32_t row, uint32_t t, float v, float vp) const {
    RopeQKVArgs b = a;
    b.q_out = a.q_out + (size_t)t * q_stride;
    b.k_cur = a.k_cur + (size_t)t * kv_stride;
    b.v_cur = a.v_cur + (size_t)t * kv_stride;
    const uint32_t p = row + a.row_base;
    if (p < a.q_rows + a.kv_rows) {
      if (row & 1) return;
      const float v2[2] = {v, vp};
      rope_store(b, (int)row, v2, 2, nullptr, (int)(pos0 + t));
    } else {
      rope_store(b, (int)row, &v, 1, nullptr, (int)(pos0 + t));
    }
  }
};
// x[t][row] += v: the residual add after W_o and W_down (model_executor.rs:213-215, 231-233).
struct PgEpiResidual {
  float* x;
  uint32_t ldx;
  __device__ void operator()(uint32_t row, uint32_t t, float v, float) const { x[(size_t)t * ldx + row] += v; }
};
// Rows (2j, 2j+1) = (gate_j, up_j): act[t][j] = silu(g) * u, silu(g) = g / (1 + exp(-g))
// (compute.rs:337-350), the decode step's EpiSwiGLU arithmetic.
struct PgEpiSwiGLU {
  float* act;
  uint32_t ld;
  __device__ void operator()(uint32_t row, uint32_t t, float v, float vp) const {
    if (row & 1) return;
    const float s = v / (1.0f + expf(-v));
    act[(size_t)t * ld + (row >> 1)] = __fmul_rn(s, vp);
  }
};

size_t prefill_xt_bytes(uint32_t T, uint32_t Kp) {
  return (size_t)((T + PG_N - 1) / PG_N) * (Kp / PG_KS) * 2 * PG_B_BYTES;
}
bool prefill_supported(int type) { return type == T_Q4_K || type == T_Q8_0; }

cudaError_t prefill_split(const Launch& L, const float* X, uint32_t ldx, uint32_t T, uint32_t K, uint32_t Kp,
                          const float* nw, float eps, void* Xt) {
  if (Kp % PG_KS || K > Kp) return cudaErrorInvalidValue;
  const uint32_t Tp = (T + PG_N - 1) / PG_N * PG_N;
  return launch_k(L, prefill_split_kernel, dim3(Tp), dim3(256), 0, X, ldx, T, K, Kp, nw, eps,
                  static_cast<__nv_bfloat16*>(Xt));
}

// The K split: a pair of CTAs per output block when the blocks alone fill at most
// half the SMs and the scratch (`ks` with room for `ks_tiles` blocks) is given.
template <class Epi>
static cudaError_t run_prefill_gemm(const Launch& L, const PackedMat& W, const void* Xt, uint32_t T, unsigned* err,
                                    Epi epi, const PrefillKSplit& ks = PrefillKSplit{}) {
  void (*k)(PackedMat, const __nv_bfloat16*, uint32_t, unsigned*, Epi, float*, unsigned*) = nullptr;
  switch (W.type) {
    case T_Q4_K: k = prefill_gemm_kernel<T_Q4_K, Epi>; break;
    case T_Q8_0: k = prefill_gemm_kernel<T_Q8_0, Epi>; break;
    default: return cudaErrorInvalidValue;
  }
  if (W.Kp % PG_KS || T == 0) return cudaErrorInvalidValue;
  cudaError_t e = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)PG_SMEM);
  if (e != cudaSuccess) return e;
  dim3 grid((W.Mp + PG_M - 1) / PG_M, (T + PG_N - 1) / PG_N, 1);
  const uint32_t blocks = grid.x * grid.y;
  if (ks.part && ks.cnt && blocks <= ks.tiles && 2 * blocks <= (uint32_t)num_sms() &&
      W.Kp / PG_KS >= 2 * PG_STAGES)
    grid.z = 2;
  return launch_k(L, k, grid, dim3(PG_THREADS), PG_SMEM, W, static_cast<const __nv_bfloat16*>(Xt), T, err, epi,
                  grid.z > 1 ? ks.part : nullptr, grid.z > 1 ? ks.cnt : nullptr);
}

cudaError_t prefill_gemm_store(const Launch& L, const PackedMat& W, const void* Xt, uint32_t T, unsigned* err,
                               float* y, uint32_t ldy) {
  return run_prefill_gemm(L, W, Xt, T, err, PgEpiStore{y, ldy});
}
cudaError_t prefill_gemm_rope(const Launch& L, const PackedMat& W, const void* Xt, uint32_t T, unsigned* err,
                              const RopeQKVArgs& a, uint32_t pos0, uint32_t q_stride, uint32_t kv_stride) {
  return run_prefill_gemm(L, W, Xt, T, err, PgEpiRope{a, pos0, q_stride, kv_stride});
}
cudaError_t prefill_gemm_residual(const Launch& L, const PackedMat& W, const void* Xt, uint32_t T, unsigned* err,
                                  float* x, uint32_t ldx, const PrefillKSplit& ks) {
  return run_prefill_gemm(L, W, Xt, T, err, PgEpiResidual{x, ldx}, ks);
}
size_t prefill_ksplit_floats(uint32_t tiles) { return (size_t)tiles * 2 * PG_M * PG_N; }
cudaError_t prefill_gemm_swiglu(const Launch& L, const PackedMat& W, const void* Xt, uint32_t T, unsigned* err,
                                float* act, uint32_t ld) {
  return run_prefill_gemm(L, W, Xt, T, err, PgEpiSwiGLU{act, ld});
}

}  // namespace rf
