// rf_attn_stream.cuh - split-K GQA decode attention over an f16 KV cache that
// streams the history through shared memory with bulk asynchronous copies.
//
// attention_reference (compute.rs:461-547) for one query token: query head h
// reads KV head h*KV/H (contiguous groups of G = H/KV heads); scores are
// dot/sqrt(hd), a stable softmax over the history plus the current position,
// then sum p*v.  Here a CTA of AS_WARPS warps owns one (KV head, split,
// sequence) unit; the split's positions are cut into tiles of TPW rows, and
// warp w takes tiles w, w + AS_WARPS, ...  Each warp runs its own pipeline:
//
//  * one lane copies a tile's K rows and V rows (contiguous in the head-major
//    cache) into one of the warp's AS_STAGES shared-memory slots with
//    cp.async.bulk, completing on the slot's mbarrier; the copies of the first
//    AS_STAGES tiles are issued before griddepcontrol.wait (the history was
//    written by earlier steps; only q and the current K/V come from the
//    kernel before), later ones as soon as a slot is read;
//  * the warp's (position, head) dot products of a tile, 32 at a time, are
//    summed across lanes by the transposing butterfly of rf_attn.cuh, so lane l
//    ends with one score of head l % G;
//  * every warp keeps its own running softmax (the max and sum of head h live in
//    the lanes l % G == h) and rescales its accumulators per tile, so warps
//    never wait for each other until the unit's end, where the four partial
//    (max, sum, output) triples are merged in shared memory.
//
// Split partials are merged by the last unit of a head to finish
// (attn_merge_tail).  Every mbarrier wait is bounded (about a second); on
// expiry the kernel sets bit 1 of *a.err (when given), waits (bounded) for its
// own copies in flight, and finishes with the values it has.
#pragma once
#include <type_traits>

#include "rf_attn.cuh"
#include "rf_tc.cuh"

namespace rf {

constexpr int AS_WARPS = ATT_WARPS;  // the merge tail's thread count
constexpr int AS_THREADS = AS_WARPS * 32;
constexpr int AS_STAGES = 2;  // two, not three: 3 CTAs share an SM (batch 8, ctx 32768: 0.70 vs 0.62 of peak)

// Positions per tile: 32 (position, head) dot products a butterfly.
template <int G>
__host__ __device__ constexpr int as_tpw() {
  return 32 / G < 16 ? 16 : 32 / G;
}
// Bytes of one tile of K (or of V).
template <int G, int HD>
__host__ __device__ constexpr uint32_t as_tile_bytes() {
  return (uint32_t)as_tpw<G>() * HD * 2;
}
// Dynamic shared memory: mbarriers (128 B), then [AS_WARPS][AS_STAGES] slots of
// a K tile and a V tile, the warps' tile weights [AS_WARPS][TPW*G], the split
// weights [ATT_MERGE_SPLITS][G], the warps' (max, sum) [AS_WARPS][2][G] and the
// last-arrival flag.
template <int G, int HD>
__host__ __device__ constexpr size_t as_smem_bytes() {
  return 128 + (size_t)AS_WARPS * AS_STAGES * 2 * as_tile_bytes<G, HD>() +
         4 * ((size_t)AS_WARPS * as_tpw<G>() * G + ATT_MERGE_SPLITS * G + AS_WARPS * 2 * G + 4);
}

// Splits of a context: at most one per 256 positions (4 tiles a warp, so a
// split's fixed costs, from its first copy to its partial, are spread over a
// pipeline of tiles), as many as fill `slots` CTAs for the (sequence, KV head)
// pairs, and no more than the workspace holds.
__host__ __device__ inline int as_nsplit(int ctx, int max_splits, int slots, int units) {
  int s = (ctx + AS_WARPS * 64 - 1) / (AS_WARPS * 64);
  const int fill = units > 0 ? slots / units : 1;
  s = s < fill ? s : fill;
  s = s < max_splits ? s : max_splits;
  return s < 1 ? 1 : s;
}

// DPL consecutive f16 of a shared-memory row as f32.
template <int DPL>
__device__ __forceinline__ void half_row(const __half* r, float (&v)[DPL]) {
  if constexpr (DPL == 4) {
    const uint2 w = *reinterpret_cast<const uint2*>(r);
    const float2 f0 = __half22float2(*reinterpret_cast<const __half2*>(&w.x));
    const float2 f1 = __half22float2(*reinterpret_cast<const __half2*>(&w.y));
    v[0] = f0.x;
    v[1 % DPL] = f0.y;
    v[2 % DPL] = f1.x;
    v[3 % DPL] = f1.y;
  } else if constexpr (DPL == 2) {
    const float2 f0 = __half22float2(*reinterpret_cast<const __half2*>(r));
    v[0] = f0.x;
    v[1 % DPL] = f0.y;
  } else {
    v[0] = __half2float(r[0]);
  }
}

template <int G, int HD>
__global__ void __launch_bounds__(AS_THREADS) attn_stream_kernel(AttnArgs a, int slots) {
  constexpr int DPL = HD / 32, TPW = as_tpw<G>(), E = TPW * G, NV = E / 32;
  constexpr uint32_t TB = as_tile_bytes<G, HD>();
  extern __shared__ __align__(128) uint8_t as_smem[];
  const uint32_t bars = tc_smem_u32(as_smem);
  uint8_t* slots_base = as_smem + 128;
  float* ew_all = reinterpret_cast<float*>(slots_base + (size_t)AS_WARPS * AS_STAGES * 2 * TB);
  float(*s_w)[G] = reinterpret_cast<float(*)[G]>(ew_all + AS_WARPS * E);
  float(*s_ml)[2][G] = reinterpret_cast<float(*)[2][G]>(ew_all + AS_WARPS * E + ATT_MERGE_SPLITS * G);
  int* s_last = reinterpret_cast<int*>(ew_all + AS_WARPS * E + ATT_MERGE_SPLITS * G + AS_WARPS * 2 * G);

  const int t = threadIdx.x, lane = t & 31, warp = t >> 5;
  const int kvh = blockIdx.x, split = blockIdx.y, b = blockIdx.z;
  // The history length is the step position, written by an earlier step.
  const int nhist = (a.d_nhist ? __ldcg(a.d_nhist) : a.nhist) + b * a.nhist_step;
  const bool has_cur = a.k_cur != nullptr;
  const int ctx = nhist + (has_cur ? 1 : 0);
  const int nsplit = as_nsplit(ctx, a.max_splits, slots, a.n_kv_heads * a.batch);
  if (split >= nsplit || ctx <= 0) return;
  const int chunk = (ctx + nsplit - 1) / nsplit;
  const int p0 = split * chunk, p1 = min(ctx, p0 + chunk);
  const int ntiles = (p1 - p0 + TPW - 1) / TPW;
  const int nt = ntiles > warp ? (ntiles - warp + AS_WARPS - 1) / AS_WARPS : 0;  // this warp's tiles
  const __half* kb =
      reinterpret_cast<const __half*>(a.kc) + (size_t)b * a.batch_stride + (size_t)kvh * a.head_stride;
  const __half* vb =
      reinterpret_cast<const __half*>(a.vc) + (size_t)b * a.batch_stride + (size_t)kvh * a.head_stride;
  uint8_t* wslots = slots_base + (size_t)warp * AS_STAGES * 2 * TB;
  const uint32_t wbar = bars + 8 * warp * AS_STAGES;
  auto tile_pos = [&](int i) { return p0 + (warp + AS_WARPS * i) * TPW; };
  // lane 0: the history rows of the warp's tile i into slot i % AS_STAGES
  auto issue = [&](int i) {
    const int s = i % AS_STAGES, pa = tile_pos(i), pb = min(min(pa + TPW, p1), nhist);
    const uint32_t bar = wbar + 8 * s;
    if (pb > pa) {
      const uint32_t bytes = (uint32_t)(pb - pa) * HD * 2;
      const uint32_t dk = tc_smem_u32(wslots + (size_t)s * 2 * TB);
      tc_mbar_expect_tx(bar, 2 * bytes);
      tc_bulk_copy_g2s(dk, kb + (size_t)pa * HD, bytes, bar);
      tc_bulk_copy_g2s(dk + TB, vb + (size_t)pa * HD, bytes, bar);
    } else {
      tc_mbar_arrive(bar);  // the tile holds only the current position
    }
  };
  if (lane == 0) {
    for (int s = 0; s < AS_STAGES; s++) tc_mbar_init(wbar + 8 * s, 1);
    tc_fence_barrier_init();
    for (int i = 0; i < nt && i < AS_STAGES; i++) issue(i);
  }
  __syncwarp();
  griddep_wait();

  const int d0 = lane * DPL;
  const float* qb = a.q + ((size_t)b * a.n_heads + (size_t)kvh * G) * HD;
  float qr[G][DPL];
#pragma unroll
  for (int h = 0; h < G; h++)
#pragma unroll
    for (int i = 0; i < DPL; i++) qr[h][i] = __ldcg(qb + (size_t)h * HD + d0 + i);
  const bool with_cur = has_cur && nhist >= p0 && nhist < p1;
  float kcur[DPL], vcur[DPL];
  cur_load<DPL>(with_cur ? a.k_cur + b * a.cur_stride + (size_t)kvh * HD : nullptr, d0, HD, kcur);
  cur_load<DPL>(with_cur ? a.v_cur + b * a.cur_stride + (size_t)kvh * HD : nullptr, d0, HD, vcur);
  const float div = sqrtf((float)HD);  // score = dot / sqrt(hd)  (compute.rs:530)

  float m_run = -INFINITY, l_run = 0.f;  // softmax state of head lane % G
  // output sums of heads (2hp, 2hp+1) as float2 pairs, so that p*v accumulates with
  // packed fma.rn.f32x2 (each half the scalar fmaf's rounding; G = 1 leaves .y at 0)
  constexpr int GP = (G + 1) / 2;
  float2 acc[GP][DPL];
#pragma unroll
  for (int hp = 0; hp < GP; hp++)
#pragma unroll
    for (int i = 0; i < DPL; i++) acc[hp][i] = make_float2(0.f, 0.f);
  float* ew = ew_all + warp * E;
  bool ok = true;
  int waited = 0;  // tiles whose copies have completed
  for (int i = 0; i < nt; i++) {
    const int s = i % AS_STAGES;
    ok = __all_sync(0xffffffffu, tc_mbar_wait(wbar + 8 * s, (uint32_t)(i / AS_STAGES) & 1u));
    if (!ok) break;
    waited = i + 1;
    const __half* kt = reinterpret_cast<const __half*>(wslots + (size_t)s * 2 * TB);
    const __half* vt = reinterpret_cast<const __half*>(wslots + (size_t)s * 2 * TB + TB);
    const int pa = tile_pos(i);
    // FULL: every position of the tile is a history row of this split (most tiles),
    // so the per-position checks drop out
    auto tile = [&](auto full_tag) {
      constexpr bool FULL = decltype(full_tag)::value;
      // scores: value c = j*G + h (position pa + j, head h), 32 at a time
      float sc[NV];
#pragma unroll
      for (int c0 = 0; c0 < E; c0 += 32) {
        float v[32];
#pragma unroll
        for (int jj = 0; jj < 32 / G; jj++) {
          const int j = c0 / G + jj, p = pa + j;
          float k[DPL];
          if (FULL || (p < nhist && p < p1)) {
            half_row<DPL>(kt + (size_t)j * HD + d0, k);
          } else {
#pragma unroll
            for (int d = 0; d < DPL; d++) k[d] = p < p1 ? kcur[d] : 0.f;
          }
#pragma unroll
          for (int h = 0; h < G; h++) {
            float dot = 0.f;
#pragma unroll
            for (int d = 0; d < DPL; d++) dot = fmaf(qr[h][d], k[d], dot);
            v[jj * G + h] = dot;
          }
        }
        warp_transpose_sum<32, 16>(v, lane);
        if constexpr (FULL) {
          sc[c0 / 32] = v[0] / div;
        } else {
          const int p = pa + (c0 + lane) / G;
          const bool valid = p < p1 && (p < nhist || with_cur);
          sc[c0 / 32] = valid ? v[0] / div : -INFINITY;
        }
      }
      // running softmax of head lane % G (softmax_reference, compute.rs:363-384)
      float mx = sc[0];
#pragma unroll
      for (int k = 1; k < NV; k++) mx = fmaxf(mx, sc[k]);
#pragma unroll
      for (int o = G; o < 32; o <<= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
      const float m_new = fmaxf(m_run, mx);
      float ls = 0.f;
#pragma unroll
      for (int k = 0; k < NV; k++) {
        const float e = expf(sc[k] - m_new);
        ew[32 * k + lane] = e;
        ls += e;
      }
#pragma unroll
      for (int o = G; o < 32; o <<= 1) ls += __shfl_xor_sync(0xffffffffu, ls, o);
      const float f = expf(m_run - m_new);
      l_run = l_run * f + ls;
      m_run = m_new;
      __syncwarp();
#pragma unroll
      for (int hp = 0; hp < GP; hp++) {
        const float f0 = __shfl_sync(0xffffffffu, f, 2 * hp);
        const float f1 = G > 1 ? __shfl_sync(0xffffffffu, f, 2 * hp + 1) : 0.f;
#pragma unroll
        for (int d = 0; d < DPL; d++) {
          acc[hp][d].x *= f0;
          acc[hp][d].y *= f1;
        }
      }
#pragma unroll
      for (int j = 0; j < TPW; j++) {
        const int p = pa + j;
        if (!FULL && p >= p1) break;
        float v[DPL];
        if (FULL || p < nhist) {
          half_row<DPL>(vt + (size_t)j * HD + d0, v);
        } else {
#pragma unroll
          for (int d = 0; d < DPL; d++) v[d] = vcur[d];
        }
        float2 e2[GP];
        if constexpr (G % 4 == 0) {
#pragma unroll
          for (int h = 0; h < G; h += 4) {
            const float4 e4 = *reinterpret_cast<const float4*>(ew + j * G + h);
            e2[h / 2] = make_float2(e4.x, e4.y);
            e2[h / 2 + 1] = make_float2(e4.z, e4.w);
          }
        } else if constexpr (G == 2) {
          e2[0] = *reinterpret_cast<const float2*>(ew + j * 2);
        } else {
          e2[0] = make_float2(ew[j], 0.f);
        }
#pragma unroll
        for (int hp = 0; hp < GP; hp++)
#pragma unroll
          for (int d = 0; d < DPL; d++) acc[hp][d] = __ffma2_rn(e2[hp], make_float2(v[d], v[d]), acc[hp][d]);
      }
    };
    if (pa + TPW <= min(p1, nhist)) tile(std::true_type{});
    else tile(std::false_type{});
    __syncwarp();  // slot s and the weights are read
    if (lane == 0 && i + AS_STAGES < nt) {
      asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
      issue(i + AS_STAGES);
    }
  }
  if (!ok) {
    // a copy did not complete in time: record it, give the copies in flight a
    // bounded wait, and finish with what was accumulated
    if (lane == 0) {
      if (a.err) atomicOr(a.err, 2u);
      for (int i = waited; i < nt && i < waited + AS_STAGES; i++)
        tc_mbar_wait(wbar + 8 * (i % AS_STAGES), (uint32_t)(i / AS_STAGES) & 1u);
    }
    __syncwarp();
  }
  griddep_launch();

  // merge the warps: (max, sum) per head, output sums into the warp's own slots
  if (lane < G) {
    s_ml[warp][0][lane] = m_run;
    s_ml[warp][1][lane] = l_run;
  }
  float* wacc = reinterpret_cast<float*>(wslots);  // [G][HD], the warp's tiles are all read
#pragma unroll
  for (int h = 0; h < G; h++)
#pragma unroll
    for (int d = 0; d < DPL; d++) wacc[h * HD + d0 + d] = (h & 1) ? acc[h / 2][d].y : acc[h / 2][d].x;
  __syncthreads();
  float* out_b = a.out + ((size_t)b * a.n_heads + (size_t)kvh * G) * HD;
  const size_t slot = ((size_t)b * a.n_kv_heads + kvh) * a.max_splits;
  float* part = a.part + (slot + split) * (size_t)G * (HD + 2);
  for (int i = t; i < G * HD; i += AS_THREADS) {
    const int h = i / HD, d = i % HD;
    float M = -INFINITY;
#pragma unroll
    for (int w = 0; w < AS_WARPS; w++) M = fmaxf(M, s_ml[w][0][h]);
    float O = 0.f, L = 0.f;
#pragma unroll
    for (int w = 0; w < AS_WARPS; w++) {
      const float m = s_ml[w][0][h];
      const float sw = m == -INFINITY ? 0.f : expf(m - M);
      O = fmaf(sw, reinterpret_cast<const float*>(slots_base + (size_t)w * AS_STAGES * 2 * TB)[i], O);
      L = fmaf(sw, s_ml[w][1][h], L);
    }
    if (nsplit == 1) {
      out_b[i] = O / L;
    } else {
      __stcg(part + (size_t)h * (HD + 2) + d, O);
      if (d == 0) {
        __stcg(part + (size_t)h * (HD + 2) + HD, M);
        __stcg(part + (size_t)h * (HD + 2) + HD + 1, L);
      }
    }
  }
  if (nsplit == 1) return;
  attn_merge_tail<DPL, G, 16>(a, b, kvh, nsplit, out_b, s_w, s_last, t, [] { __syncthreads(); });
}

}  // namespace rf
