// rf_attn.cuh - split-K GQA decode attention (one query token per sequence),
// written as a routine for a group of ATT_THREADS threads (one group per CTA of
// attn_kernel).
//
// attention_reference (compute.rs:461-547) for one query token: query head h
// reads KV head h*KV/H (contiguous groups of G = H/KV heads), so one unit loads
// each K/V row once for its G heads.  A unit is (KV head, split): the context is
// cut into nsplit chunks of about 64 positions (more per chunk only when the
// split count is capped), and a chunk is walked in passes of ATT_WARPS*PPW
// positions with a running (online) softmax.  At batch 1 the cost is latency,
// not bandwidth, so a pass issues every K row and every V row it needs before
// using any of them: one memory round trip per pass.  Lane i holds dims
// [i*DPL, i*DPL+DPL) of every row; warp w takes positions w, w+4, ... of a pass.
// The last unit of a head to finish merges the chunk partials (max-rescaled
// sums); nothing waits on another group or CTA.
#pragma once
#include <math.h>

#include "rf_device.cuh"

namespace rf {

constexpr int ATT_THREADS = 128;
constexpr int ATT_WARPS = ATT_THREADS / 32;
constexpr int ATT_CHUNK = 64;         // target positions per split
constexpr int ATT_PASS_MAX = 64;      // positions per pass, at most
constexpr int ATT_MERGE_SPLITS = 64;  // merges of up to this many splits take the parallel path

__host__ __device__ inline int attn_nsplit(int ctx, int max_splits) {
  int s = (ctx + ATT_CHUNK - 1) / ATT_CHUNK;
  s = s < 1 ? 1 : s;
  return s < max_splits ? s : max_splits;
}

// Positions per warp per pass: as many as keep the raw K and V rows of a pass in
// registers next to the query and the accumulators.
template <int DPL, int G, typename KT>
__host__ __device__ constexpr int attn_ppw() {
  return (sizeof(KT) == 4 || G * DPL > 16) ? 8 : 16;
}

// Shared memory of one group: pass scores / weights [G][ATT_PASS_MAX], warp
// partial outputs [ATT_WARPS][G][DPL*32], split weights [ATT_MERGE_SPLITS][G],
// running max, running sum and pass rescale per head, and the last-arrival flag.
template <int DPL, int G>
__host__ __device__ constexpr int attn_group_floats() {
  return G * ATT_PASS_MAX + ATT_WARPS * G * DPL * 32 + ATT_MERGE_SPLITS * G + 3 * G + 4;
}

// Barrier of the ATT_THREADS threads of group `id` (hardware barriers 1..15).
__device__ __forceinline__ void group_sync(int id) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(ATT_THREADS) : "memory");
}

// Raw words of this lane's DPL elements of a cache row: f16 pairs (RW = DPL/2
// words, odd DPL rounded up) or f32 bits (RW = DPL).  Cache rows are written by
// earlier steps and only read here.
template <typename KT, int DPL>
struct RawW {
  static constexpr int RW = sizeof(KT) == 2 ? (DPL + 1) / 2 : DPL;
};
template <int DPL, int RW>
__device__ __forceinline__ void raw_load(const __half* p, int d0, int hd, uint32_t (&r)[RW]) {
  if (DPL == 4 && d0 + 4 <= hd) {
    const uint2 v = __ldg(reinterpret_cast<const uint2*>(p + d0));
    r[0] = v.x;
    r[1 % RW] = v.y;
  } else if (DPL == 2 && d0 + 2 <= hd) {
    r[0] = __ldg(reinterpret_cast<const unsigned*>(p + d0));
  } else {
#pragma unroll
    for (int i = 0; i < RW; i++) {
      const uint32_t lo = d0 + 2 * i < hd ? __half_as_ushort(p[d0 + 2 * i]) : 0u;
      const uint32_t hi = 2 * i + 1 < DPL && d0 + 2 * i + 1 < hd ? __half_as_ushort(p[d0 + 2 * i + 1]) : 0u;
      r[i] = lo | (hi << 16);
    }
  }
}
template <int DPL, int RW>
__device__ __forceinline__ void raw_load(const float* p, int d0, int hd, uint32_t (&r)[RW]) {
#pragma unroll
  for (int i = 0; i < RW; i++) r[i] = d0 + i < hd ? __float_as_uint(__ldg(p + d0 + i)) : 0u;
}
template <int DPL, int RW, typename KT>
__device__ __forceinline__ void raw_f32(const uint32_t (&r)[RW], float (&v)[DPL]) {
  if constexpr (sizeof(KT) == 2) {
#pragma unroll
    for (int i = 0; i < DPL; i += 2) {
      const float2 f = __half22float2(*reinterpret_cast<const __half2*>(&r[i / 2]));
      v[i] = f.x;
      if (i + 1 < DPL) v[i + 1] = f.y;
    }
  } else {
#pragma unroll
    for (int i = 0; i < DPL; i++) v[i] = __uint_as_float(r[i]);
  }
}
// This lane's DPL elements of the current step's K or V (f32, written earlier in
// the same kernel, so read through L2).  The reference's attention runs before
// the step's K/V are committed to the cache, so they are used unrounded.
template <int DPL>
__device__ __forceinline__ void cur_load(const float* p, int d0, int hd, float (&v)[DPL]) {
#pragma unroll
  for (int i = 0; i < DPL; i++) v[i] = p && d0 + i < hd ? __ldcg(p + d0 + i) : 0.f;
}

// Warp sums of CNT values at once (a transposing butterfly): at each level a lane
// keeps half of the values it still holds, sends the other half to its partner
// and adds what comes back, so CNT = 32 sums take 31 shuffles in chains five
// deep (one sum at a time takes five dependent shuffles each).  Afterwards
// v[0] of lane l is the full sum of value l >> (5 - log2 CNT).
template <int CNT, int O>
__device__ __forceinline__ void warp_transpose_sum(float* v, int lane) {
  if constexpr (O >= 1) {
    if constexpr (CNT > 1) {
      constexpr int HALF = CNT / 2;
      const bool up = (lane & O) != 0;
#pragma unroll
      for (int i = 0; i < HALF; i++) {
        const float send = up ? v[i] : v[i + HALF];
        const float keep = up ? v[i + HALF] : v[i];
        v[i] = keep + __shfl_xor_sync(0xffffffffu, send, O);
      }
      warp_transpose_sum<HALF, O / 2>(v, lane);
    } else {
      v[0] += __shfl_xor_sync(0xffffffffu, v[0], O);
      warp_transpose_sum<1, O / 2>(v, lane);
    }
  }
}

// End of a split unit that has written its partial ([G][hd] sums, then (m, l)
// per head) to a.part: the last unit of (sequence b, KV head kvh) to arrive
// merges the nsplit partials (max-rescaled sums) into out_b; the others return.
// Run by ATT_THREADS threads (t = thread index, warp/lane of t); `sync` is their
// barrier, s_w [ATT_MERGE_SPLITS][G] and s_last shared scratch.
template <int DPL, int G, int MR_MAX, class Sync>
__device__ __forceinline__ void attn_merge_tail(const AttnArgs& a, int b, int kvh, int nsplit, float* out_b,
                                                float (*s_w)[G], int* s_last, int t, Sync&& sync) {
  const int lane = t & 31, warp = t >> 5, hd = a.head_dim;
  const size_t slot = ((size_t)b * a.n_kv_heads + kvh) * a.max_splits;
  // the group barrier orders every thread's partial before thread 0's arrival,
  // whose release is cumulative; its acquire, then the barrier, orders the other
  // splits' partials before every thread's loads below
  sync();
  if (t == 0) {
    unsigned prev;
    asm volatile("atom.acq_rel.gpu.global.add.u32 %0, [%1], 1;"
                 : "=r"(prev)
                 : "l"(&a.counters[(size_t)b * a.n_kv_heads + kvh])
                 : "memory");
    *s_last = prev == (unsigned)(nsplit - 1);
  }
  sync();
  if (!*s_last) {
    sync();
    return;
  }
  const float* pall = a.part + slot * (size_t)G * (hd + 2);
  if (nsplit <= ATT_MERGE_SPLITS) {
    // every output element: sum_s w_s * O_s in split order.  A thread owns EPT
    // elements and loads MR splits of all of them per round, every load of a round
    // in flight together: each round is one L2 round trip, so a caller that merges
    // tens of splits takes MR_MAX up to 16 (at most 64 values a thread); the
    // register-load kernel keeps 4, which keeps its registers where its occupancy
    // in the decode step needs them.  The first round is issued before the split
    // weights are computed (it does not depend on them), so the two overlap.
    constexpr int EPT = (G * DPL * 32 + ATT_THREADS - 1) / ATT_THREADS;  // hd <= 32*DPL
    constexpr int MR = 64 / EPT < 4 ? 4 : (64 / EPT > MR_MAX ? MR_MAX : 64 / EPT);
    float v[EPT][MR];
    auto load_round = [&](int s0) {
#pragma unroll
      for (int k = 0; k < EPT; k++) {
        const int i = t + k * ATT_THREADS, h = i / hd, d = i % hd;
#pragma unroll
        for (int j = 0; j < MR; j++)
          v[k][j] = i < G * hd && s0 + j < nsplit ? __ldcg(pall + ((size_t)(s0 + j) * G + h) * (hd + 2) + d) : 0.f;
      }
    };
    load_round(0);
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
    sync();
    float O[EPT];
#pragma unroll
    for (int k = 0; k < EPT; k++) O[k] = 0.f;
    for (int s0 = 0; s0 < nsplit; s0 += MR) {
      if (s0 > 0) load_round(s0);
#pragma unroll
      for (int k = 0; k < EPT; k++) {
        const int i = t + k * ATT_THREADS, h = i / hd;
        if (i < G * hd) {
#pragma unroll
          for (int j = 0; j < MR; j++)
            if (s0 + j < nsplit) O[k] = fmaf(s_w[s0 + j][h], v[k][j], O[k]);
        }
      }
    }
#pragma unroll
    for (int k = 0; k < EPT; k++) {
      const int i = t + k * ATT_THREADS, h = i / hd, d = i % hd;
      if (i < G * hd) out_b[(size_t)h * hd + d] = O[k];
    }
  } else {
    for (int i = t; i < G * hd; i += ATT_THREADS) {
      const int h = i / hd, d = i % hd;
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
  if (t == 0) a.counters[(size_t)b * a.n_kv_heads + kvh] = 0u;
  sync();  // shared memory may be reused after this
}

// One (KV head, split, sequence) unit, run by the ATT_THREADS threads of group
// `gid` (thread t = threadIdx.x % ATT_THREADS, barrier gid + 1).  The caller has
// made a.q, a.k_cur, a.v_cur and the history length visible.  PPW_CAP bounds
// the positions per warp of a pass (fewer registers, for callers launched with
// a tighter register budget).
template <int DPL, int G, typename KT, int PPW_CAP = ATT_PASS_MAX>
__device__ __forceinline__ void attn_unit(const AttnArgs& a, int kvh, int split, int b, float* gsm, int gid) {
  constexpr int PPW = attn_ppw<DPL, G, KT>() < PPW_CAP ? attn_ppw<DPL, G, KT>() : PPW_CAP;
  constexpr int PASS = ATT_WARPS * PPW, RW = RawW<KT, DPL>::RW;
  float(*ssc)[ATT_PASS_MAX] = reinterpret_cast<float(*)[ATT_PASS_MAX]>(gsm);
  float(*sred)[G][DPL * 32] = reinterpret_cast<float(*)[G][DPL * 32]>(gsm + G * ATT_PASS_MAX);
  float(*s_w)[G] = reinterpret_cast<float(*)[G]>(gsm + G * ATT_PASS_MAX + ATT_WARPS * G * DPL * 32);
  float* sm = gsm + G * ATT_PASS_MAX + ATT_WARPS * G * DPL * 32 + ATT_MERGE_SPLITS * G;  // running max
  float* sl = sm + G;                                                                      // running sum
  float* sf = sl + G;                                                                      // pass rescale
  int* s_last = reinterpret_cast<int*>(sf + G);
  const int bar = gid + 1;
  const int t = threadIdx.x % ATT_THREADS;
  const int lane = t & 31, warp = t >> 5;
  const int hd = a.head_dim;
  const int nhist = (a.d_nhist ? __ldcg(a.d_nhist) : a.nhist) + b * a.nhist_step;
  const bool has_cur = a.k_cur != nullptr;
  const int ctx = nhist + (has_cur ? 1 : 0);
  const int nsplit = attn_nsplit(ctx, a.max_splits);
  if (split >= nsplit || ctx <= 0) return;
  const int chunk = (ctx + nsplit - 1) / nsplit;
  const int h0 = kvh * G;
  const int p0 = split * chunk, p1 = min(ctx, p0 + chunk);
  const int d0 = lane * DPL;
  const float* qb = a.q + ((size_t)b * a.n_heads + h0) * hd;
  const KT* kb = reinterpret_cast<const KT*>(a.kc) + (size_t)b * a.batch_stride + (size_t)kvh * a.head_stride;
  const KT* vb = reinterpret_cast<const KT*>(a.vc) + (size_t)b * a.batch_stride + (size_t)kvh * a.head_stride;
  const float div = sqrtf((float)hd);  // score = dot / sqrt(hd)  (compute.rs:530)

  float qr[G][DPL];
#pragma unroll
  for (int h = 0; h < G; h++)
#pragma unroll
    for (int i = 0; i < DPL; i++) qr[h][i] = d0 + i < hd ? __ldcg(qb + (size_t)h * hd + d0 + i) : 0.f;
  // the current position, when this chunk holds it
  float kcur[DPL], vcur[DPL];
  const bool with_cur = has_cur && nhist >= p0 && nhist < p1;
  cur_load<DPL>(with_cur ? a.k_cur + b * a.cur_stride + (size_t)kvh * hd : nullptr, d0, hd, kcur);
  cur_load<DPL>(with_cur ? a.v_cur + b * a.cur_stride + (size_t)kvh * hd : nullptr, d0, hd, vcur);
  if (t < G) {
    sm[t] = -INFINITY;
    sl[t] = 0.f;
  }
  float acc[G][DPL];
#pragma unroll
  for (int h = 0; h < G; h++)
#pragma unroll
    for (int i = 0; i < DPL; i++) acc[h][i] = 0.f;

  for (int base = p0; base < p1; base += PASS) {
    const int n = min(PASS, p1 - base);
    // every cached K and V row of this warp's positions of the pass, before any is used
    uint32_t kr[PPW][RW], vr[PPW][RW];
#pragma unroll
    for (int j = 0; j < PPW; j++) {
      const int pp = base + warp + ATT_WARPS * j;
      if (pp < base + n && pp < nhist) {
        raw_load<DPL, RW>(kb + (size_t)pp * hd, d0, hd, kr[j]);
        raw_load<DPL, RW>(vb + (size_t)pp * hd, d0, hd, vr[j]);
      } else {
#pragma unroll
        for (int i = 0; i < RW; i++) kr[j][i] = vr[j][i] = 0u;
      }
    }
    // scores of the pass: the PPW*G dot products (position j, head h) of this
    // warp as value c = j*G + h, summed across the warp EC at a time
    {
      constexpr int E = PPW * G;
      constexpr int EC = E > 16 ? 32 : (E > 8 ? 16 : 8);
      constexpr int LSH = EC == 32 ? 0 : (EC == 16 ? 1 : 2);
#pragma unroll
      for (int c0 = 0; c0 < E; c0 += EC) {
        float v[EC];
#pragma unroll
        for (int e = 0; e < EC; e++) {
          const int c = c0 + e, j = c / G, h = c % G;
          float s = 0.f;
          if (c < E) {
            const bool cached = base + warp + ATT_WARPS * j < nhist;  // else the current step's row
            float k[DPL];
            raw_f32<DPL, RW, KT>(kr[j < PPW ? j : 0], k);
#pragma unroll
            for (int i = 0; i < DPL; i++) s = fmaf(qr[h < G ? h : 0][i], cached ? k[i] : kcur[i], s);
          }
          v[e] = s;
        }
        warp_transpose_sum<EC, 16>(v, lane);
        const int c = c0 + (lane >> LSH), j = c / G, h = c % G;
        if ((lane & ((1 << LSH) - 1)) == 0 && c < E && warp + ATT_WARPS * j < n)
          ssc[h][warp + ATT_WARPS * j] = v[0] / div;
      }
    }
    group_sync(bar);
    // online softmax (softmax_reference, compute.rs:363-384): the new running
    // max, weights exp(s - m) of the pass, and the rescale of what came before
    for (int h = warp; h < G; h += ATT_WARPS) {
      float m = -INFINITY;
      for (int i = lane; i < n; i += 32) m = fmaxf(m, ssc[h][i]);
#pragma unroll
      for (int o = 16; o; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
      const float m_old = sm[h], m_new = fmaxf(m_old, m);
      float l = 0.f;
      for (int i = lane; i < n; i += 32) {
        const float e = expf(ssc[h][i] - m_new);
        ssc[h][i] = e;
        l += e;
      }
#pragma unroll
      for (int o = 16; o; o >>= 1) l += __shfl_xor_sync(0xffffffffu, l, o);
      __syncwarp();
      if (lane == 0) {
        const float f = m_old == -INFINITY ? 0.f : expf(m_old - m_new);
        sf[h] = f;
        sl[h] = sl[h] * f + l;
        sm[h] = m_new;
      }
    }
    group_sync(bar);
#pragma unroll
    for (int h = 0; h < G; h++) {
      const float f = sf[h];
#pragma unroll
      for (int i = 0; i < DPL; i++) acc[h][i] *= f;
    }
#pragma unroll
    for (int j = 0; j < PPW; j++) {
      const int pp = base + warp + ATT_WARPS * j;
      if (pp < base + n) {
        float v[DPL];
        if (pp < nhist) raw_f32<DPL, RW, KT>(vr[j], v);
        else {
#pragma unroll
          for (int i = 0; i < DPL; i++) v[i] = vcur[i];
        }
#pragma unroll
        for (int h = 0; h < G; h++) {
          const float e = ssc[h][warp + ATT_WARPS * j];
#pragma unroll
          for (int i = 0; i < DPL; i++) acc[h][i] = fmaf(e, v[i], acc[h][i]);
        }
      }
    }
    group_sync(bar);  // ssc is rewritten by the next pass
  }
#pragma unroll
  for (int h = 0; h < G; h++)
#pragma unroll
    for (int i = 0; i < DPL; i++) sred[warp][h][d0 + i] = acc[h][i];
  group_sync(bar);
  float* out_b = a.out + ((size_t)b * a.n_heads + h0) * hd;
  if (nsplit == 1) {
    for (int i = t; i < G * hd; i += ATT_THREADS) {
      const int h = i / hd, d = i % hd;
      float s = 0.f;
      for (int w = 0; w < ATT_WARPS; w++) s += sred[w][h][d];
      out_b[(size_t)h * hd + d] = s / sl[h];
    }
    group_sync(bar);  // the group's shared memory is reused by its next unit
    return;
  }
  // write this chunk's partial: [G][hd] sums then (m, l) per head
  const size_t slot = ((size_t)b * a.n_kv_heads + kvh) * a.max_splits;
  float* part = a.part + (slot + split) * (size_t)G * (hd + 2);
  for (int i = t; i < G * hd; i += ATT_THREADS) {
    const int h = i / hd, d = i % hd;
    float s = 0.f;
    for (int w = 0; w < ATT_WARPS; w++) s += sred[w][h][d];
    __stcg(part + (size_t)h * (hd + 2) + d, s);
  }
  if (t < G) {
    __stcg(part + (size_t)t * (hd + 2) + hd, sm[t]);
    __stcg(part + (size_t)t * (hd + 2) + hd + 1, sl[t]);
  }
  attn_merge_tail<DPL, G, 4>(a, b, kvh, nsplit, out_b, s_w, s_last, t, [&] { group_sync(bar); });
}

}  // namespace rf
