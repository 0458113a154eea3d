// rf_gemv.cuh - batch-1 matrix-vector products of the decode engine and their
// fused epilogues (RoPE + KV append, SwiGLU, residual add, greedy argmax).
//
// Batch-1 decode reads every weight byte once per token for one multiply-add
// per element, so the GEMV is bound by HBM bandwidth when its instruction
// stream is lean enough.  For 4-bit weights on B200 it is not automatically:
// HBM delivers ~12e12 Q4_K weights/s, and at 16 integer ops per clock per SM
// sub-partition a dequantise-and-FMA loop may spend only ~1.1 integer
// instructions per weight.  The quantized kernel is built around that budget:
//
//  * One lane owns two rows (r and r+32 of a 64-row tile) and walks the tile's
//    128-byte chunks.  Every activation load is then the same address across the
//    warp (a shared-memory broadcast), every scale header is decoded once per row
//    per chunk, and no cross-lane reduction is needed.
//  * Weights are read with 256-bit loads from the tiled layout (rf_kernels.cuh),
//    so each warp-wide load is 1 KiB of consecutive bytes; the next chunk's
//    pieces are loaded while the current one is multiplied.
//  * A quant field masked in place inside its 32-bit word (bits [off, off+n),
//    off + n <= 24) reads as the float q * 2^(off-149); shared memory holds x
//    pre-multiplied by 2^(85-off) for the field position each element comes from,
//    so every product is exactly q * x * 2^-64 and one packed fma.rn.f32x2 takes
//    two elements.  The top byte of a word is brought down with one byte-permute
//    shared by two words: 17 integer ops per 16 Q4 weights.
//  * Work is split "stream-K": the 32-byte pieces of the matrix's (tile, chunk)
//    items are cut into equal contiguous ranges, one per warp of a persistent
//    grid, so every SM gets the same number of bytes whatever the matrix shape
//    and the warps' shares differ by at most one piece.  A tile whose pieces span
//    several warps is finished by the last of them to arrive (arrival counter),
//    which sums the partials in piece order: results do not depend on timing, and
//    nothing waits on another warp or CTA.
#pragma once
#include <algorithm>

#include "rf_device.cuh"

namespace rf {

constexpr float kTwo64 = 18446744073709551616.0f;  // 2^64
__device__ __forceinline__ float as_f(uint32_t bits) { return __uint_as_float(bits); }
__device__ __forceinline__ float2 ff2(float a, float b) { return make_float2(a, b); }
// 2^(85 - off): exact pre-scale of x for a field at bit `off`.
__device__ __forceinline__ float prescale(int off) { return __int_as_float((212 - off) << 23); }

// ---------------------------------------------------------------------------
// epilogues: called with the finished values of rows [row0, row0+n), n <= 2 and
// row0 even, so RoPE and SwiGLU row pairs arrive together.
//
// An epilogue with kPre = true can have its per-row inputs fetched early: the
// quantized GEMV calls pre_begin() once its inputs are visible and pre_load(row)
// for every row of the tiles its CTA may finish, keeps the values in shared
// memory while it multiplies, and passes them as `pre` (values of rows row0..);
// `pre` is null when they were not fetched.
// ---------------------------------------------------------------------------
struct EpiStore {
  static constexpr bool kPre = false;
  float* y;
  __device__ void operator()(int row0, const float* v, int n, const float* = nullptr) {
    for (int i = 0; i < n; i++) y[row0 + i] = v[i];
  }
  __device__ void pre_begin() {}
  __device__ float pre_load(uint32_t) { return 0.f; }
  __device__ void flush() {}
  __device__ void tile_done(uint32_t) {}
};

struct EpiResidual {  // out = res + W.x (res may alias out: a row is read before it is written)
  static constexpr bool kPre = true;
  const float* res;
  float* out;
  __device__ void operator()(int row0, const float* v, int n, const float* pre = nullptr) {
    for (int i = 0; i < n; i++) {
      const float r = pre ? pre[i] : (res ? __ldcg(res + row0 + i) : 0.f);
      out[row0 + i] = res ? r + v[i] : v[i];
    }
  }
  __device__ void pre_begin() {}
  __device__ float pre_load(uint32_t row) { return res ? __ldcg(res + row) : 0.f; }
  __device__ void flush() {}
  __device__ void tile_done(uint32_t) {}
};

// out = res + W.x of a row-parallel projection, pushed into a tensor-parallel sum
// over peer memory (PeerLink): every row goes to each rank's receive area at this
// rank's row of the site's parity half.  At the end of the kernel each CTA, after a
// barrier behind all of its stores, adds one arrival to this rank's counter of the
// site on every rank (a system-scope release-add); a counter grows by the
// producer's CTA count per use of the site.
struct EpiPeerPush {
  static constexpr bool kPre = true;
  const float* res;  // rank 0: the residual; other ranks: null
  PeerLink pl;
  __device__ void operator()(int row0, const float* v, int n, const float* pre = nullptr) {
    const PeerSum& P = pl.P;
    const size_t off = ((size_t)(pl.push_site & 1) * P.n_ranks + P.rank) * P.n_max;
    for (int i = 0; i < n; i++) {
      const float r = res ? (pre ? pre[i] : __ldcg(res + row0 + i)) : 0.f;
      const float o = res ? r + v[i] : v[i];
      for (int p = 0; p < P.n_ranks; p++) __stcg(P.recv[p] + off + row0 + i, o);
    }
  }
  __device__ void pre_begin() {}
  __device__ float pre_load(uint32_t row) { return res ? __ldcg(res + row) : 0.f; }
  // every thread of the CTA, after its last row
  __device__ void flush() {
    __syncthreads();
    const PeerSum& P = pl.P;
    if ((int)threadIdx.x < P.n_ranks)
      red_release_sys_add(P.flags[threadIdx.x] + ((size_t)P.rank * P.sites + pl.push_site + 1) * P.max_ctas - 1, 1u);
  }
  __device__ void tile_done(uint32_t) {}
};

// Q and K rows are packed as pairs (i, i+hd/2) of each head so that the
// half-split rotation (compute.rs:440-456) happens in registers; V rows are in
// natural order.  Q/K/V biases, when present, are added to the products first
// (bias after projection, before RoPE and the KV append: model_executor.rs:161-196).
// `pre`, when given, holds (cos, sin) of the pair and `pos` the step's position.
__device__ __forceinline__ void rope_store(const RopeQKVArgs& a, int row0, const float* v, int n,
                                           const float* pre = nullptr, int pos = -1);
// (cos, sin) component (row & 1) of the rotation of Q/K row `row` at `pos`; 0 for V rows.
__device__ __forceinline__ float rope_cs_of(const RopeQKVArgs& a, uint32_t row, int pos) {
  row += a.row_base;
  if (row >= a.q_rows + a.kv_rows) return 0.f;
  const uint32_t j = (row < a.q_rows ? row : row - a.q_rows) / 2, half = a.head_dim / 2;
  const float* c = reinterpret_cast<const float*>(a.rope_cs + (size_t)pos * half + j % half);
  return __ldg(c + (row & 1));
}
struct EpiRope {  // arguments held by value (a kernel parameter)
  static constexpr bool kPre = true;
  RopeQKVArgs a;
  int pos;
  __device__ void operator()(int row0, const float* v, int n, const float* pre = nullptr) {
    rope_store(a, row0, v, n, pre, pre ? pos : -1);
  }
  __device__ void pre_begin() { pos = __ldcg(a.d_pos); }
  __device__ float pre_load(uint32_t row) { return rope_cs_of(a, row, pos); }
  __device__ void flush() {}
  __device__ void tile_done(uint32_t) {}
};
struct EpiRopeRef {  // arguments read from memory when a row pair finishes
  static constexpr bool kPre = false;
  const RopeQKVArgs* a;
  __device__ void operator()(int row0, const float* v, int n, const float* = nullptr) { rope_store(*a, row0, v, n); }
  __device__ void pre_begin() {}
  __device__ float pre_load(uint32_t) { return 0.f; }
  __device__ void flush() {}
  __device__ void tile_done(uint32_t) {}
};
__device__ __forceinline__ void rope_store(const RopeQKVArgs& a, int row0, const float* v, int n, const float* pre,
                                           int pos) {
  {
    if (pos < 0) pos = __ldcg(a.d_pos);
    const uint32_t half = a.head_dim / 2;
    const uint32_t p = (uint32_t)row0 + a.row_base;
    if (p < a.q_rows + a.kv_rows) {
      if (n < 2) return;
      const bool isq = p < a.q_rows;
      const uint32_t j = (isq ? p : p - a.q_rows) / 2;
      const uint32_t h = j / half, i = j % half;
      const float2 cs = pre ? make_float2(pre[0], pre[1]) : a.rope_cs[(size_t)pos * half + i];
      float x0 = v[0], x1 = v[1];
      if (a.bias) {
        x0 = __fadd_rn(x0, __ldg(a.bias + p));
        x1 = __fadd_rn(x1, __ldg(a.bias + p + 1));
      }
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
      for (int s = 0; s < n; s++) {
        const uint32_t o = p + s - a.q_rows - a.kv_rows;
        const uint32_t h = o / a.head_dim, dd = o % a.head_dim;
        const float x = a.bias ? __fadd_rn(v[s], __ldg(a.bias + p + s)) : v[s];
        a.v_cur[o] = x;
        const size_t c = ((size_t)h * a.max_seq + pos) * a.head_dim + dd;
        if (a.kv_f32) ((float*)a.vcache)[c] = x;
        else ((__half*)a.vcache)[c] = __float2half_rn(x);
      }
    }
  }
}

struct EpiSwiGLU {
  static constexpr bool kPre = false;
  float* act;
  __device__ void pre_begin() {}
  __device__ float pre_load(uint32_t) { return 0.f; }
  // rows (2j, 2j+1) = (gate_j, up_j); silu(g) = g/(1+exp(-g)) then * up
  // (compute.rs:337-350, model_executor.rs:229-230)
  __device__ void operator()(int row0, const float* v, int n, const float* = nullptr) {
    if (n < 2) return;
    const float g = v[0], u = v[1];
    const float s = g / (1.0f + expf(-g));
    act[row0 >> 1] = __fmul_rn(s, u);
  }
  __device__ void flush() {}
  __device__ void tile_done(uint32_t) {}
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
  static constexpr bool kPre = false;
  float* logits;
  unsigned long long* key;
  uint32_t row_offset;
  unsigned long long best;
  __device__ void pre_begin() {}
  __device__ float pre_load(uint32_t) { return 0.f; }
  __device__ void operator()(int row0, const float* v, int n, const float* = nullptr) {
    for (int i = 0; i < n; i++) {
      if (logits) logits[row0 + i] = v[i];
      const unsigned long long k = argmax_key(v[i], row_offset + row0 + i);
      best = k > best ? k : best;
    }
  }
  // End of kernel, every lane of every warp: warp maximum, one atomic per warp.
  __device__ void flush() {
    unsigned long long b = best;
#pragma unroll
    for (int o = 16; o; o >>= 1) {
      const unsigned long long t = __shfl_xor_sync(0xffffffffu, b, o);
      b = t > b ? t : b;
    }
    if ((threadIdx.x & 31) == 0 && b) atomicMax(key, b);
  }
  __device__ void tile_done(uint32_t) {}
};

// ---------------------------------------------------------------------------
// quantized GEMV over the tiled layout
// ---------------------------------------------------------------------------
constexpr int QG_WARPS = 16;
constexpr int QG_THREADS = QG_WARPS * 32;

// Per format: CE elements per chunk, SW scale words per row and chunk, XSF the
// factor on the per-group x sums, GE elements per group, PB bytes per piece of
// the 64 rows, IB bytes per item.
template <int FMT>
struct QTraits;
// Q4_K: a chunk is one super-block; piece c is sub-block pair c (byte l: element
//       64c+l in the low nibble, 64c+32+l in the high one; quant.rs:235-248).
template <>
struct QTraits<T_Q4_K> {
  static constexpr int CE = 256, SW = 4, XSF = 1, GE = 32, PB = QT_ROWS * 32, IB = QT_ITEM_BYTES;
};
// Q4_0: a chunk is 8 blocks; piece c is blocks 2c, 2c+1 (block byte j: element j
//       low, 16+j high; value (q-8)*d, quant.rs:104-112).
template <>
struct QTraits<T_Q4_0> {
  static constexpr int CE = 256, SW = 4, XSF = 8, GE = 32, PB = QT_ROWS * 32, IB = QT_ITEM_BYTES;
};
// Q8_0: a chunk is 4 blocks; piece c is block c (value q*d, quant.rs:176-180),
//       bytes biased to q+128 on the fly.
template <>
struct QTraits<T_Q8_0> {
  static constexpr int CE = 128, SW = 2, XSF = 128, GE = 32, PB = QT_ROWS * 32, IB = QT_ITEM_BYTES;
};
// Q6_K: a chunk is half a super-block; piece c is sub-blocks 2c, 2c+1 (three
//       words each, six_bit_words; value (d*sc)*(u-32), quant.rs:376-406); the
//       header is 8 int8 scales and the f16 d.
template <>
struct QTraits<T_Q6_K> {
  static constexpr int CE = 128, SW = 3, XSF = 32, GE = 16, PB = QT_ROWS * Q6_PIECE_BYTES,
                       IB = QT_ROWS * Q6_CHUNK_BYTES;
};
// Q3_K, Q2_K: a chunk is one super-block; piece c is groups 4c..4c+3, word pair p
//       of the piece group 4c+p (elements 0-7 low nibbles, 8-15 high); values
//       d*sc*(u-4) (Q3_K, quant.rs:506-574) and d*sc*u - dmin*m (Q2_K, :443-474);
//       the header is 16 group scale bytes and d (Q2_K: d, dmin).
template <>
struct QTraits<T_Q3_K> {
  static constexpr int CE = 256, SW = 5, XSF = 4, GE = 16, PB = QT_ROWS * 32, IB = QT_ITEM_BYTES;
};
template <>
struct QTraits<T_Q2_K> {
  static constexpr int CE = 256, SW = 5, XSF = 1, GE = 16, PB = QT_ROWS * 32, IB = QT_ITEM_BYTES;
};
// Q5_K: the same words; piece c is 32-element sub-block c of the chunk (value
//       d*sc*u - dmin*m, quant.rs:303-343); the header is 4 scales, 4 mins, d, dmin.
template <>
struct QTraits<T_Q5_K> {
  static constexpr int CE = 128, SW = 3, XSF = 1, GE = 32, PB = QT_ROWS * Q6_PIECE_BYTES,
                       IB = QT_ROWS * Q6_CHUNK_BYTES;
};

// Bit offset of the field holding element k (0..7) of a word pair (A, B) in
// the decode below; high nibbles sit 4 bits above the low ones.
//   k:   0  1  2  3  4  5  6  7
//   off: 0  8 16  0  0  8 16  8
__device__ __forceinline__ int pair_off(int k) { return (k & 3) == 3 ? (k >> 2) * 8 : (k & 3) * 8; }

// Field offset of chunk element e.
template <int FMT>
__device__ __forceinline__ int qfield_off(int e) {
  if (FMT == T_Q6_K || FMT == T_Q5_K) return 6 * (e & 3);  // element t of a 16-group: field t%4 of its word
  if (FMT == T_Q8_0) return pair_off(e & 7);
  if (FMT == T_Q3_K || FMT == T_Q2_K) return pair_off(e & 7) + ((e & 15) >= 8 ? 4 : 0);  // element t of a group
  const int u = e & 63;
  const bool hi = FMT == T_Q4_K ? (u >= 32) : ((u & 31) >= 16);
  return pair_off(u & 7) + (hi ? 4 : 0);
}

// 16 nibbles of the word pair (A, B) = bytes 0..7: the low nibble of byte k
// against xl[k], the high nibble against xh[k].  P gathers the top bytes of A
// and B below bit 16.
__device__ __forceinline__ void q4_pair(uint32_t A, uint32_t B, const float4& xl0, const float4& xl1,
                                        const float4& xh0, const float4& xh1, float2& lo, float2& hi) {
  const uint32_t P = __byte_perm(A, B, 0x0073);
  lo = __ffma2_rn(ff2(as_f(A & 0xFu), as_f(A & 0xF00u)), ff2(xl0.x, xl0.y), lo);
  lo = __ffma2_rn(ff2(as_f(A & 0xF0000u), as_f(P & 0xFu)), ff2(xl0.z, xl0.w), lo);
  lo = __ffma2_rn(ff2(as_f(B & 0xFu), as_f(B & 0xF00u)), ff2(xl1.x, xl1.y), lo);
  lo = __ffma2_rn(ff2(as_f(B & 0xF0000u), as_f(P & 0xF00u)), ff2(xl1.z, xl1.w), lo);
  hi = __ffma2_rn(ff2(as_f(A & 0xF0u), as_f(A & 0xF000u)), ff2(xh0.x, xh0.y), hi);
  hi = __ffma2_rn(ff2(as_f(A & 0xF00000u), as_f(P & 0xF0u)), ff2(xh0.z, xh0.w), hi);
  hi = __ffma2_rn(ff2(as_f(B & 0xF0u), as_f(B & 0xF000u)), ff2(xh1.x, xh1.y), hi);
  hi = __ffma2_rn(ff2(as_f(B & 0xF00000u), as_f(P & 0xF000u)), ff2(xh1.z, xh1.w), hi);
}
// Half of q4_pair: the low (HI = false) or the high nibbles of bytes 0..7 of
// (A, B) against x0 (bytes 0-3) and x1 (bytes 4-7), into acc; P = byte_perm(A, B, 0x0073).
template <bool HI>
__device__ __forceinline__ void q4_half(uint32_t A, uint32_t B, uint32_t P, const float4& x0, const float4& x1,
                                        float2& acc) {
  constexpr uint32_t s = HI ? 4 : 0;
  acc = __ffma2_rn(ff2(as_f(A & (0xFu << s)), as_f(A & (0xF00u << s))), ff2(x0.x, x0.y), acc);
  acc = __ffma2_rn(ff2(as_f(A & (0xF0000u << s)), as_f(P & (0xFu << s))), ff2(x0.z, x0.w), acc);
  acc = __ffma2_rn(ff2(as_f(B & (0xFu << s)), as_f(B & (0xF00u << s))), ff2(x1.x, x1.y), acc);
  acc = __ffma2_rn(ff2(as_f(B & (0xF0000u << s)), as_f(P & (0xF00u << s))), ff2(x1.z, x1.w), acc);
}
// 8 signed bytes of (A, B), biased to q+128, against x[k].
__device__ __forceinline__ void q8_pair(uint32_t A, uint32_t B, const float4& x0, const float4& x1, float2& s) {
  constexpr uint32_t M = 0x80808080u;
  const uint32_t P = __byte_perm(A, B, 0x0073);
  s = __ffma2_rn(ff2(as_f((A ^ M) & 0xFFu), as_f((A ^ M) & 0xFF00u)), ff2(x0.x, x0.y), s);
  s = __ffma2_rn(ff2(as_f((A ^ M) & 0xFF0000u), as_f((P ^ M) & 0xFFu)), ff2(x0.z, x0.w), s);
  s = __ffma2_rn(ff2(as_f((B ^ M) & 0xFFu), as_f((B ^ M) & 0xFF00u)), ff2(x1.x, x1.y), s);
  s = __ffma2_rn(ff2(as_f((B ^ M) & 0xFF0000u), as_f((P ^ M) & 0xFF00u)), ff2(x1.z, x1.w), s);
}

// 16 six-bit fields of a Q6_K sub-block's words (A, B, C) against x[t]: P
// gathers the top bytes of A, B and C below bit 24.
__device__ __forceinline__ void q6_sub(uint32_t A, uint32_t B, uint32_t C, const float4& x0, const float4& x1,
                                       const float4& x2, const float4& x3, float2& s) {
  const uint32_t P = __byte_perm(__byte_perm(A, B, 0x0073), C, 0x0710);
  s = __ffma2_rn(ff2(as_f(A & 0x3Fu), as_f(A & 0xFC0u)), ff2(x0.x, x0.y), s);
  s = __ffma2_rn(ff2(as_f(A & 0x3F000u), as_f(A & 0xFC0000u)), ff2(x0.z, x0.w), s);
  s = __ffma2_rn(ff2(as_f(B & 0x3Fu), as_f(B & 0xFC0u)), ff2(x1.x, x1.y), s);
  s = __ffma2_rn(ff2(as_f(B & 0x3F000u), as_f(B & 0xFC0000u)), ff2(x1.z, x1.w), s);
  s = __ffma2_rn(ff2(as_f(C & 0x3Fu), as_f(C & 0xFC0u)), ff2(x2.x, x2.y), s);
  s = __ffma2_rn(ff2(as_f(C & 0x3F000u), as_f(C & 0xFC0000u)), ff2(x2.z, x2.w), s);
  s = __ffma2_rn(ff2(as_f(P & 0x3Fu), as_f(P & 0xFC0u)), ff2(x3.x, x3.y), s);
  s = __ffma2_rn(ff2(as_f(P & 0x3F000u), as_f(P & 0xFC0000u)), ff2(x3.z, x3.w), s);
}
// Signed byte k of w as a float (Q6_K sub-block scales).
__device__ __forceinline__ float sbyte_f(uint32_t w, int k) { return (float)((int)(w << (24 - 8 * k)) >> 24); }
// A Q6_K piece row (16-byte plane word 0-3 at pa, 8-byte plane words 4-5 at
// pb) and a Q6_K header row (scales at pa, d at pb), under a predicate.
__device__ __forceinline__ void ldg_q6_piece_if(bool on, const uint8_t* pa, const uint8_t* pb, uint32_t (&w)[8]) {
  asm volatile(
      "{ .reg .pred q; setp.ne.u32 q, %8, 0;\n"
      "@q ld.global.nc.L1::no_allocate.v4.b32 {%0,%1,%2,%3}, [%6];\n"
      "@q ld.global.nc.L1::no_allocate.v2.b32 {%4,%5}, [%7]; }"
      : "+r"(w[0]), "+r"(w[1]), "+r"(w[2]), "+r"(w[3]), "+r"(w[4]), "+r"(w[5])
      : "l"(pa), "l"(pb), "r"((uint32_t)on));
}
__device__ __forceinline__ void ldg_q6_hdr_if(bool on, const uint8_t* pa, const uint8_t* pb, uint32_t (&h)[3]) {
  asm volatile(
      "{ .reg .pred q; setp.ne.u32 q, %5, 0;\n"
      "@q ld.global.nc.L1::no_allocate.v2.b32 {%0,%1}, [%3];\n"
      "@q ld.global.nc.L1::no_allocate.b32 %2, [%4]; }"
      : "+r"(h[0]), "+r"(h[1]), "+r"(h[2])
      : "l"(pa), "l"(pb), "r"((uint32_t)on));
}

// A 20-byte header row (16 bytes at pa, 4 at pb) under a predicate.
__device__ __forceinline__ void ldg_hdr20_if(bool on, const uint8_t* pa, const uint8_t* pb, uint32_t (&h)[5]) {
  asm volatile(
      "{ .reg .pred q; setp.ne.u32 q, %7, 0;\n"
      "@q ld.global.nc.L1::no_allocate.v4.b32 {%0,%1,%2,%3}, [%5];\n"
      "@q ld.global.nc.L1::no_allocate.b32 %4, [%6]; }"
      : "+r"(h[0]), "+r"(h[1]), "+r"(h[2]), "+r"(h[3]), "+r"(h[4])
      : "l"(pa), "l"(pb), "r"((uint32_t)on));
}

// f16 block scale -> f32: hardware conversion, or the reference's decode when
// the matrix holds subnormal scales.
template <bool QUIRK>
__device__ __forceinline__ float scale_f(uint32_t bits16) {
  if constexpr (QUIRK) return h2f(bits16 & 0xFFFFu);
  else return __half2float(__ushort_as_half((unsigned short)(bits16 & 0xFFFFu)));
}
// Exact float of byte k of w.
__device__ __forceinline__ float byte_f(uint32_t w, int k) {
  return __uint_as_float(__byte_perm(w, 0x4B000000u, 0x7650u + k)) - 8388608.0f;
}
__device__ __forceinline__ float4 lds4(const float* p) { return *reinterpret_cast<const float4*>(p); }

// floor(a * b / c); in 32-bit arithmetic when the product fits (`narrow`), as it
// does for the piece splits of every matrix shape in use.
__device__ __forceinline__ uint64_t muldiv(uint64_t a, uint64_t b, uint64_t c, bool narrow) {
  return narrow ? (uint64_t)((uint32_t)(a * b) / (uint32_t)c) : a * b / c;
}
// a / b and a % b, likewise (a < 2^32 when narrow).
__device__ __forceinline__ uint64_t div_n(uint64_t a, uint32_t b, bool narrow) {
  return narrow ? (uint64_t)((uint32_t)a / b) : a / b;
}
__device__ __forceinline__ uint32_t mod_n(uint64_t a, uint32_t b, bool narrow) {
  return narrow ? (uint32_t)a % b : (uint32_t)(a % b);
}
// ceil(a * b / c), likewise.
__device__ __forceinline__ uint64_t muldiv_up(uint64_t a, uint64_t b, uint64_t c, bool narrow) {
  return narrow ? (uint64_t)(((uint32_t)(a * b) + (uint32_t)c - 1) / (uint32_t)c) : (a * b + c - 1) / c;
}
// Arrival on a tile counter: release (the warp's partial stores, ordered before
// this lane by a __syncwarp) and acquire (of the partials the other arrivals
// released) in one round trip.
__device__ __forceinline__ unsigned arrive_acq_rel(unsigned* p, unsigned v) {
  unsigned old;
  asm volatile("atom.acq_rel.gpu.global.add.u32 %0, [%1], %2;" : "=r"(old) : "l"(p), "r"(v) : "memory");
  return old;
}

// A GEMV that pulls its x from a tensor-parallel sum (PeerLink::pull_site): wait,
// bounded (about a second, then bit 0 of the error word), until every rank's
// arrival counter of the site holds this use's count (generation x the producer's
// CTAs), then count this CTA in; the last CTA moves the call site to the next
// generation.  One lane per rank polls; the CTA barrier after it orders the
// receive-area reads after the arrivals.
__device__ __forceinline__ void peer_pull_wait(const PeerLink& pl) {
  const PeerSum& P = pl.P;
  const int site = pl.pull_site;
  const unsigned e = *reinterpret_cast<volatile const unsigned*>(P.fgen + site) + 1;
  if (threadIdx.x < 32) {
    bool ok = true;
    if ((int)threadIdx.x < P.n_ranks)
      ok = wait_count_sys(P.flags[P.rank] + ((size_t)threadIdx.x * P.sites + site + 1) * P.max_ctas - 1,
                          e * (unsigned)pl.push_ctas);
    if (!__all_sync(0xffffffffu, ok) && threadIdx.x == 0) atomicOr(P.err, 1u);
  }
  __syncthreads();
  if (threadIdx.x == 0 && atomicAdd(P.done + site, 1u) == gridDim.x - 1) {
    P.fgen[site] = e;
    P.done[site] = 0u;
  }
}

// The quantized GEMV over every CTA of the grid.  `wait()` runs before the
// first read of x (griddepcontrol.wait: the previous kernel's completion); x and
// the residual input are read through L2.
// PULL: x comes from a tensor-parallel sum (PeerLink *pl), a separate instance so
// the plain GEMV carries none of it.
template <int FMT, bool QUIRK, int NW = QG_WARPS, bool PULL = false, class Epi, class Wait>
__device__ __forceinline__ void qgemv_body(const PackedMat& W, const float* __restrict__ x,
                                           const float* __restrict__ nw, float eps, float* __restrict__ part,
                                           unsigned* __restrict__ cnt, Epi& epi, float* smem, Wait&& wait,
                                           const PeerLink* pl = nullptr) {
  using T = QTraits<FMT>;
  constexpr int CE = T::CE, SW = T::SW, GE = T::GE, NG = CE / GE, SB = SW * 4;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  constexpr int NP = QT_PIECES;
  const uint32_t nk = W.nk, ntiles = W.Mp / QT_ROWS, tp = nk * NP;  // tp: pieces per tile
  // The work is split in pieces (item i = pieces NP*i .. NP*i+NP-1), so that the
  // warps' shares differ by at most one piece; a warp loads and decodes whole
  // items but only its pieces of the first and last one.
  const uint64_t N = (uint64_t)ntiles * nk, P = N * NP;
  const uint64_t Wt = (uint64_t)gridDim.x * NW;
  const uint64_t g0 = (uint64_t)blockIdx.x * NW;
  const bool narrow = P * Wt < (1ull << 32);
  const uint64_t pa = muldiv(P, g0 + warp, Wt, narrow), pb = muldiv(P, g0 + warp + 1, Wt, narrow);  // this warp's
  const uint64_t cpa = muldiv(P, g0, Wt, narrow), cpb = muldiv(P, g0 + NW, Wt, narrow);         // this CTA's
  const uint64_t ia = pa / NP, ib = pa < pb ? (pb + NP - 1) / NP : ia;      // items touched by the warp
  const uint64_t ca = cpa / NP, cb = (cpb + NP - 1) / NP;                   // ... by the CTA
  auto plo = [&](uint64_t i) { return i * NP < pa ? (int)(pa - i * NP) : 0; };         // first piece of item i
  auto phi = [&](uint64_t i) { return (i + 1) * NP > pb ? (int)(pb - i * NP) : NP; };  // end piece of item i
  // chunks this CTA stages: all of them, or the (possibly wrapping) window it covers
  uint32_t kc0 = 0, nst = nk;
  if (cb - ca < nk) {
    kc0 = mod_n(ca, nk, narrow);
    nst = (uint32_t)(cb - ca);
  }
  float* sx = smem;                               // [nst][CE] pre-scaled x
  float* sxs = sx + (size_t)nst * CE;             // [nst][NG] XSF * (sum of each GE elements)
  float* sws = sxs + (size_t)nst * NG;            // [NW][64] epilogue staging
  float* sslot = sws + NW * 64;             // [NW*2][64] partial tile sums of each warp
  int* stile = reinterpret_cast<int*>(sslot + NW * 2 * 64);  // [NW*2] their tiles (-1: none)
  float* sred = reinterpret_cast<float*>(stile + NW * 2);     // [40]
  float* sepi = sred + 40;                                          // [NW * 32] prefetched epilogue inputs
  float* ws = sws + warp * 64;
  // Epilogue inputs of the rows of the tiles this CTA touches (the only tiles it
  // can finish), when they fit: fetched after wait() and held in a register
  // while the CTA multiplies.
  const uint32_t etl = (uint32_t)div_n(cpa, tp, narrow);
  const uint32_t eth = cpb > cpa ? (uint32_t)div_n(cpb - 1, tp, narrow) + 1 : etl;
  const bool epre = Epi::kPre && (eth - etl) * QT_ROWS <= (uint32_t)(NW * 32);
  float epf = 0.f;

  uint32_t w[2][4][8];  // [row r / r+32][piece][word] of the chunk in flight
  uint32_t h[2][SW];    // its scale bytes
  auto load_piece = [&](uint64_t i, int c) {
    if constexpr (FMT == T_Q6_K || FMT == T_Q5_K) {
      const uint8_t* q = W.qs + i * T::IB + c * T::PB;
      ldg_q6_piece_if(true, q + lane * 16, q + QT_ROWS * 16 + lane * 8, w[0][c]);
      ldg_q6_piece_if(true, q + (lane + 32) * 16, q + QT_ROWS * 16 + (lane + 32) * 8, w[1][c]);
    } else {
      const uint8_t* q = W.qs + i * QT_ITEM_BYTES + c * (QT_ROWS * 32) + lane * 32;
      ldg256(q, w[0][c]);
      ldg256(q + 32 * 32, w[1][c]);
    }
  };
  auto load_hdr = [&](uint64_t i) {
    if constexpr (FMT == T_Q6_K || FMT == T_Q5_K) {
      const uint8_t* s = W.sc + i * (QT_ROWS * SB);
      ldg_q6_hdr_if(true, s + lane * 8, s + QT_ROWS * 8 + lane * 4, h[0]);
      ldg_q6_hdr_if(true, s + (lane + 32) * 8, s + QT_ROWS * 8 + (lane + 32) * 4, h[1]);
    } else if constexpr (FMT == T_Q3_K || FMT == T_Q2_K) {
      const uint8_t* s = W.sc + i * (QT_ROWS * SB);
      ldg_hdr20_if(true, s + lane * 16, s + QT_ROWS * 16 + lane * 4, h[0]);
      ldg_hdr20_if(true, s + (lane + 32) * 16, s + QT_ROWS * 16 + (lane + 32) * 4, h[1]);
    } else if constexpr (SW == 4) {
      const uint8_t* s = W.sc + (i * QT_ROWS + lane) * SB;
      ldg128(s, h[0]);
      ldg128(s + 32 * SB, h[1]);
    } else {
      const uint8_t* s = W.sc + (i * QT_ROWS + lane) * SB;
      ldg64(s, h[0]);
      ldg64(s + 32 * SB, h[1]);
    }
  };
  // branch-free forms for the hot path (nothing is read when `on` is false)
  auto load_piece_if = [&](bool on, uint64_t i, int c) {
    if constexpr (FMT == T_Q6_K || FMT == T_Q5_K) {
      const uint8_t* q = W.qs + i * T::IB + c * T::PB;
      ldg_q6_piece_if(on, q + lane * 16, q + QT_ROWS * 16 + lane * 8, w[0][c]);
      ldg_q6_piece_if(on, q + (lane + 32) * 16, q + QT_ROWS * 16 + (lane + 32) * 8, w[1][c]);
    } else {
      const uint8_t* q = W.qs + i * QT_ITEM_BYTES + c * (QT_ROWS * 32) + lane * 32;
      ldg256_if(on, q, w[0][c]);
      ldg256_if(on, q + 32 * 32, w[1][c]);
    }
  };
  auto load_hdr_if = [&](bool on, uint64_t i) {
    if constexpr (FMT == T_Q6_K || FMT == T_Q5_K) {
      const uint8_t* s = W.sc + i * (QT_ROWS * SB);
      ldg_q6_hdr_if(on, s + lane * 8, s + QT_ROWS * 8 + lane * 4, h[0]);
      ldg_q6_hdr_if(on, s + (lane + 32) * 8, s + QT_ROWS * 8 + (lane + 32) * 4, h[1]);
    } else if constexpr (FMT == T_Q3_K || FMT == T_Q2_K) {
      const uint8_t* s = W.sc + i * (QT_ROWS * SB);
      ldg_hdr20_if(on, s + lane * 16, s + QT_ROWS * 16 + lane * 4, h[0]);
      ldg_hdr20_if(on, s + (lane + 32) * 16, s + QT_ROWS * 16 + (lane + 32) * 4, h[1]);
    } else if constexpr (SW == 4) {
      const uint8_t* s = W.sc + (i * QT_ROWS + lane) * SB;
      ldg128_if(on, s, h[0]);
      ldg128_if(on, s + 32 * SB, h[1]);
    } else {
      const uint8_t* s = W.sc + (i * QT_ROWS + lane) * SB;
      ldg64_if(on, s, h[0]);
      ldg64_if(on, s + 32 * SB, h[1]);
    }
  };

  // The first item's weights, before wait(): with programmatic dependent launch
  // they stream in while the previous kernel finishes.
  if (ia < ib) {
    load_hdr(ia);
    const int lo = plo(ia), hi = phi(ia);
#pragma unroll
    for (int c = 0; c < NP; c++)
      if (c >= lo && c < hi) load_piece(ia, c);
  }

  wait();
  // x pulled from a tensor-parallel sum: the ranks' rows of the site's parity half,
  // summed in rank order (the order of the sum kernel, so the same values)
  const float* rb = nullptr;
  if constexpr (PULL) {
    peer_pull_wait(*pl);
    rb = pl->P.recv[pl->P.rank] + (size_t)(pl->pull_site & 1) * pl->P.n_ranks * pl->P.n_max;
  }
  auto ldx4 = [&](uint32_t i) -> float4 {  // x[i .. i+3]
    if constexpr (!PULL) return __ldcg(reinterpret_cast<const float4*>(x + i));
    float4 s4 = make_float4(0.f, 0.f, 0.f, 0.f);
    for (int r = 0; r < pl->P.n_ranks; r++) {
      const float4 t = __ldcv(reinterpret_cast<const float4*>(rb + (size_t)r * pl->P.n_max + i));
      s4.x += t.x;
      s4.y += t.y;
      s4.z += t.z;
      s4.w += t.w;
    }
    return s4;
  };
  if (lane < 2) stile[2 * warp + lane] = -1;
  if (epre) epi.pre_begin();
  // One pass over x.  The window is staged as x*nw: RMSNorm's 1/rms is applied
  // to every finished row instead (the product is linear in x), so with RMSNorm
  // the loads for the sum of squares (all of x, in the same per-thread order as
  // block_sumsq_v4, so every CTA gets the same rms) are in flight together with
  // the window's.  float4 q of the window = elements 4q..4q+3; 8 consecutive
  // threads = one 32-element group, 4 one 16-element group (warp-uniform: windows
  // are multiples of 128).
  constexpr int SU = 2;
  const uint32_t nq = nst * CE / 4;            // float4s of the window
  const uint32_t KQ = nw ? W.K / 4 : 0;        // float4s of x for the sum of squares
  const bool win_is_x = nst == nk;             // then kc0 == 0: window float4 q is x float4 q
  const uint32_t nloop = nq > KQ ? nq : KQ;
  float ss = 0.f;
  for (uint32_t q0 = (uint32_t)tid; q0 < nloop; q0 += SU * (NW * 32)) {
    float4 xv[SU], wv[SU], sv[SU];
#pragma unroll
    for (int u = 0; u < SU; u++) {
      const uint32_t q = q0 + u * (NW * 32), f = 4 * q, s = f / CE, e = f % CE;
      uint32_t kc = kc0 + s;
      if (kc >= nk) kc -= nk;
      const uint32_t gi = kc * CE + e;
      const bool in = q < nq && gi < W.K;  // K is a multiple of 32: a float4 is wholly in or out
      xv[u] = in ? ldx4(gi) : make_float4(0.f, 0.f, 0.f, 0.f);
      wv[u] = in && nw ? __ldcg(reinterpret_cast<const float4*>(nw + gi)) : make_float4(1.f, 1.f, 1.f, 1.f);
      sv[u] = !win_is_x && q < KQ ? ldx4(4 * q) : make_float4(0.f, 0.f, 0.f, 0.f);
    }
#pragma unroll
    for (int u = 0; u < SU; u++) {
      const uint32_t q = q0 + u * (NW * 32), f = 4 * q, e = f % CE;
      if (q < KQ) {
        const float4 t = win_is_x ? xv[u] : sv[u];
        if constexpr (PULL)
          if (blockIdx.x == 0) reinterpret_cast<float4*>(pl->hidden)[q] = t;  // the sum, for later residuals
        ss = fmaf(t.x, t.x, ss);
        ss = fmaf(t.y, t.y, ss);
        ss = fmaf(t.z, t.z, ss);
        ss = fmaf(t.w, t.w, ss);
      }
      if (q >= nq) continue;
      const float4 v = make_float4(xv[u].x * wv[u].x, xv[u].y * wv[u].y, xv[u].z * wv[u].z, xv[u].w * wv[u].w);
      *reinterpret_cast<float4*>(sx + f) =
          make_float4(v.x * prescale(qfield_off<FMT>(e)), v.y * prescale(qfield_off<FMT>(e + 1)),
                      v.z * prescale(qfield_off<FMT>(e + 2)), v.w * prescale(qfield_off<FMT>(e + 3)));
      float gs = ((v.x + v.y) + v.z) + v.w;
      gs += __shfl_xor_sync(0xffffffffu, gs, 1);
      gs += __shfl_xor_sync(0xffffffffu, gs, 2);
      if constexpr (GE == 32) gs += __shfl_xor_sync(0xffffffffu, gs, 4);
      if ((lane & (GE / 4 - 1)) == 0) sxs[f / GE] = gs * (float)T::XSF;
    }
  }
  float rms = 1.f;  // rms = sqrt(sum/n + eps)  (compute.rs:312-317)
  if (nw) {
#pragma unroll
    for (int o = 16; o; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
    if (lane == 0) sred[warp] = ss;
  }
  __syncthreads();
  if (nw) {
    float t = 0.f;
    for (int w2 = 0; w2 < NW; w2++) t += sred[w2];
    rms = rms_of(t, (int)W.K, eps);
  }
  griddep_launch();
  if (epre) {
    const uint32_t r = etl * QT_ROWS + tid;
    if (r < eth * QT_ROWS && r < W.M) epf = epi.pre_load(r);
  }

  // finished rows of a tile -> epilogue, two consecutive rows per lane
  // (`pre`: after the CTA barrier that publishes the prefetched inputs)
  auto emit = [&](uint32_t tile, float v0, float v1, bool pre) {
    if (nw) {  // RMSNorm's division, once per row: W.(x*nw) / rms
      v0 = v0 / rms;
      v1 = v1 / rms;
    }
    ws[lane] = v0;
    ws[32 + lane] = v1;
    __syncwarp();
    const uint32_t r = tile * QT_ROWS + 2 * lane;
    const float v[2] = {ws[2 * lane], ws[2 * lane + 1]};
    if (r < W.M) epi((int)r, v, (int)min(2u, W.M - r), pre && epre ? sepi + (r - etl * QT_ROWS) : nullptr);
    __syncwarp();
    epi.tile_done(tile);
  };
  // End of this warp's run of `len` pieces in `tile`: a whole tile goes to the
  // epilogue, a part (at most two per warp: the ends of its range) waits in
  // shared memory for the CTA-level merge.
  int nslot = 0;
  auto flush = [&](uint32_t tile, uint32_t len, float v0, float v1) {
    if (len == tp) {
      emit(tile, v0, v1, false);
      return;
    }
    float* p = sslot + (2 * warp + nslot) * 64;
    p[lane] = v0;
    p[32 + lane] = v1;
    if (lane == 0) stile[2 * warp + nslot] = (int)tile;
    nslot++;
  };

  uint32_t tile = (uint32_t)div_n(ia, nk, narrow), kc = mod_n(ia, nk, narrow), len = 0;
  float acc0 = 0.f, acc1 = 0.f;
  for (uint64_t i = ia; i < ib; i++) {
    uint32_t slot = kc + nk - kc0;
    if (slot >= nk) slot -= nk;
    const float* xc = sx + (size_t)slot * CE;
    const float* xsc = sxs + (size_t)slot * NG;
    uint32_t hc[2][SW];
#pragma unroll
    for (int s = 0; s < 2; s++)
#pragma unroll
      for (int k = 0; k < SW; k++) hc[s][k] = h[s][k];
    const bool more = i + 1 < ib;
    const int lo = plo(i), hi = phi(i), hi1 = more ? phi(i + 1) : 0;  // the next item starts at piece 0
    load_hdr_if(more, i + 1);
    float acc[2] = {0.f, 0.f};
    // Pieces outside [lo, hi) (first and last item of the warp's range) are skipped
    // with warp-uniform conditions; one copy of the code serves every item, which
    // measured faster than a separate unconditional copy for whole items.
    if constexpr (FMT == T_Q4_K) {
      // header: d, dmin (f16) | scales[12] (get_scale_min_k4, quant.rs:216-226)
      float d64[2], dmn[2];
      uint32_t scl[2], sch[2], ml[2], mh[2];
#pragma unroll
      for (int s = 0; s < 2; s++) {
        d64[s] = scale_f<QUIRK>(hc[s][0]) * kTwo64;
        dmn[s] = scale_f<QUIRK>(hc[s][0] >> 16);
        scl[s] = hc[s][1] & 0x3F3F3F3Fu;  // sc[0..3]
        ml[s] = hc[s][2] & 0x3F3F3F3Fu;   // m[0..3]
        sch[s] = (hc[s][3] & 0x0F0F0F0Fu) | ((hc[s][1] >> 2) & 0x30303030u);         // sc[4..7]
        mh[s] = ((hc[s][3] >> 4) & 0x0F0F0F0Fu) | ((hc[s][2] >> 2) & 0x30303030u);  // m[4..7]
      }
      float aS[2] = {0.f, 0.f}, aM[2] = {0.f, 0.f};
#pragma unroll
      for (int c = 0; c < NP; c++) {
        const bool on = c >= lo && c < hi;
        float2 sl[2] = {ff2(0.f, 0.f), ff2(0.f, 0.f)}, sh[2] = {ff2(0.f, 0.f), ff2(0.f, 0.f)};
        if (on) {
#pragma unroll
          for (int j = 0; j < 4; j++) {
            const float* xb = xc + 64 * c + 8 * j;
            const float4 xl0 = lds4(xb), xl1 = lds4(xb + 4), xh0 = lds4(xb + 32), xh1 = lds4(xb + 36);
#pragma unroll
            for (int s = 0; s < 2; s++)
              q4_pair(w[s][c][2 * j], w[s][c][2 * j + 1], xl0, xl1, xh0, xh1, sl[s], sh[s]);
          }
        }
        load_piece_if(c < hi1, i + 1, c);
        if (on) {
          const float xsl = xsc[2 * c], xsh = xsc[2 * c + 1];
#pragma unroll
          for (int s = 0; s < 2; s++) {
            const uint32_t scw = c < 2 ? scl[s] : sch[s], mw = c < 2 ? ml[s] : mh[s];
            const int kb = (2 * c) & 3;
            aS[s] = fmaf(byte_f(scw, kb), sl[s].x + sl[s].y, aS[s]);
            aS[s] = fmaf(byte_f(scw, kb + 1), sh[s].x + sh[s].y, aS[s]);
            aM[s] = fmaf(byte_f(mw, kb), xsl, aM[s]);
            aM[s] = fmaf(byte_f(mw, kb + 1), xsh, aM[s]);
          }
        }
      }
#pragma unroll
      for (int s = 0; s < 2; s++) acc[s] = d64[s] * aS[s] - dmn[s] * aM[s];
    } else if constexpr (FMT == T_Q4_0) {
#pragma unroll
      for (int c = 0; c < NP; c++) {
        const bool on = c >= lo && c < hi;
        float2 sb[2][2];  // [row][block of the piece]: low and high nibbles of a block sum together
#pragma unroll
        for (int s = 0; s < 2; s++)
#pragma unroll
          for (int b = 0; b < 2; b++) sb[s][b] = ff2(0.f, 0.f);
        if (on) {
#pragma unroll
          for (int j = 0; j < 4; j++) {
            const int b = j >> 1;
            const float* xb = xc + 64 * c + 32 * b + 8 * (j & 1);
            const float4 xl0 = lds4(xb), xl1 = lds4(xb + 4), xh0 = lds4(xb + 16), xh1 = lds4(xb + 20);
#pragma unroll
            for (int s = 0; s < 2; s++)
              q4_pair(w[s][c][2 * j], w[s][c][2 * j + 1], xl0, xl1, xh0, xh1, sb[s][b], sb[s][b]);
          }
        }
        load_piece_if(c < hi1, i + 1, c);
        if (!on) continue;
#pragma unroll
        for (int b = 0; b < 2; b++) {
          const float xs8 = xsc[2 * c + b];
#pragma unroll
          for (int s = 0; s < 2; s++) {
            const float d = scale_f<QUIRK>(hc[s][c] >> (16 * b));
            acc[s] = fmaf(d, fmaf(sb[s][b].x + sb[s][b].y, kTwo64, -xs8), acc[s]);
          }
        }
      }
    } else if constexpr (FMT == T_Q6_K) {
      // d*sc_j*(sum_t u_t x_t - 32 sum_t x_t) per sub-block j; u_t x_t arrive
      // scaled by 2^-64, the x sums (sxs) by 32
      float d64[2], dd[2];
#pragma unroll
      for (int s = 0; s < 2; s++) {
        dd[s] = scale_f<QUIRK>(hc[s][2]);
        d64[s] = dd[s] * kTwo64;
      }
      float aS[2] = {0.f, 0.f}, aM[2] = {0.f, 0.f};
#pragma unroll
      for (int c = 0; c < NP; c++) {
        const bool on = c >= lo && c < hi;
        float2 sb[2][2];  // [row][sub-block of the piece]
#pragma unroll
        for (int s = 0; s < 2; s++)
#pragma unroll
          for (int b = 0; b < 2; b++) sb[s][b] = ff2(0.f, 0.f);
        if (on) {
#pragma unroll
          for (int b = 0; b < 2; b++) {
            const float* xb = xc + 32 * c + 16 * b;
            const float4 x0 = lds4(xb), x1 = lds4(xb + 4), x2 = lds4(xb + 8), x3 = lds4(xb + 12);
#pragma unroll
            for (int s = 0; s < 2; s++)
              q6_sub(w[s][c][3 * b], w[s][c][3 * b + 1], w[s][c][3 * b + 2], x0, x1, x2, x3, sb[s][b]);
          }
        }
        load_piece_if(c < hi1, i + 1, c);
        if (!on) continue;
#pragma unroll
        for (int b = 0; b < 2; b++) {
          const int j = 2 * c + b;
          const float xs32 = xsc[j];
#pragma unroll
          for (int s = 0; s < 2; s++) {
            const float scf = sbyte_f(hc[s][j >> 2], j & 3);
            aS[s] = fmaf(scf, sb[s][b].x + sb[s][b].y, aS[s]);
            aM[s] = fmaf(scf, xs32, aM[s]);
          }
        }
      }
#pragma unroll
      for (int s = 0; s < 2; s++) acc[s] = d64[s] * aS[s] - dd[s] * aM[s];
    } else if constexpr (FMT == T_Q3_K || FMT == T_Q2_K) {
      // group G: sum of u x (scaled by 2^-64) with its scale byte; Q3_K subtracts 4*sc*sum(x)
      // with d (x sums staged as 4x), Q2_K m*sum(x) with dmin
      float d64[2], dm[2];
#pragma unroll
      for (int s = 0; s < 2; s++) {
        d64[s] = scale_f<QUIRK>(hc[s][4]) * kTwo64;
        dm[s] = scale_f<QUIRK>(FMT == T_Q3_K ? hc[s][4] : hc[s][4] >> 16);
      }
      float aS[2] = {0.f, 0.f}, aM[2] = {0.f, 0.f};
#pragma unroll
      for (int c = 0; c < NP; c++) {
        const bool on = c >= lo && c < hi;
        if (on) {
#pragma unroll
          for (int p = 0; p < 4; p++) {
            const int G = 4 * c + p;
            const float* xb = xc + 16 * G;
            const float xs = xsc[G];
            // low nibbles (elements 0-7) then high ones (8-15): 8 activations live at a time
            float2 sa[2] = {ff2(0.f, 0.f), ff2(0.f, 0.f)};
            {
              const float4 x0 = lds4(xb), x1 = lds4(xb + 4);
#pragma unroll
              for (int s = 0; s < 2; s++) {
                const uint32_t A = w[s][c][2 * p], B = w[s][c][2 * p + 1];
                q4_half<false>(A, B, __byte_perm(A, B, 0x0073), x0, x1, sa[s]);
              }
            }
            {
              const float4 x0 = lds4(xb + 8), x1 = lds4(xb + 12);
#pragma unroll
              for (int s = 0; s < 2; s++) {
                const uint32_t A = w[s][c][2 * p], B = w[s][c][2 * p + 1];
                q4_half<true>(A, B, __byte_perm(A, B, 0x0073), x0, x1, sa[s]);
              }
            }
#pragma unroll
            for (int s = 0; s < 2; s++) {
              const float S = sa[s].x + sa[s].y;
              if constexpr (FMT == T_Q3_K) {
                const float scf = sbyte_f(hc[s][G >> 2], G & 3);
                aS[s] = fmaf(scf, S, aS[s]);
                aM[s] = fmaf(scf, xs, aM[s]);
              } else {
                const uint32_t sb = (hc[s][G >> 2] >> (8 * (G & 3))) & 0xFFu;
                aS[s] = fmaf((float)(sb & 15u), S, aS[s]);
                aM[s] = fmaf((float)(sb >> 4), xs, aM[s]);
              }
            }
          }
        }
        load_piece_if(c < hi1, i + 1, c);
      }
#pragma unroll
      for (int s = 0; s < 2; s++) acc[s] = d64[s] * aS[s] - dm[s] * aM[s];
    } else if constexpr (FMT == T_Q5_K) {
      // sub-block c = piece c: d*sc_c*sum(u x) - dmin*m_c*sum(x); u x arrive scaled by 2^-64
      float d64[2], dmn[2];
#pragma unroll
      for (int s = 0; s < 2; s++) {
        d64[s] = scale_f<QUIRK>(hc[s][2]) * kTwo64;
        dmn[s] = scale_f<QUIRK>(hc[s][2] >> 16);
      }
      float aS[2] = {0.f, 0.f}, aM[2] = {0.f, 0.f};
#pragma unroll
      for (int c = 0; c < NP; c++) {
        const bool on = c >= lo && c < hi;
        float2 sb[2] = {ff2(0.f, 0.f), ff2(0.f, 0.f)};
        if (on) {
#pragma unroll
          for (int b = 0; b < 2; b++) {
            const float* xb = xc + 32 * c + 16 * b;
            const float4 x0 = lds4(xb), x1 = lds4(xb + 4), x2 = lds4(xb + 8), x3 = lds4(xb + 12);
#pragma unroll
            for (int s = 0; s < 2; s++)
              q6_sub(w[s][c][3 * b], w[s][c][3 * b + 1], w[s][c][3 * b + 2], x0, x1, x2, x3, sb[s]);
          }
        }
        load_piece_if(c < hi1, i + 1, c);
        if (!on) continue;
        const float xs = xsc[c];
#pragma unroll
        for (int s = 0; s < 2; s++) {
          aS[s] = fmaf(byte_f(hc[s][0], c), sb[s].x + sb[s].y, aS[s]);
          aM[s] = fmaf(byte_f(hc[s][1], c), xs, aM[s]);
        }
      }
#pragma unroll
      for (int s = 0; s < 2; s++) acc[s] = d64[s] * aS[s] - dmn[s] * aM[s];
    } else {  // Q8_0
#pragma unroll
      for (int c = 0; c < NP; c++) {
        const bool on = c >= lo && c < hi;
        float2 sa[2] = {ff2(0.f, 0.f), ff2(0.f, 0.f)};
        if (on) {
#pragma unroll
          for (int j = 0; j < 4; j++) {
            const float* xb = xc + 32 * c + 8 * j;
            const float4 x0 = lds4(xb), x1 = lds4(xb + 4);
#pragma unroll
            for (int s = 0; s < 2; s++) q8_pair(w[s][c][2 * j], w[s][c][2 * j + 1], x0, x1, sa[s]);
          }
        }
        load_piece_if(c < hi1, i + 1, c);
        if (!on) continue;
        const float xs128 = xsc[c];
#pragma unroll
        for (int s = 0; s < 2; s++) {
          const float d = scale_f<QUIRK>(hc[s][c >> 1] >> (16 * (c & 1)));
          acc[s] = fmaf(d, fmaf(sa[s].x + sa[s].y, kTwo64, -xs128), acc[s]);
        }
      }
    }
    acc0 += acc[0];
    acc1 += acc[1];
    len += hi - lo;
    if (++kc == nk || !more) {
      flush(tile, len, acc0, acc1);
      acc0 = acc1 = 0.f;
      if (kc == nk) {
        kc = 0;
        tile++;
      }
      len = 0;
    }
  }

  // CTA-level merge.  Slots 2w, 2w+1 are in chunk order, so the parts of a tile
  // are consecutive non-empty slots; the warp holding the first one sums them.
  if (epre) sepi[tid] = epf;
  __syncthreads();
  for (int i = 2 * warp; i < 2 * warp + 2; i++) {
    const int T = stile[i];
    if (T < 0) continue;
    int j = i - 1;
    while (j >= 0 && stile[j] < 0) j--;
    if (j >= 0 && stile[j] == T) continue;
    float s0 = 0.f, s1 = 0.f;
    for (int k = i; k < 2 * NW; k++) {
      const int tk = stile[k];
      if (tk < 0) continue;
      if (tk != T) break;
      s0 += sslot[k * 64 + lane];
      s1 += sslot[k * 64 + 32 + lane];
    }
    const uint64_t t0 = (uint64_t)T * tp;  // first piece of tile T
    const uint64_t a = cpa > t0 ? cpa : t0, b = cpb < t0 + tp ? cpb : t0 + tp;  // this CTA's pieces of T
    if (a == t0 && b == t0 + tp) {
      emit((uint32_t)T, s0, s1, true);
      continue;
    }
    // Across CTAs: publish this CTA's part; the CTA completing the tile sums the
    // parts in piece order (they start at piece 0 and at every CTA boundary).
    const uint32_t len_c = (uint32_t)(b - a);
    float* p = part + a * QT_ROWS;
    __stcg(p + lane, s0);
    __stcg(p + 32 + lane, s1);
    // __syncwarp orders every lane's partial before lane 0's arrival, whose
    // release is cumulative (the same idiom as a CTA barrier followed by one
    // thread's release); its acquire, then __syncwarp, orders the other parts
    // before every lane's loads below
    __syncwarp();
    unsigned old = 0;
    if (lane == 0) old = arrive_acq_rel(cnt + T, len_c);
    old = __shfl_sync(0xffffffffu, old, 0);
    if (old + len_c != tp) continue;
    __syncwarp();
    const uint64_t G = gridDim.x;
    float r0 = 0.f, r1 = 0.f;
    for (uint32_t k = 0; k < tp;) {
      uint32_t ks[8];
      int m = 0;
#pragma unroll
      for (int u = 0; u < 8; u++) {
        if (k < tp) {
          ks[u] = k;
          m = u + 1;
          const uint64_t g = muldiv_up(t0 + k + 1, G, P, narrow);  // first CTA starting after piece t0+k
          const uint64_t nb = muldiv(P, g, G, narrow);               // and its first piece
          k = nb - t0 < tp ? (uint32_t)(nb - t0) : tp;
        }
      }
      float a0[8], a1[8];
#pragma unroll
      for (int u = 0; u < 8; u++)
        if (u < m) {
          a0[u] = __ldcg(part + (t0 + ks[u]) * QT_ROWS + lane);
          a1[u] = __ldcg(part + (t0 + ks[u]) * QT_ROWS + 32 + lane);
        }
#pragma unroll
      for (int u = 0; u < 8; u++)
        if (u < m) {
          r0 += a0[u];
          r1 += a1[u];
        }
    }
    if (lane == 0) cnt[T] = 0;
    emit((uint32_t)T, r0, r1, true);
  }
}

// Dynamic shared memory qgemv_body needs for W on a grid of `grid` CTAs of `nw` warps.
inline size_t qgemv_smem_bytes(const PackedMat& W, int grid, int nw = QG_WARPS) {
  const uint64_t CE = (uint64_t)chunk_elems(W.type);
  // A CTA's pieces [cpa, cpb) number at most ceil(P/grid); the items they touch,
  // floor(cpa/NP) .. ceil(cpb/NP), at most ceil(that/NP) + 1.
  const uint64_t P = (uint64_t)(W.Mp / QT_ROWS) * W.nk * QT_PIECES;
  const uint64_t per_cta = ((P + grid - 1) / grid + QT_PIECES - 1) / QT_PIECES + 1;
  const uint64_t nst = std::min<uint64_t>(W.nk, per_cta);
  return (size_t)(nst * CE + nst * (CE / chunk_group_elems(W.type)) + nw * 64 + nw * 2 * 65 + 40 + nw * 32) *
         sizeof(float);
}

}  // namespace rf
