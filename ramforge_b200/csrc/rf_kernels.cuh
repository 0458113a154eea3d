// rf_kernels.cuh - device data layouts and kernel launchers of the decode engine.
#pragma once
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace rf {

// ggml type ids (types.rs:238-270)
enum : int {
  T_F32 = 0, T_F16 = 1, T_Q4_0 = 2, T_Q5_0 = 6, T_Q8_0 = 8, T_Q2_K = 10, T_Q3_K = 11, T_Q4_K = 12, T_Q5_K = 13,
  T_Q6_K = 14, T_Q8_K = 15
};
// Formats the engine stores as f32, decoded at load exactly as the reference's
// dequantize does (quant.rs:114-154, 579-612): matvec_q5_0/_q8_k decode a block
// and sum deq[j]*x[j] (quant.rs:1050-1490), so the f32 rows give the same products
// up to the order of the sum.
__host__ __device__ inline bool expands_to_f32(int type) { return type == T_Q5_0 || type == T_Q8_K; }
// Q3_K and Q2_K: 2- and 3-bit values held one per nibble, 16-element groups
// (each with its own scale) in one 8-byte word pair, and a 20-byte header.
__host__ __device__ inline bool nibble_group_fields(int type) { return type == T_Q3_K || type == T_Q2_K; }
// The type a matrix of GGUF `type` is stored in on the device.
__host__ __device__ inline int storage_type(int type) { return expands_to_f32(type) ? T_F32 : type; }
// Formats whose values the tiled layout holds as 6-bit fields (Q6_K: 6-bit values;
// Q5_K: 5-bit values, one spare bit each, for the same cheap decode).
__host__ __device__ inline bool six_bit_fields(int type) { return type == T_Q6_K || type == T_Q5_K; }

// Packed device form of one GGUF matrix (n_out rows of n_in elements).
//
// GGUF interleaves per-block scales with quants (Q8_0: 34-byte blocks, Q4_K:
// 144-byte super-blocks).  The engine splits every row into two byte streams at
// load time and reorders them, without changing a single bit of either:
//   qs : the quant bytes;
//   sc : the per-block scale bytes (Q8_0/Q4_0: the f16 d of every 32 elements;
//        Q4_K: the 16-byte {d, dmin, scales[12]} header of every 256 elements).
//
// Quantized types (Q4_K, Q4_0, Q8_0) use the tiled layout the GEMV streams:
// rows are grouped in tiles of 64 (the row count padded with zero rows), every
// row is cut into chunks of 128 quant bytes (256 elements for Q4_K/Q4_0, 128 for
// Q8_0; the row length padded with zero blocks), and one "item" = (tile, chunk)
// is 8 KiB of contiguous qs:
//   qs[((tile*nk + chunk)*4 + piece)*2048 + (row%64)*32 + byte%32]
// where piece = 32-byte quarter of the chunk, so one warp-wide 256-bit load reads
// 1 KiB of consecutive bytes (piece `p` of 32 consecutive rows).  The scale
// bytes of an item are contiguous too: sc[((tile*nk + chunk)*64 + row%64)*SB + b]
// with SB = 16 (Q4_K header; Q4_0: eight f16) or 8 (Q8_0: four f16) bytes.
//
// Q3_K and Q2_K re-encode their quants as nibbles (the values are kept): a chunk
// is one super-block (256 elements, 128 bytes a row, the Q4 piece layout above);
// group G (16 elements) is bytes 8(G%4)..8(G%4)+7 of piece G/4, element t of the
// group in the low (t < 8) or high nibble of byte t%8.  Q3_K holds u = q + 4
// (0..7), Q2_K the 2-bit q.  The 20 header bytes of a row and chunk are a 16-byte
// plane (one scale byte per group: Q3_K the signed scale sc-32, Q2_K the stored
// sc | m << 4) of the item's 64 rows, then a 4-byte plane (f16 d, and Q2_K's f16
// dmin; Q3_K two zero bytes).
constexpr int NG_HDR_BYTES = 20;

// Q6_K and Q5_K re-encode their quants (the values are kept, their bit positions
// are not): a chunk is 128 elements, eight 16-element groups of three 32-bit
// words each (six_bit_words), 96 bytes per row; piece p holds groups 2p and 2p+1
// (24 bytes), stored as a 16-byte plane (words 0-3 of the piece) of the item's 64
// rows followed by an 8-byte plane (words 4-5), so both warp-wide loads stay
// contiguous.  The 12 header bytes of a row and chunk are split the same way: an
// 8-byte plane of the 64 rows, then a 4-byte plane.  Q6_K: the chunk's 8 int8
// scales | f16 d, 2 zero bytes.  Q5_K: the chunk's 4 six-bit scales, 4 mins | f16
// d, f16 dmin.
//
// F32/F16 tensors stay row-major (qs_stride bytes per row, no sc).
struct PackedMat {
  int type;
  uint32_t M, K;        // rows, logical row length
  uint32_t Kp;          // row length padded to whole chunks (F32/F16: whole 32-byte units)
  uint32_t units;       // 32-byte units per row
  uint64_t qs_stride;   // quant bytes per row (padded)
  uint64_t sc_stride;   // scale bytes per row (padded; 0 for F32/F16)
  uint32_t Mp;          // rows padded to the 64-row tile (F32/F16: M)
  uint32_t nk;          // chunks per row (0 for F32/F16)
  uint32_t sbytes;      // scale bytes per row per chunk (0 for F32/F16)
  uint8_t* qs;
  uint8_t* sc;
  // Nonzero when some block scale is a subnormal half: the GEMV then decodes
  // scales the reference's way (h2f) instead of with the hardware conversion.
  // Set at load time (the host scans, or reads back the pack kernel's flag).
  int sub_scales;
};

constexpr int QT_ROWS = 64;          // rows per tile
constexpr int QT_CHUNK_BYTES = 128;  // quant bytes per row per chunk
constexpr int QT_ITEM_BYTES = QT_ROWS * QT_CHUNK_BYTES;
constexpr int QT_PIECES = 4;        // 32-byte pieces of a chunk row: the unit of the GEMV work split

constexpr int Q6_CHUNK_BYTES = 96;  // Q6_K quant bytes per row per chunk
constexpr int Q6_PIECE_BYTES = 24;
constexpr int Q6_HDR_BYTES = 12;

__host__ __device__ inline bool is_tiled(int type) {
  return type == T_Q4_K || type == T_Q4_0 || type == T_Q8_0 || six_bit_fields(type) || nibble_group_fields(type);
}
__host__ __device__ inline int chunk_elems(int type) { return type == T_Q8_0 || six_bit_fields(type) ? 128 : 256; }
__host__ __device__ inline int chunk_scale_bytes(int type) {
  return type == T_Q8_0 ? 8 : six_bit_fields(type) ? Q6_HDR_BYTES : nibble_group_fields(type) ? NG_HDR_BYTES : 16;
}
__host__ __device__ inline int chunk_quant_bytes(int type) {
  return six_bit_fields(type) ? Q6_CHUNK_BYTES : QT_CHUNK_BYTES;
}
// Elements per group of the GEMV's per-group x sums (one scale per group).
__host__ __device__ inline int chunk_group_elems(int type) {
  return type == T_Q6_K || nibble_group_fields(type) ? 16 : 32;
}

// Byte b (0 <= b < qs_stride) of row r's quant bytes.
__host__ __device__ inline uint64_t qs_byte_off(const PackedMat& W, uint32_t r, uint64_t b) {
  if (!is_tiled(W.type)) return (uint64_t)r * W.qs_stride + b;
  if (six_bit_fields(W.type)) {
    const uint64_t item = (uint64_t)(r / QT_ROWS) * W.nk + b / Q6_CHUNK_BYTES;
    const uint32_t o = (uint32_t)(b % Q6_CHUNK_BYTES), p = o / Q6_PIECE_BYTES, pb = o % Q6_PIECE_BYTES;
    const uint64_t base = item * (QT_ROWS * Q6_CHUNK_BYTES) + (uint64_t)p * (QT_ROWS * Q6_PIECE_BYTES);
    return pb < 16 ? base + (r % QT_ROWS) * 16 + pb : base + QT_ROWS * 16 + (r % QT_ROWS) * 8 + (pb - 16);
  }
  const uint64_t item = (uint64_t)(r / QT_ROWS) * W.nk + b / QT_CHUNK_BYTES;
  return (item * 4 + (b / 32) % 4) * (QT_ROWS * 32) + (uint64_t)(r % QT_ROWS) * 32 + b % 32;
}
// Byte b (0 <= b < sc_stride) of row r's scale bytes.
__host__ __device__ inline uint64_t sc_byte_off(const PackedMat& W, uint32_t r, uint64_t b) {
  const uint64_t item = (uint64_t)(r / QT_ROWS) * W.nk + b / W.sbytes;
  if (six_bit_fields(W.type) || nibble_group_fields(W.type)) {  // an A-byte plane, then a 4-byte plane
    const uint32_t A = W.sbytes - 4, o = (uint32_t)(b % W.sbytes);
    const uint64_t base = item * (QT_ROWS * (uint64_t)W.sbytes);
    return o < A ? base + (r % QT_ROWS) * A + o : base + QT_ROWS * A + (r % QT_ROWS) * 4 + (o - A);
  }
  return (item * QT_ROWS + r % QT_ROWS) * W.sbytes + b % W.sbytes;
}

// 6-bit value q+32 of element e (0..255) of a GGUF Q6_K block (BlockQ6K::dequantize,
// quant.rs:376-406: low nibble from ql, high bit pair from qh).
__host__ __device__ inline uint32_t q6k_value(const uint8_t* blk, int e) {
  const int h = e >> 7, l = e & 31, k = (e >> 5) & 3;
  const uint8_t lq = blk[64 * h + l + 32 * (k & 1)];
  const uint32_t lo = k < 2 ? (lq & 15u) : (uint32_t)(lq >> 4);
  return lo | ((uint32_t)((blk[128 + 32 * h + l] >> (2 * k)) & 3) << 4);
}
// 5-bit value q + 16*high of element e (0..255) of a GGUF Q5_K block
// (BlockQ5K::dequantize, quant.rs:303-343): nibble of qs[32g + l] (low for the
// first 32 elements of group g = e/64, high for the next 32), high bit 2g or 2g+1
// of qh[8g + l/8] (the reference's indexing).
__host__ __device__ inline uint32_t q5k_value(const uint8_t* blk, int e) {
  const int g = e >> 6, hi = (e >> 5) & 1, l = e & 31;
  const uint32_t nib = (blk[48 + 32 * g + l] >> (4 * hi)) & 15u;
  return nib | ((uint32_t)((blk[16 + 8 * g + l / 8] >> (2 * g + hi)) & 1) << 4);
}
// get_scale_min of Q4_K/Q5_K (quant.rs:288-299): 6-bit scale and min of sub-block j.
__host__ __device__ inline void k4_scale_min(const uint8_t* s, int j, uint32_t* sc, uint32_t* m) {
  if (j < 4) {
    *sc = s[j] & 63u;
    *m = s[j + 4] & 63u;
  } else {
    *sc = (s[j + 4] & 0xFu) | ((uint32_t)(s[j - 4] >> 6) << 4);
    *m = (uint32_t)(s[j + 4] >> 4) | ((uint32_t)(s[j] >> 6) << 4);
  }
}
// The three packed words of 16 values u0..u15 (< 64): A = u0..u3 at bits 0/6/12/18,
// B = u4..u7, C = u8..u11 likewise, and the top bytes of A, B, C together hold
// u12..u15 at bits 0/6/12/18 of A[31:24] | B[31:24] << 8 | C[31:24] << 16.  Every
// field then lies below bit 24.
__host__ __device__ inline void six_bit_words(const uint32_t u[16], uint32_t out[3]) {
  const uint32_t T = u[12] | (u[13] << 6) | (u[14] << 12) | (u[15] << 18);
  for (int k = 0; k < 3; k++)
    out[k] = u[4 * k] | (u[4 * k + 1] << 6) | (u[4 * k + 2] << 12) | (u[4 * k + 3] << 18) | (((T >> (8 * k)) & 0xFFu) << 24);
}
// Nibble u of element e (0..255) of a GGUF Q3_K block (BlockQ3K::dequantize,
// quant.rs:506-574): q = 2 bits of qs[32n + 16h + l] at 2j, minus 4 when hmask bit
// 4n + j of hmask[16h + l] is clear, for group 8n + 2j + h; u = q + 4.
__host__ __device__ inline uint32_t q3k_nibble(const uint8_t* blk, int e) {
  const int n = e >> 7, j = (e >> 5) & 3, h = (e >> 4) & 1, l = e & 15;
  const uint32_t low = (blk[32 + 32 * n + 16 * h + l] >> (2 * j)) & 3u;
  return low + ((blk[16 * h + l] >> (4 * n + j)) & 1u) * 4u;
}
// Signed scale sc - 32 of group G (0..15) of a Q3_K block: the 12 scale bytes
// unpack to 16 six-bit values, of which group 8n + 2j + h uses value j + 4h (the
// reference uses the first eight in both halves).
__host__ __device__ inline int q3k_group_scale(const uint8_t* blk, int G) {
  const uint8_t* sb = blk + 96;
  auto rd = [&](int o) {
    return (uint32_t)sb[o] | ((uint32_t)sb[o + 1] << 8) | ((uint32_t)sb[o + 2] << 16) | ((uint32_t)sb[o + 3] << 24);
  };
  const uint32_t k1 = 0x03030303u, k2 = 0x0F0F0F0Fu, a0 = rd(0), a1 = rd(4), t = rd(8);
  const uint32_t aux[4] = {(a0 & k2) | ((t & k1) << 4), (a1 & k2) | (((t >> 2) & k1) << 4),
                           ((a0 >> 4) & k2) | (((t >> 4) & k1) << 4), ((a1 >> 4) & k2) | (((t >> 6) & k1) << 4)};
  const int k = ((G >> 1) & 3) + 4 * (G & 1);
  return (int)(int8_t)(uint8_t)(aux[k >> 2] >> (8 * (k & 3))) - 32;
}
// 2-bit q of element e of a GGUF Q2_K block (BlockQ2K::dequantize, quant.rs:443-474):
// bits 2j of qs[32n + 16h + l] for group 8n + 2j + h (scale byte of that group).
__host__ __device__ inline uint32_t q2k_nibble(const uint8_t* blk, int e) {
  const int n = e >> 7, j = (e >> 5) & 3, h = (e >> 4) & 1, l = e & 15;
  return (blk[16 + 32 * n + 16 * h + l] >> (2 * j)) & 3u;
}
// Scatter GGUF Q3_K or Q2_K block k (one chunk) of a row into packed row r of g.
// Used by the device and the host packers alike.
__host__ __device__ inline void nibble_group_pack_block(const PackedMat& g, uint8_t* Q, uint8_t* C, uint32_t r,
                                                        uint32_t k, const uint8_t* s) {
  const bool q3 = g.type == T_Q3_K;
  for (int G = 0; G < 16; G++) {
    for (int t = 0; t < 8; t++) {
      const int e = 16 * G + t;
      const uint32_t lo = q3 ? q3k_nibble(s, e) : q2k_nibble(s, e), hi = q3 ? q3k_nibble(s, e + 8) : q2k_nibble(s, e + 8);
      Q[qs_byte_off(g, r, (uint64_t)k * QT_CHUNK_BYTES + 32 * (G / 4) + 8 * (G % 4) + t)] = (uint8_t)(lo | (hi << 4));
    }
    C[sc_byte_off(g, r, (uint64_t)k * NG_HDR_BYTES + G)] = q3 ? (uint8_t)(int8_t)q3k_group_scale(s, G) : s[G];
  }
  const uint64_t hb = (uint64_t)k * NG_HDR_BYTES + 16;
  if (q3) {
    C[sc_byte_off(g, r, hb)] = s[108];
    C[sc_byte_off(g, r, hb + 1)] = s[109];
  } else {
    for (int i = 0; i < 4; i++) C[sc_byte_off(g, r, hb + i)] = s[80 + i];
  }
}

// Scatter GGUF Q6_K or Q5_K block k (256 elements at s) of a row into packed row r
// of g (quant bytes into Q, header bytes into C; the zero padding is left as is).
// Used by the device and the host packers alike.
__host__ __device__ inline void six_bit_pack_block(const PackedMat& g, uint8_t* Q, uint8_t* C, uint32_t r, uint32_t k,
                                                   const uint8_t* s) {
  const bool q5 = g.type == T_Q5_K;
  for (int j = 0; j < 16; j++) {
    uint32_t u[16], w[3];
    for (int t = 0; t < 16; t++) u[t] = q5 ? q5k_value(s, 16 * j + t) : q6k_value(s, 16 * j + t);
    six_bit_words(u, w);
    const uint64_t b = (uint64_t)(2 * k + j / 8) * Q6_CHUNK_BYTES + 12 * (j % 8);
    for (int t = 0; t < 3; t++) {
      uint8_t* p = Q + qs_byte_off(g, r, b + 4 * t);  // a word never straddles a plane
      for (int i = 0; i < 4; i++) p[i] = (uint8_t)(w[t] >> (8 * i));
    }
  }
  for (int h = 0; h < 2; h++) {
    const uint64_t hb = (uint64_t)(2 * k + h) * Q6_HDR_BYTES;
    if (q5) {  // sub-blocks 4h..4h+3: scales, mins, then d and dmin as stored
      for (int i = 0; i < 4; i++) {
        uint32_t sc, m;
        k4_scale_min(s + 4, 4 * h + i, &sc, &m);
        C[sc_byte_off(g, r, hb + i)] = (uint8_t)sc;
        C[sc_byte_off(g, r, hb + 4 + i)] = (uint8_t)m;
      }
      for (int i = 0; i < 4; i++) C[sc_byte_off(g, r, hb + 8 + i)] = s[i];
    } else {
      for (int i = 0; i < 8; i++) C[sc_byte_off(g, r, hb + i)] = s[192 + 8 * h + i];
      C[sc_byte_off(g, r, hb + 8)] = s[208];
      C[sc_byte_off(g, r, hb + 9)] = s[209];
    }
  }
}
// Device bytes of the two streams.
inline uint64_t packed_qs_bytes(const PackedMat& W) { return (uint64_t)W.Mp * W.qs_stride; }
inline uint64_t packed_sc_bytes(const PackedMat& W) { return (uint64_t)W.Mp * W.sc_stride; }

__host__ __device__ inline int elems_per_unit(int type) {
  switch (type) {
    case T_F32: return 8;
    case T_F16: return 16;
    case T_Q8_0: return 32;
    default: return 64;
  }
}
__host__ __device__ inline int block_elems(int type) {
  switch (type) {
    case T_F32: case T_F16: return 1;
    case T_Q4_0: case T_Q5_0: case T_Q8_0: return 32;
    case T_Q2_K: case T_Q3_K: case T_Q4_K: case T_Q5_K: case T_Q6_K: case T_Q8_K: return 256;
    default: return 0;
  }
}
__host__ __device__ inline int block_bytes(int type) {
  switch (type) {
    case T_F32: return 4;
    case T_F16: return 2;
    case T_Q4_0: return 18;
    case T_Q8_0: return 34;
    case T_Q5_0: return 22;
    case T_Q2_K: return 84;
    case T_Q3_K: return 110;
    case T_Q4_K: return 144;
    case T_Q5_K: return 176;
    case T_Q6_K: return 210;
    case T_Q8_K: return 292;
    default: return 0;
  }
}
// Padded row length for a type: whole chunks (quantized) or whole units (F32/F16).
inline uint32_t padded_k(int type, uint32_t K) {
  const uint32_t q = (uint32_t)(is_tiled(type) ? chunk_elems(type) : elems_per_unit(type));
  return (K + q - 1) / q * q;
}
bool packed_geometry(int type, uint32_t M, uint32_t K, PackedMat* out);  // fills all but pointers

// Split-K scratch of the quantized GEMV: partial row sums of tiles whose chunks
// are spread over several warps, and one arrival counter per tile (zero at rest:
// the warp that completes a tile resets it).  Kernels of one stream may share it.
struct GemvScratch {
  float* part;
  unsigned* cnt;
  uint64_t part_floats;
  uint32_t n_cnt;
};
// Scratch a matrix needs (0 / 0 for F32/F16).
void gemv_scratch_need(const PackedMat& W, uint64_t* part_floats, uint32_t* n_cnt);

// ---- launch helpers -------------------------------------------------------
// Every engine kernel is launched with programmatic dependent launch so its
// weight prefetch overlaps the previous kernel's tail.
struct Launch {
  cudaStream_t stream;
  bool pdl;
  bool wide = false;  // quantized GEMVs as one 16-warp CTA per SM for every epilogue (tensor parallel)
};

// Repack GGUF rows (device bytes) into a PackedMat. src_row_of[dst] selects the
// GGUF row for each packed row (NULL = identity).  *d_sub (device word, may be
// NULL) is set to 1 when a block scale is a subnormal half, else 0.
cudaError_t launch_pack(const uint8_t* gguf, const int* src_row_of, PackedMat dst, unsigned* d_sub, cudaStream_t s);
// Host scan of packed scale bytes: true when any block scale is a subnormal half.
bool has_subnormal_scales(const PackedMat& W, const uint8_t* sc_host);

// ---- GEMV families -------------------------------------------------------
// All take x (f32, K elements) and optionally RMSNorm it on the fly with
// norm_w/eps (rms_norm_reference, compute.rs:291-319).  Quantized matrices need
// the split-K scratch (gemv_scratch_need); F32/F16 ones ignore it.
struct PeerLink;  // a GEMV's part in a tensor-parallel sum over peer memory (below)
cudaError_t gemv_store(const Launch& L, const PackedMat& W, const GemvScratch* ws, const float* x, const float* norm_w,
                       float eps, float* y);
// out[row] = (res ? res[row] : 0) + (W.x)[row]   (residual add, model_executor.rs:213-215, 231-233)
cudaError_t gemv_residual(const Launch& L, const PackedMat& W, const GemvScratch* ws, const float* x, const float* res,
                          float* out);

struct RopeQKVArgs {
  uint32_t q_rows, kv_rows, head_dim, max_seq;
  const float2* rope_cs;  // [max_seq][head_dim/2] (cos, sin)
  const int* d_pos;       // current position (device)
  float* q_out;           // [q_rows]
  float* k_cur;           // [kv_rows]
  float* v_cur;           // [kv_rows]
  void* kcache;           // [kv_heads][max_seq][head_dim]
  void* vcache;
  int kv_f32;
  // Packed [Q;K;V] row of the matrix's row 0: 0 for the fused matrix (or [Q;K]),
  // q_rows + kv_rows for a separate V matrix.
  uint32_t row_base;
  // Q/K/V biases in packed [Q;K;V] row order, added before RoPE (null: none).
  const float* bias;
};
// Fused: RMSNorm(attn_norm) -> packed [Q;K;V] matvec -> RoPE on Q/K pairs -> K/V append.
// With `pull`, x is the sum over ranks of a peer sum's rows instead (PeerLink).
cudaError_t gemv_qkv_rope(const Launch& L, const PackedMat& W, const GemvScratch* ws, const float* x,
                          const float* norm_w, float eps, const RopeQKVArgs& a, const PeerLink* pull = nullptr);
// Fused: RMSNorm(ffn_norm) -> packed [gate_j; up_j] matvec -> act[j] = silu(g)*u.
cudaError_t gemv_swiglu(const Launch& L, const PackedMat& W, const GemvScratch* ws, const float* x,
                        const float* norm_w, float eps, float* act, const PeerLink* pull = nullptr);
// Fused LM head: optional RMSNorm(output_norm) -> logits (nullable) -> packed
// argmax key (atomicMax of (ordered value, ~global_row)).
cudaError_t gemv_argmax(const Launch& L, const PackedMat& W, const GemvScratch* ws, const float* x,
                        const float* norm_w, float eps, float* logits, unsigned long long* key, uint32_t row_offset);
// Batched standalone GEMV: y[b][row] = (W . x[b])[row] for b < batch, x[b] at
// x + b*K, y[b] at y + b*M.
cudaError_t gemv_batched(cudaStream_t s, const PackedMat& W, const GemvScratch* ws, const float* x, int batch,
                         float* y);

// ---- batched prompt GEMM on the tensor cores (rf_prefill.cu) ---------------------
// Formats the tensor-core GEMM dequantizes (Q4_K, Q8_0); other matrices keep the
// token-by-token path.
bool prefill_supported(int type);
// Bytes of the split activation buffer for T tokens of padded row length Kp.
size_t prefill_xt_bytes(uint32_t T, uint32_t Kp);
// X [T][K] f32 (row stride ldx), RMS-normalised per token with nw/eps when nw is
// set, split into bf16 hi/lo in the GEMM's tiled operand layout (Kp >= K, a
// multiple of 64; the padding is zero).
cudaError_t prefill_split(const Launch& L, const float* X, uint32_t ldx, uint32_t T, uint32_t K, uint32_t Kp,
                          const float* nw, float eps, void* Xt);
// y[t][row] = (W . x_t)[row] for t < T on the tensor cores (3 bf16 products per
// element pair: hi*hi + hi*lo + lo*hi, f32 accumulation); err (may be null) gets
// bit 0 when a bounded wait gave up.
cudaError_t prefill_gemm_store(const Launch& L, const PackedMat& W, const void* Xt, uint32_t T, unsigned* err,
                               float* y, uint32_t ldy);
// The same GEMM with the decode step's epilogues, for a prompt chunk of T tokens:
//  rope: Q/K/V rows (packed order, a.row_base as in the step) of token t at
//        position pos0 + t: bias, RoPE, K/V into the cache; Q, K, V rows into
//        a.q_out / a.k_cur / a.v_cur + t * (q_stride or kv_stride);
//  residual: x[t][row] += (W . x_t)[row];
//  swiglu: act[t][j] = silu(gate_j) * up_j over the interleaved gate/up rows.
cudaError_t prefill_gemm_rope(const Launch& L, const PackedMat& W, const void* Xt, uint32_t T, unsigned* err,
                              const RopeQKVArgs& a, uint32_t pos0, uint32_t q_stride, uint32_t kv_stride);
// Scratch of the residual GEMM's K split: `tiles` output blocks of two [128 x 128]
// f32 partials (prefill_ksplit_floats(tiles) floats) and one arrival counter each
// (zero at rest; the last arrival resets it).  Without it the GEMM runs unsplit.
struct PrefillKSplit {
  float* part = nullptr;
  unsigned* cnt = nullptr;
  uint32_t tiles = 0;
};
size_t prefill_ksplit_floats(uint32_t tiles);
cudaError_t prefill_gemm_residual(const Launch& L, const PackedMat& W, const void* Xt, uint32_t T, unsigned* err,
                                  float* x, uint32_t ldx, const PrefillKSplit& ks = PrefillKSplit{});
cudaError_t prefill_gemm_swiglu(const Launch& L, const PackedMat& W, const void* Xt, uint32_t T, unsigned* err,
                                float* act, uint32_t ld);
// x[t] <- the dequantized embedding row of tokens[t] (device array), t < T.
cudaError_t launch_embed_rows(const Launch& L, const PackedMat& E, const uint32_t* tokens, uint32_t T, float* x);

// ---- tensor-parallel sum over NVLink peer memory ------------------------------
// The sum of the ranks' partial vectors after a row-parallel projection, as one
// kernel over peer memory instead of a library all-reduce: every rank stores its
// partial straight into each rank's receive area (NVLink peer stores through
// cudaIpc mappings), raises one flag per slice on each rank, waits for the other
// ranks' flags of its slices and sums the ranks' partials in rank order (the same
// result on every rank).  A flag holds the call site's generation, so flags of
// earlier steps never match; waits are bounded and report through `err`.
constexpr int RF_MAX_TP = 8;
constexpr int PS_THREADS = 256, PS_ELEMS = 4 * PS_THREADS;  // elements a CTA sums
struct PeerSum {
  float* recv[RF_MAX_TP];      // rank p's receive area: [2 (site parity)][n_ranks][n_max]
  unsigned* flags[RF_MAX_TP];  // rank p's flags: [n_ranks][sites][max_ctas]
  unsigned* epoch;             // this rank: generation of each call site [sites]
  unsigned* done;              // this rank: CTAs finished per call site [sites]
  unsigned* err;               // this rank: bit 0 = a wait gave up
  unsigned* fgen;              // this rank: generation of each call site's fused sum (PeerLink) [sites]
  int rank, n_ranks, n_max, sites, max_ctas;
};
// Bytes of one rank's area (receive | flags | epoch | done | err), and its layout.
size_t peer_sum_area_bytes(int n_ranks, int n_max, int sites);
void peer_sum_bind(PeerSum* P, int p, void* area_of_p, bool own);
// out[i] = sum over ranks of partial[i] (i < n, n a multiple of 4); call site
// `site` < P.sites, consecutive sites of one step alternate parity.
cudaError_t launch_peer_sum(const Launch& L, const PeerSum& P, const float* partial, float* out, int n, int site);
// One peer sum whose second rank never arrives (a local phantom area): its
// bounded wait gives up and sets bit 0 of *err_out.
cudaError_t peer_sum_selftest(unsigned* err_out);

// The same sum fused into the GEMVs on either side of it, so no kernel runs for
// it.  The row-parallel GEMV (push_site >= 0) stores its rows (plus the residual
// on rank 0) into every rank's receive area, and each of its CTAs, after its
// stores, adds one arrival to this rank's counter of the site on every rank
// (system-scope release-add; the counter is the first flag word of the site).
// The next GEMV (pull_site >= 0) waits, bounded, until every rank's counter holds
// fused generation x push_ctas, stages x as the ranks' rows summed in rank order (the
// sum kernel's order), and its CTA 0 writes that sum to `hidden` (the residual of
// the next row-parallel product).  Generations advance as in the kernel above;
// the counters grow by push_ctas per use and are compared modulo 2^32.  The fused
// sum keeps its own generation per site (fgen) and its counter in the site's last
// flag slot, apart from the sum kernel's, so an engine may use both on one site.
struct PeerLink {
  PeerSum P;
  int push_site = -1, pull_site = -1;
  int push_ctas = 0;  // CTAs of the pushing GEMV (its launch's grid)
  float* hidden = nullptr;
};
// CTAs a quantized GEMV launch has on this device (the pushing GEMV's arrival count).
int gemv_ctas(const Launch& L, const PackedMat& W, bool residual_epilogue);
// out = res + W.x pushed into the peer sum of pl.push_site (res: rank 0's residual or null).
cudaError_t gemv_peer_push(const Launch& L, const PackedMat& W, const GemvScratch* ws, const float* x,
                           const float* res, const PeerLink& pl);

// ---- attention -------------------------------------------------------------
struct AttnArgs {
  const float* q;          // [batch][H][hd]
  const void* kc;          // cache base; head stride = head_stride elems, batch stride = batch_stride
  const void* vc;
  uint64_t head_stride, batch_stride;
  const float* k_cur;      // [KV][hd] current position (engine) or NULL
  const float* v_cur;
  const int* d_nhist;      // history length on device (engine) or NULL
  int nhist;               // history length when d_nhist == NULL
  int n_heads, n_kv_heads, head_dim, batch;
  int max_splits;
  float* part;             // [batch][KV][max_splits][G][hd + 2]
  unsigned* counters;      // [batch][KV], zero at rest
  float* out;              // [batch][H][hd]
  int kv_f32;
  unsigned* err;           // bit 1 set when a bounded wait gave up (may be NULL)
  int max_ctx;             // with d_nhist: the longest context the launch may serve (kernel choice)
  // Prompt chunks: sequence b's history is nhist + b * nhist_step positions of one
  // shared cache (batch_stride 0) and its current K/V row is k_cur/v_cur + b * cur_stride.
  int nhist_step;
  uint64_t cur_stride;
};
// Contexts from which launch_attention streams the history through shared memory.
constexpr int kAttnStreamMinCtx = 1024;
size_t attn_part_floats(int batch, int n_kv_heads, int max_splits, int G, int hd);
cudaError_t launch_attention(const Launch& L, const AttnArgs& a);

// ---- small kernels -------------------------------------------------------------
// hidden <- dequantized row *d_token of the embedding; also resets *key to 0.
cudaError_t launch_embed(const Launch& L, const PackedMat& E, const uint32_t* d_token, float* hidden,
                         unsigned long long* key);
cudaError_t launch_rmsnorm(const Launch& L, const float* x, const float* w, float eps, uint32_t n, float* y);
// token <- argmax index of *key; hist[*d_pos] <- token (when in range); *d_pos += 1.
cudaError_t launch_finalize(const Launch& L, const unsigned long long* key, uint32_t* d_token, int* d_pos,
                            uint32_t* hist, int hist_len);
// Dequantize rows [r0, r0+n) of a packed matrix into f32 (debug / parity dumps).
cudaError_t launch_dequant_rows(const PackedMat& W, uint32_t r0, uint32_t n, float* out, cudaStream_t s);
// f16/f32 KV read in reference layout: out[p][h][d] for p in [start,end).
cudaError_t launch_kv_gather(const void* cache, int kv_f32, uint32_t kv_heads, uint32_t max_seq, uint32_t hd,
                             uint32_t start, uint32_t end, float* out, cudaStream_t s);

}  // namespace rf
