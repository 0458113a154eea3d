// rf_kernels.cuh - device data layouts and kernel launchers of the decode engine.
#pragma once
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace rf {

// ggml type ids (types.rs:238-270)
enum : int { T_F32 = 0, T_F16 = 1, T_Q4_0 = 2, T_Q8_0 = 8, T_Q4_K = 12 };

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

__host__ __device__ inline bool is_tiled(int type) { return type == T_Q4_K || type == T_Q4_0 || type == T_Q8_0; }
__host__ __device__ inline int chunk_elems(int type) { return type == T_Q8_0 ? 128 : 256; }
__host__ __device__ inline int chunk_scale_bytes(int type) { return type == T_Q8_0 ? 8 : 16; }

// Byte b (0 <= b < qs_stride) of row r's quant bytes.
__host__ __device__ inline uint64_t qs_byte_off(const PackedMat& W, uint32_t r, uint64_t b) {
  if (!is_tiled(W.type)) return (uint64_t)r * W.qs_stride + b;
  const uint64_t item = (uint64_t)(r / QT_ROWS) * W.nk + b / QT_CHUNK_BYTES;
  return (item * 4 + (b / 32) % 4) * (QT_ROWS * 32) + (uint64_t)(r % QT_ROWS) * 32 + b % 32;
}
// Byte b (0 <= b < sc_stride) of row r's scale bytes.
__host__ __device__ inline uint64_t sc_byte_off(const PackedMat& W, uint32_t r, uint64_t b) {
  const uint64_t item = (uint64_t)(r / QT_ROWS) * W.nk + b / W.sbytes;
  return (item * QT_ROWS + r % QT_ROWS) * W.sbytes + b % W.sbytes;
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
    case T_Q4_0: case T_Q8_0: return 32;
    case T_Q4_K: return 256;
    default: return 0;
  }
}
__host__ __device__ inline int block_bytes(int type) {
  switch (type) {
    case T_F32: return 4;
    case T_F16: return 2;
    case T_Q4_0: return 18;
    case T_Q8_0: return 34;
    case T_Q4_K: return 144;
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
};
// Fused: RMSNorm(attn_norm) -> packed [Q;K;V] matvec -> RoPE on Q/K pairs -> K/V append.
cudaError_t gemv_qkv_rope(const Launch& L, const PackedMat& W, const GemvScratch* ws, const float* x,
                          const float* norm_w, float eps, const RopeQKVArgs& a);
// Fused: RMSNorm(ffn_norm) -> packed [gate_j; up_j] matvec -> act[j] = silu(g)*u.
cudaError_t gemv_swiglu(const Launch& L, const PackedMat& W, const GemvScratch* ws, const float* x,
                        const float* norm_w, float eps, float* act);
// Fused LM head: optional RMSNorm(output_norm) -> logits (nullable) -> packed
// argmax key (atomicMax of (ordered value, ~global_row)).
cudaError_t gemv_argmax(const Launch& L, const PackedMat& W, const GemvScratch* ws, const float* x,
                        const float* norm_w, float eps, float* logits, unsigned long long* key, uint32_t row_offset);
// Batched standalone GEMV: y[b][row] = (W . x[b])[row] for b < batch, x[b] at
// x + b*K, y[b] at y + b*M.
cudaError_t gemv_batched(cudaStream_t s, const PackedMat& W, const GemvScratch* ws, const float* x, int batch,
                         float* y);

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
  int rank, n_ranks, n_max, sites, max_ctas;
};
// Bytes of one rank's area (receive | flags | epoch | done | err), and its layout.
size_t peer_sum_area_bytes(int n_ranks, int n_max, int sites);
void peer_sum_bind(PeerSum* P, int p, void* area_of_p, bool own);
// out[i] = sum over ranks of partial[i] (i < n, n a multiple of 4); call site
// `site` < P.sites, consecutive sites of one step alternate parity.
cudaError_t launch_peer_sum(const Launch& L, const PeerSum& P, const float* partial, float* out, int n, int site);

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
};
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
// ---- the persistent decode-step kernel (rf_step.cu) ------------------------------
// One cooperative launch runs a whole token step: embedding row, every layer
// (QKV+RoPE+KV append | attention | Wo+residual | gate/up+SwiGLU | down+residual),
// then either the LM head + greedy argmax + advance (decode) or the final
// RMSNorm into final_hidden (forward).  Phases are separated by grid barriers
// whose waits are bounded (err bit 0 on expiry); each GEMV phase issues its
// first weight loads before its barrier.
struct StepLayer {
  PackedMat qkv, wo, gateup, down;
  const float* attn_norm;
  const float* ffn_norm;
  RopeQKVArgs rope;  // the QKV epilogue of this layer (its K/V cache, shapes, buffers)
  AttnArgs attn;     // the attention of this layer
};
struct StepArgs {
  const StepLayer* layers;  // device array [n_layers]
  int n_layers;
  int decode;
  PackedMat embd, lm;
  const float* out_norm;
  float eps;
  uint32_t n_embd, q_rows, kv_rows, head_dim, max_seq, n_heads, n_kv_heads;
  const float2* rope_cs;
  float *hidden, *final_hidden, *q, *k_cur, *v_cur, *att, *act, *logits;  // logits may be NULL
  uint32_t* d_token;
  int* d_pos;
  uint32_t* hist;
  int hist_len;
  unsigned long long* key;
  uint32_t vocab_off;
  GemvScratch gws;
  float* attn_part;
  unsigned* attn_counters;
  int max_splits;
  unsigned* bar;  // arrival counter (zeroed by launch_step_kernel)
  unsigned* err;  // bit 0: a barrier wait gave up
  unsigned long long* stamps;  // NULL, or [barriers + 1] globaltimer ns: kernel start, then each barrier's end
};
// Dynamic shared memory of the step kernel for these shapes, or 0 when the
// kernel has no instance for them (layer / LM-head types, head_dim, GQA group,
// f16 KV cache, no subnormal scales) or they do not fit one CTA per SM.
size_t step_kernel_smem(const StepArgs& a, const StepLayer& layer0);
cudaError_t launch_step_kernel(cudaStream_t s, const StepArgs& a, const StepLayer& layer0, size_t smem);
// Runs one step-kernel barrier on the current device with `phantom` extra
// expected arrivals (none of which come) and returns the error word.
cudaError_t barrier_selftest(unsigned phantom, unsigned* err_out);

// f16/f32 KV read in reference layout: out[p][h][d] for p in [start,end).
cudaError_t launch_kv_gather(const void* cache, int kv_f32, uint32_t kv_heads, uint32_t max_seq, uint32_t hd,
                             uint32_t start, uint32_t end, float* out, cudaStream_t s);

}  // namespace rf
