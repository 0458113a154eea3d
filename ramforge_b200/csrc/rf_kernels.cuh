// rf_kernels.cuh - device data layouts and kernel launchers of the decode engine.
#pragma once
#include <cuda.h>  // CUtensorMap (types only; the encoder is fetched from the driver at run time)
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace rf {

// ggml type ids (types.rs:238-270)
enum : int { T_F32 = 0, T_F16 = 1, T_Q4_0 = 2, T_Q8_0 = 8, T_Q4_K = 12 };

// Packed device form of one GGUF matrix (n_out rows of n_in elements).
//
// GGUF interleaves per-block scales with quants (Q8_0: 34-byte blocks, Q4_K:
// 144-byte super-blocks), which leaves quants at 2- or 16-byte alignment.  The
// engine splits every row into two byte streams at load time, without changing
// a single bit of either:
//   qs : the quant bytes of the row, blocks concatenated in GGUF order, padded to
//        a multiple of 32 bytes so each lane reads one 256-bit "unit" per load;
//   sc : the per-block scale bytes of the row (Q8_0/Q4_0: the f16 d of every 32
//        elements; Q4_K: the 16-byte {d, dmin, scales[12]} header of every
//        256 elements).
// A unit covers EPU elements: Q8_0 32 (one block), Q4_0 64 (two blocks), Q4_K
// 64 (one sub-block pair of a super-block), F16 16, F32 8.
struct PackedMat {
  int type;
  uint32_t M, K;        // rows, logical row length
  uint32_t Kp;          // row length padded to a whole number of units / blocks
  uint32_t units;       // 32-byte units per row
  uint64_t qs_stride;   // bytes per row of qs
  uint64_t sc_stride;   // bytes per row of sc (0 for F32/F16)
  uint8_t* qs;
  uint8_t* sc;
};

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
// Padded row length for a type: a multiple of the unit and of the block.
inline uint32_t padded_k(int type, uint32_t K) {
  uint32_t q = (uint32_t)(type == T_Q4_K ? 256 : elems_per_unit(type));
  return (K + q - 1) / q * q;
}
bool packed_geometry(int type, uint32_t M, uint32_t K, PackedMat* out);  // fills all but pointers

// TMA descriptors of a packed quantized matrix for the pipelined GEMV: 64-row x
// 16-unit boxes of qs (512 B per row) and the matching scale bytes.  ok == false
// (F32/F16, or rows whose scale stride is not a multiple of 16 bytes) selects the
// register-streaming GEMV instead.
struct GemvMaps {
  CUtensorMap qs, sc;
  uint32_t sc_chunk_bytes;
  bool ok;
};
// Builds the descriptors for the device pointers in W (false: not TMA-eligible).
bool make_gemv_maps(const PackedMat& W, GemvMaps* out);

// ---- launch helpers -------------------------------------------------------
// Every engine kernel is launched with programmatic dependent launch so its
// weight prefetch overlaps the previous kernel's tail.
struct Launch {
  cudaStream_t stream;
  bool pdl;
};

// Repack GGUF rows (device bytes) into a PackedMat. src_row_of[dst] selects the
// GGUF row for each packed row (NULL = identity).
cudaError_t launch_pack(const uint8_t* gguf, const int* src_row_of, PackedMat dst, cudaStream_t s);

// ---- GEMV families -------------------------------------------------------
// All take x (f32, K elements) and optionally RMSNorm it on the fly with
// norm_w/eps (rms_norm_reference, compute.rs:291-319).
cudaError_t gemv_store(const Launch& L, const PackedMat& W, const GemvMaps* maps, const float* x, const float* norm_w, float eps,
                       float* y);
// out[row] = (res ? res[row] : 0) + (W.x)[row]   (residual add, model_executor.rs:213-215, 231-233)
cudaError_t gemv_residual(const Launch& L, const PackedMat& W, const GemvMaps* maps, const float* x, const float* res, float* out);

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
cudaError_t gemv_qkv_rope(const Launch& L, const PackedMat& W, const GemvMaps* maps, const float* x, const float* norm_w, float eps,
                          const RopeQKVArgs& a);
// Fused: RMSNorm(ffn_norm) -> packed [gate_j; up_j] matvec -> act[j] = silu(g)*u.
cudaError_t gemv_swiglu(const Launch& L, const PackedMat& W, const GemvMaps* maps, const float* x, const float* norm_w, float eps,
                        float* act);
// Fused LM head: optional RMSNorm(output_norm) -> logits (nullable) -> packed
// argmax key (atomicMax of (ordered value, ~global_row)).
cudaError_t gemv_argmax(const Launch& L, const PackedMat& W, const GemvMaps* maps, const float* x, const float* norm_w, float eps,
                        float* logits, unsigned long long* key, uint32_t row_offset);
// Batched standalone GEMV: y[b][row] for b < batch (x read through L1).
cudaError_t gemv_batched(cudaStream_t s, const PackedMat& W, const float* x, int batch, float* y);

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
// f16/f32 KV read in reference layout: out[p][h][d] for p in [start,end).
cudaError_t launch_kv_gather(const void* cache, int kv_f32, uint32_t kv_heads, uint32_t max_seq, uint32_t hd,
                             uint32_t start, uint32_t end, float* out, cudaStream_t s);

}  // namespace rf
