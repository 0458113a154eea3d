// rfsynth.h - seeded synthetic Llama GGUF generator and GGUF block encoders.
// Host-only helper library (librfsynth.so) used by the tests and the benchmark
// to produce the benchmark configurations' models; it is not part of the
// decode engine's drop-in boundary (include/rfcuda.h).
#ifndef RF_SYNTH_H
#define RF_SYNTH_H
#include <stddef.h>
#include <stdint.h>
#ifdef __cplusplus
extern "C" {
#endif

enum { RFS_F32 = 0, RFS_F16 = 1, RFS_Q4_0 = 2, RFS_Q8_0 = 8, RFS_Q4_K = 12, RFS_Q6_K = 14 };

typedef struct {
  const char* arch; /* "llama" (default) or "qwen2" */
  uint32_t vocab_size, context_length, n_embd, n_layers, n_ff, n_heads, n_kv_heads;
  float rms_eps, rope_theta;
  int layer_type; /* type of the 7 per-layer matrices */
  int embd_type;  /* token_embd.weight */
  int out_type;   /* output.weight; -1 = absent (tied to token_embd) */
  uint64_t seed;
  float weight_std;
  int v_type;         /* attn_v.weight type; -1 = layer_type (Q4_K_M-style mixes use Q6_K) */
  int down_type;      /* ffn_down.weight type; -1 = layer_type */
  float qkv_bias_std; /* > 0: F32 blk.N.attn_{q,k,v}.bias of N(0, qkv_bias_std) (qwen2); 0 = none */
} rfs_llama_spec;

/* out[i] = N(0, stddev) sample #(start+i) of stream (seed, stream). */
void rfs_fill_normal(uint64_t seed, uint64_t stream, float stddev, uint64_t start, float* out, size_t n);
size_t rfs_row_bytes(int type, size_t n);
/* Quantise rows x[rows][cols] into GGUF blocks. */
int rfs_quantize(int type, const float* x, size_t rows, size_t cols, uint8_t* out, int threads);
/* Size in bytes of the GGUF image for `spec` (0 = invalid spec). */
uint64_t rfs_llama_gguf_size(const rfs_llama_spec* spec);
/* Write the GGUF image into out[cap]. 0 on success. */
int rfs_llama_gguf_write(const rfs_llama_spec* spec, uint8_t* out, uint64_t cap, int threads);

#ifdef __cplusplus
}
#endif
#endif
