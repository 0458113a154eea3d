/*
 * oracle.h - CPU restatement of RAMforge's legacy decode hot path.
 *
 * TEST INFRASTRUCTURE ONLY.  This library is the parity checker for the
 * B200 engine (librfcuda.so).  Only tests/, __graft_entry__.smoke() and the
 * cpu_baseline / --impl reference legs of bench.py may load it.  The product
 * path never links, loads or calls anything here.
 *
 * The reference (NeonMC23/RAMforge) is pure Rust and cannot be compiled in
 * this image (no cargo/rustc), so this is a line-by-line restatement of its
 * arithmetic in C11, compiled with -O2 -ffp-contract=off against glibc libm
 * (the same libm Rust's f32::{powf,exp,sin,cos} resolve to on linux-gnu).
 * Each function cites the reference file:line it follows.  The restatement
 * is pinned against the reference's own known-answer tests
 * (tests/test_oracle_golden.py).
 */
#ifndef RF_ORACLE_H
#define RF_ORACLE_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ggml type ids (crates/ramforge-core/src/types.rs:238-270). */
enum {
  ORC_F32 = 0, ORC_F16 = 1, ORC_Q4_0 = 2, ORC_Q5_0 = 6, ORC_Q8_0 = 8,
  ORC_Q2_K = 10, ORC_Q3_K = 11, ORC_Q4_K = 12, ORC_Q5_K = 13, ORC_Q6_K = 14, ORC_Q8_K = 15
};

/* ---- block-level primitives ---------------------------------------- */
float orc_f16_to_f32(uint16_t bits);
uint16_t orc_f32_to_f16(float f); /* IEEE RNE, used by the kv_f16 mode */
/* Bytes of one row of `n` elements of `type`; 0 when n is not a block multiple. */
size_t orc_row_bytes(int type, size_t n);
/* Decode one row (dequantize_row_* / f32 / f16 copy). Returns 0 on success. */
int orc_dequant_row(int type, const uint8_t* bytes, size_t nbytes, size_t n, float* out);

/* ---- numeric core (crates/ramforge-core/src/compute.rs) ------------- */
/* y[out] = W[out][in] . x  in the runtime kernel order of `type`
 * (Q4_0 fused interleave, Q8_0/Q4_K dequant-then-dot, F32 sequential).
 * threads > 1 partitions rows only; per-row order (and result) is unchanged. */
int orc_matvec(int type, const uint8_t* w, size_t wbytes, size_t in, size_t out,
               const float* x, float* y, int threads);
/* quantized_matvec_reference: decode a full row, then sequential dot. */
int orc_matvec_reference(int type, const uint8_t* w, size_t wbytes, size_t in, size_t out,
                         const float* x, float* y);
int orc_rmsnorm(const float* x, const float* w, float eps, size_t n, float* y);
int orc_rope(float* q, float* k, size_t pos, size_t head_dim, size_t n_heads,
             size_t n_kv_heads, float theta);
/* attention_reference: history [hist][kv_heads][head_dim]; returns output [H][hd]. */
int orc_attention(const float* q, const float* k_hist, const float* v_hist,
                  const float* k_cur, const float* v_cur, size_t hist, size_t n_heads,
                  size_t n_kv_heads, size_t head_dim, float* out);
int orc_softmax(float* v, size_t n);
void orc_silu(const float* x, float* y, size_t n);
void orc_swiglu(const float* g, const float* u, float* y, size_t n);
uint32_t orc_argmax(const float* logits, size_t n);

/* ---- model ----------------------------------------------------------- */
typedef struct orc_model orc_model;
typedef struct {
  uint32_t vocab_size, context_length, n_embd, n_layers, n_ff, n_heads, n_kv_heads, head_dim;
  float rms_eps, rope_theta;
} orc_config;

/* Parse a GGUF image held in memory (caller keeps `data` alive). kv_f16 != 0
 * rounds every committed K/V history entry to f16 (the GPU cache format);
 * kv_f16 == 0 is the reference's f32 cache.  max_seq bounds the KV cache.
 * threads: row partitioning for matvecs (1 = the reference's dispatch for
 * Q8_0/Q4_K; results do not depend on it). */
orc_model* orc_model_open(const uint8_t* data, size_t len, int kv_f16, uint32_t max_seq,
                          int threads);
void orc_model_close(orc_model* m);
const char* orc_last_error(void);
int orc_model_config(const orc_model* m, orc_config* cfg);
/* forward_single_streaming: pos must equal the KV length; writes final_hidden
 * (output-normed hidden, n_embd floats, may be NULL). */
int orc_forward(orc_model* m, uint32_t token, uint32_t pos, float* final_hidden);
/* compute_logits over a final hidden vector (n_embd) -> logits (vocab). */
int orc_logits(orc_model* m, const float* final_hidden, float* logits);
/* Optional per-layer hidden dump of the last forward: [n_layers][n_embd]. */
int orc_last_layer_hiddens(const orc_model* m, float* out);
/* Bounded CPU-baseline samples: one layer of a token forward (no commit) and a
 * row slice of the LM head. */
int orc_layer_step(orc_model* m, uint32_t layer, uint32_t pos, float* hidden);
int orc_logits_rows(orc_model* m, const float* final_hidden, uint32_t r0, uint32_t r1, float* out);
uint32_t orc_kv_len(const orc_model* m);
void orc_kv_reset(orc_model* m);
int orc_kv_fill_synthetic(orc_model* m, uint32_t n, uint32_t seed);
/* K or V history of one layer, reference layout [pos][kv_head][head_dim], f32. */
int orc_kv_read(const orc_model* m, uint32_t layer, int which_v, uint32_t start, uint32_t end,
                float* out);
/* Greedy generate (inference.rs generate_impl): prompt processed token by token,
 * then n_new greedy tokens.  out_tokens receives n_new tokens; optional
 * out_logits receives [n_new][vocab] logits that produced them; optional
 * out_margin receives top1 - top2 per generated token. */
int orc_generate(orc_model* m, const uint32_t* prompt, uint32_t n_prompt, uint32_t n_new,
                 uint32_t* out_tokens, float* out_logits, float* out_margin);

#ifdef __cplusplus
}
#endif
#endif
