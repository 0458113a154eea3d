/*
 * rfcuda.h - C ABI of librfcuda.so, the B200 (sm_100a) decode engine that
 * replaces RAMforge's legacy CPU executor on the per-token hot path.
 *
 * Conventions (mirroring the reference's Rust contracts):
 *   - every call returns int: RF_OK (0) or a negative RF_E* code; the reason is
 *     in rf_last_error() (thread-local), never a panic or abort
 *     (reference: Result<_, String> throughout, e.g. streaming_model.rs:909-919);
 *   - the caller owns host buffers (activations, logits); the engine owns device
 *     weights, the KV cache and its scratch (reference: caller-owned &mut [f32]
 *     scratch in model_executor.rs:102-121, model-owned persistent weights);
 *   - one host thread drives one engine (reference: one thread per engine,
 *     layer cache behind a Mutex, streaming_model.rs:141);
 *   - matrices use the ggml convention ne0 = input (row length), ne1 = output
 *     rows, rows stored contiguously (reference: compute.rs:7-15).
 * Reference paths are crates/<crate>/src/<file>:<line> in NeonMC23/RAMforge.
 */
#ifndef RFCUDA_H
#define RFCUDA_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define RF_ABI_VERSION 3

/* status codes */
#define RF_OK 0
#define RF_EINVAL (-1)       /* bad argument / shape / position (arity mismatch errors) */
#define RF_ENOMEM (-2)       /* byte budget exceeded or a device/pinned allocation failed */
#define RF_ECUDA (-3)        /* CUDA runtime error */
#define RF_EFORMAT (-4)      /* malformed GGUF / unsupported tensor type */
#define RF_ESTATE (-5)       /* wrong state, e.g. layer not loaded, KV cache full */
#define RF_EUNSUPPORTED (-6) /* valid request this build does not implement */
#define RF_ENCCL (-7)        /* NCCL (tensor-parallel) failure */
#define RF_ETIMEOUT (-8)     /* a bounded device-side wait gave up */

/* ggml tensor type ids (types.rs:238-270) accepted by the engine */
#define RF_TYPE_F32 0
#define RF_TYPE_F16 1
#define RF_TYPE_Q4_0 2
#define RF_TYPE_Q8_0 8
#define RF_TYPE_Q2_K 10
#define RF_TYPE_Q3_K 11
#define RF_TYPE_Q4_K 12
#define RF_TYPE_Q5_K 13
#define RF_TYPE_Q6_K 14
/* accepted and stored as f32, decoded at load exactly as the reference's dequantize
 * (quant.rs:114-154, 579-612): its matvec for these decodes then sums in f32 */
#define RF_TYPE_Q5_0 6
#define RF_TYPE_Q8_K 15

/* per-layer tensor roles, the nine tensors of StreamingLayerWeights
 * (model_executor.rs:33-48; names blk.N.<role>.weight, model.rs:182-192) */
#define RF_ROLE_ATTN_NORM 0
#define RF_ROLE_ATTN_Q 1
#define RF_ROLE_ATTN_K 2
#define RF_ROLE_ATTN_V 3
#define RF_ROLE_ATTN_OUTPUT 4
#define RF_ROLE_FFN_NORM 5
#define RF_ROLE_FFN_GATE 6
#define RF_ROLE_FFN_UP 7
#define RF_ROLE_FFN_DOWN 8
/* optional qwen2 Q/K/V biases (StreamingLayerWeights::attn_{q,k,v}_bias,
 * model_executor.rs:43-47): all three or none, vectors (ne1 = 0 or 1) in F32/F16 of
 * n_heads*head_dim, n_kv_heads*head_dim, n_kv_heads*head_dim elements */
#define RF_ROLE_ATTN_Q_BIAS 9
#define RF_ROLE_ATTN_K_BIAS 10
#define RF_ROLE_ATTN_V_BIAS 11
/* persistent tensors (persistent.rs:20-80) */
#define RF_ROLE_TOKEN_EMBD 16
#define RF_ROLE_OUTPUT_NORM 17
#define RF_ROLE_OUTPUT 18

/* LlamaConfig (runtime/src/model.rs:25-37); head_dim = n_embd / n_heads (model.rs:148). */
typedef struct rf_model_config {
  uint32_t vocab_size, context_length, n_embd, n_layers, n_ff, n_heads, n_kv_heads, head_dim;
  float rms_eps, rope_theta;
} rf_model_config;

/* GPU runtime configuration: the reference's RuntimeConfig (runtime_config.rs:15-23)
 * plus the device-side knobs.  Zero-initialise and set what you need. */
typedef struct rf_runtime_config {
  int device;                 /* CUDA ordinal */
  int tp_rank, tp_size;       /* tensor parallelism (tp_size 0/1 = single GPU) */
  const uint8_t* nccl_id;     /* 128-byte id from rf_tp_unique_id (tp_size > 1) */
  uint32_t max_seq_len;       /* KV capacity in positions; 0 = context_length */
  uint64_t vram_budget_bytes; /* byte budget for everything the engine allocates; 0 = device free memory */
  int ring_slots;             /* out-of-core VRAM ring depth; 0 = all layers resident (non-resident
                                 layers then load and release synchronously each step) */
  int kv_f32;                 /* 1 = f32 KV cache (reference format); 0 = f16 (default) */
  int disable_graphs;         /* 1 = launch kernels eagerly instead of replaying a CUDA graph */
} rf_runtime_config;

/* One host tensor handed to rf_layer_load / rf_persistent_load. */
typedef struct rf_tensor_view {
  int role;          /* RF_ROLE_* */
  int ggml_type;     /* RF_TYPE_* */
  uint64_t ne0, ne1; /* ne1 = 1 for vectors */
  const void* host;  /* GGUF block bytes */
  uint64_t bytes;
} rf_tensor_view;

/* ResidencyStats (residency.rs:7-40) for the device weight store and ring. */
typedef struct rf_residency_stats {
  uint64_t layer_loads, layer_releases, cache_hits, cache_misses, evictions;
  uint64_t peak_bytes, h2d_bytes;
  uint64_t ring_copies;      /* layer images copied into ring slots */
  uint64_t host_image_bytes; /* pinned host images of streamed layers (not charged to the VRAM budget) */
  /* engines created from a file: coalesced reads of streamed layers' tensors
   * (layer_read.rs:50 plans), the bytes they read and the gap bytes among them */
  uint64_t file_reads, file_read_bytes, file_gap_bytes;
  /* persistent tensors (token_embd, output) that should_keep_resident (persistent.rs:468)
   * kept out of device memory under an explicit VRAM budget: held in mapped pinned host
   * memory and read by the kernels over the host link */
  uint64_t host_mapped_bytes;
} rf_residency_stats;

/* One rank's slice of a tensor-parallel engine: Q/K/V and gate/up are split by
 * rows (KV head groups, FFN rows), Wo/Wdown by columns, the LM head by vocab rows. */
typedef struct rf_tp_shard {
  uint32_t q_heads, q_head_offset, kv_heads, kv_head_offset;
  uint32_t ff_rows, ff_offset, vocab_rows, vocab_offset;
} rf_tp_shard;

typedef struct rf_engine rf_engine;

const char* rf_last_error(void);
int rf_abi_version(void);

/* ---- host-only helpers (no GPU needed) ------------------------------------ */
/* parse_gguf_file (gguf.rs:196) + LlamaConfig::from_gguf (model.rs:40-161) on an
 * in-memory GGUF image. */
int rf_gguf_read_config(const void* gguf, uint64_t len, rf_model_config* out);
/* The shard an engine of tp_size ranks gives rank tp_rank (RF_EINVAL when the
 * model does not split evenly or a slice would cut a quant block of `ggml_type`). */
int rf_tp_shard_plan(const rf_model_config* cfg, int tp_size, int tp_rank, int ggml_type, rf_tp_shard* out);

/* should_keep_resident (persistent.rs:468): 1 when a persistent tensor of
 * resident_bytes stays resident under a budget of budget_total bytes (at most a
 * quarter of it), else 0.  Overflow-free for any inputs. */
int rf_should_keep_resident(uint64_t resident_bytes, uint64_t budget_total);

/* A tensor's bytes in a GGUF file. */
typedef struct rf_tensor_extent {
  uint64_t file_offset, byte_length;
} rf_tensor_extent;
/* One read of a layer's plan: a contiguous file range holding `count` tensors
 * (entries first..first+count-1 of the plan's placements); gap_bytes are the
 * alignment/metadata bytes between them that the read carries along. */
typedef struct rf_read_range {
  uint64_t file_offset, byte_length, logical_bytes, gap_bytes;
  uint32_t first, count;
} rf_read_range;
/* Where tensor `index` (of the extents given) lands: range `range`, at
 * offset_in_range bytes into it. */
typedef struct rf_planned_tensor {
  uint32_t index, range;
  uint64_t offset_in_range;
} rf_planned_tensor;
typedef struct rf_read_plan_totals {
  uint64_t logical_tensor_count, logical_bytes, physical_bytes, gap_bytes;
  uint64_t reusable_group_buffer_bytes; /* 0: none (LayerReadPlan::reusable_group_buffer_bytes) */
} rf_read_plan_totals;
/* build_layer_read_plan (layer_read.rs:50-132): tensors sorted by file offset
 * (ties by index) are merged into one read while the gap to the previous tensor
 * is at most 4 KiB and the merged span at most 64 MiB.  Overlapping or overflowing
 * extents are RF_EINVAL; RF_ENOMEM when range_cap is too small.  placed has n
 * entries, in the reads' order. */
int rf_layer_read_plan(const rf_tensor_extent* tensors, uint32_t n, rf_read_range* ranges, uint32_t range_cap,
                       uint32_t* n_ranges, rf_planned_tensor* placed, rf_read_plan_totals* totals);

/* ---- engine lifecycle -------------------------------------------------- */
/* Empty engine for explicit layer/persistent loads (StreamingLlamaModel::load
 * without a data source, streaming_model.rs:156-182). */
int rf_engine_create(const rf_model_config* cfg, const rf_runtime_config* rt, rf_engine** out);
/* Parse a GGUF image in host memory (parse_gguf_file gguf.rs:196 +
 * LlamaConfig::from_gguf model.rs:40 + validate_required_tensors model.rs:168),
 * upload persistent weights and, when rt->ring_slots == 0, every layer.  The
 * image must stay alive while the engine may stream layers from it. */
int rf_engine_create_from_gguf(const void* gguf, uint64_t len, const rf_runtime_config* rt, rf_engine** out);
/* Same, from a file path (GgufDataSource::open, datasource.rs:97); the file is mapped. */
int rf_engine_create_from_file(const char* path, const rf_runtime_config* rt, rf_engine** out);
void rf_engine_destroy(rf_engine* e);
int rf_engine_config(const rf_engine* e, rf_model_config* out);

/* ---- weights (layer load/compute/release) --------------------------------- */
/* Persistent weight upload (PersistentWeight, persistent.rs:20-80). */
int rf_persistent_load(rf_engine* e, const rf_tensor_view* view);
/* load_layer (streaming_model.rs:581-847): copies and packs the nine tensors of one
 * layer (and its Q/K/V biases, when given) into device memory, charging the byte
 * budget "layer:<i>:weights".  A partial bias set or a bias of the wrong shape is
 * RF_EFORMAT (validate_qkv_bias, streaming_model.rs:1654-1696), with nothing charged.
 * V may have another type than Q and K (it then runs as its own matrix). */
int rf_layer_load(rf_engine* e, int layer, const rf_tensor_view* views, int n_views);
/* load_layer from the engine's own GGUF source (engines created from a GGUF). */
int rf_layer_load_gguf(rf_engine* e, int layer);
/* release_layer (streaming_model.rs:849-873): frees the layer and its charge. */
int rf_layer_release(rf_engine* e, int layer);
int rf_layer_is_resident(const rf_engine* e, int layer);
/* ModelExecutor::execute_layer (model_executor.rs:102-236) on the engine's
 * device hidden state at position pos (== KV length). The layer's K/V is written
 * at slot pos and becomes history when rf_kv_commit advances the length
 * (the deferred commit of streaming_model.rs:1289-1295). */
int rf_layer_compute(rf_engine* e, int layer, uint32_t pos);

/* ---- hidden state, token forward, logits ----------------------------------- */
/* hidden <- token_embd row (get_embedding, tensor.rs:701 / persistent.rs:80). */
int rf_embed(rf_engine* e, uint32_t token);
int rf_hidden_write(rf_engine* e, const float* host, uint32_t n);
int rf_hidden_read(rf_engine* e, float* host, uint32_t n);
/* KvCache::increment_seq_len (kv_cache.rs:415). */
int rf_kv_commit(rf_engine* e);
/* forward_single_streaming (streaming_model.rs:909-1305): pos must equal the KV
 * length (else RF_EINVAL, streaming_model.rs:921); final_hidden (n_embd floats,
 * output-normed) may be NULL. */
int rf_forward_token(rf_engine* e, uint32_t token, uint32_t pos, float* final_hidden);
/* The prompt-token loop of generate_impl (inference.rs:578-592, one
 * forward_single_streaming per prompt token) as batched passes: tokens at
 * positions [KV length, KV length + n_tokens) go through every layer in chunks of
 * 256 as tensor-core GEMMs (Q4_K and Q8_0 weights dequantized in shared memory,
 * activations split into bf16 high and low parts, f32 accumulation) with one
 * attention launch per layer and chunk.  Their K/V are committed, and the last
 * token's hidden state is left as rf_forward_token leaves it (rf_compute_logits
 * then gives its logits).  Results match the token-by-token forward within the
 * GEMM's about 2^-16 relative error per product.  RF_EUNSUPPORTED (nothing
 * changed) under tensor parallelism, with streamed layers, or when a layer matrix
 * is not Q4_K/Q8_0; RF_ETIMEOUT when a GEMM's bounded wait gave up. */
int rf_prefill(rf_engine* e, const uint32_t* tokens, uint32_t n_tokens);
/* compute_logits (streaming_model.rs:1334-1371) on the last forward's hidden plus the
 * greedy pick (Sampler::sample_checked greedy branch, sampling.rs:45-56: first
 * maximum wins).  logits (vocab floats) and argmax may each be NULL. */
int rf_compute_logits(rf_engine* e, float* logits, uint32_t* argmax);
/* One greedy decode step at pos = KV length: forward(token) + logits + argmax,
 * replayed as one CUDA graph. */
int rf_decode_step(rf_engine* e, uint32_t token, uint32_t* next_token);
/* generate_impl greedy path (inference.rs:445-759): prompt token by token, then
 * n_new greedy tokens into out (n_new entries). */
int rf_generate(rf_engine* e, const uint32_t* prompt, uint32_t n_prompt, uint32_t n_new, uint32_t* out);

/* ---- measurement hooks (the Profiler's per-event timers, profile.rs:8-60) --------- */
/* Kernels of this library one decode step launches: 5 per layer + embedding,
 * output norm, LM head with argmax, token advance, plus 2 per layer (the peer
 * sums) under tensor parallelism over peer memory. */
int rf_step_kernel_count(const rf_engine* e, uint32_t* out);
/* Failure-detection check of the bounded wait of the tensor-parallel peer sum,
 * on one GPU: a two-rank sum whose second rank is a local area that never
 * raises its flag.  The wait gives up after about a second and *err_word is 1
 * (0 would mean the phantom rank's flag arrived).  No counterpart in the
 * reference (its executor is CPU code). */
int rf_selftest_wait(int device, uint32_t* err_word);
/* n_steps greedy decode steps from `token` at pos = KV length, token fed back on
 * the device (rf_generate's loop), bracketed by CUDA events on the engine stream:
 * *device_ms = their elapsed device time.  out_tokens (n_steps) may be NULL. */
int rf_decode_timed(rf_engine* e, uint32_t token, uint32_t n_steps, uint32_t* out_tokens, float* device_ms);
/* Average device time per launch of each per-layer kernel class
 * (0 QKV+RoPE, 1 attention, 2 Wo+residual, 3 gate/up+SwiGLU, 4 down+residual),
 * each class launched over every resident layer in turn, `iters` rounds, captured
 * into one CUDA graph and replayed between events on the engine stream (device
 * time, no host launch time).  Runs at pos = KV length without committing. */
int rf_bench_layer_kernels(rf_engine* e, uint32_t iters, float* avg_ms5);

/* ---- KV cache (KvCache, kv_cache.rs:20-510) ------------------------------------ */
int rf_kv_reset(rf_engine* e);                        /* clear (kv_cache.rs clear / inference.rs:405-409) */
int rf_kv_seq_len(const rf_engine* e, uint32_t* out); /* seq_len */
/* get_k_range / get_v_range (kv_cache.rs:452-480): positions [start,end) of this
 * rank's KV heads as f32 in the reference layout [pos][kv_head][head_dim]. */
int rf_kv_read(const rf_engine* e, int layer, int which_v, uint32_t start, uint32_t end, float* host);

/* ---- byte budget and residency (MemoryBudget memory.rs:39-388, StagingPlan
 *      staging_plan.rs:46-77, should_keep_resident persistent.rs:468) ----------- */
int rf_budget_total(const rf_engine* e, uint64_t* out);
int rf_budget_used(const rf_engine* e, uint64_t* out);
int rf_budget_available(const rf_engine* e, uint64_t* out);
/* Choose which layers stay resident (mask[i] != 0) and the ring depth used for the
 * others; vram_weight_budget_bytes caps resident layer weights plus ring slots.
 * With ring_slots > 0 (and a GGUF source) every step streams the non-resident
 * layers: each is packed once into pinned host memory, then copied with
 * cudaMemcpyAsync on a side stream into one of ring_slots device slots
 * ("ring:slot:<i>" budget charges), overlapping the compute of the layers before
 * it (StagingPlan's transfer/compute overlap, staging_plan.rs:46-77, which the
 * reference leaves unsupported).  With ring_slots == 0 they load, compute and
 * release in turn (load_layer/release_layer, streaming_model.rs:1081-1270).  Kept
 * layers that are not loaded (an engine created with ring_slots > 0 uploads none)
 * are loaded from the GGUF source. */
int rf_set_residency_plan(rf_engine* e, const uint8_t* resident_mask, int ring_slots,
                          uint64_t vram_weight_budget_bytes);
/* The planner's choice for a weight budget (a MemoryBudget mapped onto a resident
 * set, the role of the reference's plan/StagingPlan, staging_plan.rs:46-77): when
 * every layer image fits vram_weight_budget_bytes (or it is 0) all layers stay
 * resident and no ring is used; else the first layers that fit beside ring_slots
 * slots of the largest image stay resident and the rest stream through the ring
 * (ring_slots 0: load, compute, release).  Applies the plan with
 * rf_set_residency_plan; mask_out (n_layers entries, may be NULL) receives it.
 * RF_ENOMEM when the ring slots alone exceed the budget. */
int rf_plan_residency(rf_engine* e, uint64_t vram_weight_budget_bytes, int ring_slots, uint8_t* mask_out);
/* LayerCache (layer_cache.rs:25-175) for layers the plan streams without a ring:
 * after its step a loaded layer stays in device memory as the most recently used
 * entry while the cached layers' bytes fit capacity_bytes, evicting least
 * recently used ones first (residency stats: evictions, cache_hits); a layer
 * larger than the capacity is released.  0 (the default) caches nothing; a new
 * capacity or residency plan empties the cache. */
int rf_set_layer_cache(rf_engine* e, uint64_t capacity_bytes);
int rf_residency_stats_get(const rf_engine* e, rf_residency_stats* out);

/* ---- tensor parallelism -------------------------------------------------------- */
/* 128-byte NCCL unique id for rank 0 to distribute (ncclGetUniqueId). */
int rf_tp_unique_id(uint8_t* out128);
/* *out = 1 when the row-parallel projections' sums run over NVLink peer memory
 * (one kernel each, cudaIpc-mapped receive areas), 0 when they use NCCL
 * all-reduce (single GPU, a peer mapping unavailable, or RF_PEER_SUM=0).  No
 * counterpart in the reference (CPU only). */
int rf_tp_peer_sum(const rf_engine* e, int* out);

/* ---- standalone ops on device pointers (benchmark configs 2 and 3) ---------------
 * A packed matrix is the device form of one GGUF weight (quantized_matvec_dispatch,
 * compute_dispatch.rs:90-254 / quantized_matvec_reference compute.rs:185-229). */
typedef struct rf_matrix rf_matrix;
/* Pack GGUF block bytes (host or device pointer, `on_device`) of an out x in
 * matrix of ggml_type on the current device. */
int rf_matrix_create(int ggml_type, const void* gguf_bytes, uint64_t bytes, int on_device, uint32_t n_out,
                     uint32_t n_in, rf_matrix** out);
void rf_matrix_destroy(rf_matrix* m);
uint64_t rf_matrix_device_bytes(const rf_matrix* m);
/* y[b][out] = W . x[b][in] for b < batch (1..8); dX, dY device pointers; stream
 * is a cudaStream_t (NULL = legacy default stream). */
int rf_qmatvec(const rf_matrix* m, const float* dX, float* dY, int batch, void* stream);
/* Y[t][out] = W . X[t] for t < n_tokens (any positive count): the batched form
 * of quantized_matvec_dispatch (compute_dispatch.rs:90-254) on the tensor cores,
 * for prompt batches.  dX [n_tokens][in] f32, dY [n_tokens][out] f32, device
 * pointers; Q4_K and Q8_0 matrices (RF_EUNSUPPORTED otherwise).  Each weight and
 * activation is split into bf16 hi + lo and multiplied as hi*hi + hi*lo + lo*hi
 * with f32 accumulation (relative error near 2^-16 against the f32 reference).
 * The split activations live in a per-device workspace the library grows. */
int rf_qgemm(const rf_matrix* m, const float* dX, float* dY, int n_tokens, void* stream);
/* Error word of rf_qgemm on the current device (synchronises it, reads, clears):
 * bit 0 = a bounded wait of the GEMM gave up, so some output since the last read
 * is unspecified.  No counterpart in the reference. */
int rf_qgemm_error_word(uint32_t* word);
/* Single-token GQA decode attention (attention_reference compute.rs:461-547)
 * for `batch` sequences: dQ [batch][H][hd] f32, dK/dV [batch][KV][ctx][hd] f16,
 * dOut [batch][H][hd] f32; softmax over all ctx positions with scale 1/sqrt(hd).
 * Split-K scratch comes from a per-device workspace the library allocates once. */
int rf_decode_attention(const float* dQ, const uint16_t* dK, const uint16_t* dV, int ctx, int n_heads,
                        int n_kv_heads, int head_dim, int batch, float* dOut, void* stream);
/* rf_decode_attention that allocates no device memory.  No counterpart in the
 * reference.  For callers that cannot call cudaMalloc: processes whose device
 * memory is already owned by another allocator (a framework's caching pool or
 * a fixed arena), where a fresh cudaMalloc fails or fragments that pool, and
 * latency-critical loops that cannot afford the device synchronisation
 * cudaMalloc/cudaFree may imply.  The split-K scratch is a fixed 16 MiB
 * array in the library, held on every GPU that loads it until exit; shapes
 * that need more return RF_EINVAL.  Every call looks the array's address up in
 * the current context (so it stays valid across a cudaDeviceReset); the first
 * call on a device may load the library's device code, so make it before any
 * stream capture.  All calls share the array: calls that overlap on the GPU
 * race.  Same arguments as rf_decode_attention; results equal its results
 * within the attention tolerance (max|o - o_ref| <= 1e-4 * max|o_ref|), and
 * exactly when the fixed scratch holds the split count rf_decode_attention
 * uses; for larger shapes the scratch forces fewer context splits, which
 * changes the f32 summation order. */
int rf_decode_attention_noalloc(const float* dQ, const uint16_t* dK, const uint16_t* dV, int ctx, int n_heads,
                                int n_kv_heads, int head_dim, int batch, float* dOut, void* stream);

#ifdef __cplusplus
}
#endif
#endif /* RFCUDA_H */
