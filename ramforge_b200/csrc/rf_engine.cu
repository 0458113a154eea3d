// rf_engine.cu - the decode engine behind include/rfcuda.h.
//
// One engine drives one GPU (one tensor-parallel rank).  Everything the decode
// step touches lives in HBM: packed layer weights, persistent embedding /
// output weights, the f16 KV cache (head-major [kv_head][pos][head_dim] so a
// CTA reads one head's history contiguously), activation scratch and the
// step's inputs (token id, position) as device words.  Because the position is
// a device word, the whole token step - embedding, every layer, output norm,
// LM head with argmax and the token/position advance - is one CUDA graph that
// is replayed unchanged for every token.
#include <dlfcn.h>
#include <errno.h>
#include <fcntl.h>
#include <math.h>
#include <nccl.h>
#include <string.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include <algorithm>
#include <memory>
#include <string>
#include <vector>

#include "rf_attn.cuh"
#include "rf_common.h"

using namespace rf;

// ---------------------------------------------------------------------------
// NCCL, loaded on demand (only tensor-parallel engines need it)
// ---------------------------------------------------------------------------
namespace {
struct NcclApi {
  ncclResult_t (*getUniqueId)(ncclUniqueId*) = nullptr;
  ncclResult_t (*commInitRank)(ncclComm_t*, int, ncclUniqueId, int) = nullptr;
  ncclResult_t (*allReduce)(const void*, void*, size_t, ncclDataType_t, ncclRedOp_t, ncclComm_t, cudaStream_t) = nullptr;
  ncclResult_t (*allGather)(const void*, void*, size_t, ncclDataType_t, ncclComm_t, cudaStream_t) = nullptr;
  ncclResult_t (*commDestroy)(ncclComm_t) = nullptr;
  const char* (*errStr)(ncclResult_t) = nullptr;
  bool ok = false;
};
NcclApi* nccl() {
  static NcclApi api;
  static bool tried = false;
  if (!tried) {
    tried = true;
    void* h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
    if (!h) h = dlopen("libnccl.so", RTLD_NOW | RTLD_GLOBAL);
    if (h) {
      api.getUniqueId = (decltype(api.getUniqueId))dlsym(h, "ncclGetUniqueId");
      api.commInitRank = (decltype(api.commInitRank))dlsym(h, "ncclCommInitRank");
      api.allReduce = (decltype(api.allReduce))dlsym(h, "ncclAllReduce");
      api.allGather = (decltype(api.allGather))dlsym(h, "ncclAllGather");
      api.commDestroy = (decltype(api.commDestroy))dlsym(h, "ncclCommDestroy");
      api.errStr = (decltype(api.errStr))dlsym(h, "ncclGetErrorString");
      api.ok = api.getUniqueId && api.commInitRank && api.allReduce && api.allGather && api.commDestroy && api.errStr;
    }
  }
  return api.ok ? &api : nullptr;
}
#define RF_NCCL(expr)                                                                           \
  do {                                                                                          \
    ncclResult_t _r = (expr);                                                                   \
    if (_r != ncclSuccess) return set_error(RF_ENCCL, "%s failed: %s", #expr, nccl()->errStr(_r)); \
  } while (0)

inline uint64_t align256(uint64_t x) { return (x + 255) & ~255ull; }

const char* kRoleNames[9] = {"attn_norm", "attn_q", "attn_k", "attn_v", "attn_output",
                             "ffn_norm", "ffn_gate", "ffn_up", "ffn_down"};
// A layer's tensor views: the nine weights (roles 0-8) and the optional qwen2
// Q/K/V biases (roles 9-11, StreamingLayerWeights::attn_{q,k,v}_bias,
// model_executor.rs:33-48).
constexpr int kLayerViews = 12;
// Prompt tokens one batched pass handles (two 128-token column blocks of the
// tensor-core GEMM), and the context splits of its attention.
constexpr uint32_t kPrefillChunk = 256;
constexpr int kPrefillSplits = 4;
const char* kBiasNames[3] = {"attn_q", "attn_k", "attn_v"};

struct Layer {
  bool resident = false;
  void* block = nullptr;
  uint64_t bytes = 0;
  PackedMat qkv{}, wo{}, gateup{}, down{};
  // V on its own when its type differs from Q/K's (then qkv holds [Q;K]); M = 0: V is in qkv
  PackedMat vmat{};
  float* attn_norm = nullptr;
  float* ffn_norm = nullptr;
  float* qkv_bias = nullptr;  // [Q;K;V] biases in packed row order (qwen2), or null
};

// A layer's weights as one contiguous device image (packed Q/K/V, W_o, gate/up,
// down, then the two norms; each part 256-byte aligned).  `tmpl` holds the
// matrices' geometry with pointers as offsets from the image base, so the same
// image can live in the layer's own allocation or in any ring slot.
struct LayerImage {
  std::vector<uint8_t> bytes;
  Layer tmpl;
};
// A streamed layer's image in pinned host memory (the source of its ring copies).
struct StreamImage {
  uint8_t* host = nullptr;
  uint64_t bytes = 0;
  Layer tmpl;
};

struct StepIO {  // device words read by the step kernels
  uint32_t token;
  int pos;
};
}  // namespace

struct rf_engine {
  rf_model_config cfg{};
  rf_runtime_config rt{};
  int dev = 0;
  int tp = 1, rank = 0;
  // local (this rank's) shard geometry
  uint32_t qh_local = 0, kvh_local = 0, q_local = 0, kv_local = 0, ff_local = 0;
  uint32_t qh_off = 0, kvh_off = 0, ff_off = 0, vocab_local = 0, vocab_off = 0, vocab_chunk = 0;
  uint32_t max_seq = 0, seq_len = 0;
  int max_splits = 0;
  Budget budget;
  cudaStream_t stream = nullptr;
  // GGUF source (optional)
  Gguf gguf;
  const uint8_t* src = nullptr;
  uint64_t src_len = 0;
  void* map_addr = nullptr;
  uint64_t map_len = 0;
  int src_fd = -1;  // the GGUF file, when the engine was created from a path: streamed layers are read from it
  bool created = false;  // creation (and its initial layer loads) finished
  uint8_t* read_stage = nullptr;  // pinned staging of a streamed layer's coalesced reads (reused)
  uint64_t read_stage_bytes = 0;
  // persistent weights
  PackedMat embd{}, out{};
  bool tied = false, have_embd = false, have_out = false, have_onorm = false;
  void* embd_block = nullptr;
  void* out_block = nullptr;
  // persistent tensors the residency policy keeps in mapped pinned host memory
  void* embd_host = nullptr;
  void* out_host = nullptr;
  uint64_t embd_host_bytes = 0, out_host_bytes = 0;
  float* out_norm = nullptr;
  std::vector<Layer> layers;
  std::vector<uint8_t> plan_resident;  // residency plan (1 = keep resident)
  // LayerCache (layer_cache.rs:25-175): layers the plan streams that stay loaded
  // after their step, least recently used first, within cache_capacity bytes
  uint64_t cache_capacity = 0, cache_used = 0;
  std::vector<int> cache_lru;
  // KV cache
  void* kv_block = nullptr;
  std::vector<void*> kc, vc;
  // scratch
  void* scratch = nullptr;
  float *hidden = nullptr, *final_hidden = nullptr, *partial = nullptr, *q = nullptr, *k_cur = nullptr,
        *v_cur = nullptr, *att = nullptr, *act = nullptr, *logits = nullptr, *logits_all = nullptr,
        *attn_part = nullptr;
  unsigned* attn_counters = nullptr;
  GemvScratch gws{};  // split-K partials + tile counters of the quantized GEMV
  // out-of-core ring: pinned host images of streamed layers, device slots fed by
  // a copy stream, and the events ordering copies against the layers' kernels
  std::vector<StreamImage> simg;
  cudaStream_t copy_stream = nullptr;
  std::vector<void*> ring;
  uint64_t ring_slot_bytes = 0;
  std::vector<cudaEvent_t> ring_free, ring_ready;
  StepIO* d_io = nullptr;
  uint32_t* d_hist = nullptr;  // token produced at each position (device-side greedy history)
  unsigned long long* d_key = nullptr;
  float2* rope_cs = nullptr;
  // pinned host words
  StepIO* h_io = nullptr;
  uint32_t* h_tok = nullptr;
  unsigned long long* h_key = nullptr;
  // graphs
  cudaGraphExec_t g_forward = nullptr, g_decode = nullptr;
  unsigned* h_err = nullptr;  // pinned copy of the peer-sum error word, read after each synchronisation
  // NCCL
  ncclComm_t comm = nullptr;
  // tensor-parallel sums over NVLink peer memory (PeerSum); NCCL when unavailable
  PeerSum ps{};
  bool ps_ok = false;
  void* ps_area = nullptr;
  std::vector<void*> ps_peer;  // peer areas mapped through cudaIpc
  // batched prompt (rf_prefill): buffers of one chunk of kPrefillChunk tokens,
  // allocated on the first call and charged as "scratch:prefill"
  void* pf_block = nullptr;
  float *pf_x = nullptr, *pf_q = nullptr, *pf_k = nullptr, *pf_v = nullptr, *pf_att = nullptr, *pf_act = nullptr,
        *pf_part = nullptr;
  unsigned *pf_cnt = nullptr, *pf_err = nullptr;
  uint32_t* pf_tok = nullptr;
  void* pf_xt = nullptr;
  PrefillKSplit pf_ks;  // K split of the W_o / W_down GEMMs
  rf_residency_stats stats{};
};

namespace {

int dev_alloc(rf_engine* e, const std::string& charge, uint64_t bytes, void** out) {
  RF_TRY(e->budget.allocate(charge, bytes));
  cudaError_t err = cudaMalloc(out, bytes);
  if (err != cudaSuccess) {
    e->budget.release(charge);
    *out = nullptr;
    return set_error(RF_ENOMEM, "cudaMalloc(%llu) for '%s' failed: %s", (unsigned long long)bytes, charge.c_str(),
                     cudaGetErrorString(err));
  }
  return RF_OK;
}
void dev_free(rf_engine* e, const std::string& charge, void** p) {
  if (*p) {
    cudaFree(*p);
    *p = nullptr;
    e->budget.release(charge);
  }
}

// Host -> device copy ordered on the engine stream and finished on return (the
// engine stream is non-blocking, so a legacy-stream copy would not order against
// its kernels, and a copy from pageable memory may return before its DMA ends).
cudaError_t h2d_sync(rf_engine* e, void* dst, const void* src, uint64_t bytes) {
  cudaError_t ce = cudaMemcpyAsync(dst, src, bytes, cudaMemcpyHostToDevice, e->stream);
  return ce == cudaSuccess ? cudaStreamSynchronize(e->stream) : ce;
}

void drop_graphs(rf_engine* e) {
  if (e->g_forward) cudaGraphExecDestroy(e->g_forward);
  if (e->g_decode) cudaGraphExecDestroy(e->g_decode);
  e->g_forward = e->g_decode = nullptr;
}

// Build the RoPE (cos, sin) table on the host with the reference's f32
// expression: angle = theta^(-2i/hd) * pos (compute.rs:446-450), evaluated by the
// same glibc powf/cosf/sinf the Rust f32 methods call.
std::vector<float2> rope_table(uint32_t max_seq, uint32_t hd, float theta) {
  const uint32_t half = hd / 2;
  std::vector<float> inv(half);
  for (uint32_t i = 0; i < half; i++) {
    const float ex = -2.0f * (float)i / (float)hd;
    inv[i] = powf(theta, ex);
  }
  std::vector<float2> t((size_t)max_seq * half);
  for (uint32_t p = 0; p < max_seq; p++)
    for (uint32_t i = 0; i < half; i++) {
      const float angle = inv[i] * (float)p;
      t[(size_t)p * half + i] = make_float2(cosf(angle), sinf(angle));
    }
  return t;
}

int validate_config(const rf_model_config& c, int tp) {
  if (!c.n_embd || !c.n_layers || !c.n_heads || !c.n_kv_heads || !c.vocab_size || !c.n_ff)
    return set_error(RF_EINVAL, "model config has a zero dimension");
  if (c.n_heads % c.n_kv_heads) return set_error(RF_EINVAL, "GQA requires n_heads %% n_kv_heads == 0");
  if (!c.head_dim || c.head_dim % 2 || c.head_dim > 128)
    return set_error(RF_EUNSUPPORTED, "head_dim %u unsupported (even, <= 128)", c.head_dim);
  const uint32_t G = c.n_heads / c.n_kv_heads;
  if (G != 1 && G != 2 && G != 4 && G != 8) return set_error(RF_EUNSUPPORTED, "GQA group %u unsupported", G);
  if (c.n_kv_heads % tp || c.n_ff % tp) return set_error(RF_EINVAL, "tp %d must divide n_kv_heads and n_ff", tp);
  return RF_OK;
}

// Vocabulary rows per rank: an even split rounded up to whole 64-row tiles of
// the packed LM head, so every shard starts on a tile (the last one is shorter).
uint32_t vocab_chunk_of(const rf_model_config& c, int tp) {
  if (tp <= 1) return c.vocab_size;
  return ((c.vocab_size + tp - 1) / tp + QT_ROWS - 1) / QT_ROWS * QT_ROWS;
}

int shard_plan(const rf_model_config& c, int tp, int rank, int block, rf_tp_shard* o) {
  if (tp < 1 || rank < 0 || rank >= tp) return set_error(RF_EINVAL, "tp_rank %d / tp_size %d invalid", rank, tp);
  RF_TRY(validate_config(c, tp));
  const uint32_t G = c.n_heads / c.n_kv_heads;
  o->kv_heads = c.n_kv_heads / tp;
  o->kv_head_offset = o->kv_heads * rank;
  o->q_heads = o->kv_heads * G;
  o->q_head_offset = o->kv_head_offset * G;
  o->ff_rows = c.n_ff / tp;
  o->ff_offset = o->ff_rows * rank;
  const uint32_t chunk = vocab_chunk_of(c, tp);
  o->vocab_offset = std::min(c.vocab_size, chunk * rank);
  o->vocab_rows = std::min(c.vocab_size, o->vocab_offset + chunk) - o->vocab_offset;
  if (o->vocab_rows == 0)
    return set_error(RF_EINVAL, "tp %d: a vocabulary of %u rows leaves rank %d no whole 64-row tile", tp,
                     c.vocab_size, rank);
  if (tp > 1 && block > 1) {  // row-parallel column slices must not cut a quant block
    const uint32_t q_cols = o->q_heads * c.head_dim;
    if (q_cols % block || o->ff_rows % block)
      return set_error(RF_EINVAL, "tp %d: shard widths (%u attention columns, %u FFN columns) are not multiples of "
                       "the %d-element quant block", tp, q_cols, o->ff_rows, block);
  }
  return RF_OK;
}

int setup_geometry(rf_engine* e) {
  const rf_model_config& c = e->cfg;
  e->tp = e->rt.tp_size > 1 ? e->rt.tp_size : 1;
  e->rank = e->tp > 1 ? e->rt.tp_rank : 0;
  rf_tp_shard sh{};
  RF_TRY(shard_plan(c, e->tp, e->rank, 1, &sh));
  e->kvh_local = sh.kv_heads;
  e->kvh_off = sh.kv_head_offset;
  e->qh_local = sh.q_heads;
  e->qh_off = sh.q_head_offset;
  e->q_local = e->qh_local * c.head_dim;
  e->kv_local = e->kvh_local * c.head_dim;
  e->ff_local = sh.ff_rows;
  e->ff_off = sh.ff_offset;
  e->vocab_chunk = vocab_chunk_of(c, e->tp);
  e->vocab_off = sh.vocab_offset;
  e->vocab_local = sh.vocab_rows;
  e->max_seq = e->rt.max_seq_len ? e->rt.max_seq_len : c.context_length;
  if (!e->max_seq) return set_error(RF_EINVAL, "max_seq_len is zero");
  // attention splits: one per 64 positions of the longest context this engine
  // holds (so the attention grid has no more units than a step can use), at most
  // 64 (512 positions a split past 32k)
  e->max_splits = std::min<int>(attn_nsplit((int)e->max_seq, 1 << 30), std::max<int>(64, (int)((e->max_seq + 511) / 512)));
  return RF_OK;
}

// Peer-memory tensor-parallel sums (PeerSum): every rank exports one area through
// cudaIpc, the handles travel by an NCCL all-gather, and every rank maps the
// others'.  The ranks agree (an NCCL min) before using it, so either all ranks
// sum over peer memory or all use NCCL all-reduce.  RF_PEER_SUM=0 forces NCCL.
int setup_peer_sum(rf_engine* e) {
  e->ps_ok = false;
  const char* env = getenv("RF_PEER_SUM");
  bool ok = !(env && env[0] == '0') && e->tp <= RF_MAX_TP && e->cfg.n_embd % 4 == 0;
  PeerSum& P = e->ps;
  P = PeerSum{};
  P.rank = e->rank;
  P.n_ranks = e->tp;
  P.n_max = (int)e->cfg.n_embd;
  P.sites = 2 * (int)e->cfg.n_layers;
  const size_t bytes = peer_sum_area_bytes(P.n_ranks, P.n_max, P.sites);
  uint8_t* d_x = nullptr;  // [tp][64] handle bytes, then one int for the agreement
  RF_CUDA(cudaMalloc(&d_x, 64ull * e->tp + 64));
  std::vector<cudaIpcMemHandle_t> h(e->tp);
  memset(h.data(), 0, sizeof(cudaIpcMemHandle_t) * h.size());
  if (ok && dev_alloc(e, "scratch:peer_sum", bytes, &e->ps_area) != RF_OK) ok = false;
  if (ok)
    ok = cudaMemsetAsync(e->ps_area, 0, bytes, e->stream) == cudaSuccess &&
         cudaStreamSynchronize(e->stream) == cudaSuccess && cudaIpcGetMemHandle(&h[e->rank], e->ps_area) == cudaSuccess;
  cudaGetLastError();
  int rc = RF_OK;
  cudaError_t ce = h2d_sync(e, d_x + 64ull * e->rank, &h[e->rank], sizeof(cudaIpcMemHandle_t));
  if (ce == cudaSuccess) {
    const ncclResult_t r = nccl()->allGather(d_x + 64ull * e->rank, d_x, 64, ncclUint8, e->comm, e->stream);
    if (r != ncclSuccess) rc = set_error(RF_ENCCL, "peer-sum handle exchange failed: %s", nccl()->errStr(r));
  }
  if (!rc && ce == cudaSuccess) ce = cudaMemcpyAsync(h.data(), d_x, 64ull * e->tp, cudaMemcpyDeviceToHost, e->stream);
  if (!rc && ce == cudaSuccess) ce = cudaStreamSynchronize(e->stream);
  e->ps_peer.assign(e->tp, nullptr);
  for (int p = 0; !rc && ce == cudaSuccess && ok && p < e->tp; p++) {
    if (p == e->rank) continue;
    if (cudaIpcOpenMemHandle(&e->ps_peer[p], h[p], cudaIpcMemLazyEnablePeerAccess) != cudaSuccess) {
      cudaGetLastError();
      e->ps_peer[p] = nullptr;
      ok = false;
    }
  }
  // agreement: the minimum over ranks of ok
  int flag = ok ? 1 : 0;
  if (!rc && ce == cudaSuccess) ce = h2d_sync(e, d_x + 64ull * e->tp, &flag, sizeof flag);
  if (!rc && ce == cudaSuccess) {
    const ncclResult_t r =
        nccl()->allReduce(d_x + 64ull * e->tp, d_x + 64ull * e->tp, 1, ncclInt32, ncclMin, e->comm, e->stream);
    if (r != ncclSuccess) rc = set_error(RF_ENCCL, "peer-sum agreement failed: %s", nccl()->errStr(r));
  }
  if (!rc && ce == cudaSuccess)
    ce = cudaMemcpyAsync(&flag, d_x + 64ull * e->tp, sizeof flag, cudaMemcpyDeviceToHost, e->stream);
  if (!rc && ce == cudaSuccess) ce = cudaStreamSynchronize(e->stream);
  cudaFree(d_x);
  if (!rc && ce != cudaSuccess) rc = set_error(RF_ECUDA, "peer-sum setup failed: %s", cudaGetErrorString(ce));
  if (rc || flag != 1) {  // every rank falls back to NCCL
    for (void* q : e->ps_peer)
      if (q) cudaIpcCloseMemHandle(q);
    e->ps_peer.clear();
    if (e->ps_area) dev_free(e, "scratch:peer_sum", &e->ps_area);
    return rc;
  }
  for (int p = 0; p < e->tp; p++) peer_sum_bind(&P, p, p == e->rank ? e->ps_area : e->ps_peer[p], p == e->rank);
  e->ps_ok = true;
  return RF_OK;
}

int engine_init_device(rf_engine* e) {
  const rf_model_config& c = e->cfg;
  RF_CUDA(cudaSetDevice(e->dev));
  RF_CUDA(cudaStreamCreateWithFlags(&e->stream, cudaStreamNonBlocking));
  size_t free_b = 0, total_b = 0;
  RF_CUDA(cudaMemGetInfo(&free_b, &total_b));
  e->budget = Budget(e->rt.vram_budget_bytes ? e->rt.vram_budget_bytes : (uint64_t)free_b);
  e->layers.assign(c.n_layers, Layer{});
  e->plan_resident.assign(c.n_layers, 1);
  e->simg.assign(c.n_layers, StreamImage{});
  // KV cache: per layer K and V, [kv_head_local][max_seq][head_dim]
  const uint64_t esz = e->rt.kv_f32 ? 4 : 2;
  const uint64_t per = align256((uint64_t)e->kvh_local * e->max_seq * c.head_dim * esz);
  RF_TRY(dev_alloc(e, "kv_cache", per * 2 * c.n_layers, &e->kv_block));
  e->kc.resize(c.n_layers);
  e->vc.resize(c.n_layers);
  for (uint32_t l = 0; l < c.n_layers; l++) {
    e->kc[l] = (uint8_t*)e->kv_block + per * (2 * l);
    e->vc[l] = (uint8_t*)e->kv_block + per * (2 * l + 1);
  }
  // scratch
  const uint32_t G = c.n_heads / c.n_kv_heads;
  const uint64_t part_f = attn_part_floats(1, e->kvh_local, e->max_splits, G, c.head_dim);
  // GEMV split-K scratch for any matrix this rank can hold, sized for the
  // smallest chunk (128 elements, Q8_0): one 64-row partial per piece
  uint64_t gpart = 0;
  uint32_t gcnt = 0;
  const uint32_t shapes[5][2] = {{e->q_local + 2 * e->kv_local, c.n_embd},
                                 {c.n_embd, e->q_local},
                                 {2 * e->ff_local, c.n_embd},
                                 {c.n_embd, e->ff_local},
                                 {e->vocab_local, c.n_embd}};
  for (auto& sh : shapes) {
    const uint64_t mp = (sh[0] + QT_ROWS - 1) / QT_ROWS * QT_ROWS;
    gpart = std::max<uint64_t>(gpart, mp * ((sh[1] + 127) / 128) * QT_PIECES);
    gcnt = std::max<uint32_t>(gcnt, (uint32_t)(mp / QT_ROWS));
  }
  e->gws.part_floats = gpart;
  e->gws.n_cnt = gcnt;
  // the residual GEMMs split K over CTA pairs only when their blocks fill at most
  // half the SMs, so half the SM count bounds the blocks that need scratch
  const uint32_t ks_tiles = (uint32_t)std::max(1, num_sms() / 2);
  struct Item { void** p; uint64_t bytes; };
  const uint64_t vl_pad = (uint64_t)e->vocab_chunk;
  std::vector<Item> items = {
      {(void**)&e->hidden, 4ull * c.n_embd},        {(void**)&e->final_hidden, 4ull * c.n_embd},
      {(void**)&e->partial, 4ull * c.n_embd},       {(void**)&e->q, 4ull * e->q_local},
      {(void**)&e->k_cur, 4ull * e->kv_local},      {(void**)&e->v_cur, 4ull * e->kv_local},
      {(void**)&e->att, 4ull * e->q_local},         {(void**)&e->act, 4ull * e->ff_local},
      {(void**)&e->logits, 4ull * vl_pad},          {(void**)&e->logits_all, 4ull * vl_pad * e->tp},
      {(void**)&e->attn_part, 4ull * part_f},       {(void**)&e->attn_counters, 4ull * e->kvh_local},
      {(void**)&e->gws.part, 4ull * gpart},         {(void**)&e->gws.cnt, 4ull * gcnt},
      {(void**)&e->d_io, sizeof(StepIO)},           {(void**)&e->d_key, 8},
      {(void**)&e->d_hist, 4ull * e->max_seq},
      {(void**)&e->rope_cs, 8ull * e->max_seq * (c.head_dim / 2)}};
  uint64_t total = 0;
  for (auto& it : items) total += align256(it.bytes);
  RF_TRY(dev_alloc(e, "scratch:activations", total, &e->scratch));
  // zeroed on the engine stream: a legacy-stream memset is not ordered against
  // the engine stream's copies and kernels
  RF_CUDA(cudaMemsetAsync(e->scratch, 0, total, e->stream));
  RF_CUDA(cudaStreamSynchronize(e->stream));
  uint64_t off = 0;
  for (auto& it : items) {
    *it.p = (uint8_t*)e->scratch + off;
    off += align256(it.bytes);
  }
  auto tab = rope_table(e->max_seq, c.head_dim, c.rope_theta);
  RF_CUDA(h2d_sync(e, e->rope_cs, tab.data(), tab.size() * sizeof(float2)));
  // one pinned {token, pos} slot per position: asynchronous steps never share a source slot
  RF_CUDA(cudaMallocHost((void**)&e->h_io, sizeof(StepIO) * (e->max_seq + 1)));
  RF_CUDA(cudaMallocHost((void**)&e->h_tok, 4 * 4096));
  RF_CUDA(cudaMallocHost((void**)&e->h_key, 8));
  RF_CUDA(cudaMallocHost((void**)&e->h_err, 8));
  e->h_err[0] = 0;
  if (e->tp > 1) {
    if (!nccl()) return set_error(RF_ENCCL, "tensor parallelism needs libnccl.so.2, which could not be loaded");
    if (!e->rt.nccl_id) return set_error(RF_EINVAL, "tp_size > 1 requires nccl_id");
    ncclUniqueId id;
    memcpy(&id, e->rt.nccl_id, sizeof id);
    RF_NCCL(nccl()->commInitRank(&e->comm, e->tp, id, e->rank));
    RF_TRY(setup_peer_sum(e));
  }
  return RF_OK;
}

// ---- weight packing ----------------------------------------------------------------
struct View {
  int type = -1;
  int ndims = 2;
  uint64_t ne0 = 0, ne1 = 0, bytes = 0;
  const uint8_t* host = nullptr;
};

int check_view(const View& v, const char* what, uint64_t ne0, uint64_t ne1) {
  if (!v.host) return set_error(RF_EINVAL, "missing tensor %s", what);
  if (v.ne0 != ne0 || v.ne1 != ne1)
    return set_error(RF_EINVAL, "%s shape mismatch: expected [%llu, %llu], got [%llu, %llu]", what,
                     (unsigned long long)ne0, (unsigned long long)ne1, (unsigned long long)v.ne0,
                     (unsigned long long)v.ne1);
  const int qk = block_elems(v.type);
  if (!qk) return set_error(RF_EFORMAT, "%s: tensor type %d is not supported by the engine", what, v.type);
  if (ne0 % qk) return set_error(RF_EFORMAT, "%s: row length %llu not a multiple of %d", what, (unsigned long long)ne0, qk);
  const uint64_t need = ne0 / qk * block_bytes(v.type) * ne1;
  if (v.bytes < need)
    return set_error(RF_EINVAL, "%s truncated: expected %llu bytes, got %llu", what, (unsigned long long)need,
                     (unsigned long long)v.bytes);
  return RF_OK;
}

uint64_t row_bytes_of(const View& v) { return v.ne0 / block_elems(v.type) * block_bytes(v.type); }

// A matrix view of a format the engine stores as f32 (expands_to_f32) decoded into
// `store` (the reference's dequantize, value for value) and described as F32; any
// other view is passed through.
int expand_view(const View& v, std::vector<float>* store, View* out) {
  *out = v;
  if (!v.host || !expands_to_f32(v.type)) return RF_OK;
  store->resize(v.ne0 * v.ne1);
  RF_TRY(expand_rows_f32(v.type, v.host, row_bytes_of(v), v.ne1, (uint32_t)v.ne0, store->data()));
  out->type = T_F32;
  out->host = reinterpret_cast<const uint8_t*>(store->data());
  out->bytes = 4ull * v.ne0 * v.ne1;
  return RF_OK;
}

// f32 copy of a norm vector (F32 or F16 storage; TensorData F16 rows are f32 after load)
int norm_to_f32(const View& v, uint32_t n, std::vector<float>* out) {
  out->resize(n);
  if (v.type == T_F32) memcpy(out->data(), v.host, 4ull * n);
  else if (v.type == T_F16) {
    for (uint32_t i = 0; i < n; i++) {
      uint16_t h;
      memcpy(&h, v.host + 2ull * i, 2);
      const float f = __half2float(__ushort_as_half(h));
      (*out)[i] = (h & 0x7C00u) ? f : f * 0.5f;  // reference f16 decode (tensor.rs:1017-1041)
    }
  } else {
    return set_error(RF_EUNSUPPORTED, "norm weights of type %d are not supported", v.type);
  }
  return RF_OK;
}

std::vector<int> iota_rows(uint32_t start, uint32_t n) {
  std::vector<int> r(n);
  for (uint32_t i = 0; i < n; i++) r[i] = (int)(start + i);
  return r;
}
// Packed order pairing dimension i with i+hd/2 of every head in [h0, h0+nh).
std::vector<int> rope_pair_rows(uint32_t h0, uint32_t nh, uint32_t hd) {
  std::vector<int> r;
  r.reserve((size_t)nh * hd);
  const uint32_t half = hd / 2;
  for (uint32_t h = 0; h < nh; h++)
    for (uint32_t i = 0; i < half; i++) {
      r.push_back((int)((h0 + h) * hd + i));
      r.push_back((int)((h0 + h) * hd + i + half));
    }
  return r;
}

// Place a packed matrix in a layer image at *off: qs | sc (each 256-byte aligned).
void image_put(const HostPacked& hp, std::vector<uint8_t>* img, uint64_t* off, PackedMat* dst) {
  *dst = hp.geo;
  dst->qs = reinterpret_cast<uint8_t*>(*off);
  memcpy(img->data() + *off, hp.qs.data(), hp.qs.size());
  *off += align256(hp.qs.size());
  dst->sc = reinterpret_cast<uint8_t*>(*off);
  if (!hp.sc.empty()) memcpy(img->data() + *off, hp.sc.data(), hp.sc.size());
  *off += align256(hp.sc.size() ? hp.sc.size() : 16);
  dst->sub_scales = has_subnormal_scales(hp.geo, hp.sc.data()) ? 1 : 0;
}
uint64_t packed_bytes(const HostPacked& hp) { return align256(hp.qs.size()) + align256(hp.sc.size() ? hp.sc.size() : 16); }

// Image pointers (offsets) -> addresses inside the image at `base`.
void bind_layer(Layer* L, const Layer& tmpl, uint8_t* base) {
  auto rebase = [base](PackedMat m) {
    m.qs = base + reinterpret_cast<uintptr_t>(m.qs);
    m.sc = base + reinterpret_cast<uintptr_t>(m.sc);
    return m;
  };
  L->qkv = rebase(tmpl.qkv);
  L->wo = rebase(tmpl.wo);
  L->gateup = rebase(tmpl.gateup);
  L->down = rebase(tmpl.down);
  L->vmat = tmpl.vmat.M ? rebase(tmpl.vmat) : PackedMat{};
  L->attn_norm = reinterpret_cast<float*>(base + reinterpret_cast<uintptr_t>(tmpl.attn_norm));
  L->ffn_norm = reinterpret_cast<float*>(base + reinterpret_cast<uintptr_t>(tmpl.ffn_norm));
  L->qkv_bias = tmpl.qkv_bias ? reinterpret_cast<float*>(base + reinterpret_cast<uintptr_t>(tmpl.qkv_bias)) : nullptr;
  L->bytes = tmpl.bytes;
}

// validate_qkv_bias (streaming_model.rs:1654-1696): the three biases come all or
// none, each 1-D of the projection's output size.
int validate_qkv_bias(const View* v, int l, uint64_t qd, uint64_t kvd) {
  const bool p[3] = {v[9].host != nullptr, v[10].host != nullptr, v[11].host != nullptr};
  const int count = (int)p[0] + (int)p[1] + (int)p[2];
  if (count == 0) return RF_OK;
  if (count != 3)
    return set_error(RF_EFORMAT,
                     "layer %d has an incomplete Q/K/V bias set (q.bias: %s, k.bias: %s, v.bias: %s); refusing to "
                     "run inference with partial biases",
                     l, p[0] ? "true" : "false", p[1] ? "true" : "false", p[2] ? "true" : "false");
  const uint64_t want[3] = {qd, kvd, kvd};
  for (int i = 0; i < 3; i++) {
    const View& b = v[9 + i];
    if (b.ndims != 1 || b.ne0 != want[i])
      return set_error(RF_EFORMAT, "invalid blk.%d.%s.bias shape: expected 1D [%llu], got %s[%llu, %llu]", l,
                       kBiasNames[i], (unsigned long long)want[i], b.ndims == 1 ? "1D " : "",
                       (unsigned long long)b.ne0, (unsigned long long)b.ne1);
    if (b.type != T_F32 && b.type != T_F16)
      return set_error(RF_EUNSUPPORTED, "blk.%d.%s.bias: tensor type %d is not supported", l, kBiasNames[i], b.type);
    if (b.bytes < want[i] * (b.type == T_F32 ? 4 : 2))
      return set_error(RF_EINVAL, "blk.%d.%s.bias truncated", l, kBiasNames[i]);
  }
  return RF_OK;
}

// load_layer's packing (streaming_model.rs:581-847) into a host image: this
// rank's rows of Q/K/V (RoPE pairs adjacent), W_o, interleaved gate/up and
// down, in the tiled layout, plus the norms as f32.
int build_layer_image(rf_engine* e, int l, const View* vin /*[kLayerViews]*/, LayerImage* out) {
  const rf_model_config& c = e->cfg;
  const uint32_t hd = c.head_dim, qd = c.n_heads * hd, kvd = c.n_kv_heads * hd;
  RF_TRY(check_view(vin[0], "attn_norm", c.n_embd, 1));
  RF_TRY(check_view(vin[1], "attn_q", c.n_embd, qd));
  RF_TRY(check_view(vin[2], "attn_k", c.n_embd, kvd));
  RF_TRY(check_view(vin[3], "attn_v", c.n_embd, kvd));
  RF_TRY(check_view(vin[4], "attn_output", qd, c.n_embd));
  RF_TRY(check_view(vin[5], "ffn_norm", c.n_embd, 1));
  RF_TRY(check_view(vin[6], "ffn_gate", c.n_embd, c.n_ff));
  RF_TRY(check_view(vin[7], "ffn_up", c.n_embd, c.n_ff));
  RF_TRY(check_view(vin[8], "ffn_down", c.n_ff, c.n_embd));
  RF_TRY(validate_qkv_bias(vin, l, qd, kvd));
  // matrices in formats stored as f32 are decoded here; from now on they are F32
  std::vector<float> xs[kLayerViews];
  View v[kLayerViews];
  for (int j = 0; j < kLayerViews; j++) RF_TRY(expand_view(vin[j], &xs[j], &v[j]));
  if (v[1].type != v[2].type)
    return set_error(RF_EUNSUPPORTED, "layer %d: Q and K of different types are not supported", l);
  // V of another type (e.g. Q6_K beside Q4_K Q/K) is its own matrix, run as a
  // second launch of the same epilogue
  const bool split_v = v[3].type != v[1].type;
  if (v[6].type != v[7].type) return set_error(RF_EUNSUPPORTED, "layer %d: gate/up of different types", l);
  const uint32_t qk_o = block_elems(v[4].type), qk_d = block_elems(v[8].type);
  if ((e->qh_off * hd) % qk_o || e->q_local % qk_o || e->ff_off % qk_d || e->ff_local % qk_d)
    return set_error(RF_EINVAL, "tensor-parallel shard of layer %d does not fall on block boundaries", l);
  HostPacked qkv, vm, wo, gu, dn;
  const std::vector<int> qrows = rope_pair_rows(e->qh_off, e->qh_local, hd),
                         krows = rope_pair_rows(e->kvh_off, e->kvh_local, hd),
                         vrows = iota_rows(e->kvh_off * hd, e->kv_local);
  RF_TRY(host_packed_init(v[1].type, e->q_local + (split_v ? 1 : 2) * e->kv_local, c.n_embd, &qkv));
  RF_TRY(pack_rows(v[1].host, row_bytes_of(v[1]), 0, qrows, &qkv, 0, 1));
  RF_TRY(pack_rows(v[2].host, row_bytes_of(v[2]), 0, krows, &qkv, e->q_local, 1));
  if (split_v) {
    RF_TRY(host_packed_init(v[3].type, e->kv_local, c.n_embd, &vm));
    RF_TRY(pack_rows(v[3].host, row_bytes_of(v[3]), 0, vrows, &vm, 0, 1));
  } else {
    RF_TRY(pack_rows(v[3].host, row_bytes_of(v[3]), 0, vrows, &qkv, e->q_local + e->kv_local, 1));
  }
  // biases in the packed row order of this rank's Q/K/V rows
  const bool has_bias = v[9].host != nullptr;
  const uint32_t nbias = e->q_local + 2 * e->kv_local;
  std::vector<float> bias;
  if (has_bias) {
    std::vector<float> bq, bk, bv;
    RF_TRY(norm_to_f32(v[9], qd, &bq));
    RF_TRY(norm_to_f32(v[10], kvd, &bk));
    RF_TRY(norm_to_f32(v[11], kvd, &bv));
    bias.resize(nbias);
    for (uint32_t i = 0; i < e->q_local; i++) bias[i] = bq[qrows[i]];
    for (uint32_t i = 0; i < e->kv_local; i++) bias[e->q_local + i] = bk[krows[i]];
    for (uint32_t i = 0; i < e->kv_local; i++) bias[e->q_local + e->kv_local + i] = bv[vrows[i]];
  }
  RF_TRY(host_packed_init(v[4].type, c.n_embd, e->q_local, &wo));
  RF_TRY(pack_rows(v[4].host, row_bytes_of(v[4]), e->qh_off * hd / qk_o, iota_rows(0, c.n_embd), &wo, 0, 1));
  RF_TRY(host_packed_init(v[6].type, 2 * e->ff_local, c.n_embd, &gu));
  RF_TRY(pack_rows(v[6].host, row_bytes_of(v[6]), 0, iota_rows(e->ff_off, e->ff_local), &gu, 0, 2));
  RF_TRY(pack_rows(v[7].host, row_bytes_of(v[7]), 0, iota_rows(e->ff_off, e->ff_local), &gu, 1, 2));
  RF_TRY(host_packed_init(v[8].type, c.n_embd, e->ff_local, &dn));
  RF_TRY(pack_rows(v[8].host, row_bytes_of(v[8]), e->ff_off / qk_d, iota_rows(0, c.n_embd), &dn, 0, 1));
  std::vector<float> an, fn;
  RF_TRY(norm_to_f32(v[0], c.n_embd, &an));
  RF_TRY(norm_to_f32(v[5], c.n_embd, &fn));
  const uint64_t total = packed_bytes(qkv) + (split_v ? packed_bytes(vm) : 0) + packed_bytes(wo) + packed_bytes(gu) +
                         packed_bytes(dn) + 2 * align256(4ull * c.n_embd) + (has_bias ? align256(4ull * nbias) : 0);
  out->bytes.assign(total, 0);
  Layer& t = out->tmpl;
  t = Layer{};
  uint64_t off = 0;
  image_put(qkv, &out->bytes, &off, &t.qkv);
  if (split_v) image_put(vm, &out->bytes, &off, &t.vmat);
  image_put(wo, &out->bytes, &off, &t.wo);
  image_put(gu, &out->bytes, &off, &t.gateup);
  image_put(dn, &out->bytes, &off, &t.down);
  t.attn_norm = reinterpret_cast<float*>(off);
  memcpy(out->bytes.data() + off, an.data(), 4ull * c.n_embd);
  off += align256(4ull * c.n_embd);
  t.ffn_norm = reinterpret_cast<float*>(off);
  memcpy(out->bytes.data() + off, fn.data(), 4ull * c.n_embd);
  off += align256(4ull * c.n_embd);
  if (has_bias) {
    t.qkv_bias = reinterpret_cast<float*>(off);
    memcpy(out->bytes.data() + off, bias.data(), 4ull * nbias);
  }
  t.bytes = total;
  return RF_OK;
}

int load_layer_views(rf_engine* e, int l, const View* v /*[kLayerViews]*/) {
  LayerImage img;
  RF_TRY(build_layer_image(e, l, v, &img));
  Layer& L = e->layers[l];
  const std::string charge = "layer:" + std::to_string(l) + ":weights";
  RF_TRY(dev_alloc(e, charge, img.tmpl.bytes, &L.block));
  cudaError_t ce = h2d_sync(e, L.block, img.bytes.data(), img.tmpl.bytes);
  if (ce != cudaSuccess) {  // release_layer on every error path (streaming_model.rs:1170-1270)
    dev_free(e, charge, &L.block);
    return set_error(RF_ECUDA, "layer %d upload failed: %s", l, cudaGetErrorString(ce));
  }
  void* block = L.block;
  bind_layer(&L, img.tmpl, (uint8_t*)block);
  L.block = block;
  L.resident = true;
  e->stats.layer_loads++;
  e->stats.h2d_bytes += img.tmpl.bytes;
  e->stats.peak_bytes = e->budget.peak();
  drop_graphs(e);
  return RF_OK;
}

View view_from_gguf(const GgufTensor* t) {
  View v;
  if (!t) return v;
  v.type = (int)t->type;
  v.ndims = (int)t->dims.size();
  v.ne0 = t->dims.size() > 0 ? t->dims[0] : 1;
  v.ne1 = t->dims.size() > 1 ? t->dims[1] : 1;
  v.bytes = t->nbytes;
  v.host = t->data;
  return v;
}

int lm_head(rf_engine* e, PackedMat* W);

int load_persistent(rf_engine* e, int role, const View& v0) {
  const rf_model_config& c = e->cfg;
  if (role == RF_ROLE_OUTPUT_NORM) {
    RF_TRY(check_view(v0, "output_norm", c.n_embd, 1));
    std::vector<float> w;
    RF_TRY(norm_to_f32(v0, c.n_embd, &w));
    void* p = nullptr;
    if (!e->out_norm) {
      RF_TRY(dev_alloc(e, "persistent:output_norm", 4ull * c.n_embd, &p));
      e->out_norm = (float*)p;
    }
    RF_CUDA(h2d_sync(e, e->out_norm, w.data(), 4ull * c.n_embd));
    e->have_onorm = true;
  } else if (role == RF_ROLE_TOKEN_EMBD || role == RF_ROLE_OUTPUT) {
    const bool is_embd = role == RF_ROLE_TOKEN_EMBD;
    // get_embedding expects [n_embd, vocab] (tensor.rs:706-714)
    RF_TRY(check_view(v0, is_embd ? "token_embd" : "output", c.n_embd, c.vocab_size));
    std::vector<float> xs;
    View v;
    RF_TRY(expand_view(v0, &xs, &v));
    HostPacked hp;
    const uint32_t rows = is_embd ? c.vocab_size : e->vocab_local;
    const uint32_t r0 = is_embd ? 0 : e->vocab_off;
    RF_TRY(host_packed_init(v.type, rows, c.n_embd, &hp));
    RF_TRY(pack_rows(v.host, row_bytes_of(v), 0, iota_rows(r0, rows), &hp, 0, 1));
    const std::string charge = is_embd ? "persistent:token_embd" : "persistent:output";
    void** blk = is_embd ? &e->embd_block : &e->out_block;
    void** hblk = is_embd ? &e->embd_host : &e->out_host;
    dev_free(e, charge, blk);
    if (*hblk) {
      e->stats.host_mapped_bytes -= is_embd ? e->embd_host_bytes : e->out_host_bytes;
      cudaFreeHost(*hblk);
      *hblk = nullptr;
    }
    const uint64_t pbytes = packed_bytes(hp);
    std::vector<uint8_t> img(pbytes);
    uint64_t off = 0;
    PackedMat* dst = is_embd ? &e->embd : &e->out;
    image_put(hp, &img, &off, dst);
    uint8_t* base = nullptr;
    // PersistentWeight's policy (should_keep_resident, persistent.rs:468; applied at
    // streaming_model.rs:1586): under an explicit VRAM budget a tensor larger than a
    // quarter of it is not kept in device memory.  Here it stays in mapped pinned
    // host memory and the same kernels read it over the host link (the streamed
    // embedding row and output projection of persistent.rs:80-209, 286-466).
    if (e->rt.vram_budget_bytes && !rf_should_keep_resident(pbytes, e->budget.total())) {
      RF_CUDA(cudaHostAlloc(hblk, pbytes, cudaHostAllocMapped));
      memcpy(*hblk, img.data(), pbytes);
      void* dptr = nullptr;
      RF_CUDA(cudaHostGetDevicePointer(&dptr, *hblk, 0));
      base = (uint8_t*)dptr;
      (is_embd ? e->embd_host_bytes : e->out_host_bytes) = pbytes;
      e->stats.host_mapped_bytes += pbytes;
    } else {
      RF_TRY(dev_alloc(e, charge, pbytes, blk));
      RF_CUDA(h2d_sync(e, *blk, img.data(), img.size()));
      base = (uint8_t*)*blk;
      e->stats.h2d_bytes += pbytes;
    }
    dst->qs = base + reinterpret_cast<uintptr_t>(dst->qs);
    dst->sc = base + reinterpret_cast<uintptr_t>(dst->sc);
    if (is_embd) e->have_embd = true;
    else { e->have_out = true; e->tied = false; }
  } else {
    return set_error(RF_EINVAL, "unknown persistent role %d", role);
  }
  drop_graphs(e);
  return RF_OK;
}

// The LM head matrix: output.weight, or the tied embedding rows of this rank
// (compute_logits uses token_embd when output.weight is absent, streaming_model.rs:1353).
int lm_head(rf_engine* e, PackedMat* W) {
  if (e->have_out) { *W = e->out; return RF_OK; }
  if (!e->have_embd) return set_error(RF_ESTATE, "no output or token_embd weights loaded");
  // rows [vocab_off, vocab_off + vocab_local) of the embedding: whole 64-row
  // tiles (shard_plan aligns vocabulary shards), so the sub-matrix is a suffix of
  // the same layout
  if (is_tiled(e->embd.type) && e->vocab_off % QT_ROWS)
    return set_error(RF_ESTATE, "vocabulary shard offset %u is not a multiple of %d rows", e->vocab_off, QT_ROWS);
  *W = e->embd;
  W->M = e->vocab_local;
  if (is_tiled(W->type)) W->Mp = (W->M + QT_ROWS - 1) / QT_ROWS * QT_ROWS;
  else W->Mp = W->M;
  W->qs = e->embd.qs + (uint64_t)e->vocab_off * e->embd.qs_stride;
  W->sc = e->embd.sc + (uint64_t)e->vocab_off * e->embd.sc_stride;
  return RF_OK;
}

int release_layer_impl(rf_engine* e, int l) {
  Layer& L = e->layers[l];
  if (!L.resident) return set_error(RF_ESTATE, "layer %d is not loaded", l);
  auto cached = std::find(e->cache_lru.begin(), e->cache_lru.end(), l);
  if (cached != e->cache_lru.end()) {  // released while in the layer cache
    e->cache_lru.erase(cached);
    e->cache_used -= L.bytes;
  }
  dev_free(e, "layer:" + std::to_string(l) + ":weights", &L.block);
  L = Layer{};
  e->stats.layer_releases++;
  drop_graphs(e);
  return RF_OK;
}

// Layer l's views from the GGUF: the nine weights (load_layer's map,
// streaming_model.rs:581-847) and, when present, the Q/K/V biases (:829-831).
int gguf_layer_views(rf_engine* e, int l, View* v /*[kLayerViews]*/) {
  for (int j = 0; j < 9; j++) {
    const std::string name = "blk." + std::to_string(l) + "." + kRoleNames[j] + ".weight";
    const GgufTensor* t = e->gguf.find(name);
    if (!t || !t->data) return set_error(RF_EFORMAT, "missing tensor '%s'", name.c_str());
    v[j] = view_from_gguf(t);
  }
  for (int j = 0; j < 3; j++) {
    const GgufTensor* t = e->gguf.find("blk." + std::to_string(l) + "." + kBiasNames[j] + ".bias");
    v[9 + j] = t && t->data ? view_from_gguf(t) : View{};
  }
  return RF_OK;
}

int read_layer_views(rf_engine* e, int l, View* v);

int load_layer_gguf(rf_engine* e, int l) {
  if (!e->src) return set_error(RF_ESTATE, "engine has no GGUF source");
  View v[kLayerViews];
  RF_TRY(gguf_layer_views(e, l, v));
  // engines created from a path read a loaded layer through its coalesced read
  // plan; the first load of every layer at creation uses the mapped file
  if (e->src_fd >= 0 && e->created) RF_TRY(read_layer_views(e, l, v));
  return load_layer_views(e, l, v);
}

// ---- the step ----------------------------------------------------------------------
// One layer: execute_layer's block order (model_executor.rs:147-233) as five
// fused kernels.  Row-parallel projections finish with a sum over ranks.
// Kernel class k of layer l: 0 QKV+RoPE+KV append, 1 attention, 2 Wo+residual,
// 3 gate/up+SwiGLU, 4 down+residual (2 and 4 end with the rank all-reduce).
// QKV epilogue arguments of layer l: RoPE on the packed Q/K pairs, K/V append at
// the step position.
RopeQKVArgs rope_args(rf_engine* e, int l) {
  RopeQKVArgs ra{};
  ra.q_rows = e->q_local;
  ra.kv_rows = e->kv_local;
  ra.head_dim = e->cfg.head_dim;
  ra.max_seq = e->max_seq;
  ra.rope_cs = e->rope_cs;
  ra.d_pos = &e->d_io->pos;
  ra.q_out = e->q;
  ra.k_cur = e->k_cur;
  ra.v_cur = e->v_cur;
  ra.kcache = e->kc[l];
  ra.vcache = e->vc[l];
  ra.kv_f32 = e->rt.kv_f32;
  ra.row_base = 0;
  ra.bias = e->layers[l].qkv_bias;
  return ra;
}

// Attention of layer l over the history (length = the step position) and the
// current K/V.
AttnArgs attn_args(rf_engine* e, int l) {
  AttnArgs aa{};
  aa.q = e->q;
  aa.kc = e->kc[l];
  aa.vc = e->vc[l];
  aa.head_stride = (uint64_t)e->max_seq * e->cfg.head_dim;
  aa.batch_stride = 0;
  aa.k_cur = e->k_cur;
  aa.v_cur = e->v_cur;
  aa.d_nhist = &e->d_io->pos;
  aa.n_heads = (int)e->qh_local;
  aa.n_kv_heads = (int)e->kvh_local;
  aa.head_dim = (int)e->cfg.head_dim;
  aa.batch = 1;
  aa.max_splits = e->max_splits;
  aa.part = e->attn_part;
  aa.counters = e->attn_counters;
  aa.out = e->att;
  aa.kv_f32 = e->rt.kv_f32;
  aa.max_ctx = (int)e->max_seq;
  return aa;
}

// hidden = the sum over ranks of e->partial (row-parallel projection at call site
// `site` of the step): over peer memory, or an NCCL all-reduce.
int tp_sum(rf_engine* e, const Launch& La, int site) {
  if (e->ps_ok) {
    RF_CUDA(launch_peer_sum(La, e->ps, e->partial, e->hidden, (int)e->cfg.n_embd, site));
  } else {
    RF_NCCL(nccl()->allReduce(e->partial, e->hidden, e->cfg.n_embd, ncclFloat32, ncclSum, e->comm, e->stream));
  }
  return RF_OK;
}

bool all_resident(const rf_engine* e) {
  for (auto& L : e->layers)
    if (!L.resident) return false;
  return true;
}

// Whether the rank sum after W_o (k = 2) or W_down (k = 4) of layer l runs inside
// the GEMVs on either side of it (PeerLink) instead of as its own kernel: under
// tensor parallelism over peer memory, when the producing and the consuming
// matrices are tiled.  The last layer's W_down keeps the sum kernel (the output
// RMSNorm reads the sum).
bool fuse_sum(const rf_engine* e, int l, int k) {
  if (e->tp == 1 || !e->ps_ok) return false;
  const Layer& L = e->layers[l];
  if (k == 2) return is_tiled(L.wo.type) && is_tiled(L.gateup.type);
  return l + 1 < (int)e->layers.size() && is_tiled(L.down.type) && is_tiled(e->layers[l + 1].qkv.type);
}
PeerLink peer_link(const rf_engine* e) {
  PeerLink pl;
  pl.P = e->ps;
  pl.hidden = e->hidden;
  return pl;
}

// Kernel class k of layer l.  `fused`: inside a whole step, where the rank sums
// run inside the GEMVs around them (fuse_sum); every other caller (single layers,
// per-class timing, streamed steps) gets the sum kernel after each row-parallel product.
int enqueue_layer_kernel(rf_engine* e, int l, int k, bool pdl = false, bool fused = false) {
  const rf_model_config& c = e->cfg;
  Layer& L = e->layers[l];
  const Launch La{e->stream, pdl, e->tp > 1};
  if (k == 0) {
    RopeQKVArgs ra = rope_args(e, l);
    if (fused && l > 0 && fuse_sum(e, l - 1, 4)) {
      PeerLink pl = peer_link(e);
      pl.pull_site = 2 * (l - 1) + 1;
      pl.push_ctas = gemv_ctas(La, e->layers[l - 1].down, true);
      RF_CUDA(gemv_qkv_rope(La, L.qkv, &e->gws, e->hidden, L.attn_norm, c.rms_eps, ra, &pl));
    } else {
      RF_CUDA(gemv_qkv_rope(La, L.qkv, &e->gws, e->hidden, L.attn_norm, c.rms_eps, ra));
    }
    if (L.vmat.M) {  // V of its own type: the same epilogue from the V rows on
      ra.row_base = e->q_local + e->kv_local;
      RF_CUDA(gemv_qkv_rope(La, L.vmat, &e->gws, e->hidden, L.attn_norm, c.rms_eps, ra));
    }
  } else if (k == 1) {
    RF_CUDA(launch_attention(La, attn_args(e, l)));
  } else if (k == 2 || k == 4) {
    const PackedMat& W = k == 2 ? L.wo : L.down;
    const float* x = k == 2 ? e->att : e->act;
    const int site = 2 * l + (k == 4 ? 1 : 0);
    if (e->tp == 1) {
      RF_CUDA(gemv_residual(La, W, &e->gws, x, e->hidden, e->hidden));
    } else if (fused && fuse_sum(e, l, k)) {
      PeerLink pl = peer_link(e);
      pl.push_site = site;
      RF_CUDA(gemv_peer_push(La, W, &e->gws, x, e->rank == 0 ? e->hidden : nullptr, pl));
    } else {
      RF_CUDA(gemv_residual(La, W, &e->gws, x, e->rank == 0 ? e->hidden : nullptr, e->partial));
      RF_TRY(tp_sum(e, La, site));
    }
  } else {
    if (fused && fuse_sum(e, l, 2)) {
      PeerLink pl = peer_link(e);
      pl.pull_site = 2 * l;
      pl.push_ctas = gemv_ctas(La, L.wo, true);
      RF_CUDA(gemv_swiglu(La, L.gateup, &e->gws, e->hidden, L.ffn_norm, c.rms_eps, e->act, &pl));
    } else {
      RF_CUDA(gemv_swiglu(La, L.gateup, &e->gws, e->hidden, L.ffn_norm, c.rms_eps, e->act));
    }
  }
  return RF_OK;
}

int enqueue_layer(rf_engine* e, int l, bool pdl, bool fused = false) {
  for (int k = 0; k < 5; k++) RF_TRY(enqueue_layer_kernel(e, l, k, pdl, fused));
  return RF_OK;
}


// embedding -> every layer -> output RMSNorm into final_hidden.
int enqueue_forward(rf_engine* e, bool pdl) {
  const Launch La{e->stream, pdl};
  RF_CUDA(launch_embed(La, e->embd, &e->d_io->token, e->hidden, e->d_key));
  for (uint32_t l = 0; l < e->cfg.n_layers; l++) RF_TRY(enqueue_layer(e, (int)l, pdl, true));
  RF_CUDA(launch_rmsnorm(La, e->hidden, e->out_norm, e->cfg.rms_eps, e->cfg.n_embd, e->final_hidden));
  return RF_OK;
}

// LM head + greedy argmax (+ rank max) on final_hidden.
int enqueue_logits(rf_engine* e, bool pdl, bool want_logits) {
  PackedMat W;
  RF_TRY(lm_head(e, &W));
  const Launch La{e->stream, pdl};
  RF_CUDA(cudaMemsetAsync(e->d_key, 0, 8, e->stream));
  RF_CUDA(gemv_argmax(La, W, &e->gws, e->final_hidden, nullptr, 0.f, want_logits ? e->logits : nullptr, e->d_key,
                      e->vocab_off));
  if (e->tp > 1) RF_NCCL(nccl()->allReduce(e->d_key, e->d_key, 1, ncclUint64, ncclMax, e->comm, e->stream));
  return RF_OK;
}

int enqueue_decode(rf_engine* e, bool pdl) {
  RF_TRY(enqueue_forward(e, pdl));
  RF_TRY(enqueue_logits(e, pdl, false));
  RF_CUDA(launch_finalize(Launch{e->stream, pdl}, e->d_key, &e->d_io->token, &e->d_io->pos, e->d_hist, (int)e->max_seq));
  return RF_OK;
}

int ensure_ready(rf_engine* e) {
  if (!e->have_embd) return set_error(RF_ESTATE, "token_embd is not loaded");
  if (!e->have_onorm) return set_error(RF_ESTATE, "output_norm is not loaded");
  if (!all_resident(e)) {
    if (!e->src) return set_error(RF_ESTATE, "a layer is not resident and the engine has no GGUF source");
  }
  return RF_OK;
}

// ---- batched prompt (rf_prefill) ----------------------------------------------------
// A prompt chunk of T tokens goes through each layer as four tensor-core GEMMs
// (rf_prefill.cu) with the decode step's epilogues, and one attention launch whose
// sequence b is token b over the cache positions before it plus its own K/V.  The
// results equal the token-by-token forward (inference.rs:578-592) up to the
// GEMM's split-bf16 products (about 2^-16 relative per product).

// Why the engine cannot prefill in batches (RF_OK when it can).
int prefill_check(rf_engine* e) {
  if (e->tp > 1) return set_error(RF_EUNSUPPORTED, "batched prefill runs on one GPU (tp_size %d)", e->tp);
  if (!all_resident(e)) return set_error(RF_EUNSUPPORTED, "batched prefill needs every layer resident");
  for (size_t l = 0; l < e->layers.size(); l++) {
    const Layer& L = e->layers[l];
    const PackedMat* ms[5] = {&L.qkv, &L.wo, &L.gateup, &L.down, &L.vmat};
    for (int i = 0; i < 5; i++) {
      if (i == 4 && !ms[i]->M) continue;
      if (!prefill_supported(ms[i]->type))
        return set_error(RF_EUNSUPPORTED, "layer %zu holds a matrix of type %d; batched prefill covers Q4_K and Q8_0",
                         l, ms[i]->type);
    }
  }
  return RF_OK;
}

int ensure_prefill_buffers(rf_engine* e) {
  if (e->pf_block) return RF_OK;
  const rf_model_config& c = e->cfg;
  const uint64_t T = kPrefillChunk, G = c.n_heads / c.n_kv_heads;
  uint32_t kp = 0;
  for (const Layer& L : e->layers)
    for (const PackedMat* m : {&L.qkv, &L.wo, &L.gateup, &L.down, &L.vmat}) kp = std::max(kp, m->Kp);
  // the residual GEMMs split K over CTA pairs only when their blocks fill at most
  // half the SMs, so half the SM count bounds the blocks that need scratch
  const uint32_t ks_tiles = (uint32_t)std::max(1, num_sms() / 2);
  struct Item { void** p; uint64_t bytes; };
  std::vector<Item> items = {
      {(void**)&e->pf_x, 4 * T * c.n_embd},          {(void**)&e->pf_q, 4 * T * e->q_local},
      {(void**)&e->pf_k, 4 * T * e->kv_local},       {(void**)&e->pf_v, 4 * T * e->kv_local},
      {(void**)&e->pf_att, 4 * T * e->q_local},      {(void**)&e->pf_act, 4 * T * e->ff_local},
      {(void**)&e->pf_part, 4 * attn_part_floats((int)T, (int)e->kvh_local, kPrefillSplits, (int)G, (int)c.head_dim)},
      {(void**)&e->pf_cnt, 4 * T * e->kvh_local},    {(void**)&e->pf_err, 4},
      {(void**)&e->pf_tok, 4 * T},                   {(void**)&e->pf_xt, prefill_xt_bytes((uint32_t)T, kp)},
      {(void**)&e->pf_ks.part, 4 * prefill_ksplit_floats(ks_tiles)},
      {(void**)&e->pf_ks.cnt, 4ull * ks_tiles}};
  uint64_t total = 0;
  for (auto& it : items) total += align256(it.bytes);
  RF_TRY(dev_alloc(e, "scratch:prefill", total, &e->pf_block));
  RF_CUDA(cudaMemsetAsync(e->pf_block, 0, total, e->stream));  // attention counters start at zero
  RF_CUDA(cudaStreamSynchronize(e->stream));
  uint64_t off = 0;
  for (auto& it : items) {
    *it.p = (uint8_t*)e->pf_block + off;
    off += align256(it.bytes);
  }
  e->pf_ks.tiles = ks_tiles;
  return RF_OK;
}

// Tokens at positions [pos0, pos0 + T) (already in pf_tok) through every layer;
// their K/V go into the cache, the hidden states stay in pf_x.
int enqueue_prefill_chunk(rf_engine* e, uint32_t T, uint32_t pos0) {
  const rf_model_config& c = e->cfg;
  const Launch La{e->stream, false};
  const uint32_t d = c.n_embd;
  RF_CUDA(launch_embed_rows(La, e->embd, e->pf_tok, T, e->pf_x));
  for (uint32_t l = 0; l < c.n_layers; l++) {
    Layer& L = e->layers[l];
    // RMSNorm(attn_norm) -> [Q;K;V] -> bias, RoPE, K/V append (model_executor.rs:147-196)
    RF_CUDA(prefill_split(La, e->pf_x, d, T, d, L.qkv.Kp, L.attn_norm, c.rms_eps, e->pf_xt));
    RopeQKVArgs ra = rope_args(e, (int)l);
    ra.q_out = e->pf_q;
    ra.k_cur = e->pf_k;
    ra.v_cur = e->pf_v;
    RF_CUDA(prefill_gemm_rope(La, L.qkv, e->pf_xt, T, e->pf_err, ra, pos0, e->q_local, e->kv_local));
    if (L.vmat.M) {  // V of its own type: the same epilogue from the V rows on
      if (L.vmat.Kp != L.qkv.Kp)
        RF_CUDA(prefill_split(La, e->pf_x, d, T, d, L.vmat.Kp, L.attn_norm, c.rms_eps, e->pf_xt));
      ra.row_base = e->q_local + e->kv_local;
      RF_CUDA(prefill_gemm_rope(La, L.vmat, e->pf_xt, T, e->pf_err, ra, pos0, e->q_local, e->kv_local));
    }
    // attention: token b over cache positions [0, pos0 + b) and its own K/V
    AttnArgs aa = attn_args(e, (int)l);
    aa.q = e->pf_q;
    aa.k_cur = e->pf_k;
    aa.v_cur = e->pf_v;
    aa.cur_stride = e->kv_local;
    aa.d_nhist = nullptr;
    aa.nhist = (int)pos0;
    aa.nhist_step = 1;
    aa.batch = (int)T;
    aa.batch_stride = 0;
    aa.max_splits = kPrefillSplits;
    aa.part = e->pf_part;
    aa.counters = e->pf_cnt;
    aa.out = e->pf_att;
    RF_CUDA(launch_attention(La, aa));
    // W_o + residual
    RF_CUDA(prefill_split(La, e->pf_att, e->q_local, T, e->q_local, L.wo.Kp, nullptr, 0.f, e->pf_xt));
    RF_CUDA(prefill_gemm_residual(La, L.wo, e->pf_xt, T, e->pf_err, e->pf_x, d, e->pf_ks));
    // RMSNorm(ffn_norm) -> [gate;up] -> SwiGLU
    RF_CUDA(prefill_split(La, e->pf_x, d, T, d, L.gateup.Kp, L.ffn_norm, c.rms_eps, e->pf_xt));
    RF_CUDA(prefill_gemm_swiglu(La, L.gateup, e->pf_xt, T, e->pf_err, e->pf_act, e->ff_local));
    // W_down + residual
    RF_CUDA(prefill_split(La, e->pf_act, e->ff_local, T, e->ff_local, L.down.Kp, nullptr, 0.f, e->pf_xt));
    RF_CUDA(prefill_gemm_residual(La, L.down, e->pf_xt, T, e->pf_err, e->pf_x, d, e->pf_ks));
  }
  return RF_OK;
}

// Make every layer resident, loading from the GGUF source where needed.
// Layers the residency plan marks non-resident are loaded for the step and
// released afterwards (load -> compute -> release, streaming_model.rs:1081-1270).
// Layer l, which the plan streams, has just been used: keep it loaded as the
// most recently used entry of the layer cache when its bytes fit the capacity
// after evicting least recently used entries (LayerCache::insert_loaded,
// layer_cache.rs:72-135); else release it (load -> compute -> release).
int cache_layer(rf_engine* e, int l, bool loaded_now) {
  auto it = std::find(e->cache_lru.begin(), e->cache_lru.end(), l);
  if (it != e->cache_lru.end()) {  // a hit: move to the back
    e->cache_lru.erase(it);
    e->cache_lru.push_back(l);
    return RF_OK;
  }
  const uint64_t bytes = e->layers[l].bytes;
  if (!loaded_now) return RF_OK;
  RF_CUDA(cudaStreamSynchronize(e->stream));  // the step's kernels may still read what is released below
  if (!bytes || bytes > e->cache_capacity) return release_layer_impl(e, l);
  while (e->cache_used + bytes > e->cache_capacity && !e->cache_lru.empty()) {
    const int victim = e->cache_lru.front();
    e->cache_lru.erase(e->cache_lru.begin());
    e->cache_used -= e->layers[victim].bytes;
    RF_TRY(release_layer_impl(e, victim));
    e->stats.evictions++;
  }
  e->cache_lru.push_back(l);
  e->cache_used += bytes;
  return RF_OK;
}

// Drop every cached layer (capacity change, residency plan change).
int cache_clear(rf_engine* e) {
  RF_CUDA(cudaStreamSynchronize(e->stream));
  for (int l : e->cache_lru)
    if (e->layers[l].resident && !e->plan_resident[l]) RF_TRY(release_layer_impl(e, l));
  e->cache_lru.clear();
  e->cache_used = 0;
  return RF_OK;
}

int run_stepwise(rf_engine* e, bool decode) {
  const Launch La{e->stream, false};
  RF_CUDA(launch_embed(La, e->embd, &e->d_io->token, e->hidden, e->d_key));
  for (uint32_t l = 0; l < e->cfg.n_layers; l++) {
    bool loaded_now = false;
    if (!e->layers[l].resident) {
      e->stats.cache_misses++;
      RF_TRY(load_layer_gguf(e, (int)l));
      loaded_now = true;
    } else {
      e->stats.cache_hits++;
    }
    RF_TRY(enqueue_layer(e, (int)l, false));
    if (!e->plan_resident[l]) RF_TRY(cache_layer(e, (int)l, loaded_now));
  }
  RF_CUDA(launch_rmsnorm(La, e->hidden, e->out_norm, e->cfg.rms_eps, e->cfg.n_embd, e->final_hidden));
  if (decode) {
    RF_TRY(enqueue_logits(e, false, false));
    RF_CUDA(launch_finalize(La, e->d_key, &e->d_io->token, &e->d_io->pos, e->d_hist, (int)e->max_seq));
  }
  return RF_OK;
}

// ---- out-of-core ring ---------------------------------------------------------------
// Layers the residency plan leaves out stream through `ring_slots` device slots:
// their packed images are built once into pinned host memory, and each step
// copies them with cudaMemcpyAsync on a side stream.  A slot's copy waits for the
// kernels of the layer that used it before (ring_free), a layer's kernels wait
// for its copy (ring_ready), and the copy of the layer `ring_slots` ahead is
// issued as soon as a layer's kernels are queued, so transfers overlap the
// compute of the layers in between.  The slots are charged to the byte budget
// ("ring:slot:<i>"), the pinned images are host memory and are not.
// A streamed layer's tensors read from the GGUF file (GgufDataSource::
// read_coalesced_tensor_range_into, datasource.rs:411, over build_layer_read_plan,
// layer_read.rs:50): the plan's coalesced ranges are pread into one reused pinned
// staging buffer and the views are pointed into it.
int read_layer_views(rf_engine* e, int l, View* v /*[kLayerViews], from gguf_layer_views*/) {
  std::vector<rf_tensor_extent> ext;
  std::vector<int> role;
  for (int j = 0; j < kLayerViews; j++)
    if (v[j].host) {
      ext.push_back({(uint64_t)(v[j].host - e->src), v[j].bytes});
      role.push_back(j);
    }
  ReadPlan plan;
  RF_TRY(build_read_plan(ext.data(), (uint32_t)ext.size(), &plan));
  const uint64_t need = plan.totals.physical_bytes;
  if (need > e->read_stage_bytes) {
    if (e->read_stage) cudaFreeHost(e->read_stage);
    e->read_stage = nullptr;
    e->read_stage_bytes = 0;
    RF_CUDA(cudaHostAlloc((void**)&e->read_stage, need, cudaHostAllocDefault));
    e->read_stage_bytes = need;
  }
  std::vector<uint64_t> base(plan.ranges.size());
  uint64_t off = 0;
  for (size_t r = 0; r < plan.ranges.size(); r++) {
    const rf_read_range& rr = plan.ranges[r];
    base[r] = off;
    uint64_t done = 0;
    while (done < rr.byte_length) {
      const ssize_t got = pread(e->src_fd, e->read_stage + off + done, (size_t)(rr.byte_length - done),
                                (off_t)(rr.file_offset + done));
      if (got < 0 && errno == EINTR) continue;
      if (got <= 0)
        return set_error(RF_EFORMAT, "reading layer %d: %llu bytes at file offset %llu failed", l,
                         (unsigned long long)rr.byte_length, (unsigned long long)rr.file_offset);
      done += (uint64_t)got;
    }
    off += rr.byte_length;
  }
  for (const rf_planned_tensor& p : plan.placed) v[role[p.index]].host = e->read_stage + base[p.range] + p.offset_in_range;
  e->stats.file_reads += plan.ranges.size();
  e->stats.file_read_bytes += plan.totals.physical_bytes;
  e->stats.file_gap_bytes += plan.totals.gap_bytes;
  return RF_OK;
}

int ensure_stream_image(rf_engine* e, int l) {
  StreamImage& si = e->simg[l];
  if (si.host) return RF_OK;
  if (!e->src) return set_error(RF_ESTATE, "layer %d is not resident and the engine has no GGUF source", l);
  View v[kLayerViews];
  RF_TRY(gguf_layer_views(e, l, v));
  if (e->src_fd >= 0) RF_TRY(read_layer_views(e, l, v));
  LayerImage img;
  RF_TRY(build_layer_image(e, l, v, &img));
  RF_CUDA(cudaHostAlloc((void**)&si.host, img.tmpl.bytes, cudaHostAllocDefault));
  memcpy(si.host, img.bytes.data(), img.tmpl.bytes);
  si.bytes = img.tmpl.bytes;
  si.tmpl = img.tmpl;
  e->stats.host_image_bytes += si.bytes;
  return RF_OK;
}

void free_ring(rf_engine* e) {
  if (e->stream) cudaStreamSynchronize(e->stream);
  if (e->copy_stream) cudaStreamSynchronize(e->copy_stream);
  for (size_t i = 0; i < e->ring.size(); i++) dev_free(e, "ring:slot:" + std::to_string(i), &e->ring[i]);
  for (auto ev : e->ring_free) cudaEventDestroy(ev);
  for (auto ev : e->ring_ready) cudaEventDestroy(ev);
  e->ring.clear();
  e->ring_free.clear();
  e->ring_ready.clear();
  e->ring_slot_bytes = 0;
}

int ensure_ring(rf_engine* e, uint64_t slot_bytes) {
  const int R = e->rt.ring_slots;
  if ((int)e->ring.size() == R && e->ring_slot_bytes >= slot_bytes) return RF_OK;
  free_ring(e);
  if (!e->copy_stream) RF_CUDA(cudaStreamCreateWithFlags(&e->copy_stream, cudaStreamNonBlocking));
  e->ring.assign(R, nullptr);
  e->ring_free.assign(R, nullptr);
  e->ring_ready.assign(R, nullptr);
  for (int i = 0; i < R; i++) {
    int rc = dev_alloc(e, "ring:slot:" + std::to_string(i), slot_bytes, &e->ring[i]);
    if (rc) {
      free_ring(e);
      return rc;
    }
    RF_CUDA(cudaEventCreateWithFlags(&e->ring_free[i], cudaEventDisableTiming));
    RF_CUDA(cudaEventCreateWithFlags(&e->ring_ready[i], cudaEventDisableTiming));
    RF_CUDA(cudaEventRecord(e->ring_free[i], e->stream));
  }
  e->ring_slot_bytes = slot_bytes;
  return RF_OK;
}

// One step with the non-resident layers streamed through the ring.
int run_ring(rf_engine* e, bool decode) {
  const int R = e->rt.ring_slots;
  std::vector<int> S;  // streamed layers, in order
  uint64_t maxb = 0;
  for (uint32_t l = 0; l < e->cfg.n_layers; l++)
    if (!e->layers[l].resident) {
      RF_TRY(ensure_stream_image(e, (int)l));
      S.push_back((int)l);
      maxb = std::max(maxb, e->simg[l].bytes);
    }
  RF_TRY(ensure_ring(e, maxb));
  auto issue = [&](size_t j) -> int {
    const int slot = (int)(j % R);
    const StreamImage& si = e->simg[S[j]];
    RF_CUDA(cudaStreamWaitEvent(e->copy_stream, e->ring_free[slot], 0));
    RF_CUDA(cudaMemcpyAsync(e->ring[slot], si.host, si.bytes, cudaMemcpyHostToDevice, e->copy_stream));
    RF_CUDA(cudaEventRecord(e->ring_ready[slot], e->copy_stream));
    e->stats.ring_copies++;
    e->stats.h2d_bytes += si.bytes;
    return RF_OK;
  };
  const Launch La{e->stream, false};
  RF_CUDA(launch_embed(La, e->embd, &e->d_io->token, e->hidden, e->d_key));
  for (size_t j = 0; j < S.size() && j < (size_t)R; j++) RF_TRY(issue(j));
  size_t j = 0;
  for (uint32_t l = 0; l < e->cfg.n_layers; l++) {
    Layer& L = e->layers[l];
    if (L.resident) {
      e->stats.cache_hits++;
      RF_TRY(enqueue_layer(e, (int)l, false));
      continue;
    }
    e->stats.cache_misses++;
    const int slot = (int)(j % R);
    RF_CUDA(cudaStreamWaitEvent(e->stream, e->ring_ready[slot], 0));
    bind_layer(&L, e->simg[l].tmpl, (uint8_t*)e->ring[slot]);  // the layer stays non-resident
    const int rc = enqueue_layer(e, (int)l, false);
    L = Layer{};
    RF_TRY(rc);
    RF_CUDA(cudaEventRecord(e->ring_free[slot], e->stream));
    if (j + R < S.size()) RF_TRY(issue(j + R));
    j++;
  }
  RF_CUDA(launch_rmsnorm(La, e->hidden, e->out_norm, e->cfg.rms_eps, e->cfg.n_embd, e->final_hidden));
  if (decode) {
    RF_TRY(enqueue_logits(e, false, false));
    RF_CUDA(launch_finalize(La, e->d_key, &e->d_io->token, &e->d_io->pos, e->d_hist, (int)e->max_seq));
  }
  return RF_OK;
}

int capture(rf_engine* e, bool decode, cudaGraphExec_t* out) {
  cudaGraph_t g = nullptr;
  RF_CUDA(cudaStreamBeginCapture(e->stream, cudaStreamCaptureModeThreadLocal));
  int rc = decode ? enqueue_decode(e, true) : enqueue_forward(e, true);
  cudaError_t ce = cudaStreamEndCapture(e->stream, &g);
  if (rc) {
    if (g) cudaGraphDestroy(g);
    return rc;
  }
  if (ce != cudaSuccess) return set_error(RF_ECUDA, "graph capture failed: %s", cudaGetErrorString(ce));
  ce = cudaGraphInstantiate(out, g, 0);
  cudaGraphDestroy(g);
  if (ce != cudaSuccess) return set_error(RF_ECUDA, "graph instantiate failed: %s", cudaGetErrorString(ce));
  return RF_OK;
}

// After a synchronisation of the engine stream: a tensor-parallel peer-sum wait
// that gave up fails the call.  The error word is copied into pinned host memory
// on the stream and read after it drains.
int check_async_errors(rf_engine* e) {
  if (!e->ps_ok) return RF_OK;
  RF_CUDA(cudaMemcpyAsync(e->h_err, e->ps.err, 4, cudaMemcpyDeviceToHost, e->stream));
  RF_CUDA(cudaStreamSynchronize(e->stream));
  const unsigned perr = e->h_err[0];
  if (!perr) return RF_OK;
  RF_CUDA(cudaMemsetAsync(e->ps.err, 0, 4, e->stream));
  RF_CUDA(cudaStreamSynchronize(e->stream));
  e->h_err[0] = 0;
  return set_error(RF_ETIMEOUT, "a tensor-parallel peer sum waited too long for another rank (0x%x)", perr);
}

// Launch one token step (forward, or decode = forward + logits + advance).
int launch_step(rf_engine* e, bool decode) {
  if (!all_resident(e)) return e->rt.ring_slots > 0 && e->src ? run_ring(e, decode) : run_stepwise(e, decode);
  if (e->rt.disable_graphs) return decode ? enqueue_decode(e, true) : enqueue_forward(e, true);
  cudaGraphExec_t* g = decode ? &e->g_decode : &e->g_forward;
  if (!*g) RF_TRY(capture(e, decode, g));
  e->stats.cache_hits += e->cfg.n_layers;
  RF_CUDA(cudaGraphLaunch(*g, e->stream));
  return RF_OK;
}

// Queue the step inputs.  The copy reads pinned slot `pos`, which no other
// in-flight step uses (positions are distinct until the KV cache is reset, and
// every entry point that reuses positions synchronises before returning).
int set_io(rf_engine* e, uint32_t token, uint32_t pos) {
  StepIO* slot = e->h_io + std::min<uint32_t>(pos, e->max_seq);
  slot->token = token;
  slot->pos = (int)pos;
  RF_CUDA(cudaMemcpyAsync(e->d_io, slot, sizeof(StepIO), cudaMemcpyHostToDevice, e->stream));
  return RF_OK;
}

int check_step(rf_engine* e, uint32_t token, uint32_t pos) {
  if (pos != e->seq_len)
    return set_error(RF_EINVAL, "KV position/history mismatch: position %u requires cache history %u, got %u", pos,
                     pos, e->seq_len);
  if (e->seq_len >= e->max_seq) return set_error(RF_ESTATE, "KV cache full (%u positions)", e->max_seq);
  if (token >= e->cfg.vocab_size)
    return set_error(RF_EINVAL, "token_id %u out of bounds for vocab %u", token, e->cfg.vocab_size);
  return ensure_ready(e);
}

// n greedy decode steps starting from `token` at pos = KV length.  Each step's
// argmax is the next step's token on the device (finalize_kernel), and lands in
// d_hist[pos]; the host copies the n tokens once at the end.  With device_ms the
// n steps are bracketed by events on the engine stream.
int decode_loop(rf_engine* e, uint32_t token, uint32_t n, uint32_t* out, float* device_ms) {
  if (n == 0) {
    if (device_ms) *device_ms = 0.f;
    return RF_OK;
  }
  if ((uint64_t)e->seq_len + n > e->max_seq) return set_error(RF_ESTATE, "KV cache full");
  const uint32_t p0 = e->seq_len;
  RF_TRY(set_io(e, token, p0));
  cudaEvent_t a = nullptr, b = nullptr;
  if (device_ms) {
    RF_CUDA(cudaEventCreate(&a));
    RF_CUDA(cudaEventCreate(&b));
    RF_CUDA(cudaEventRecord(a, e->stream));
  }
  int rc = RF_OK;
  for (uint32_t t = 0; t < n && !rc; t++) {
    rc = launch_step(e, true);
    if (!rc) e->seq_len++;
  }
  if (device_ms && !rc) {
    cudaError_t ce = cudaEventRecord(b, e->stream);
    if (ce == cudaSuccess) ce = cudaEventSynchronize(b);
    if (ce == cudaSuccess) ce = cudaEventElapsedTime(device_ms, a, b);
    if (ce != cudaSuccess) rc = set_error(RF_ECUDA, "decode timing failed: %s", cudaGetErrorString(ce));
  }
  if (a) cudaEventDestroy(a);
  if (b) cudaEventDestroy(b);
  if (rc) return rc;
  if (out) RF_CUDA(cudaMemcpyAsync(out, e->d_hist + p0, 4ull * n, cudaMemcpyDeviceToHost, e->stream));
  RF_CUDA(cudaStreamSynchronize(e->stream));
  return check_async_errors(e);
}

int engine_finish_create(rf_engine* e) {
  RF_TRY(setup_geometry(e));
  RF_TRY(engine_init_device(e));
  return RF_OK;
}

int create_from_image(const uint8_t* p, uint64_t len, const rf_runtime_config* rt, rf_engine* e) {
  e->rt = rt ? *rt : rf_runtime_config{};
  e->dev = e->rt.device;
  e->src = p;
  e->src_len = len;
  RF_TRY(parse_gguf(p, len, &e->gguf));
  RF_TRY(llama_config_from_gguf(e->gguf, &e->cfg));
  // validate_required_tensors (model.rs:168-200)
  for (const char* n : {"token_embd.weight", "output_norm.weight"})
    if (!e->gguf.find(n)) return set_error(RF_EFORMAT, "Unsupported or incomplete model: missing tensor '%s'", n);
  RF_TRY(engine_finish_create(e));
  RF_TRY(load_persistent(e, RF_ROLE_TOKEN_EMBD, view_from_gguf(e->gguf.find("token_embd.weight"))));
  RF_TRY(load_persistent(e, RF_ROLE_OUTPUT_NORM, view_from_gguf(e->gguf.find("output_norm.weight"))));
  if (const GgufTensor* o = e->gguf.find("output.weight")) RF_TRY(load_persistent(e, RF_ROLE_OUTPUT, view_from_gguf(o)));
  else e->tied = true;
  if (e->rt.ring_slots == 0)
    for (uint32_t l = 0; l < e->cfg.n_layers; l++) RF_TRY(load_layer_gguf(e, (int)l));
  return RF_OK;
}

void destroy(rf_engine* e) {
  if (!e) return;
  cudaSetDevice(e->dev);
  if (e->stream) cudaStreamSynchronize(e->stream);
  drop_graphs(e);
  for (size_t l = 0; l < e->layers.size(); l++)
    if (e->layers[l].block) cudaFree(e->layers[l].block);
  if (e->embd_block) cudaFree(e->embd_block);
  if (e->out_block) cudaFree(e->out_block);
  if (e->embd_host) cudaFreeHost(e->embd_host);
  if (e->out_host) cudaFreeHost(e->out_host);
  if (e->out_norm) cudaFree(e->out_norm);
  if (e->kv_block) cudaFree(e->kv_block);
  if (e->scratch) cudaFree(e->scratch);
  if (e->pf_block) cudaFree(e->pf_block);
  if (e->copy_stream) cudaStreamSynchronize(e->copy_stream);
  for (auto p : e->ring)
    if (p) cudaFree(p);
  for (auto ev : e->ring_free) cudaEventDestroy(ev);
  for (auto ev : e->ring_ready) cudaEventDestroy(ev);
  if (e->copy_stream) cudaStreamDestroy(e->copy_stream);
  for (auto& si : e->simg)
    if (si.host) cudaFreeHost(si.host);
  if (e->h_io) cudaFreeHost(e->h_io);
  if (e->h_tok) cudaFreeHost(e->h_tok);
  if (e->h_key) cudaFreeHost(e->h_key);
  if (e->h_err) cudaFreeHost(e->h_err);
  for (void* q : e->ps_peer)
    if (q) cudaIpcCloseMemHandle(q);
  if (e->ps_area) cudaFree(e->ps_area);
  if (e->comm && nccl()) nccl()->commDestroy(e->comm);
  if (e->stream) cudaStreamDestroy(e->stream);
  if (e->map_addr) munmap(e->map_addr, e->map_len);
  if (e->src_fd >= 0) close(e->src_fd);
  if (e->read_stage) cudaFreeHost(e->read_stage);
  delete e;
}

#define ENGINE_GUARD(e)                                                \
  do {                                                                 \
    if (!(e)) return set_error(RF_EINVAL, "null engine");              \
    cudaError_t _se = cudaSetDevice((e)->dev);                         \
    if (_se != cudaSuccess)                                            \
      return set_error(RF_ECUDA, "cudaSetDevice: %s", cudaGetErrorString(_se)); \
  } while (0)

// Bytes of layer l's device image (build_layer_image's layout) for this rank,
// from its GGUF tensor types (layers of a mixed-format model differ).
uint64_t layer_image_bytes(rf_engine* e, int l) {
  const rf_model_config& c = e->cfg;
  const std::string pre = "blk." + std::to_string(l) + ".";
  auto type_of = [&](const char* role) -> int {  // the device storage type
    const GgufTensor* t = e->gguf.find(pre + role + ".weight");
    return t ? storage_type((int)t->type) : -1;
  };
  auto mat = [](int type, uint32_t M, uint32_t K) -> uint64_t {
    PackedMat g{};
    if (type < 0 || !packed_geometry(type, M, K, &g)) return 0;
    const uint64_t sc = packed_sc_bytes(g);
    return align256(packed_qs_bytes(g)) + align256(sc ? sc : 16);
  };
  const bool split_v = type_of("attn_v") != type_of("attn_q");
  const bool bias = e->gguf.find(pre + "attn_q.bias") != nullptr;
  return mat(type_of("attn_q"), e->q_local + (split_v ? 1 : 2) * e->kv_local, c.n_embd) +
         (split_v ? mat(type_of("attn_v"), e->kv_local, c.n_embd) : 0) +
         mat(type_of("attn_output"), c.n_embd, e->q_local) + mat(type_of("ffn_gate"), 2 * e->ff_local, c.n_embd) +
         mat(type_of("ffn_down"), c.n_embd, e->ff_local) + 2 * align256(4ull * c.n_embd) +
         (bias ? align256(4ull * (e->q_local + 2 * e->kv_local)) : 0);
}

// Whether layer l's V is a matrix of its own (its GGUF type differs from Q's);
// false when the engine has no GGUF source (then only loaded layers tell).
bool layer_v_split(rf_engine* e, int l) {
  if (!e->src) return false;
  const std::string pre = "blk." + std::to_string(l) + ".";
  const GgufTensor* q = e->gguf.find(pre + "attn_q.weight");
  const GgufTensor* v = e->gguf.find(pre + "attn_v.weight");
  return q && v && storage_type((int)q->type) != storage_type((int)v->type);
}

}  // namespace

// ===========================================================================
// C ABI
// ===========================================================================
extern "C" {

const char* rf_last_error(void) { return last_error(); }
int rf_abi_version(void) { return RF_ABI_VERSION; }

int rf_gguf_read_config(const void* gguf, uint64_t len, rf_model_config* out) {
  if (!gguf || !out) return set_error(RF_EINVAL, "null argument");
  Gguf g;
  RF_TRY(parse_gguf((const uint8_t*)gguf, len, &g));
  return llama_config_from_gguf(g, out);
}

int rf_tp_shard_plan(const rf_model_config* cfg, int tp_size, int tp_rank, int ggml_type, rf_tp_shard* out) {
  if (!cfg || !out) return set_error(RF_EINVAL, "null argument");
  rf_model_config c = *cfg;
  if (!c.head_dim && c.n_heads) c.head_dim = c.n_embd / c.n_heads;
  const int block = block_elems(ggml_type);
  if (!block) return set_error(RF_EINVAL, "unknown ggml type %d", ggml_type);
  return shard_plan(c, tp_size, tp_rank, block, out);
}

int rf_engine_create(const rf_model_config* cfg, const rf_runtime_config* rt, rf_engine** out) {
  if (!cfg || !out) return set_error(RF_EINVAL, "null argument");
  *out = nullptr;
  rf_engine* e = new rf_engine();
  e->cfg = *cfg;
  if (!e->cfg.head_dim && e->cfg.n_heads) e->cfg.head_dim = e->cfg.n_embd / e->cfg.n_heads;
  e->rt = rt ? *rt : rf_runtime_config{};
  e->dev = e->rt.device;
  int rc = engine_finish_create(e);
  if (rc) { destroy(e); return rc; }
  *out = e;
  return RF_OK;
}

int rf_engine_create_from_gguf(const void* gguf, uint64_t len, const rf_runtime_config* rt, rf_engine** out) {
  if (!gguf || !out) return set_error(RF_EINVAL, "null argument");
  *out = nullptr;
  rf_engine* e = new rf_engine();
  int rc = create_from_image((const uint8_t*)gguf, len, rt, e);
  if (rc) { destroy(e); return rc; }
  *out = e;
  return RF_OK;
}

int rf_engine_create_from_file(const char* path, const rf_runtime_config* rt, rf_engine** out) {
  if (!path || !out) return set_error(RF_EINVAL, "null argument");
  *out = nullptr;
  int fd = open(path, O_RDONLY);
  if (fd < 0) return set_error(RF_EINVAL, "cannot open '%s'", path);
  struct stat st;
  if (fstat(fd, &st) != 0 || st.st_size <= 0) { close(fd); return set_error(RF_EFORMAT, "cannot stat '%s'", path); }
  void* m = mmap(nullptr, (size_t)st.st_size, PROT_READ, MAP_PRIVATE, fd, 0);
  if (m == MAP_FAILED) {
    close(fd);
    return set_error(RF_EFORMAT, "cannot map '%s'", path);
  }
  rf_engine* e = new rf_engine();
  e->map_addr = m;
  e->map_len = (uint64_t)st.st_size;
  e->src_fd = fd;
  int rc = create_from_image((const uint8_t*)m, (uint64_t)st.st_size, rt, e);
  if (rc) { destroy(e); return rc; }
  e->created = true;
  *out = e;
  return RF_OK;
}

void rf_engine_destroy(rf_engine* e) { destroy(e); }

int rf_engine_config(const rf_engine* e, rf_model_config* out) {
  if (!e || !out) return set_error(RF_EINVAL, "null argument");
  *out = e->cfg;
  return RF_OK;
}

int rf_persistent_load(rf_engine* e, const rf_tensor_view* v) {
  ENGINE_GUARD(e);
  if (!v) return set_error(RF_EINVAL, "null view");
  View w;
  w.type = v->ggml_type;
  w.ne0 = v->ne0;
  w.ne1 = v->ne1 ? v->ne1 : 1;
  w.bytes = v->bytes;
  w.host = (const uint8_t*)v->host;
  return load_persistent(e, v->role, w);
}

int rf_layer_load(rf_engine* e, int layer, const rf_tensor_view* views, int n_views) {
  ENGINE_GUARD(e);
  if (layer < 0 || layer >= (int)e->cfg.n_layers) return set_error(RF_EINVAL, "layer %d out of range", layer);
  if (!views || n_views <= 0) return set_error(RF_EINVAL, "no tensor views");
  if (e->layers[layer].resident) return set_error(RF_ESTATE, "layer %d is already loaded", layer);
  View v[kLayerViews];
  for (int i = 0; i < n_views; i++) {
    const rf_tensor_view& t = views[i];
    if (t.role < 0 || t.role >= kLayerViews)
      return set_error(RF_EINVAL, "view %d has role %d (not a layer tensor)", i, t.role);
    v[t.role].type = t.ggml_type;
    v[t.role].ndims = t.ne1 > 1 ? 2 : 1;  // ne1 = 0 or 1: a vector
    v[t.role].ne0 = t.ne0;
    v[t.role].ne1 = t.ne1 ? t.ne1 : 1;
    v[t.role].bytes = t.bytes;
    v[t.role].host = (const uint8_t*)t.host;
  }
  return load_layer_views(e, layer, v);
}

int rf_layer_load_gguf(rf_engine* e, int layer) {
  ENGINE_GUARD(e);
  if (layer < 0 || layer >= (int)e->cfg.n_layers) return set_error(RF_EINVAL, "layer %d out of range", layer);
  if (e->layers[layer].resident) return set_error(RF_ESTATE, "layer %d is already loaded", layer);
  return load_layer_gguf(e, layer);
}

int rf_layer_release(rf_engine* e, int layer) {
  ENGINE_GUARD(e);
  if (layer < 0 || layer >= (int)e->cfg.n_layers) return set_error(RF_EINVAL, "layer %d out of range", layer);
  RF_CUDA(cudaStreamSynchronize(e->stream));
  return release_layer_impl(e, layer);
}

int rf_layer_is_resident(const rf_engine* e, int layer) {
  if (!e || layer < 0 || layer >= (int)e->cfg.n_layers) return 0;
  return e->layers[layer].resident ? 1 : 0;
}

int rf_layer_compute(rf_engine* e, int layer, uint32_t pos) {
  ENGINE_GUARD(e);
  if (layer < 0 || layer >= (int)e->cfg.n_layers) return set_error(RF_EINVAL, "layer %d out of range", layer);
  if (!e->layers[layer].resident) return set_error(RF_ESTATE, "layer %d is not loaded", layer);
  if (pos != e->seq_len)
    return set_error(RF_EINVAL, "KV position/history mismatch: position %u, history %u", pos, e->seq_len);
  if (e->seq_len >= e->max_seq) return set_error(RF_ESTATE, "KV cache full");
  e->h_io->pos = (int)pos;
  RF_CUDA(cudaMemcpyAsync(&e->d_io->pos, &e->h_io->pos, 4, cudaMemcpyHostToDevice, e->stream));
  RF_TRY(enqueue_layer(e, layer, false));
  RF_CUDA(cudaStreamSynchronize(e->stream));
  return RF_OK;
}

int rf_embed(rf_engine* e, uint32_t token) {
  ENGINE_GUARD(e);
  if (!e->have_embd) return set_error(RF_ESTATE, "token_embd is not loaded");
  if (token >= e->cfg.vocab_size) return set_error(RF_EINVAL, "token_id %u out of bounds", token);
  e->h_io->token = token;
  RF_CUDA(cudaMemcpyAsync(&e->d_io->token, &e->h_io->token, 4, cudaMemcpyHostToDevice, e->stream));
  RF_CUDA(launch_embed(Launch{e->stream, false}, e->embd, &e->d_io->token, e->hidden, e->d_key));
  RF_CUDA(cudaStreamSynchronize(e->stream));
  return RF_OK;
}

int rf_hidden_write(rf_engine* e, const float* host, uint32_t n) {
  ENGINE_GUARD(e);
  if (!host || n != e->cfg.n_embd) return set_error(RF_EINVAL, "hidden size mismatch: expected %u", e->cfg.n_embd);
  RF_CUDA(h2d_sync(e, e->hidden, host, 4ull * n));
  return RF_OK;
}

int rf_hidden_read(rf_engine* e, float* host, uint32_t n) {
  ENGINE_GUARD(e);
  if (!host || n != e->cfg.n_embd) return set_error(RF_EINVAL, "hidden size mismatch: expected %u", e->cfg.n_embd);
  RF_CUDA(cudaStreamSynchronize(e->stream));
  RF_CUDA(cudaMemcpy(host, e->hidden, 4ull * n, cudaMemcpyDeviceToHost));
  return RF_OK;
}

int rf_kv_commit(rf_engine* e) {
  ENGINE_GUARD(e);
  if (e->seq_len >= e->max_seq) return set_error(RF_ESTATE, "KV cache full");
  e->seq_len++;
  return RF_OK;
}

int rf_forward_token(rf_engine* e, uint32_t token, uint32_t pos, float* final_hidden) {
  ENGINE_GUARD(e);
  RF_TRY(check_step(e, token, pos));
  RF_TRY(set_io(e, token, pos));
  RF_TRY(launch_step(e, false));
  e->seq_len++;
  if (final_hidden) {
    RF_CUDA(cudaMemcpyAsync(final_hidden, e->final_hidden, 4ull * e->cfg.n_embd, cudaMemcpyDeviceToHost, e->stream));
  }
  RF_CUDA(cudaStreamSynchronize(e->stream));
  return check_async_errors(e);
}

int rf_prefill(rf_engine* e, const uint32_t* tokens, uint32_t n_tokens) {
  ENGINE_GUARD(e);
  if (!tokens || n_tokens == 0) return set_error(RF_EINVAL, "empty prompt");
  if ((uint64_t)e->seq_len + n_tokens > e->max_seq)
    return set_error(RF_ESTATE, "prompt of %u tokens at position %u exceeds the KV capacity %u", n_tokens, e->seq_len,
                     e->max_seq);
  for (uint32_t i = 0; i < n_tokens; i++)
    if (tokens[i] >= e->cfg.vocab_size) return set_error(RF_EINVAL, "token_id %u out of bounds", tokens[i]);
  RF_TRY(ensure_ready(e));
  RF_TRY(prefill_check(e));
  RF_TRY(ensure_prefill_buffers(e));
  const uint32_t d = e->cfg.n_embd;
  uint32_t last = 0;
  for (uint32_t c0 = 0; c0 < n_tokens; c0 += kPrefillChunk) {
    const uint32_t T = std::min(kPrefillChunk, n_tokens - c0);
    RF_CUDA(h2d_sync(e, e->pf_tok, tokens + c0, 4ull * T));
    RF_TRY(enqueue_prefill_chunk(e, T, e->seq_len));
    e->seq_len += T;
    last = T - 1;
  }
  // the last token's state, as rf_forward_token leaves it: hidden and the
  // output-normed final_hidden that rf_compute_logits reads
  const Launch La{e->stream, false};
  RF_CUDA(cudaMemcpyAsync(e->hidden, e->pf_x + (size_t)last * d, 4ull * d, cudaMemcpyDeviceToDevice, e->stream));
  RF_CUDA(launch_rmsnorm(La, e->pf_x + (size_t)last * d, e->out_norm, e->cfg.rms_eps, d, e->final_hidden));
  // the GEMMs' bounded waits report through pf_err (bit 0)
  RF_CUDA(cudaMemcpyAsync(&e->h_err[1], e->pf_err, 4, cudaMemcpyDeviceToHost, e->stream));
  RF_CUDA(cudaStreamSynchronize(e->stream));
  const unsigned err = e->h_err[1];
  if (err) {
    RF_CUDA(cudaMemsetAsync(e->pf_err, 0, 4, e->stream));
    RF_CUDA(cudaStreamSynchronize(e->stream));
    return set_error(RF_ETIMEOUT, "a tensor-core GEMM of the batched prefill gave up waiting (error word 0x%x)", err);
  }
  return check_async_errors(e);
}

int rf_compute_logits(rf_engine* e, float* logits, uint32_t* argmax) {
  ENGINE_GUARD(e);
  RF_TRY(enqueue_logits(e, false, logits != nullptr));
  if (logits) {
    if (e->tp > 1) {
      RF_NCCL(nccl()->allGather(e->logits, e->logits_all, e->vocab_chunk, ncclFloat32, e->comm, e->stream));
      RF_CUDA(cudaMemcpyAsync(logits, e->logits_all, 4ull * e->cfg.vocab_size, cudaMemcpyDeviceToHost, e->stream));
    } else {
      RF_CUDA(cudaMemcpyAsync(logits, e->logits, 4ull * e->cfg.vocab_size, cudaMemcpyDeviceToHost, e->stream));
    }
  }
  RF_CUDA(cudaMemcpyAsync(e->h_key, e->d_key, 8, cudaMemcpyDeviceToHost, e->stream));
  RF_CUDA(cudaStreamSynchronize(e->stream));
  if (argmax) *argmax = ~(uint32_t)(*e->h_key & 0xFFFFFFFFull);
  return RF_OK;
}

int rf_decode_step(rf_engine* e, uint32_t token, uint32_t* next_token) {
  ENGINE_GUARD(e);
  RF_TRY(check_step(e, token, e->seq_len));
  RF_TRY(set_io(e, token, e->seq_len));
  RF_TRY(launch_step(e, true));
  e->seq_len++;
  RF_CUDA(cudaMemcpyAsync(e->h_tok, &e->d_io->token, 4, cudaMemcpyDeviceToHost, e->stream));
  RF_CUDA(cudaStreamSynchronize(e->stream));
  RF_TRY(check_async_errors(e));
  if (next_token) *next_token = e->h_tok[0];
  return RF_OK;
}

int rf_generate(rf_engine* e, const uint32_t* prompt, uint32_t n_prompt, uint32_t n_new, uint32_t* out) {
  ENGINE_GUARD(e);
  if (!prompt || n_prompt == 0) return set_error(RF_EINVAL, "empty prompt");
  if (n_new && !out) return set_error(RF_EINVAL, "null output");
  if ((uint64_t)e->seq_len + n_prompt + n_new > e->max_seq + 1ull)
    return set_error(RF_ESTATE, "prompt + generation exceed the KV capacity %u", e->max_seq);
  for (uint32_t i = 0; i < n_prompt; i++)
    if (prompt[i] >= e->cfg.vocab_size) return set_error(RF_EINVAL, "token_id %u out of bounds", prompt[i]);
  RF_TRY(ensure_ready(e));
  // prompt tokens except the last: forward only (inference.rs:578-592)
  for (uint32_t i = 0; i + 1 < n_prompt; i++) {
    RF_TRY(set_io(e, prompt[i], e->seq_len));
    RF_TRY(launch_step(e, false));
    e->seq_len++;
  }
  if (n_new == 0) {
    RF_TRY(set_io(e, prompt[n_prompt - 1], e->seq_len));
    RF_TRY(launch_step(e, false));
    e->seq_len++;
    RF_CUDA(cudaStreamSynchronize(e->stream));
    return check_async_errors(e);
  }
  // The last prompt token and every generated token but the last go through
  // decode steps whose argmax feeds the next step on the device (the reference
  // forwards each sampled token except the final one, inference.rs:595-712).
  return decode_loop(e, prompt[n_prompt - 1], n_new, out, nullptr);
}

int rf_decode_timed(rf_engine* e, uint32_t token, uint32_t n_steps, uint32_t* out_tokens, float* device_ms) {
  ENGINE_GUARD(e);
  if (token >= e->cfg.vocab_size) return set_error(RF_EINVAL, "token_id %u out of bounds", token);
  if ((uint64_t)e->seq_len + n_steps > e->max_seq)
    return set_error(RF_ESTATE, "%u steps exceed the KV capacity %u at length %u", n_steps, e->max_seq, e->seq_len);
  RF_TRY(ensure_ready(e));
  return decode_loop(e, token, n_steps, out_tokens, device_ms);
}

int rf_step_kernel_count(const rf_engine* ec, uint32_t* out) {
  if (!ec || !out) return set_error(RF_EINVAL, "null argument");
  rf_engine* e = const_cast<rf_engine*>(ec);
  // embed, 5 per layer (6 with a separate V matrix), output norm, LM head, advance, and under tensor
  // parallelism over peer memory the sum kernels of the rank sums not fused into the GEMVs (NCCL's own
  // kernels are not counted)
  uint32_t n = 5u * e->cfg.n_layers + 4u;
  for (uint32_t l = 0; l < e->cfg.n_layers; l++) {
    n += e->layers[l].vmat.M || layer_v_split(e, (int)l) ? 1u : 0u;
    if (e->ps_ok) n += (fuse_sum(e, (int)l, 2) ? 0u : 1u) + (fuse_sum(e, (int)l, 4) ? 0u : 1u);
  }
  *out = n;
  return RF_OK;
}

int rf_selftest_wait(int device, uint32_t* err_word) {
  if (!err_word) return set_error(RF_EINVAL, "null argument");
  RF_CUDA(cudaSetDevice(device));
  unsigned w = 0;
  RF_CUDA(peer_sum_selftest(&w));
  *err_word = w;
  return RF_OK;
}

int rf_bench_layer_kernels(rf_engine* e, uint32_t iters, float* avg_ms5) {
  ENGINE_GUARD(e);
  if (!avg_ms5 || iters == 0) return set_error(RF_EINVAL, "bad arguments");
  if (!all_resident(e)) return set_error(RF_ESTATE, "every layer must be resident");
  if (e->seq_len >= e->max_seq) return set_error(RF_ESTATE, "KV cache full");
  e->h_io->pos = (int)e->seq_len;
  RF_CUDA(cudaMemcpyAsync(&e->d_io->pos, &e->h_io->pos, 4, cudaMemcpyHostToDevice, e->stream));
  cudaEvent_t a, b;
  RF_CUDA(cudaEventCreate(&a));
  RF_CUDA(cudaEventCreate(&b));
  int rc = RF_OK;
  // Each kernel class over all layers, `iters` times, captured into one graph and
  // replayed: the launches are serialised on the device with no host time between
  // them, so the average is the kernel's own device time (plus the graph's
  // kernel-to-kernel gap), not the host's launch rate.
  for (int k = 0; k < 5 && !rc; k++) {
    cudaGraph_t g = nullptr;
    cudaGraphExec_t ge = nullptr;
    cudaError_t ce = cudaStreamBeginCapture(e->stream, cudaStreamCaptureModeThreadLocal);
    if (ce == cudaSuccess) {
      for (uint32_t it = 0; it < iters && !rc; it++)
        for (uint32_t l = 0; l < e->cfg.n_layers && !rc; l++) rc = enqueue_layer_kernel(e, (int)l, k);
      ce = cudaStreamEndCapture(e->stream, &g);
    }
    if (ce == cudaSuccess && !rc) ce = cudaGraphInstantiate(&ge, g, 0);
    if (ce == cudaSuccess && !rc) ce = cudaGraphLaunch(ge, e->stream);  // warm-up
    if (ce == cudaSuccess && !rc) ce = cudaEventRecord(a, e->stream);
    if (ce == cudaSuccess && !rc) ce = cudaGraphLaunch(ge, e->stream);
    if (ce == cudaSuccess && !rc) ce = cudaEventRecord(b, e->stream);
    if (ce == cudaSuccess && !rc) ce = cudaEventSynchronize(b);
    float ms = 0.f;
    if (ce == cudaSuccess && !rc) ce = cudaEventElapsedTime(&ms, a, b);
    if (ge) cudaGraphExecDestroy(ge);
    if (g) cudaGraphDestroy(g);
    if (ce != cudaSuccess && !rc) rc = set_error(RF_ECUDA, "kernel timing failed: %s", cudaGetErrorString(ce));
    avg_ms5[k] = ms / (float)(iters * e->cfg.n_layers);
  }
  cudaEventDestroy(a);
  cudaEventDestroy(b);
  return rc;
}

int rf_kv_reset(rf_engine* e) {
  ENGINE_GUARD(e);
  e->seq_len = 0;
  return RF_OK;
}

int rf_kv_seq_len(const rf_engine* e, uint32_t* out) {
  if (!e || !out) return set_error(RF_EINVAL, "null argument");
  *out = e->seq_len;
  return RF_OK;
}

int rf_kv_read(const rf_engine* ec, int layer, int which_v, uint32_t start, uint32_t end, float* host) {
  rf_engine* e = const_cast<rf_engine*>(ec);
  ENGINE_GUARD(e);
  if (layer < 0 || layer >= (int)e->cfg.n_layers || start > end || end > e->seq_len || !host)
    return set_error(RF_EINVAL, "KV read range [%u,%u) of layer %d invalid (history %u)", start, end, layer, e->seq_len);
  if (end == start) return RF_OK;
  const uint64_t n = (uint64_t)(end - start) * e->kvh_local * e->cfg.head_dim;
  float* tmp = nullptr;
  RF_CUDA(cudaMalloc(&tmp, n * 4));
  cudaError_t ce = launch_kv_gather(which_v ? e->vc[layer] : e->kc[layer], e->rt.kv_f32, e->kvh_local, e->max_seq,
                                    e->cfg.head_dim, start, end, tmp, e->stream);
  if (ce == cudaSuccess) ce = cudaMemcpyAsync(host, tmp, n * 4, cudaMemcpyDeviceToHost, e->stream);
  if (ce == cudaSuccess) ce = cudaStreamSynchronize(e->stream);
  cudaFree(tmp);
  if (ce != cudaSuccess) return set_error(RF_ECUDA, "KV read failed: %s", cudaGetErrorString(ce));
  return RF_OK;
}

int rf_budget_total(const rf_engine* e, uint64_t* out) {
  if (!e || !out) return set_error(RF_EINVAL, "null argument");
  *out = e->budget.total();
  return RF_OK;
}
int rf_budget_used(const rf_engine* e, uint64_t* out) {
  if (!e || !out) return set_error(RF_EINVAL, "null argument");
  *out = e->budget.used();
  return RF_OK;
}
int rf_budget_available(const rf_engine* e, uint64_t* out) {
  if (!e || !out) return set_error(RF_EINVAL, "null argument");
  *out = e->budget.available();
  return RF_OK;
}


int rf_set_residency_plan(rf_engine* e, const uint8_t* mask, int ring_slots, uint64_t vram_weight_budget_bytes) {
  ENGINE_GUARD(e);
  if (!mask) return set_error(RF_EINVAL, "null residency mask");
  if (ring_slots < 0) return set_error(RF_EINVAL, "ring_slots must be >= 0");
  RF_TRY(cache_clear(e));
  uint64_t resident_bytes = 0, slot_bytes = 0;
  for (uint32_t l = 0; l < e->cfg.n_layers; l++) {
    if (mask[l]) resident_bytes += e->layers[l].resident ? e->layers[l].bytes : layer_image_bytes(e, (int)l);
    if (!mask[l]) slot_bytes = std::max(slot_bytes, layer_image_bytes(e, (int)l));
  }
  const uint64_t need = resident_bytes + (uint64_t)ring_slots * slot_bytes;
  if (vram_weight_budget_bytes && need > vram_weight_budget_bytes)
    return set_error(RF_ENOMEM, "resident layers and %d ring slots need %llu bytes, weight budget is %llu", ring_slots,
                     (unsigned long long)need, (unsigned long long)vram_weight_budget_bytes);
  RF_CUDA(cudaStreamSynchronize(e->stream));
  for (uint32_t l = 0; l < e->cfg.n_layers; l++) {
    e->plan_resident[l] = mask[l] ? 1 : 0;
    if (!mask[l] && e->layers[l].resident) {
      RF_TRY(release_layer_impl(e, (int)l));
      e->stats.evictions++;
    }
  }
  // layers the plan keeps that are not loaded yet (an engine created with a ring
  // uploads none) are loaded now from the GGUF source
  for (uint32_t l = 0; l < e->cfg.n_layers; l++)
    if (mask[l] && !e->layers[l].resident && e->src) RF_TRY(load_layer_gguf(e, (int)l));
  if (ring_slots != e->rt.ring_slots) free_ring(e);
  e->rt.ring_slots = ring_slots;
  return RF_OK;
}

int rf_plan_residency(rf_engine* e, uint64_t vram_weight_budget_bytes, int ring_slots, uint8_t* mask_out) {
  ENGINE_GUARD(e);
  if (ring_slots < 0) return set_error(RF_EINVAL, "ring_slots must be >= 0");
  const uint32_t L = e->cfg.n_layers;
  std::vector<uint64_t> img(L);
  uint64_t slot = 0, all = 0;
  for (uint32_t l = 0; l < L; l++) {
    img[l] = layer_image_bytes(e, (int)l);
    slot = std::max(slot, img[l]);
    all += img[l];
  }
  std::vector<uint8_t> mask(L, 0);
  int slots = ring_slots;
  if (!vram_weight_budget_bytes || all <= vram_weight_budget_bytes) {
    std::fill(mask.begin(), mask.end(), 1);  // everything fits: no ring
    slots = 0;
  } else {
    const uint64_t ring = (uint64_t)ring_slots * slot;
    if (ring > vram_weight_budget_bytes)
      return set_error(RF_ENOMEM, "%d ring slots of %llu bytes exceed the weight budget %llu", ring_slots,
                       (unsigned long long)slot, (unsigned long long)vram_weight_budget_bytes);
    uint64_t used = ring;
    for (uint32_t l = 0; l < L && used + img[l] <= vram_weight_budget_bytes; l++) {
      mask[l] = 1;
      used += img[l];
    }
  }
  if (mask_out) std::copy(mask.begin(), mask.end(), mask_out);
  return rf_set_residency_plan(e, mask.data(), slots, vram_weight_budget_bytes);
}

int rf_set_layer_cache(rf_engine* e, uint64_t capacity_bytes) {
  ENGINE_GUARD(e);
  RF_TRY(cache_clear(e));
  e->cache_capacity = capacity_bytes;
  return RF_OK;
}

int rf_residency_stats_get(const rf_engine* e, rf_residency_stats* out) {
  if (!e || !out) return set_error(RF_EINVAL, "null argument");
  *out = e->stats;
  out->peak_bytes = e->budget.peak();
  return RF_OK;
}

int rf_tp_peer_sum(const rf_engine* e, int* out) {
  if (!e || !out) return set_error(RF_EINVAL, "null argument");
  *out = e->ps_ok ? 1 : 0;
  return RF_OK;
}

int rf_tp_unique_id(uint8_t* out128) {
  if (!out128) return set_error(RF_EINVAL, "null argument");
  if (!nccl()) return set_error(RF_ENCCL, "libnccl.so.2 could not be loaded");
  ncclUniqueId id;
  RF_NCCL(nccl()->getUniqueId(&id));
  memcpy(out128, &id, sizeof id);
  return RF_OK;
}

}  // extern "C"
