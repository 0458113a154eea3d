// rf_ops.cu - standalone device-pointer ops of include/rfcuda.h: packed
// matrices + quantized matvec (benchmark config 2) and batched GQA decode
// attention (benchmark config 3).
#include <mutex>
#include <unordered_map>

#include "rf_common.h"

using namespace rf;

struct rf_matrix {
  PackedMat m{};
  void* block = nullptr;
  uint64_t bytes = 0;
  int device = 0;
};

namespace {
// Per-device split-K workspace for rf_decode_attention: partial sums and the
// per-(sequence, KV head) arrival counters (zero at rest; the last CTA of a
// head resets its counter).  Grown on demand, never shrunk.
struct AttnWorkspace {
  float* part = nullptr;
  size_t part_floats = 0;
  unsigned* counters = nullptr;
  size_t n_counters = 0;
};
std::mutex g_ws_mu;
std::unordered_map<int, AttnWorkspace> g_ws;

// Fixed scratch of rf_decode_attention_noalloc: the split-K partial sums
// followed by the per-(sequence, KV head) arrival counters, 16 MiB per device
// that loads this library, held until the process exits.  Device code could
// name it directly; host code must ask the runtime for its device address.
constexpr size_t kNoAllocScratchFloats = size_t(4) << 20;  // 16 MiB
static __device__ __align__(256) float g_noalloc_scratch[kNoAllocScratchFloats];

// Device address of g_noalloc_scratch in the current device's current context.
// Looked up on every call rather than cached: after a cudaDeviceReset the
// library's device code is loaded again into the new context and the array gets
// a new address, which a cached pointer would miss.  The lookup allocates
// nothing; the first one in a context may load the device code, which is why the
// first call should come before any stream capture.
int noalloc_scratch(float** out) {
  void* p = nullptr;
  cudaError_t ce = cudaGetSymbolAddress(&p, g_noalloc_scratch);
  if (ce != cudaSuccess || !p)
    return set_error(RF_ECUDA, "cudaGetSymbolAddress(no-allocation scratch) failed: %s", cudaGetErrorString(ce));
  *out = (float*)p;
  return RF_OK;
}

// Per-device split-K scratch of rf_qmatvec (GemvScratch), grown on demand.
struct GemvWorkspace {
  float* part = nullptr;
  uint64_t part_floats = 0;
  unsigned* cnt = nullptr;
  uint32_t n_cnt = 0;
};
std::mutex g_gws_mu;
std::unordered_map<int, GemvWorkspace> g_gws;

int gemv_workspace(int dev, const PackedMat& W, GemvScratch* out) {
  uint64_t pf = 0;
  uint32_t nc = 0;
  gemv_scratch_need(W, &pf, &nc);
  std::lock_guard<std::mutex> lk(g_gws_mu);
  GemvWorkspace& w = g_gws[dev];
  if (w.part_floats < pf) {
    if (w.part) cudaFree(w.part);
    w.part = nullptr;
    w.part_floats = 0;
    RF_CUDA(cudaMalloc(&w.part, pf * sizeof(float)));
    w.part_floats = pf;
  }
  if (w.n_cnt < nc) {
    if (w.cnt) cudaFree(w.cnt);
    w.cnt = nullptr;
    w.n_cnt = 0;
    RF_CUDA(cudaMalloc(&w.cnt, nc * sizeof(unsigned)));
    RF_CUDA(cudaMemset(w.cnt, 0, nc * sizeof(unsigned)));
    RF_CUDA(cudaDeviceSynchronize());  // zero before any caller stream (possibly non-blocking) uses them
    w.n_cnt = nc;
  }
  *out = GemvScratch{w.part, w.cnt, w.part_floats, w.n_cnt};
  return RF_OK;
}

int workspace(int dev, size_t part_floats, size_t n_counters, AttnWorkspace** out) {
  std::lock_guard<std::mutex> lk(g_ws_mu);
  AttnWorkspace& w = g_ws[dev];
  if (w.part_floats < part_floats) {
    if (w.part) cudaFree(w.part);
    w.part = nullptr;
    w.part_floats = 0;
    RF_CUDA(cudaMalloc(&w.part, part_floats * sizeof(float)));
    w.part_floats = part_floats;
  }
  if (w.n_counters < n_counters) {
    if (w.counters) cudaFree(w.counters);
    w.counters = nullptr;
    w.n_counters = 0;
    RF_CUDA(cudaMalloc(&w.counters, n_counters * sizeof(unsigned)));
    RF_CUDA(cudaMemset(w.counters, 0, n_counters * sizeof(unsigned)));
    RF_CUDA(cudaDeviceSynchronize());  // zero before any caller stream (possibly non-blocking) uses them
    w.n_counters = n_counters;
  }
  *out = &w;
  return RF_OK;
}
}  // namespace

extern "C" {

int rf_matrix_create(int type, const void* bytes, uint64_t nbytes, int on_device, uint32_t n_out, uint32_t n_in,
                     rf_matrix** out) {
  if (!bytes || !out) return set_error(RF_EINVAL, "null argument");
  *out = nullptr;
  if (expands_to_f32(type)) {  // stored as f32: decode on the host, then an F32 matrix
    const uint32_t qk = block_elems(type);
    if (n_out == 0 || n_in == 0 || n_in % qk)
      return set_error(RF_EINVAL, "type %d cannot hold a %u x %u matrix", type, n_out, n_in);
    const uint64_t rb = (uint64_t)(n_in / qk) * block_bytes(type);
    if (nbytes < rb * n_out)
      return set_error(RF_EINVAL, "weight truncated: expected %llu bytes, got %llu", (unsigned long long)(rb * n_out),
                       (unsigned long long)nbytes);
    std::vector<uint8_t> staged;
    const uint8_t* src = (const uint8_t*)bytes;
    if (on_device) {
      staged.resize(rb * n_out);
      RF_CUDA(cudaMemcpy(staged.data(), bytes, staged.size(), cudaMemcpyDeviceToHost));
      src = staged.data();
    }
    std::vector<float> f((size_t)n_in * n_out);
    RF_TRY(expand_rows_f32(type, src, rb, n_out, n_in, f.data()));
    return rf_matrix_create(T_F32, f.data(), 4ull * f.size(), 0, n_out, n_in, out);
  }
  PackedMat g;
  if (!packed_geometry(type, n_out, n_in, &g))
    return set_error(RF_EINVAL, "type %d cannot hold a %u x %u matrix", type, n_out, n_in);
  const uint64_t row_bytes = (uint64_t)(n_in / block_elems(type)) * block_bytes(type);
  if (nbytes < row_bytes * n_out)
    return set_error(RF_EINVAL, "weight truncated: expected %llu bytes, got %llu",
                     (unsigned long long)(row_bytes * n_out), (unsigned long long)nbytes);
  rf_matrix* m = new rf_matrix();
  cudaGetDevice(&m->device);
  // qs | sc | one word for the pack kernel's subnormal-scale flag
  const uint64_t qs_b = (packed_qs_bytes(g) + 255) & ~255ull, sc_b = (packed_sc_bytes(g) + 255) & ~255ull;
  m->bytes = qs_b + (sc_b ? sc_b : 256) + 256;
  cudaError_t ce = cudaMalloc(&m->block, m->bytes);
  if (ce != cudaSuccess) {
    delete m;
    return set_error(RF_ENOMEM, "cudaMalloc(%llu) failed: %s", (unsigned long long)m->bytes, cudaGetErrorString(ce));
  }
  m->m = g;
  m->m.qs = (uint8_t*)m->block;
  m->m.sc = (uint8_t*)m->block + qs_b;
  unsigned* flag = (unsigned*)((uint8_t*)m->block + qs_b + (sc_b ? sc_b : 256));
  if (on_device) {
    ce = launch_pack((const uint8_t*)bytes, nullptr, m->m, flag, 0);
    if (ce == cudaSuccess) ce = cudaDeviceSynchronize();
    unsigned f = 0;
    if (ce == cudaSuccess) ce = cudaMemcpy(&f, flag, sizeof f, cudaMemcpyDeviceToHost);
    m->m.sub_scales = f ? 1 : 0;
  } else {
    HostPacked hp;
    std::vector<int> rows(n_out);
    for (uint32_t r = 0; r < n_out; r++) rows[r] = (int)r;
    int rc = host_packed_init(type, n_out, n_in, &hp);
    if (!rc) rc = pack_rows((const uint8_t*)bytes, row_bytes, 0, rows, &hp, 0, 1);
    if (rc) {
      cudaFree(m->block);
      delete m;
      return rc;
    }
    ce = cudaMemcpy(m->m.qs, hp.qs.data(), hp.qs.size(), cudaMemcpyHostToDevice);
    if (ce == cudaSuccess && !hp.sc.empty()) ce = cudaMemcpy(m->m.sc, hp.sc.data(), hp.sc.size(), cudaMemcpyHostToDevice);
    // a copy from pageable memory may return before its DMA ends: finish it
    // before the caller's streams (possibly non-blocking) read the matrix
    if (ce == cudaSuccess) ce = cudaDeviceSynchronize();
    m->m.sub_scales = has_subnormal_scales(hp.geo, hp.sc.data()) ? 1 : 0;
  }
  if (ce != cudaSuccess) {
    cudaFree(m->block);
    delete m;
    return set_error(RF_ECUDA, "packing failed: %s", cudaGetErrorString(ce));
  }
  *out = m;
  return RF_OK;
}

void rf_matrix_destroy(rf_matrix* m) {
  if (!m) return;
  int cur = 0;
  cudaGetDevice(&cur);
  cudaSetDevice(m->device);
  cudaFree(m->block);
  cudaSetDevice(cur);
  delete m;
}

uint64_t rf_matrix_device_bytes(const rf_matrix* m) { return m ? m->bytes : 0; }

int rf_qmatvec(const rf_matrix* m, const float* dX, float* dY, int batch, void* stream) {
  if (!m || !dX || !dY) return set_error(RF_EINVAL, "null argument");
  if (batch < 1 || batch > 8) return set_error(RF_EINVAL, "batch %d out of range 1..8", batch);
  cudaStream_t s = (cudaStream_t)stream;
  int cur = 0;
  RF_CUDA(cudaGetDevice(&cur));
  if (cur != m->device) return set_error(RF_EINVAL, "matrix lives on device %d, current device is %d", m->device, cur);
  GemvScratch ws{};
  RF_TRY(gemv_workspace(cur, m->m, &ws));
  RF_CUDA(gemv_batched(s, m->m, &ws, dX, batch, dY));
  return RF_OK;
}

// rf_qgemm's per-device workspace: the split activations and an error word.
struct QgemmWorkspace {
  void* xt = nullptr;
  size_t xt_bytes = 0;
  unsigned* err = nullptr;
};
std::mutex g_qg_mu;
std::unordered_map<int, QgemmWorkspace> g_qg;

int rf_qgemm(const rf_matrix* m, const float* dX, float* dY, int n_tokens, void* stream) {
  if (!m || !dX || !dY) return set_error(RF_EINVAL, "null argument");
  if (n_tokens < 1) return set_error(RF_EINVAL, "n_tokens %d must be positive", n_tokens);
  if (!prefill_supported(m->m.type))
    return set_error(RF_EUNSUPPORTED, "the tensor-core GEMM covers Q4_K and Q8_0 matrices, not type %d", m->m.type);
  cudaStream_t s = (cudaStream_t)stream;
  int cur = 0;
  RF_CUDA(cudaGetDevice(&cur));
  if (cur != m->device) return set_error(RF_EINVAL, "matrix lives on device %d, current device is %d", m->device, cur);
  const size_t need = prefill_xt_bytes((uint32_t)n_tokens, m->m.Kp);
  void* xt = nullptr;
  unsigned* err = nullptr;
  {
    std::lock_guard<std::mutex> lk(g_qg_mu);
    QgemmWorkspace& w = g_qg[cur];
    if (!w.err) {
      RF_CUDA(cudaMalloc(&w.err, sizeof(unsigned)));
      RF_CUDA(cudaMemset(w.err, 0, sizeof(unsigned)));
      RF_CUDA(cudaDeviceSynchronize());
    }
    if (w.xt_bytes < need) {
      if (w.xt) cudaFree(w.xt);
      w.xt = nullptr;
      w.xt_bytes = 0;
      RF_CUDA(cudaMalloc(&w.xt, need));
      w.xt_bytes = need;
    }
    xt = w.xt;
    err = w.err;
  }
  RF_CUDA(prefill_split(Launch{s, false}, dX, m->m.K, (uint32_t)n_tokens, m->m.K, m->m.Kp, nullptr, 0.f, xt));
  RF_CUDA(prefill_gemm_store(Launch{s, false}, m->m, xt, (uint32_t)n_tokens, err, dY, m->m.M));
  return RF_OK;
}

int rf_qgemm_error_word(uint32_t* word) {
  if (!word) return set_error(RF_EINVAL, "null argument");
  int dev = 0;
  RF_CUDA(cudaGetDevice(&dev));
  unsigned* err = nullptr;
  {
    std::lock_guard<std::mutex> lk(g_qg_mu);
    auto it = g_qg.find(dev);
    if (it != g_qg.end()) err = it->second.err;
  }
  *word = 0;
  if (!err) return RF_OK;
  RF_CUDA(cudaDeviceSynchronize());
  unsigned w = 0;
  RF_CUDA(cudaMemcpy(&w, err, sizeof w, cudaMemcpyDeviceToHost));
  if (w) RF_CUDA(cudaMemset(err, 0, sizeof w));
  RF_CUDA(cudaDeviceSynchronize());
  *word = w;
  return RF_OK;
}

int rf_decode_attention(const float* dQ, const uint16_t* dK, const uint16_t* dV, int ctx, int n_heads, int n_kv_heads,
                        int head_dim, int batch, float* dOut, void* stream) {
  if (!dQ || !dK || !dV || !dOut) return set_error(RF_EINVAL, "null argument");
  if (ctx <= 0 || batch <= 0 || n_kv_heads <= 0 || n_heads % n_kv_heads || head_dim <= 0 || head_dim > 128)
    return set_error(RF_EINVAL, "invalid attention shape");
  const int G = n_heads / n_kv_heads;
  if (G != 1 && G != 2 && G != 4 && G != 8) return set_error(RF_EUNSUPPORTED, "GQA group %d unsupported", G);
  int dev = 0;
  RF_CUDA(cudaGetDevice(&dev));
  const int max_splits = std::max(64, (ctx + 511) / 512);
  AttnWorkspace* w = nullptr;
  RF_TRY(workspace(dev, attn_part_floats(batch, n_kv_heads, max_splits, G, head_dim),
                   (size_t)batch * n_kv_heads, &w));
  AttnArgs a{};
  a.q = dQ;
  a.kc = dK;
  a.vc = dV;
  a.head_stride = (uint64_t)ctx * head_dim;
  a.batch_stride = (uint64_t)n_kv_heads * ctx * head_dim;
  a.k_cur = nullptr;
  a.v_cur = nullptr;
  a.d_nhist = nullptr;
  a.nhist = ctx;
  a.n_heads = n_heads;
  a.n_kv_heads = n_kv_heads;
  a.head_dim = head_dim;
  a.batch = batch;
  a.max_splits = max_splits;
  a.part = w->part;
  a.counters = w->counters;
  a.out = dOut;
  a.kv_f32 = 0;
  RF_CUDA(launch_attention(Launch{(cudaStream_t)stream, false}, a));
  return RF_OK;
}

// rf_decode_attention for callers that cannot allocate device memory: the
// split-K partials and counters live in g_noalloc_scratch instead of a
// workspace grown with cudaMalloc.  Every call looks up the array's device
// address in the current context (cudaGetSymbolAddress); make the first call on
// a device before any stream capture.  Calls share the array: the
// counters are cleared (cudaMemsetAsync, no allocation) before every launch,
// and calls that overlap on the GPU race on the scratch.  Shapes whose scratch
// exceeds kNoAllocScratchFloats are rejected with RF_EINVAL.
int rf_decode_attention_noalloc(const float* dQ, const uint16_t* dK, const uint16_t* dV, int ctx, int n_heads,
                                int n_kv_heads, int head_dim, int batch, float* dOut, void* stream) {
  if (!dQ || !dK || !dV || !dOut) return set_error(RF_EINVAL, "null argument");
  if (ctx <= 0 || batch <= 0 || n_kv_heads <= 0 || n_heads % n_kv_heads || head_dim <= 0 || head_dim > 128)
    return set_error(RF_EINVAL, "invalid attention shape");
  const int G = n_heads / n_kv_heads;
  if (G != 1 && G != 2 && G != 4 && G != 8) return set_error(RF_EUNSUPPORTED, "GQA group %d unsupported", G);
  float* scratch = nullptr;
  RF_TRY(noalloc_scratch(&scratch));
  const size_t n_counters = (size_t)batch * n_kv_heads;
  const size_t per_split = attn_part_floats(batch, n_kv_heads, 1, G, head_dim);
  const int min_splits = (ctx + 511) / 512;  // every split covers at most 512 positions
  int max_splits = std::max(64, min_splits);
  if (per_split * (size_t)max_splits + n_counters > kNoAllocScratchFloats) {
    const size_t fit = per_split ? (kNoAllocScratchFloats - std::min(n_counters, kNoAllocScratchFloats)) / per_split : 0;
    if (fit < (size_t)min_splits)
      return set_error(RF_EINVAL,
                       "rf_decode_attention_noalloc: batch %d x %d KV heads x ctx %d needs %zu bytes of scratch; "
                       "its fixed scratch holds %zu bytes",
                       batch, n_kv_heads, ctx, (per_split * (size_t)min_splits + n_counters) * 4,
                       kNoAllocScratchFloats * 4);
    max_splits = (int)std::min<size_t>(fit, (size_t)max_splits);
  }
  unsigned* counters = reinterpret_cast<unsigned*>(scratch + per_split * (size_t)max_splits);
  RF_CUDA(cudaMemsetAsync(counters, 0, n_counters * sizeof(unsigned), (cudaStream_t)stream));
  AttnArgs a{};
  a.q = dQ;
  a.kc = dK;
  a.vc = dV;
  a.head_stride = (uint64_t)ctx * head_dim;
  a.batch_stride = (uint64_t)n_kv_heads * ctx * head_dim;
  a.nhist = ctx;
  a.n_heads = n_heads;
  a.n_kv_heads = n_kv_heads;
  a.head_dim = head_dim;
  a.batch = batch;
  a.max_splits = max_splits;
  a.part = scratch;
  a.counters = counters;
  a.out = dOut;
  RF_CUDA(launch_attention(Launch{(cudaStream_t)stream, false}, a));
  return RF_OK;
}

}  // extern "C"
