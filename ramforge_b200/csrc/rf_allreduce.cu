// rf_allreduce.cu - the tensor-parallel sum over NVLink peer memory (PeerSum in
// rf_kernels.cuh): one kernel per row-parallel projection in place of a library
// all-reduce.
#include "rf_device.cuh"

namespace rf {

namespace {

__global__ void __launch_bounds__(PS_THREADS) peer_sum_kernel(PeerSum P, const float* __restrict__ partial,
                                                              float* __restrict__ out, int n, int site) {
  griddep_wait();
  // The next kernel may start now: it waits for this one's completion before it
  // reads the sum, and meanwhile its weight prefetch overlaps the exchange.
  griddep_launch();
  const int b = blockIdx.x, par = site & 1;
  const unsigned e = *reinterpret_cast<volatile unsigned*>(P.epoch + site) + 1;  // this call's generation
  const int i0 = b * PS_ELEMS + threadIdx.x * 4;
  const bool in = i0 < n;
  // 1. this rank's slice into every rank's receive area (row `rank`)
  if (in) {
    const float4 v = __ldcg(reinterpret_cast<const float4*>(partial + i0));
    for (int p = 0; p < P.n_ranks; p++)
      __stcg(reinterpret_cast<float4*>(P.recv[p] + ((size_t)par * P.n_ranks + P.rank) * P.n_max + i0), v);
  }
  __syncthreads();  // the CTA's peer stores, then the flags' release (system scope) orders them
  // 2. flag slice b on every rank, then wait for every rank's flag of slice b here
  if (threadIdx.x < P.n_ranks) {
    const int p = threadIdx.x;
    st_release_sys(P.flags[p] + ((size_t)P.rank * P.sites + site) * P.max_ctas + b, e);
    const unsigned* f = P.flags[P.rank] + ((size_t)p * P.sites + site) * P.max_ctas + b;
    if (!wait_flag_sys(f, e)) atomicOr(P.err, 1u);
  }
  __syncthreads();
  // 3. the ranks' partials in rank order
  if (in) {
    float4 s = make_float4(0.f, 0.f, 0.f, 0.f);
    for (int p = 0; p < P.n_ranks; p++) {
      const float4 t = __ldcv(reinterpret_cast<const float4*>(P.recv[P.rank] + ((size_t)par * P.n_ranks + p) * P.n_max + i0));
      s.x += t.x;
      s.y += t.y;
      s.z += t.z;
      s.w += t.w;
    }
    *reinterpret_cast<float4*>(out + i0) = s;
  }
  // 4. the last CTA moves the call site to the next generation
  __syncthreads();
  if (threadIdx.x == 0 && atomicAdd(P.done + site, 1u) == gridDim.x - 1) {
    P.epoch[site] = e;
    P.done[site] = 0u;
  }
}
}  // namespace

static size_t recv_bytes(int n_ranks, int n_max) { return ((size_t)2 * n_ranks * n_max * sizeof(float) + 255) & ~size_t(255); }
// flag slots per call site: one per CTA of the sum kernel (PS_ELEMS elements) or
// per 64-row tile of a GEMV that pushes its rows (PeerLink), whichever is more
static int max_ctas_of(int n_max) { return (n_max + QT_ROWS - 1) / QT_ROWS; }
static size_t flag_words(int n_ranks, int n_max, int sites) { return (size_t)n_ranks * sites * max_ctas_of(n_max); }

size_t peer_sum_area_bytes(int n_ranks, int n_max, int sites) {
  return recv_bytes(n_ranks, n_max) + 4 * (flag_words(n_ranks, n_max, sites) + 3 * (size_t)sites + 1);
}

void peer_sum_bind(PeerSum* P, int p, void* area, bool own) {
  uint8_t* a = static_cast<uint8_t*>(area);
  P->recv[p] = reinterpret_cast<float*>(a);
  P->flags[p] = reinterpret_cast<unsigned*>(a + recv_bytes(P->n_ranks, P->n_max));
  P->max_ctas = max_ctas_of(P->n_max);
  if (own) {
    unsigned* w = P->flags[p] + flag_words(P->n_ranks, P->n_max, P->sites);
    P->epoch = w;
    P->done = w + P->sites;
    P->err = w + 2 * P->sites;
    P->fgen = w + 2 * P->sites + 1;
  }
}

cudaError_t launch_peer_sum(const Launch& L, const PeerSum& P, const float* partial, float* out, int n, int site) {
  if (n <= 0 || n % 4 || n > P.n_max || site < 0 || site >= P.sites || P.n_ranks > RF_MAX_TP)
    return cudaErrorInvalidValue;
  return launch_k(L, peer_sum_kernel, dim3((n + PS_ELEMS - 1) / PS_ELEMS), dim3(PS_THREADS), 0, P, partial, out, n,
                  site);
}

// Check of the peer sum's bounded wait on one GPU: a two-rank sum whose second
// rank is a second local area that no kernel ever flags.  The wait for that
// rank's flag gives up after about a second, sets bit 0 of the error word and
// the kernel finishes; *err_out gets the word.
cudaError_t peer_sum_selftest(unsigned* err_out) {
  const int n_max = PS_ELEMS, sites = 2;
  // each area and the vectors start on a 256-byte boundary (float4 accesses)
  const size_t bytes = (peer_sum_area_bytes(2, n_max, sites) + 255) & ~size_t(255);
  uint8_t* mem = nullptr;
  cudaError_t e = cudaMalloc(&mem, 2 * bytes + 2 * n_max * sizeof(float));
  if (e != cudaSuccess) return e;
  e = cudaMemset(mem, 0, 2 * bytes + 2 * n_max * sizeof(float));
  PeerSum P{};
  P.rank = 0;
  P.n_ranks = 2;
  P.n_max = n_max;
  P.sites = sites;
  peer_sum_bind(&P, 0, mem, true);
  peer_sum_bind(&P, 1, mem + bytes, false);
  float* partial = reinterpret_cast<float*>(mem + 2 * bytes);
  float* out = partial + n_max;
  if (e == cudaSuccess) e = launch_peer_sum(Launch{nullptr, false}, P, partial, out, n_max, 0);
  if (e == cudaSuccess) e = cudaDeviceSynchronize();
  unsigned w = 0;
  if (e == cudaSuccess) e = cudaMemcpy(&w, P.err, sizeof w, cudaMemcpyDeviceToHost);
  if (e == cudaSuccess) *err_out = w;
  cudaFree(mem);
  return e;
}

}  // namespace rf
