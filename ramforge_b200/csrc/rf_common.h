// rf_common.h - host-side shared pieces of librfcuda.so: error reporting, the
// byte budget, GGUF parsing and host-side weight packing.
#pragma once
#include <cuda_runtime.h>
#include <stdarg.h>
#include <stdint.h>

#include <map>
#include <string>
#include <vector>

#include "../../include/rfcuda.h"
#include "rf_kernels.cuh"

namespace rf {

// ---- errors: thread-local message + negative status (Result<_, String>) ----
int set_error(int code, const char* fmt, ...);
const char* last_error();

#define RF_CUDA(expr)                                                                         \
  do {                                                                                        \
    cudaError_t _e = (expr);                                                                  \
    if (_e != cudaSuccess)                                                                    \
      return ::rf::set_error(RF_ECUDA, "%s failed: %s (%s:%d)", #expr, cudaGetErrorString(_e), \
                             __FILE__, __LINE__);                                             \
  } while (0)
#define RF_TRY(expr)      \
  do {                    \
    int _rc = (expr);     \
    if (_rc) return _rc;  \
  } while (0)

// ---- MemoryBudget (ramforge-core/src/memory.rs:39-388) -------------------
// Named byte charges against a fixed total: allocate fails on zero size, on a
// duplicate name and when the charge does not fit; release fails on unknown
// names.  peak tracks the high-water mark.
class Budget {
 public:
  explicit Budget(uint64_t total = 0) : total_(total) {}
  uint64_t total() const { return total_; }
  uint64_t used() const { return used_; }
  uint64_t peak() const { return peak_; }
  uint64_t available() const { return total_ > used_ ? total_ - used_ : 0; }
  bool can_allocate(uint64_t b) const { return b <= available(); }
  int allocate(const std::string& name, uint64_t bytes);
  int release(const std::string& name);
  bool has(const std::string& name) const { return charges_.count(name) != 0; }
  uint64_t charge(const std::string& name) const {
    auto it = charges_.find(name);
    return it == charges_.end() ? 0 : it->second;
  }

 private:
  uint64_t total_ = 0, used_ = 0, peak_ = 0;
  std::map<std::string, uint64_t> charges_;
};

// ---- GGUF (ramforge-core/src/gguf.rs:196-330) ----------------------------
struct GgufMeta {
  uint32_t vtype = 0;
  bool has_u = false, has_f = false;
  uint64_t u = 0;
  double f = 0;
  std::string str;
  uint64_t arr_len = 0;
};
struct GgufTensor {
  std::string name;
  std::vector<uint64_t> dims;
  uint32_t type = 0;
  uint64_t offset = 0, nbytes = 0;
  const uint8_t* data = nullptr;
};
struct Gguf {
  uint32_t version = 0;
  uint64_t alignment = 32, data_start = 0;
  std::map<std::string, GgufMeta> meta;
  std::vector<GgufTensor> tensors;
  const GgufTensor* find(const std::string& n) const;
};
int parse_gguf(const uint8_t* p, uint64_t len, Gguf* out);
// LlamaConfig::from_gguf (runtime/src/model.rs:40-161)
int llama_config_from_gguf(const Gguf& g, rf_model_config* cfg);

// ---- coalesced layer reads (runtime/src/layer_read.rs:6-132) -------------------
constexpr uint64_t kMaxCoalescedGap = 4 * 1024;           // MAX_COALESCED_GAP_BYTES
constexpr uint64_t kMaxCoalescedSpan = 64ull * 1024 * 1024;  // MAX_COALESCED_SPAN_BYTES
struct ReadPlan {
  std::vector<rf_read_range> ranges;
  std::vector<rf_planned_tensor> placed;
  rf_read_plan_totals totals{};
};
int build_read_plan(const rf_tensor_extent* t, uint32_t n, ReadPlan* out);

// ---- host packing: GGUF rows -> PackedMat byte streams --------------------
struct HostPacked {
  PackedMat geo;  // geometry (pointers unused)
  std::vector<uint8_t> qs, sc;
};
// Size a zeroed host image of an M x K packed matrix of `type`.
int host_packed_init(int type, uint32_t M, uint32_t K, HostPacked* out);
// Copy rows into a packed image: packed row dst_row0 + r*dst_row_step takes GGUF
// source row src_rows[r] (rows of src_row_bytes), starting at block src_blk_off
// (a column slice for row-parallel shards).  Multi-threaded, pure byte shuffle.
int pack_rows(const uint8_t* src, uint64_t src_row_bytes, uint32_t src_blk_off, const std::vector<int>& src_rows,
              HostPacked* out, uint32_t dst_row0, uint32_t dst_row_step);
// Decode `rows` GGUF rows of a format the engine stores as f32 (expands_to_f32),
// K elements each (rows of src_row_bytes), into out[rows][K]: the reference's
// block dequantize, value for value.  Multi-threaded.
int expand_rows_f32(int type, const uint8_t* src, uint64_t src_row_bytes, uint64_t rows, uint32_t K, float* out);

}  // namespace rf
