// rf_common.cpp - errors, byte budget, GGUF parsing, LlamaConfig, host packing.
#include "rf_common.h"

#include <stdio.h>
#include <string.h>

#include <algorithm>
#include <cmath>
#include <thread>

namespace rf {

static thread_local std::string g_err;

int set_error(int code, const char* fmt, ...) {
  char buf[1024];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof buf, fmt, ap);
  va_end(ap);
  g_err = buf;
  return code;
}
const char* last_error() { return g_err.c_str(); }

// ---- Budget ----------------------------------------------------------------
// MemoryBudget::allocate (memory.rs:93-122) / release (memory.rs:131-152).
int Budget::allocate(const std::string& name, uint64_t bytes) {
  if (bytes == 0) return set_error(RF_EINVAL, "invalid allocation size 0 for '%s'", name.c_str());
  if (charges_.count(name)) return set_error(RF_EINVAL, "allocation '%s' already exists", name.c_str());
  if (!can_allocate(bytes))
    return set_error(RF_ENOMEM,
                     "insufficient VRAM budget for '%s': requested %llu, available %llu (total %llu, used %llu)",
                     name.c_str(), (unsigned long long)bytes, (unsigned long long)available(),
                     (unsigned long long)total_, (unsigned long long)used_);
  charges_[name] = bytes;
  used_ += bytes;
  peak_ = std::max(peak_, used_);
  return RF_OK;
}
int Budget::release(const std::string& name) {
  auto it = charges_.find(name);
  if (it == charges_.end()) return set_error(RF_EINVAL, "allocation '%s' not found", name.c_str());
  used_ -= it->second;
  charges_.erase(it);
  return RF_OK;
}

// ---- GGUF ---------------------------------------------------------------------
namespace {
struct Reader {
  const uint8_t* p;
  uint64_t len, pos = 0;
  bool err = false;
  bool take(void* dst, uint64_t n) {
    if (err || pos + n > len || pos + n < pos) {
      err = true;
      return false;
    }
    if (dst) memcpy(dst, p + pos, n);
    pos += n;
    return true;
  }
  uint32_t u32() { uint32_t v = 0; take(&v, 4); return v; }
  uint64_t u64() { uint64_t v = 0; take(&v, 8); return v; }
  bool str(std::string* s) {
    uint64_t n = u64();
    if (err || n > 10ull * 1024 * 1024 || pos + n > len) { err = true; return false; }  // MAX_STRING_LEN (gguf.rs:12)
    if (s) s->assign((const char*)p + pos, n);
    pos += n;
    return true;
  }
};

// read_metadata_value (gguf.rs:130-151); integer/float views as MetadataValue::as_u64
// (types.rs:86-98) and the get_f32_arch match (runtime/src/model.rs:79-98).
void read_scalar(Reader& r, uint32_t t, GgufMeta* m) {
  uint8_t b1 = 0; uint16_t b2 = 0; uint32_t b4 = 0; uint64_t b8 = 0;
  switch (t) {
    case 0: r.take(&b1, 1); m->u = b1; m->has_u = true; break;
    case 1: r.take(&b1, 1); m->u = (uint64_t)(int64_t)(int8_t)b1; m->has_u = true; break;
    case 2: r.take(&b2, 2); m->u = b2; m->has_u = true; break;
    case 3: r.take(&b2, 2); m->u = (uint64_t)(int64_t)(int16_t)b2; m->has_u = true; break;
    case 4: r.take(&b4, 4); m->u = b4; m->has_u = true; m->f = b4; m->has_f = true; break;
    case 5: r.take(&b4, 4); m->u = (uint64_t)(int64_t)(int32_t)b4; m->has_u = true; m->f = (int32_t)b4; m->has_f = true; break;
    case 6: { float f = 0; r.take(&f, 4); m->f = f; m->has_f = true; break; }
    case 7: r.take(&b1, 1); break;
    case 8: r.str(&m->str); break;
    case 10: r.take(&b8, 8); m->u = b8; m->has_u = true; m->f = (double)b8; m->has_f = true; break;
    case 11: r.take(&b8, 8); m->u = b8; m->has_u = true; m->f = (double)(int64_t)b8; m->has_f = true; break;
    case 12: { double d = 0; r.take(&d, 8); m->f = d; m->has_f = true; break; }
    default: r.err = true;
  }
}

// GgmlType::type_info (types.rs:354-376) for the types the engine accepts: the
// block table of rf_kernels.cuh (block_elems / block_bytes).
bool type_info(uint32_t type, uint64_t* qk, uint64_t* bsz) {
  if (type > 255 || !block_elems((int)type)) return false;
  *qk = (uint64_t)block_elems((int)type);
  *bsz = (uint64_t)block_bytes((int)type);
  return true;
}
}  // namespace

const GgufTensor* Gguf::find(const std::string& n) const {
  for (auto& t : tensors)
    if (t.name == n) return &t;
  return nullptr;
}

int parse_gguf(const uint8_t* p, uint64_t len, Gguf* g) {
  Reader r{p, len};
  char magic[4];
  if (!r.take(magic, 4) || memcmp(magic, "GGUF", 4)) return set_error(RF_EFORMAT, "invalid GGUF magic");
  g->version = r.u32();
  if (g->version < 1 || g->version > 3) return set_error(RF_EFORMAT, "unsupported GGUF version %u", g->version);
  const uint64_t nt = r.u64(), nkv = r.u64();
  if (r.err || nt > 10000000ull || nkv > 100000ull) return set_error(RF_EFORMAT, "GGUF header counts out of range");
  for (uint64_t i = 0; i < nkv; i++) {
    std::string key;
    r.str(&key);
    GgufMeta m;
    m.vtype = r.u32();
    if (r.err) return set_error(RF_EFORMAT, "truncated GGUF metadata");
    if (m.vtype == 9) {  // read_array_value (gguf.rs:153-194)
      const uint32_t at = r.u32();
      const uint64_t n = r.u64();
      if (at == 9 || n > 10000000ull) return set_error(RF_EFORMAT, "unsupported GGUF array");
      m.arr_len = n;
      for (uint64_t j = 0; j < n && !r.err; j++) {
        GgufMeta tmp;
        read_scalar(r, at, &tmp);
      }
    } else {
      read_scalar(r, m.vtype, &m);
    }
    if (r.err) return set_error(RF_EFORMAT, "truncated or invalid GGUF metadata value for '%s'", key.c_str());
    g->meta[key] = m;
  }
  auto al = g->meta.find("general.alignment");
  g->alignment = (al != g->meta.end() && al->second.has_u) ? al->second.u : 32;  // gguf.rs:251-255
  g->tensors.resize(nt);
  for (auto& t : g->tensors) {
    r.str(&t.name);
    const uint32_t nd = r.u32();
    if (r.err || nd > 8) return set_error(RF_EFORMAT, "invalid tensor info");  // MAX_DIMENSIONS (gguf.rs:13)
    t.dims.resize(nd);
    for (auto& d : t.dims) d = r.u64();
    t.type = r.u32();
    t.offset = r.u64();
    if (r.err) return set_error(RF_EFORMAT, "truncated tensor info");
  }
  uint64_t ds = r.pos;
  if (g->alignment && ds % g->alignment) ds += g->alignment - ds % g->alignment;  // align_offset (model.rs:197)
  g->data_start = ds;
  for (auto& t : g->tensors) {
    uint64_t ne = 1, qk = 0, bsz = 0;
    for (auto d : t.dims) ne *= d;
    if (!type_info(t.type, &qk, &bsz)) continue;  // unknown types stay unresolved
    t.nbytes = (ne + qk - 1) / qk * bsz;
    if (ds + t.offset + t.nbytes > len || ds + t.offset < ds)
      return set_error(RF_EFORMAT, "tensor '%s' extends past the end of the GGUF image", t.name.c_str());
    t.data = p + ds + t.offset;
  }
  return RF_OK;
}

int llama_config_from_gguf(const Gguf& g, rf_model_config* c) {
  auto arch_it = g.meta.find("general.architecture");
  std::string arch = arch_it != g.meta.end() ? arch_it->second.str : "unknown";
  if (arch != "llama" && arch != "qwen2")
    return set_error(RF_EFORMAT, "unsupported execution architecture '%s' (supported: [llama, qwen2])",
                     arch.c_str());
  const char* pre[4] = {arch.c_str(), "llama", "qwen2", "general"};
  auto get_u = [&](const char* sfx, uint64_t* v) {  // get_u64_arch (model.rs:54-77)
    for (auto pf : pre) {
      auto it = g.meta.find(std::string(pf) + "." + sfx);
      if (it != g.meta.end() && it->second.has_u) { *v = it->second.u; return true; }
    }
    return false;
  };
  auto get_f = [&](const char* sfx, float* v) {  // get_f32_arch (model.rs:79-98)
    for (auto pf : pre) {
      auto it = g.meta.find(std::string(pf) + "." + sfx);
      if (it != g.meta.end() && it->second.has_f) { *v = (float)it->second.f; return true; }
    }
    return false;
  };
  uint64_t v = 0;
  memset(c, 0, sizeof *c);
  if (get_u("vocab_size", &v)) c->vocab_size = (uint32_t)v;
  else {
    auto t = g.meta.find("tokenizer.ggml.tokens");
    if (t == g.meta.end()) return set_error(RF_EFORMAT, "missing vocab_size (tried %s.vocab_size)", arch.c_str());
    c->vocab_size = (uint32_t)t->second.arr_len;
  }
  if (!get_u("context_length", &v)) return set_error(RF_EFORMAT, "missing %s.context_length", arch.c_str());
  c->context_length = (uint32_t)v;
  if (!get_u("embedding_length", &v)) return set_error(RF_EFORMAT, "missing %s.embedding_length", arch.c_str());
  c->n_embd = (uint32_t)v;
  if (!get_u("block_count", &v)) return set_error(RF_EFORMAT, "missing %s.block_count", arch.c_str());
  c->n_layers = (uint32_t)v;
  if (!get_u("feed_forward_length", &v) && !get_u("intermediate_size", &v))
    return set_error(RF_EFORMAT, "missing %s.feed_forward_length", arch.c_str());
  c->n_ff = (uint32_t)v;
  if (!get_u("attention.head_count", &v)) return set_error(RF_EFORMAT, "missing %s.attention.head_count", arch.c_str());
  c->n_heads = (uint32_t)v;
  c->n_kv_heads = get_u("attention.head_count_kv", &v) ? (uint32_t)v : c->n_heads;
  if (!get_f("attention.layer_norm_rms_epsilon", &c->rms_eps) && !get_f("attention.layer_norm_epsilon", &c->rms_eps))
    c->rms_eps = 1e-5f;  // model.rs:142-144
  if (!get_f("rope.freq_base", &c->rope_theta)) c->rope_theta = 10000.0f;  // model.rs:146
  if (c->n_heads == 0 || c->n_kv_heads == 0) return set_error(RF_EFORMAT, "zero attention heads");
  c->head_dim = c->n_embd / c->n_heads;  // model.rs:148
  return RF_OK;
}

// ---- host packing ---------------------------------------------------------------
int host_packed_init(int type, uint32_t M, uint32_t K, HostPacked* out) {
  if (!packed_geometry(type, M, K, &out->geo))
    return set_error(RF_EINVAL, "type %d cannot hold a %u x %u matrix", type, M, K);
  out->qs.assign(packed_qs_bytes(out->geo), 0);
  out->sc.assign(packed_sc_bytes(out->geo), 0);
  return RF_OK;
}

int pack_rows(const uint8_t* src, uint64_t src_row_bytes, uint32_t src_blk_off, const std::vector<int>& src_rows,
              HostPacked* out, uint32_t dst_row0, uint32_t dst_row_step) {
  const PackedMat& g = out->geo;
  const uint32_t qk = block_elems(g.type), bsz = block_bytes(g.type), nblk = g.K / qk;
  if ((uint64_t)(src_blk_off + nblk) * bsz > src_row_bytes)
    return set_error(RF_EINVAL, "packing slice exceeds the source row");
  const size_t n = src_rows.size();
  if (n && (uint64_t)dst_row0 + (uint64_t)(n - 1) * dst_row_step >= g.M)
    return set_error(RF_EINVAL, "packing rows exceed the destination");
  uint8_t* Q = out->qs.data();
  uint8_t* C = out->sc.data();
  auto work = [&](size_t a, size_t b) {
    for (size_t r = a; r < b; r++) {
      const uint8_t* s = src + (uint64_t)src_rows[r] * src_row_bytes + (uint64_t)src_blk_off * bsz;
      const uint32_t dr = (uint32_t)(dst_row0 + (uint64_t)r * dst_row_step);
      switch (g.type) {
        case T_F32:
        case T_F16: memcpy(Q + qs_byte_off(g, dr, 0), s, (size_t)nblk * bsz); break;
        case T_Q8_0:
          for (uint32_t k = 0; k < nblk; k++, s += 34) {
            memcpy(C + sc_byte_off(g, dr, 2ull * k), s, 2);
            memcpy(Q + qs_byte_off(g, dr, 32ull * k), s + 2, 32);
          }
          break;
        case T_Q4_0:
          for (uint32_t k = 0; k < nblk; k++, s += 18) {
            memcpy(C + sc_byte_off(g, dr, 2ull * k), s, 2);
            memcpy(Q + qs_byte_off(g, dr, 16ull * k), s + 2, 16);
          }
          break;
        case T_Q4_K:
          for (uint32_t k = 0; k < nblk; k++, s += 144) {
            memcpy(C + sc_byte_off(g, dr, 16ull * k), s, 16);
            for (int p = 0; p < 4; p++) memcpy(Q + qs_byte_off(g, dr, 128ull * k + 32 * p), s + 16 + 32 * p, 32);
          }
          break;
        case T_Q6_K:
          for (uint32_t k = 0; k < nblk; k++, s += 210) six_bit_pack_block(g, Q, C, dr, k, s);
          break;
        case T_Q5_K:
          for (uint32_t k = 0; k < nblk; k++, s += 176) six_bit_pack_block(g, Q, C, dr, k, s);
          break;
        case T_Q3_K:
          for (uint32_t k = 0; k < nblk; k++, s += 110) nibble_group_pack_block(g, Q, C, dr, k, s);
          break;
        case T_Q2_K:
          for (uint32_t k = 0; k < nblk; k++, s += 84) nibble_group_pack_block(g, Q, C, dr, k, s);
          break;
      }
    }
  };
  const size_t nt = std::min<size_t>(std::max(1u, std::thread::hardware_concurrency()), 32);
  if (n < 256 || nt <= 1) {
    work(0, n);
  } else {
    std::vector<std::thread> ts;
    const size_t per = (n + nt - 1) / nt;
    for (size_t t = 0; t < nt; t++) {
      const size_t a = t * per, b = std::min(n, a + per);
      if (a < b) ts.emplace_back(work, a, b);
    }
    for (auto& t : ts) t.join();
  }
  return RF_OK;
}


// ---- formats stored as f32: the reference's block decodes --------------------------
namespace {
// f16 -> f32 as the reference reads block scales (quant.rs:40-65): IEEE, except that
// a subnormal half comes out at half its IEEE value.
float ref_f16(const uint8_t* p) {
  const uint32_t h = (uint32_t)p[0] | ((uint32_t)p[1] << 8), e = (h >> 10) & 31, m = h & 1023;
  float v;
  if (e == 0) v = std::ldexp((float)m, -25);
  else if (e == 31) v = m ? NAN : INFINITY;
  else v = std::ldexp((float)(m | 1024), (int)e - 25);
  return (h & 0x8000) ? -v : v;
}
uint32_t rd_u32(const uint8_t* p) {
  return (uint32_t)p[0] | ((uint32_t)p[1] << 8) | ((uint32_t)p[2] << 16) | ((uint32_t)p[3] << 24);
}
// BlockQ5_0::dequantize (quant.rs:140-151): q = nibble | high bit << 4, value (q-16)*d.
void dq_q5_0(const uint8_t* b, float* o) {
  const float d = ref_f16(b);
  const uint32_t qh = rd_u32(b + 2);
  for (int j = 0; j < 16; j++) {
    const int q0 = (int)((b[6 + j] & 0xFu) | (((qh >> j) << 4) & 0x10u)) - 16;
    const int q1 = (int)((b[6 + j] >> 4) | ((qh >> (j + 12)) & 0x10u)) - 16;
    o[j] = (float)q0 * d;
    o[16 + j] = (float)q1 * d;
  }
}
// BlockQ8K::dequantize (quant.rs:605-609): f32 d, value d*q.
void dq_q8_k(const uint8_t* b, float* o) {
  float d;
  memcpy(&d, b, 4);
  for (int i = 0; i < 256; i++) o[i] = d * (float)(int8_t)b[4 + i];
}
}  // namespace

int expand_rows_f32(int type, const uint8_t* src, uint64_t src_row_bytes, uint64_t rows, uint32_t K, float* out) {
  if (!expands_to_f32(type)) return set_error(RF_EINVAL, "type %d is not expanded to f32", type);
  const uint32_t qk = block_elems(type), bsz = block_bytes(type);
  if (K % qk || (uint64_t)(K / qk) * bsz > src_row_bytes) return set_error(RF_EINVAL, "bad row for type %d", type);
  auto work = [&](uint64_t a, uint64_t b) {
    for (uint64_t r = a; r < b; r++)
      for (uint32_t k = 0; k < K / qk; k++) {
        const uint8_t* blk = src + r * src_row_bytes + (uint64_t)k * bsz;
        float* o = out + r * K + (uint64_t)k * qk;
        switch (type) {
          case T_Q5_0: dq_q5_0(blk, o); break;
          case T_Q8_K: dq_q8_k(blk, o); break;
        }
      }
  };
  const uint64_t nt = std::min<uint64_t>(std::max(1u, std::thread::hardware_concurrency()), 32);
  if (rows < 256 || nt <= 1) {
    work(0, rows);
  } else {
    std::vector<std::thread> ts;
    const uint64_t per = (rows + nt - 1) / nt;
    for (uint64_t t = 0; t < nt; t++) {
      const uint64_t a = t * per, b = std::min(rows, a + per);
      if (a < b) ts.emplace_back(work, a, b);
    }
    for (auto& t : ts) t.join();
  }
  return RF_OK;
}

}  // namespace rf

namespace rf {

// Tensors sorted by (file offset, index); each joins the current read when the
// gap to it is at most kMaxCoalescedGap and the grown span at most
// kMaxCoalescedSpan, else it starts a new read (layer_read.rs:50-132).
int build_read_plan(const rf_tensor_extent* t, uint32_t n, ReadPlan* out) {
  *out = ReadPlan{};
  std::vector<uint32_t> order(n);
  uint64_t logical = 0;
  for (uint32_t i = 0; i < n; i++) {
    order[i] = i;
    if (t[i].file_offset + t[i].byte_length < t[i].file_offset)
      return set_error(RF_EINVAL, "tensor %u file range overflows", i);
    if (logical + t[i].byte_length < logical) return set_error(RF_EINVAL, "layer logical byte count overflows");
    logical += t[i].byte_length;
  }
  std::sort(order.begin(), order.end(), [&](uint32_t a, uint32_t b) {
    return t[a].file_offset != t[b].file_offset ? t[a].file_offset < t[b].file_offset : a < b;
  });
  for (uint32_t idx : order) {
    const uint64_t start = t[idx].file_offset, end = start + t[idx].byte_length;
    if (!out->ranges.empty()) {
      rf_read_range& cur = out->ranges.back();
      const uint64_t cur_end = cur.file_offset + cur.byte_length;
      if (start < cur_end) return set_error(RF_EINVAL, "tensor ranges overlap at index %u", idx);
      const uint64_t gap = start - cur_end, span = end - cur.file_offset;
      if (gap <= kMaxCoalescedGap && span <= kMaxCoalescedSpan) {
        out->placed.push_back({idx, (uint32_t)(out->ranges.size() - 1), start - cur.file_offset});
        cur.byte_length = span;
        cur.logical_bytes += t[idx].byte_length;
        cur.gap_bytes += gap;
        cur.count++;
        continue;
      }
    }
    out->ranges.push_back({start, t[idx].byte_length, t[idx].byte_length, 0, (uint32_t)out->placed.size(), 1});
    out->placed.push_back({idx, (uint32_t)(out->ranges.size() - 1), 0});
  }
  rf_read_plan_totals& tot = out->totals;
  tot.logical_tensor_count = n;
  tot.logical_bytes = logical;
  bool grouped = out->ranges.size() > 1;
  uint64_t max_span = 0;
  for (const rf_read_range& r : out->ranges) {
    tot.physical_bytes += r.byte_length;
    tot.gap_bytes += r.gap_bytes;
    grouped = grouped && r.count > 1;
    max_span = std::max(max_span, r.byte_length);
  }
  tot.reusable_group_buffer_bytes = grouped ? max_span : 0;
  return RF_OK;
}

}  // namespace rf

extern "C" int rf_should_keep_resident(uint64_t resident_bytes, uint64_t budget_total) {
  return resident_bytes <= budget_total / 4 ? 1 : 0;
}

extern "C" int rf_layer_read_plan(const rf_tensor_extent* tensors, uint32_t n, rf_read_range* ranges,
                                  uint32_t range_cap, uint32_t* n_ranges, rf_planned_tensor* placed,
                                  rf_read_plan_totals* totals) {
  if ((n && !tensors) || !n_ranges) return rf::set_error(RF_EINVAL, "null argument");
  rf::ReadPlan plan;
  RF_TRY(rf::build_read_plan(tensors, n, &plan));
  *n_ranges = (uint32_t)plan.ranges.size();
  if (plan.ranges.size() > range_cap || (plan.ranges.size() && !ranges))
    return rf::set_error(RF_ENOMEM, "the plan has %zu reads, room for %u", plan.ranges.size(), range_cap);
  std::copy(plan.ranges.begin(), plan.ranges.end(), ranges);
  if (placed) std::copy(plan.placed.begin(), plan.placed.end(), placed);
  if (totals) *totals = plan.totals;
  return RF_OK;
}
