// rfsynth.cpp - seeded synthetic Llama GGUF models and GGUF block encoders.
//
// The reference ships no quantiser or GGUF writer: its tests assemble GGUFs
// byte by byte (crates/ramforge-runtime/src/inference.rs:782-995).  This file
// is the build's own writer for the benchmark configurations:
//   * GGUF v3 layout as parse_gguf_file reads it (crates/ramforge-core/src/gguf.rs:196-330):
//     header, metadata KV, tensor infos, data section aligned to 32 bytes,
//     every tensor offset aligned to 32 relative to the data start;
//   * Q8_0 / Q4_0 / Q4_K / Q6_K encoders written from the block layouts the
//     decoders read (crates/ramforge-core/src/quant.rs:84-255, 376-406).  Encoder quality does
//     not matter for parity: the engine and the checker read the same bytes.
// Weights are N(0, std) from a counter-based generator (splitmix64 + Box-Muller
// in double precision), so any row of any tensor can be produced independently
// and generation parallelises over rows.
#include <algorithm>
#include <cmath>
#include <cstdint>
#include <cstring>
#include <string>
#include <thread>
#include <vector>

#include "rfsynth.h"

namespace {

inline uint64_t splitmix64(uint64_t x) {
  x += 0x9E3779B97F4A7C15ull;
  x = (x ^ (x >> 30)) * 0xBF58476D1CE4E5B9ull;
  x = (x ^ (x >> 27)) * 0x94D049BB133111EBull;
  return x ^ (x >> 31);
}

// Normal pair for counter p of stream key: Marsaglia's polar method, where the
// k-th attempt of pair p draws its two uniforms from hash(key, p, k), so every
// pair is still addressable independently of the others.
inline void normal_pair(uint64_t key, uint64_t p, double* z0, double* z1) {
  for (uint64_t k = 0;; k++) {
    const uint64_t h = splitmix64(key ^ (p * 0xD1B54A32D192ED03ull) ^ (k * 0xA0761D6478BD642Full));
    const double u = (double)(int64_t)(h & 0xFFFFFFFFull) * (1.0 / 2147483648.0) - 1.0;
    const double v = (double)(int64_t)(h >> 32) * (1.0 / 2147483648.0) - 1.0;
    const double s = u * u + v * v;
    if (s > 0.0 && s < 1.0) {
      const double f = std::sqrt(-2.0 * std::log(s) / s);
      *z0 = u * f;
      *z1 = v * f;
      return;
    }
  }
}

inline uint64_t stream_key(uint64_t seed, uint64_t stream) {
  return splitmix64(splitmix64(seed) ^ (stream * 0x9E3779B97F4A7C15ull + 0x632BE59BD9B4E019ull));
}

uint16_t f32_to_f16(float f) {
  uint32_t x;
  std::memcpy(&x, &f, 4);
  uint32_t sign = (x >> 16) & 0x8000u, ax = x & 0x7FFFFFFFu;
  if (ax >= 0x7F800000u) return (uint16_t)(sign | 0x7C00u | (ax > 0x7F800000u ? 0x200u : 0u));
  if (ax >= 0x477FF000u) return (uint16_t)(sign | 0x7C00u);
  if (ax < 0x38800000u) {
    if (ax < 0x33000000u) return (uint16_t)sign;
    uint32_t e = ax >> 23, m = (ax & 0x7FFFFFu) | 0x800000u, sh = 126u - e;
    uint32_t q = m >> sh, rem = m & ((1u << sh) - 1u), half = 1u << (sh - 1u);
    if (rem > half || (rem == half && (q & 1u))) q++;
    return (uint16_t)(sign | q);
  }
  uint32_t e = (ax >> 23) - 112u, m = ax & 0x7FFFFFu;
  uint32_t q = (e << 10) | (m >> 13), rem = m & 0x1FFFu;
  if (rem > 0x1000u || (rem == 0x1000u && (q & 1u))) q++;
  return (uint16_t)(sign | q);
}

float f16_to_f32(uint16_t h) {
  uint32_t sign = (uint32_t)(h & 0x8000u) << 16, e = (h >> 10) & 0x1Fu, m = h & 0x3FFu, o;
  if (e == 0) {
    if (m == 0) o = sign;
    else {
      int s = 0;
      while (!(m & 0x400u)) { m <<= 1; s++; }
      o = sign | ((uint32_t)(113 - s) << 23) | ((m & 0x3FFu) << 13);
    }
  } else if (e == 31) o = sign | 0x7F800000u | (m << 13);
  else o = sign | ((e + 112u) << 23) | (m << 13);
  float f;
  std::memcpy(&f, &o, 4);
  return f;
}

inline void put16(uint8_t* p, uint16_t v) { p[0] = (uint8_t)v; p[1] = (uint8_t)(v >> 8); }

// Q8_0: d = amax/127 (stored f16), q = round(x/d).
void enc_q8_0(const float* x, uint8_t* b) {
  float amax = 0.f;
  for (int i = 0; i < 32; i++) amax = std::max(amax, std::fabs(x[i]));
  uint16_t dh = f32_to_f16(amax / 127.f);
  float d = f16_to_f32(dh);
  put16(b, dh);
  const float id = d > 0.f ? 1.0f / d : 0.f;
  for (int i = 0; i < 32; i++) {
    int q = (int)std::lrintf(x[i] * id);
    q = std::min(127, std::max(-127, q));
    b[2 + i] = (uint8_t)(int8_t)q;
  }
}

// Q4_0: d = amax/7 (stored f16), nibble = round(x/d) + 8; byte j = lo(elem j) | hi(elem 16+j).
void enc_q4_0(const float* x, uint8_t* b) {
  float amax = 0.f;
  for (int i = 0; i < 32; i++) amax = std::max(amax, std::fabs(x[i]));
  uint16_t dh = f32_to_f16(amax / 7.f);
  float d = f16_to_f32(dh);
  put16(b, dh);
  const float id = d > 0.f ? 1.0f / d : 0.f;
  auto qz = [&](float v) {
    int q = (int)std::lrintf(v * id) + 8;
    return std::min(15, std::max(0, q));
  };
  for (int j = 0; j < 16; j++) b[2 + j] = (uint8_t)(qz(x[j]) | (qz(x[16 + j]) << 4));
}

// Q4_K: per 32-element sub-block an affine range [lo, hi] with lo <= 0; sub-block
// scale (hi-lo)/15 and min -lo are quantised to 6 bits against f16 super-scales
// d = max scale/63, dmin = max min/63, packed as get_scale_min reads them
// (quant.rs:216-226): s[k] = sc_k | (sc_{k+4}>>4)<<6, s[k+4] = m_k | (m_{k+4}>>4)<<6,
// s[k+8] = (sc_{k+4} & 15) | (m_{k+4} & 15)<<4.
void enc_q4_k(const float* x, uint8_t* b) {
  float scale[8], mn[8];
  for (int j = 0; j < 8; j++) {
    float lo = 0.f, hi = 0.f;
    for (int l = 0; l < 32; l++) { lo = std::min(lo, x[32 * j + l]); hi = std::max(hi, x[32 * j + l]); }
    scale[j] = (hi - lo) / 15.f;
    mn[j] = -lo;
  }
  float ms = *std::max_element(scale, scale + 8), mm = *std::max_element(mn, mn + 8);
  uint16_t dh = f32_to_f16(ms / 63.f), mh = f32_to_f16(mm / 63.f);
  float d = f16_to_f32(dh), dmin = f16_to_f32(mh);
  put16(b, dh);
  put16(b + 2, mh);
  uint8_t sc[8], m[8];
  for (int j = 0; j < 8; j++) {
    int s = d > 0.f ? (int)std::lrint(scale[j] / d) : 0;
    int t = dmin > 0.f ? (int)std::lrint(mn[j] / dmin) : 0;
    sc[j] = (uint8_t)std::min(63, std::max(0, s));
    m[j] = (uint8_t)std::min(63, std::max(0, t));
  }
  uint8_t* s = b + 4;
  for (int k = 0; k < 4; k++) {
    s[k] = (uint8_t)((sc[k] & 63) | ((sc[k + 4] >> 4) << 6));
    s[k + 4] = (uint8_t)((m[k] & 63) | ((m[k + 4] >> 4) << 6));
    s[k + 8] = (uint8_t)((sc[k + 4] & 15) | ((m[k + 4] & 15) << 4));
  }
  uint8_t q[256];
  for (int j = 0; j < 8; j++) {
    const float S = d * (float)sc[j], M = dmin * (float)m[j], iS = S > 0.f ? 1.0f / S : 0.f;
    for (int l = 0; l < 32; l++) {
      int v = (int)std::lrintf((x[32 * j + l] + M) * iS);
      q[32 * j + l] = (uint8_t)std::min(15, std::max(0, v));
    }
  }
  uint8_t* qs = b + 16;
  for (int g = 0; g < 4; g++)
    for (int l = 0; l < 32; l++) qs[32 * g + l] = (uint8_t)(q[64 * g + l] | (q[64 * g + 32 + l] << 4));
}

// Q6_K: per 16-element sub-block a symmetric scale amax/31, quantised to int8
// against the f16 super-scale d = max scale/127; value (d*sc)*q with q in
// [-32, 31] stored as q+32.  Bytes as BlockQ6K::dequantize reads them
// (quant.rs:376-406): for half h and l < 32, element 128h+l+32k takes the
// low (k < 2) or high nibble of ql[64h + l + 32(k&1)] and bits 2k..2k+1 of
// qh[32h + l]; sub-block j of the super-block uses scales[j]; d at byte 208.
void enc_q6_k(const float* x, uint8_t* b) {
  float scale[16];
  for (int j = 0; j < 16; j++) {
    float amax = 0.f;
    for (int l = 0; l < 16; l++) amax = std::max(amax, std::fabs(x[16 * j + l]));
    scale[j] = amax / 31.f;
  }
  const float ms = *std::max_element(scale, scale + 16);
  const uint16_t dh = f32_to_f16(ms / 127.f);
  const float d = f16_to_f32(dh);
  int8_t sc[16];
  for (int j = 0; j < 16; j++) {
    const int s = d > 0.f ? (int)std::lrint(scale[j] / d) : 0;
    sc[j] = (int8_t)std::min(127, std::max(-128, s));
  }
  uint8_t u[256];
  for (int j = 0; j < 16; j++) {
    const float S = d * (float)sc[j], iS = S != 0.f ? 1.0f / S : 0.f;
    for (int l = 0; l < 16; l++) {
      const int q = (int)std::lrintf(x[16 * j + l] * iS);
      u[16 * j + l] = (uint8_t)(std::min(31, std::max(-32, q)) + 32);
    }
  }
  uint8_t* ql = b;
  uint8_t* qh = b + 128;
  for (int h = 0; h < 2; h++)
    for (int l = 0; l < 32; l++) {
      const uint8_t* v = u + 128 * h + l;  // v[32k]: element 128h + l + 32k
      ql[64 * h + l] = (uint8_t)((v[0] & 15) | ((v[64] & 15) << 4));
      ql[64 * h + 32 + l] = (uint8_t)((v[32] & 15) | ((v[96] & 15) << 4));
      qh[32 * h + l] = (uint8_t)((v[0] >> 4) | ((v[32] >> 4) << 2) | ((v[64] >> 4) << 4) | ((v[96] >> 4) << 6));
    }
  for (int j = 0; j < 16; j++) b[192 + j] = (uint8_t)sc[j];
  put16(b + 208, dh);
}

size_t block_elems(int type) {
  switch (type) {
    case RFS_F32: case RFS_F16: return 1;
    case RFS_Q4_0: case RFS_Q8_0: return 32;
    case RFS_Q4_K: case RFS_Q6_K: return 256;
    default: return 0;
  }
}
size_t block_bytes(int type) {
  switch (type) {
    case RFS_F32: return 4;
    case RFS_F16: return 2;
    case RFS_Q4_0: return 18;
    case RFS_Q8_0: return 34;
    case RFS_Q4_K: return 144;
    case RFS_Q6_K: return 210;
    default: return 0;
  }
}

void encode_row(int type, const float* x, size_t n, uint8_t* out) {
  size_t qk = block_elems(type), bs = block_bytes(type);
  for (size_t i = 0; i < n / qk; i++) {
    const float* xb = x + i * qk;
    uint8_t* ob = out + i * bs;
    switch (type) {
      case RFS_F32: std::memcpy(ob, xb, 4); break;
      case RFS_F16: put16(ob, f32_to_f16(xb[0])); break;
      case RFS_Q4_0: enc_q4_0(xb, ob); break;
      case RFS_Q8_0: enc_q8_0(xb, ob); break;
      case RFS_Q4_K: enc_q4_k(xb, ob); break;
      case RFS_Q6_K: enc_q6_k(xb, ob); break;
    }
  }
}

template <class F>
void parallel_rows(size_t rows, int threads, F&& fn) {
  if (threads <= 1 || rows < 64) { fn(0, rows); return; }
  std::vector<std::thread> ts;
  size_t per = (rows + threads - 1) / threads;
  for (int t = 0; t < threads; t++) {
    size_t a = t * per, b = std::min(rows, a + per);
    if (a >= b) break;
    ts.emplace_back([&, a, b] { fn(a, b); });
  }
  for (auto& t : ts) t.join();
}

struct TensorPlan {
  std::string name;
  uint64_t ne0, ne1;  // ne0 = row length (in), ne1 = rows (out); ne1 == 1 for 1-D
  int ndims, type;
  bool ones;          // norm weights: constant 1.0
  uint64_t offset, bytes, stream;
  float stddev;       // 0: the spec's weight_std
};

std::vector<TensorPlan> plan_llama(const rfs_llama_spec* s) {
  std::vector<TensorPlan> t;
  uint64_t hd = s->n_embd / s->n_heads, qd = hd * s->n_heads, kvd = hd * s->n_kv_heads;
  uint64_t stream = 0;
  auto add = [&](const std::string& n, uint64_t ne0, uint64_t ne1, int nd, int ty, bool ones, float sd = 0.f) {
    t.push_back({n, ne0, ne1, nd, ty, ones, 0, 0, stream++, sd});
  };
  const int vt = s->v_type >= 0 ? s->v_type : s->layer_type, dt = s->down_type >= 0 ? s->down_type : s->layer_type;
  add("token_embd.weight", s->n_embd, s->vocab_size, 2, s->embd_type, false);
  for (uint32_t l = 0; l < s->n_layers; l++) {
    std::string p = "blk." + std::to_string(l) + ".";
    add(p + "attn_norm.weight", s->n_embd, 1, 1, RFS_F32, true);
    add(p + "attn_q.weight", s->n_embd, qd, 2, s->layer_type, false);
    add(p + "attn_k.weight", s->n_embd, kvd, 2, s->layer_type, false);
    add(p + "attn_v.weight", s->n_embd, kvd, 2, vt, false);
    if (s->qkv_bias_std > 0.f) {
      add(p + "attn_q.bias", qd, 1, 1, RFS_F32, false, s->qkv_bias_std);
      add(p + "attn_k.bias", kvd, 1, 1, RFS_F32, false, s->qkv_bias_std);
      add(p + "attn_v.bias", kvd, 1, 1, RFS_F32, false, s->qkv_bias_std);
    }
    add(p + "attn_output.weight", qd, s->n_embd, 2, s->layer_type, false);
    add(p + "ffn_norm.weight", s->n_embd, 1, 1, RFS_F32, true);
    add(p + "ffn_gate.weight", s->n_embd, s->n_ff, 2, s->layer_type, false);
    add(p + "ffn_up.weight", s->n_embd, s->n_ff, 2, s->layer_type, false);
    add(p + "ffn_down.weight", s->n_ff, s->n_embd, 2, dt, false);
  }
  add("output_norm.weight", s->n_embd, 1, 1, RFS_F32, true);
  if (s->out_type >= 0) add("output.weight", s->n_embd, s->vocab_size, 2, s->out_type, false);
  return t;
}

struct Writer {
  std::vector<uint8_t> b;
  void u32(uint32_t v) { uint8_t x[4]; std::memcpy(x, &v, 4); b.insert(b.end(), x, x + 4); }
  void u64(uint64_t v) { uint8_t x[8]; std::memcpy(x, &v, 8); b.insert(b.end(), x, x + 8); }
  void f32(float v) { uint8_t x[4]; std::memcpy(x, &v, 4); b.insert(b.end(), x, x + 4); }
  void str(const std::string& s) { u64(s.size()); b.insert(b.end(), s.begin(), s.end()); }
  void kv_u32(const std::string& k, uint32_t v) { str(k); u32(4); u32(v); }
  void kv_f32(const std::string& k, float v) { str(k); u32(6); f32(v); }
  void kv_str(const std::string& k, const std::string& v) { str(k); u32(8); str(v); }
};

// Header + metadata + tensor infos (data start is this size rounded up to 32).
std::vector<uint8_t> build_header(const rfs_llama_spec* s, std::vector<TensorPlan>& plan, uint64_t* data_bytes) {
  uint64_t off = 0;
  for (auto& t : plan) {
    uint64_t ne = t.ne0 * t.ne1;
    t.bytes = ne / block_elems(t.type) * block_bytes(t.type);
    t.offset = off;
    off += (t.bytes + 31) / 32 * 32;
  }
  *data_bytes = off;
  Writer w;
  w.b.insert(w.b.end(), {'G', 'G', 'U', 'F'});
  w.u32(3);
  w.u64(plan.size());
  std::string a = s->arch ? s->arch : "llama";
  w.u64(11);
  w.kv_str("general.architecture", a);
  w.kv_u32("general.alignment", 32);
  w.kv_u32(a + ".vocab_size", s->vocab_size);
  w.kv_u32(a + ".context_length", s->context_length);
  w.kv_u32(a + ".embedding_length", s->n_embd);
  w.kv_u32(a + ".block_count", s->n_layers);
  w.kv_u32(a + ".feed_forward_length", s->n_ff);
  w.kv_u32(a + ".attention.head_count", s->n_heads);
  w.kv_u32(a + ".attention.head_count_kv", s->n_kv_heads);
  w.kv_f32(a + ".attention.layer_norm_rms_epsilon", s->rms_eps);
  w.kv_f32(a + ".rope.freq_base", s->rope_theta);
  for (auto& t : plan) {
    w.str(t.name);
    w.u32(t.ndims);
    w.u64(t.ne0);
    if (t.ndims == 2) w.u64(t.ne1);
    w.u32(t.type);
    w.u64(t.offset);
  }
  while (w.b.size() % 32) w.b.push_back(0);
  return w.b;
}

bool spec_ok(const rfs_llama_spec* s) {
  if (!s || !s->n_heads || !s->n_kv_heads || s->n_heads % s->n_kv_heads || s->n_embd % s->n_heads) return false;
  uint64_t hd = s->n_embd / s->n_heads;
  if (hd % 2) return false;
  for (int ty : {s->layer_type, s->embd_type}) {
    size_t qk = block_elems(ty);
    if (!qk || s->n_embd % qk || s->n_ff % qk || (hd * s->n_heads) % qk) return false;
  }
  if (s->out_type >= 0 && (!block_elems(s->out_type) || s->n_embd % block_elems(s->out_type))) return false;
  if (s->v_type >= 0 && (!block_elems(s->v_type) || s->n_embd % block_elems(s->v_type))) return false;
  if (s->down_type >= 0 && (!block_elems(s->down_type) || s->n_ff % block_elems(s->down_type))) return false;
  return true;
}

}  // namespace

extern "C" {

void rfs_fill_normal(uint64_t seed, uint64_t stream, float stddev, uint64_t start, float* out, size_t n) {
  const uint64_t key = stream_key(seed, stream);
  const double sd = (double)stddev;
  size_t i = 0;
  double z0, z1;
  if (n && (start & 1)) {  // odd first element: second half of its pair
    normal_pair(key, start >> 1, &z0, &z1);
    out[i++] = (float)(z1 * sd);
  }
  for (; i + 1 < n; i += 2) {
    normal_pair(key, (start + i) >> 1, &z0, &z1);
    out[i] = (float)(z0 * sd);
    out[i + 1] = (float)(z1 * sd);
  }
  if (i < n) {
    normal_pair(key, (start + i) >> 1, &z0, &z1);
    out[i] = (float)(z0 * sd);
  }
}

size_t rfs_row_bytes(int type, size_t n) {
  size_t qk = block_elems(type);
  if (!qk || n % qk) return 0;
  return n / qk * block_bytes(type);
}

int rfs_quantize(int type, const float* x, size_t rows, size_t cols, uint8_t* out, int threads) {
  size_t rb = rfs_row_bytes(type, cols);
  if (!rb) return -1;
  parallel_rows(rows, threads, [&](size_t a, size_t b) {
    for (size_t r = a; r < b; r++) encode_row(type, x + r * cols, cols, out + r * rb);
  });
  return 0;
}

uint64_t rfs_llama_gguf_size(const rfs_llama_spec* s) {
  if (!spec_ok(s)) return 0;
  auto plan = plan_llama(s);
  uint64_t data = 0;
  auto hdr = build_header(s, plan, &data);
  return hdr.size() + data;
}

int rfs_llama_gguf_write(const rfs_llama_spec* s, uint8_t* out, uint64_t cap, int threads) {
  if (!spec_ok(s)) return -1;
  auto plan = plan_llama(s);
  uint64_t data = 0;
  auto hdr = build_header(s, plan, &data);
  if (hdr.size() + data > cap) return -2;
  std::memcpy(out, hdr.data(), hdr.size());
  uint8_t* ds = out + hdr.size();
  std::memset(ds, 0, data);
  for (auto& t : plan) {
    uint8_t* dst = ds + t.offset;
    size_t rb = rfs_row_bytes(t.type, t.ne0);
    uint64_t key_stream = t.stream;
    parallel_rows(t.ne1, threads, [&](size_t a, size_t b) {
      std::vector<float> row(t.ne0);
      for (size_t r = a; r < b; r++) {
        if (t.ones) std::fill(row.begin(), row.end(), 1.0f);
        else rfs_fill_normal(s->seed, key_stream, t.stddev > 0.f ? t.stddev : s->weight_std, (uint64_t)r * t.ne0,
                             row.data(), t.ne0);
        encode_row(t.type, row.data(), t.ne0, dst + r * rb);
      }
    });
  }
  return 0;
}

}  // extern "C"
