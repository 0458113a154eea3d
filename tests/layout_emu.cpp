// layout_emu.cpp - test infrastructure: the tiled Q6_K / Q5_K / Q3_K / Q2_K layouts
// and the quantized GEMV's decode, emulated on the CPU.
//
// The packing helpers are the engine's own (rf_kernels.cuh, shared by its host and
// device packers).  The emulation then reads the packed bytes with the addressing the
// GEMV kernel uses (item, piece and header-plane offsets computed directly, not through
// qs_byte_off / sc_byte_off), decodes each quant field with the masked-in-place float
// trick, and applies the per-group scale arithmetic of rf_gemv.cuh, so a change to
// either side that breaks their agreement shows up here without a GPU.
// Built by tests/test_packed_layout.py; the oracle is the checker.
#include <cmath>
#include <cstdint>
#include <cstring>
#include <vector>

#include "rf_kernels.cuh"

using namespace rf;

namespace {
float asf(uint32_t b) {
  float f;
  memcpy(&f, &b, 4);
  return f;
}
// f16 as the reference reads block scales: IEEE, a subnormal half at half its value
float ref_h2f(uint32_t h) {
  const uint32_t e = (h >> 10) & 31, m = h & 1023;
  float v = e == 0 ? std::ldexp((float)m, -25) : std::ldexp((float)(m | 1024), (int)e - 25);
  return (h & 0x8000) ? -v : v;
}
float prescale(int off) { return asf((uint32_t)(212 - off) << 23); }  // 2^(85-off)
int pair_off(int k) { return (k & 3) == 3 ? (k >> 2) * 8 : (k & 3) * 8; }
const float kTwo64 = 18446744073709551616.0f;
}  // namespace

extern "C" int emu_gemv(int type, const uint8_t* raw, uint32_t M, uint32_t K, const float* x, float* y) {
  if (!six_bit_fields(type) && !nibble_group_fields(type)) return -1;
  const uint32_t bsz = block_bytes(type), nblk = K / 256;
  PackedMat W{};
  W.type = type;
  W.M = M;
  W.K = W.Kp = K;
  W.Mp = (M + QT_ROWS - 1) / QT_ROWS * QT_ROWS;
  W.nk = K / chunk_elems(type);
  W.sbytes = chunk_scale_bytes(type);
  W.qs_stride = (uint64_t)W.nk * chunk_quant_bytes(type);
  W.sc_stride = (uint64_t)W.nk * W.sbytes;
  std::vector<uint8_t> Q((size_t)W.Mp * W.qs_stride, 0), C((size_t)W.Mp * W.sc_stride, 0);
  for (uint32_t r = 0; r < M; r++)
    for (uint32_t k = 0; k < nblk; k++) {
      const uint8_t* s = raw + ((uint64_t)r * nblk + k) * bsz;
      if (six_bit_fields(type)) six_bit_pack_block(W, Q.data(), C.data(), r, k, s);
      else nibble_group_pack_block(W, Q.data(), C.data(), r, k, s);
    }
  const uint32_t SB = W.sbytes, A = SB - 4, CE = chunk_elems(type);
  for (uint32_t r = 0; r < M; r++) {
    double acc = 0;
    const uint32_t lr = r % QT_ROWS;
    for (uint32_t ch = 0; ch < W.nk; ch++) {
      const uint64_t item = (uint64_t)(r / QT_ROWS) * W.nk + ch;
      const uint8_t* hs = C.data() + item * QT_ROWS * SB;  // header planes of the item
      uint32_t h[5] = {0, 0, 0, 0, 0};
      memcpy(h, hs + lr * A, A);
      memcpy(&h[A / 4], hs + QT_ROWS * A + lr * 4, 4);
      const uint32_t dw = h[A / 4];
      const float* xc = x + (uint64_t)ch * CE;
      float aS = 0.f, aM = 0.f;
      if (six_bit_fields(type)) {  // pieces: 16-byte plane then 8-byte plane of the 64 rows
        for (int c = 0; c < 4; c++) {
          const uint8_t* q = Q.data() + item * QT_ROWS * Q6_CHUNK_BYTES + (uint64_t)c * QT_ROWS * Q6_PIECE_BYTES;
          uint32_t w[6];
          memcpy(w, q + lr * 16, 16);
          memcpy(w + 4, q + QT_ROWS * 16 + lr * 8, 8);
          float S[2] = {0.f, 0.f}, X[2] = {0.f, 0.f};
          for (int b = 0; b < 2; b++) {
            const uint32_t a0 = w[3 * b], a1 = w[3 * b + 1], a2 = w[3 * b + 2];
            const uint32_t P = (a0 >> 24) | ((a1 >> 24) << 8) | ((a2 >> 24) << 16);
            const uint32_t src[4] = {a0, a1, a2, P};
            for (int t = 0; t < 16; t++) {
              const int off = 6 * (t & 3);
              const float xv = xc[32 * c + 16 * b + t];
              S[b] = std::fma(asf(src[t / 4] & (63u << off)), xv * prescale(off), S[b]);
              X[b] += xv;
            }
          }
          if (type == T_Q6_K) {  // two 16-element sub-blocks, int8 scales, value d*sc*(u-32)
            for (int b = 0; b < 2; b++) {
              const int j = 2 * c + b;
              const float sc = (float)(int8_t)(h[j >> 2] >> (8 * (j & 3)));
              aS = std::fma(sc, S[b], aS);
              aM = std::fma(sc, 32.f * X[b], aM);
            }
          } else {  // Q5_K: one 32-element sub-block, value d*sc*u - dmin*m
            aS = std::fma((float)((h[0] >> (8 * c)) & 255), S[0] + S[1], aS);
            aM = std::fma((float)((h[1] >> (8 * c)) & 255), X[0] + X[1], aM);
          }
        }
        const float d = ref_h2f(dw & 0xFFFF), dm = type == T_Q6_K ? d : ref_h2f(dw >> 16);
        acc += (double)(d * kTwo64 * aS) - (double)(dm * aM);
      } else {  // Q3_K / Q2_K: the Q4 pieces, one 16-element group per word pair
        for (int c = 0; c < 4; c++) {
          const uint8_t* q = Q.data() + item * QT_ITEM_BYTES + (uint64_t)c * QT_ROWS * 32 + lr * 32;
          uint32_t w[8];
          memcpy(w, q, 32);
          for (int p = 0; p < 4; p++) {
            const int G = 4 * c + p;
            const uint32_t a0 = w[2 * p], a1 = w[2 * p + 1];
            const uint32_t P = (a0 >> 24) | ((a1 >> 24) << 8);
            float S = 0.f, X = 0.f;
            for (int t = 0; t < 16; t++) {
              const int k = t & 7, off = pair_off(k) + (t >= 8 ? 4 : 0);
              const uint32_t word = (k & 3) == 3 ? P : (k < 4 ? a0 : a1);
              const float xv = xc[16 * G + t];
              S = std::fma(asf(word & (0xFu << off)), xv * prescale(off), S);
              X += xv;
            }
            const uint32_t sb = (h[G >> 2] >> (8 * (G & 3))) & 255;
            if (type == T_Q3_K) {
              aS = std::fma((float)(int8_t)sb, S, aS);
              aM = std::fma((float)(int8_t)sb, 4.f * X, aM);
            } else {
              aS = std::fma((float)(sb & 15), S, aS);
              aM = std::fma((float)(sb >> 4), X, aM);
            }
          }
        }
        const float d = ref_h2f(dw & 0xFFFF), dm = type == T_Q3_K ? d : ref_h2f(dw >> 16);
        acc += (double)(d * kTwo64 * aS) - (double)(dm * aM);
      }
    }
    y[r] = (float)acc;
  }
  return 0;
}
