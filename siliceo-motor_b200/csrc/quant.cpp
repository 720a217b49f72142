// Block quantizers for the GGUF types of a Q4_K_M file (Q4_K, Q6_K and the
// Q5_0 / Q8_0 fallbacks for rows that are not a multiple of 256).
//
// The reference has no quantizer for these types, only dequantizers
// (crates/s-gguf/src/dequant.rs:66-206); these encoders write the block
// layouts those dequantizers read. Scale search is a plain min/max fit per
// sub-block: any valid encoding is acceptable, because the oracle and the
// engine dequantize the same bytes.
#include <algorithm>
#include <cmath>
#include <cstdint>
#include <cstring>

#include "common.hpp"

namespace sm {

static inline void wr16(uint8_t* p, uint16_t v) { p[0] = (uint8_t)v; p[1] = (uint8_t)(v >> 8); }
static inline int iround(float x) { return (int)lrintf(x); }

// Q4_K: [d fp16][dmin fp16][scales 12][qs 128]; x = d*sc*q - dmin*m, q in 0..15.
void quantize_q4_k_block(const float* x, uint8_t* out) {
  float scale[8], minv[8];
  for (int j = 0; j < 8; j++) {
    float mn = x[32 * j], mx = x[32 * j];
    for (int l = 1; l < 32; l++) { mn = std::min(mn, x[32 * j + l]); mx = std::max(mx, x[32 * j + l]); }
    if (mn > 0.f) mn = 0.f;
    scale[j] = (mx - mn) / 15.f;
    minv[j] = -mn;
  }
  float ms = 0.f, mm = 0.f;
  for (int j = 0; j < 8; j++) { ms = std::max(ms, scale[j]); mm = std::max(mm, minv[j]); }
  uint16_t dh = f32_to_fp16(ms / 63.f), mh = f32_to_fp16(mm / 63.f);
  float d = fp16_to_f32_ref(dh), dmin = fp16_to_f32_ref(mh);
  uint8_t sc[8], m[8];
  for (int j = 0; j < 8; j++) {
    sc[j] = (uint8_t)std::clamp(d > 0.f ? iround(scale[j] / d) : 0, 0, 63);
    m[j] = (uint8_t)std::clamp(dmin > 0.f ? iround(minv[j] / dmin) : 0, 0, 63);
  }
  wr16(out, dh);
  wr16(out + 2, mh);
  uint8_t* s = out + 4;
  for (int i = 0; i < 4; i++) {
    s[i] = (uint8_t)((sc[i] & 63) | ((sc[i + 4] >> 4) << 6));
    s[i + 4] = (uint8_t)((m[i] & 63) | ((m[i + 4] >> 4) << 6));
    s[i + 8] = (uint8_t)((sc[i + 4] & 0xF) | ((m[i + 4] & 0xF) << 4));
  }
  uint8_t q[256];
  for (int j = 0; j < 8; j++) {
    float dj = d * (float)sc[j], mj = dmin * (float)m[j];
    for (int l = 0; l < 32; l++) {
      int v = dj > 0.f ? iround((x[32 * j + l] + mj) / dj) : 0;
      q[32 * j + l] = (uint8_t)std::clamp(v, 0, 15);
    }
  }
  uint8_t* qs = out + 16;
  for (int g = 0; g < 4; g++)
    for (int l = 0; l < 32; l++) qs[32 * g + l] = (uint8_t)(q[64 * g + l] | (q[64 * g + 32 + l] << 4));
}

// Q6_K: [ql 128][qh 64][scales 16 x i8][d fp16]; x = d*sc*(q-32), q in 0..63.
void quantize_q6_k_block(const float* x, uint8_t* out) {
  float scale[16];
  float amax_s = 0.f, smax = 0.f;
  for (int j = 0; j < 16; j++) {
    float am = 0.f, xm = 0.f;
    for (int l = 0; l < 16; l++) {
      float v = x[16 * j + l];
      if (std::fabs(v) > am) { am = std::fabs(v); xm = v; }
    }
    scale[j] = -xm / 32.f;  // the largest-magnitude value maps to q-32 = -32
    if (std::fabs(scale[j]) > amax_s) { amax_s = std::fabs(scale[j]); smax = scale[j]; }
  }
  (void)smax;
  uint16_t dh = f32_to_fp16(amax_s / 127.f);
  float d = fp16_to_f32_ref(dh);
  int8_t sc[16];
  for (int j = 0; j < 16; j++) sc[j] = (int8_t)std::clamp(d > 0.f ? iround(scale[j] / d) : 0, -127, 127);
  uint8_t q[256];
  for (int j = 0; j < 16; j++) {
    float dj = d * (float)sc[j];
    for (int l = 0; l < 16; l++) {
      int v = dj != 0.f ? iround(x[16 * j + l] / dj) : 0;
      q[16 * j + l] = (uint8_t)(std::clamp(v, -32, 31) + 32);
    }
  }
  uint8_t* ql = out;
  uint8_t* qh = out + 128;
  for (int n = 0; n < 2; n++)
    for (int l = 0; l < 32; l++) {
      uint8_t q1 = q[n * 128 + l], q2 = q[n * 128 + l + 32], q3 = q[n * 128 + l + 64], q4 = q[n * 128 + l + 96];
      ql[n * 64 + l] = (uint8_t)((q1 & 0xF) | ((q3 & 0xF) << 4));
      ql[n * 64 + l + 32] = (uint8_t)((q2 & 0xF) | ((q4 & 0xF) << 4));
      qh[n * 32 + l] = (uint8_t)((q1 >> 4) | ((q2 >> 4) << 2) | ((q3 >> 4) << 4) | ((q4 >> 4) << 6));
    }
  std::memcpy(out + 192, sc, 16);
  wr16(out + 208, dh);
}

// Q5_0: [d fp16][qh u32][qs 16]; x = d*(q-16), q in 0..31.
void quantize_q5_0_block(const float* x, uint8_t* out) {
  float am = 0.f, xm = 0.f;
  for (int l = 0; l < 32; l++)
    if (std::fabs(x[l]) > am) { am = std::fabs(x[l]); xm = x[l]; }
  uint16_t dh = f32_to_fp16(xm / -16.f);
  float d = fp16_to_f32_ref(dh);
  uint8_t q[32];
  for (int l = 0; l < 32; l++) q[l] = (uint8_t)std::clamp(d != 0.f ? iround(x[l] / d) + 16 : 16, 0, 31);
  uint32_t qh = 0;
  for (int l = 0; l < 16; l++) {
    out[6 + l] = (uint8_t)((q[l] & 0xF) | ((q[l + 16] & 0xF) << 4));
    qh |= (uint32_t)(q[l] >> 4) << l;
    qh |= (uint32_t)(q[l + 16] >> 4) << (l + 16);
  }
  wr16(out, dh);
  std::memcpy(out + 2, &qh, 4);
}

// Q8_0: [d fp16][qs 32 x i8]; x = q*d.
void quantize_q8_0_block(const float* x, uint8_t* out) {
  float am = 0.f;
  for (int l = 0; l < 32; l++) am = std::max(am, std::fabs(x[l]));
  uint16_t dh = f32_to_fp16(am / 127.f);
  float d = fp16_to_f32_ref(dh);
  wr16(out, dh);
  for (int l = 0; l < 32; l++) out[2 + l] = (uint8_t)(int8_t)std::clamp(d > 0.f ? iround(x[l] / d) : 0, -127, 127);
}

// Quantizes n elements (a multiple of the block size) of type t into out.
bool quantize_row(uint32_t t, const float* x, uint64_t n, uint8_t* out) {
  switch (t) {
    case QT_F32: std::memcpy(out, x, n * 4); return true;
    case QT_Q4K: for (uint64_t b = 0; b < n / 256; b++) quantize_q4_k_block(x + 256 * b, out + 144 * b); return n % 256 == 0;
    case QT_Q6K: for (uint64_t b = 0; b < n / 256; b++) quantize_q6_k_block(x + 256 * b, out + 210 * b); return n % 256 == 0;
    case QT_Q5_0: for (uint64_t b = 0; b < n / 32; b++) quantize_q5_0_block(x + 32 * b, out + 22 * b); return n % 32 == 0;
    case QT_Q8_0: for (uint64_t b = 0; b < n / 32; b++) quantize_q8_0_block(x + 32 * b, out + 34 * b); return n % 32 == 0;
    default: return false;
  }
}

}  // namespace sm
