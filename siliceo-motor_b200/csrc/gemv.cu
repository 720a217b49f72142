// Dequant-fused GEMV for GGUF Q4_K / Q6_K / Q8_0 / Q5_0 weights, batch 1..32,
// and the bit-exact dequantizer.
//
// Reference semantics: y[s,o] = sum_d W[o,d] * x[s,d] with W the f32 values of
// dequantize() (crates/s-models/src/qwen2.rs:663-674; the reference's fused
// GPU kernels crates/s-backend-cuda/kernels/src/lib.rs:709-876 do the same one
// thread per output). Here a warp owns R rows: its lanes stride over the
// row's 16-byte units with 128-bit streaming loads, and the partial sums are
// combined with warp shuffles. Within a sub-block the scale is factored out
// (sum x*(d*sc*q - dmin*m) = d*sc*sum(q*x) - dmin*m*sum(x)), so the inner
// loop is one exact int->float conversion and one FMA per weight; the result
// differs from the reference's sequential sum by rounding only.
#include <cuda_fp16.h>

#include <mutex>

#include "device.cuh"

namespace sm {

constexpr int GEMV_WARPS = 4;

// ----------------------------------------------------------- dequant ----
__device__ __forceinline__ uint32_t rd16(const uint8_t* p) { return (uint32_t)p[0] | ((uint32_t)p[1] << 8); }

__device__ __forceinline__ void scale_min_k4(int j, const uint8_t* s, uint32_t* d, uint32_t* m) {
  if (j < 4) {  // dequant.rs:41-49
    *d = s[j] & 63;
    *m = s[j + 4] & 63;
  } else {
    *d = (s[j + 4] & 0x0F) | ((s[j - 4] >> 6) << 4);
    *m = (s[j + 4] >> 4) | ((s[j] >> 6) << 4);
  }
}

// Element e of row o, with the reference's f32 operations (no contraction).
__device__ float dequant_elem(const DWDesc& w, uint32_t o, uint32_t e) {
  const uint8_t* row = w.body + (size_t)o * w.body_stride;
  switch (w.type) {
    case 12: {  // Q4_K, dequant.rs:98-124
      const uint32_t blk = e >> 8, l = e & 255, g = l >> 6, within = l & 63, w31 = within & 31;
      const KqPos ps = kq_pos(blk, w.n_in >> 8, q4k_group_bytes(8));
      const uint8_t* h = row + q4k_hdr_off(ps);
      float d = fp16_ref(rd16(h)), dmin = fp16_ref(rd16(h + 2));
      uint32_t is = 2 * g + (within >= 32), sc, m;
      scale_min_k4((int)is, h + 4, &sc, &m);
      uint32_t qb = row[q4k_qs_off(ps, g, w31 >> 4) + (w31 & 15)];
      uint32_t q = within < 32 ? (qb & 0x0F) : (qb >> 4);
      float d1 = __fmul_rn(d, (float)sc), m1 = __fmul_rn(dmin, (float)m);
      return __fsub_rn(__fmul_rn(d1, (float)q), m1);
    }
    case 14: {  // Q6_K, dequant.rs:178-206
      const uint32_t blk = e >> 8, l = e & 255, n = l >> 7, wl = l & 127, k = wl >> 5, ll = wl & 31, is = ll >> 4;
      const KqPos ps = kq_pos(blk, w.n_in >> 8, q6k_group_bytes(8));
      float d = fp16_ref(rd16(row + q6k_d_off(ps)));
      if (!isfinite(d)) return 0.0f;
      uint32_t qlb = row[q6k_q_off(ps, n, is, (k & 1) ? 1 : 0) + (ll & 15)];
      uint32_t nib = (k & 2) ? (qlb >> 4) : (qlb & 0x0F);
      uint32_t hb = (row[q6k_q_off(ps, n, is, 2) + (ll & 15)] >> (2 * k)) & 3;
      int32_t q = (int32_t)(nib | (hb << 4)) - 32;
      float sc = (float)(int8_t)row[q6k_sc_off(ps) + n * 8 + is + 2 * k];
      return __fmul_rn(__fmul_rn(d, sc), (float)q);
    }
    case 8: {  // Q8_0, dequant.rs:66-71
      uint32_t blk = e >> 5, l = e & 31;
      float d = fp16_ref(rd16(w.aux + (size_t)o * w.aux_stride + blk * 2));
      return __fmul_rn((float)(int8_t)row[blk * 32 + l], d);
    }
    case 6: {  // Q5_0, dequant.rs:79-94
      uint32_t blk = e >> 5, l = e & 31;
      const uint8_t* a = w.aux + (size_t)o * w.aux_stride + blk * 8;
      uint32_t qh = (uint32_t)a[0] | ((uint32_t)a[1] << 8) | ((uint32_t)a[2] << 16) | ((uint32_t)a[3] << 24);
      float d = fp16_ref(rd16(a + 4));
      uint32_t qb = row[blk * 16 + (l & 15)];
      int32_t q = (int32_t)((l < 16 ? (qb & 0x0F) : (qb >> 4)) | (((qh >> l) & 1u) << 4)) - 16;
      return __fmul_rn(d, (float)q);
    }
    case 0:
      return reinterpret_cast<const float*>(row)[e];
  }
  return 0.0f;
}

__global__ void dequant_kernel(DWDesc w, float* out) {
  size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
  size_t n = (size_t)w.n_out * w.n_in;
  if (i >= n) return;
  uint32_t o = (uint32_t)(i / w.n_in), e = (uint32_t)(i % w.n_in);
  out[i] = dequant_elem(w, o, e);
}

// Embedding lookup (qwen2.rs:468-472): row tok of the table, dequantized exactly.
__global__ void embed_kernel(DWDesc w, const uint32_t* tokens, float* x, uint32_t ldx) {
  uint32_t r = blockIdx.y, tok = tokens[r];
  for (uint32_t e = blockIdx.x * blockDim.x + threadIdx.x; e < w.n_in; e += gridDim.x * blockDim.x)
    x[(size_t)r * ldx + e] = dequant_elem(w, tok, e);
}

// -------------------------------------------------------------- GEMV ----
// Each unit function adds, for R rows and up to BT columns, one lane's share
// of a row: acc[r][b] += sum over the unit's weights of W*x.

// Q4_K unit = 16 bytes of qs (32 weights: 16 of sub-block 2j, 16 of 2j+1)
// plus the block header (d, dmin, 12 scale bytes) read as one 16-byte load.
template <int R, int BT>
__device__ __forceinline__ void unit_q4k(const uint8_t* const* rowp, int u, uint32_t nb, const float* x, uint32_t ldx,
                                         int ncols, float (&acc)[R][BT]) {
  const int blk = u >> 3, p = u & 7, j = p >> 1;
  const KqPos ps = kq_pos((uint32_t)blk, nb, q4k_group_bytes(8));
  const uint32_t ho = q4k_hdr_off(ps), qo = q4k_qs_off(ps, (uint32_t)j, (uint32_t)(p & 1));
  uint4 hd[R], qs[R];
#pragma unroll
  for (int r = 0; r < R; r++) {
    hd[r] = ld_stream(rowp[r] + ho);
    qs[r] = ld_stream(rowp[r] + qo);
  }
  float d1[R], m1[R], d2[R], m2[R];
#pragma unroll
  for (int r = 0; r < R; r++) {
    const float d = fp16_ref(hd[r].x & 0xFFFFu), dmin = fp16_ref(hd[r].x >> 16);
    uint32_t sa, ma, sb, mb;
    if (j < 2) {  // sub-blocks 2j, 2j+1 < 4
      const int s0 = 16 * j;
      sa = (hd[r].y >> s0) & 63u;
      ma = (hd[r].z >> s0) & 63u;
      sb = (hd[r].y >> (s0 + 8)) & 63u;
      mb = (hd[r].z >> (s0 + 8)) & 63u;
    } else {  // sub-blocks 4..7
      const int s0 = 16 * (j - 2);
      const uint32_t a0 = (hd[r].w >> s0) & 0xFFu, a1 = (hd[r].w >> (s0 + 8)) & 0xFFu;
      sa = (a0 & 0xF) | (((hd[r].y >> (s0 + 6)) & 3u) << 4);
      ma = (a0 >> 4) | (((hd[r].z >> (s0 + 6)) & 3u) << 4);
      sb = (a1 & 0xF) | (((hd[r].y >> (s0 + 14)) & 3u) << 4);
      mb = (a1 >> 4) | (((hd[r].z >> (s0 + 14)) & 3u) << 4);
    }
    d1[r] = d * (float)sa;
    m1[r] = dmin * (float)ma;
    d2[r] = d * (float)sb;
    m2[r] = dmin * (float)mb;
  }
  const int base = blk * 256 + 64 * j + 16 * (p & 1);
#pragma unroll
  for (int b = 0; b < BT; b++) {
    if (b >= ncols) break;
    const float* xb = x + (size_t)b * ldx + base;
    float xl[16], xh[16];
#pragma unroll
    for (int i = 0; i < 4; i++) {
      float4 a = ldg4(xb + 4 * i), c = ldg4(xb + 32 + 4 * i);
      xl[4 * i] = a.x; xl[4 * i + 1] = a.y; xl[4 * i + 2] = a.z; xl[4 * i + 3] = a.w;
      xh[4 * i] = c.x; xh[4 * i + 1] = c.y; xh[4 * i + 2] = c.z; xh[4 * i + 3] = c.w;
    }
    float sxl = 0.f, sxh = 0.f;
#pragma unroll
    for (int i = 0; i < 16; i++) { sxl += xl[i]; sxh += xh[i]; }
#pragma unroll
    for (int r = 0; r < R; r++) {
      const uint32_t wv[4] = {qs[r].x, qs[r].y, qs[r].z, qs[r].w};
      float sl0 = 0.f, sl1 = 0.f, sh0 = 0.f, sh1 = 0.f;
#pragma unroll
      for (int i = 0; i < 4; i++) {
        const uint32_t lo = wv[i] & 0x0F0F0F0Fu, hi = (wv[i] >> 4) & 0x0F0F0F0Fu;
        sl0 = fmaf(byte_f<0>(lo, 8388608.f), xl[4 * i + 0], sl0);
        sl1 = fmaf(byte_f<1>(lo, 8388608.f), xl[4 * i + 1], sl1);
        sl0 = fmaf(byte_f<2>(lo, 8388608.f), xl[4 * i + 2], sl0);
        sl1 = fmaf(byte_f<3>(lo, 8388608.f), xl[4 * i + 3], sl1);
        sh0 = fmaf(byte_f<0>(hi, 8388608.f), xh[4 * i + 0], sh0);
        sh1 = fmaf(byte_f<1>(hi, 8388608.f), xh[4 * i + 1], sh1);
        sh0 = fmaf(byte_f<2>(hi, 8388608.f), xh[4 * i + 2], sh0);
        sh1 = fmaf(byte_f<3>(hi, 8388608.f), xh[4 * i + 3], sh1);
      }
      acc[r][b] += (d1[r] * (sl0 + sl1) - m1[r] * sxl) + (d2[r] * (sh0 + sh1) - m2[r] * sxh);
    }
  }
}

// Q6_K unit = 64 weights of one block: half n, 16-column slice c, all four
// 32-row groups (ql 2 x 16 B + qh 16 B + 4 scale bytes + d).
template <int R, int BT>
__device__ __forceinline__ void unit_q6k(const uint8_t* const* rowp, int u, uint32_t nb, const float* x, uint32_t ldx,
                                         int ncols, float (&acc)[R][BT]) {
  const int blk = u >> 2, n = (u >> 1) & 1, c = u & 1;
  const KqPos ps = kq_pos((uint32_t)blk, nb, q6k_group_bytes(8));
  uint4 qa[R], qb[R], qh[R];
  float ds[R][4];
#pragma unroll
  for (int r = 0; r < R; r++) {
    const uint8_t* b = rowp[r];
    qa[r] = ld_stream(b + q6k_q_off(ps, n, c, 0));
    qb[r] = ld_stream(b + q6k_q_off(ps, n, c, 1));
    qh[r] = ld_stream(b + q6k_q_off(ps, n, c, 2));
    const uint2 scw = __ldg(reinterpret_cast<const uint2*>(b + q6k_sc_off(ps) + n * 8));
    float d = fp16_ref(__ldg(reinterpret_cast<const unsigned short*>(b + q6k_d_off(ps))));
    if (!isfinite(d)) d = 0.f;  // the reference skips such a block (kernels/src/lib.rs:845)
    const uint32_t s0 = c ? (scw.x >> 8) : scw.x, s1 = c ? (scw.y >> 8) : scw.y;
    ds[r][0] = d * (float)(int8_t)(s0 & 0xFF);
    ds[r][1] = d * (float)(int8_t)((s0 >> 16) & 0xFF);
    ds[r][2] = d * (float)(int8_t)(s1 & 0xFF);
    ds[r][3] = d * (float)(int8_t)((s1 >> 16) & 0xFF);
  }
  const int base = blk * 256 + n * 128 + c * 16;
#pragma unroll
  for (int b = 0; b < BT; b++) {
    if (b >= ncols) break;
    const float* xb = x + (size_t)b * ldx + base;
    float xv[4][16];
#pragma unroll
    for (int g = 0; g < 4; g++)
#pragma unroll
      for (int i = 0; i < 4; i++) {
        float4 a = ldg4(xb + 32 * g + 4 * i);
        xv[g][4 * i] = a.x; xv[g][4 * i + 1] = a.y; xv[g][4 * i + 2] = a.z; xv[g][4 * i + 3] = a.w;
      }
#pragma unroll
    for (int r = 0; r < R; r++) {
      const uint32_t av[4] = {qa[r].x, qa[r].y, qa[r].z, qa[r].w};
      const uint32_t bv[4] = {qb[r].x, qb[r].y, qb[r].z, qb[r].w};
      const uint32_t hv[4] = {qh[r].x, qh[r].y, qh[r].z, qh[r].w};
      float s[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
      for (int i = 0; i < 4; i++) {
        const uint32_t w1 = (av[i] & 0x0F0F0F0Fu) | ((hv[i] << 4) & 0x30303030u);
        const uint32_t w2 = (bv[i] & 0x0F0F0F0Fu) | ((hv[i] << 2) & 0x30303030u);
        const uint32_t w3 = ((av[i] >> 4) & 0x0F0F0F0Fu) | (hv[i] & 0x30303030u);
        const uint32_t w4 = ((bv[i] >> 4) & 0x0F0F0F0Fu) | ((hv[i] >> 2) & 0x30303030u);
        const uint32_t ww[4] = {w1, w2, w3, w4};
#pragma unroll
        for (int g = 0; g < 4; g++) {
          s[g] = fmaf(byte_f<0>(ww[g], 8388640.f), xv[g][4 * i + 0], s[g]);
          s[g] = fmaf(byte_f<1>(ww[g], 8388640.f), xv[g][4 * i + 1], s[g]);
          s[g] = fmaf(byte_f<2>(ww[g], 8388640.f), xv[g][4 * i + 2], s[g]);
          s[g] = fmaf(byte_f<3>(ww[g], 8388640.f), xv[g][4 * i + 3], s[g]);
        }
      }
      acc[r][b] += (ds[r][0] * s[0] + ds[r][1] * s[1]) + (ds[r][2] * s[2] + ds[r][3] * s[3]);
    }
  }
}

// Q8_0 unit = 16 int8 weights (half a block) + d.
template <int R, int BT>
__device__ __forceinline__ void unit_q80(const uint8_t* const* rowp, const uint8_t* const* auxp, int u, const float* x,
                                         uint32_t ldx, int ncols, float (&acc)[R][BT]) {
  const int blk = u >> 1, h = u & 1;
  uint4 q[R];
  float d[R];
#pragma unroll
  for (int r = 0; r < R; r++) {
    q[r] = ld_stream(rowp[r] + (size_t)blk * 32 + h * 16);
    d[r] = fp16_ref(__ldg(reinterpret_cast<const unsigned short*>(auxp[r]) + blk));
  }
  const int base = blk * 32 + h * 16;
#pragma unroll
  for (int b = 0; b < BT; b++) {
    if (b >= ncols) break;
    const float* xb = x + (size_t)b * ldx + base;
    float xv[16];
#pragma unroll
    for (int i = 0; i < 4; i++) {
      float4 a = ldg4(xb + 4 * i);
      xv[4 * i] = a.x; xv[4 * i + 1] = a.y; xv[4 * i + 2] = a.z; xv[4 * i + 3] = a.w;
    }
#pragma unroll
    for (int r = 0; r < R; r++) {
      const uint32_t wv[4] = {q[r].x ^ 0x80808080u, q[r].y ^ 0x80808080u, q[r].z ^ 0x80808080u, q[r].w ^ 0x80808080u};
      float s0 = 0.f, s1 = 0.f;
#pragma unroll
      for (int i = 0; i < 4; i++) {
        s0 = fmaf(byte_f<0>(wv[i], 8388736.f), xv[4 * i + 0], s0);
        s1 = fmaf(byte_f<1>(wv[i], 8388736.f), xv[4 * i + 1], s1);
        s0 = fmaf(byte_f<2>(wv[i], 8388736.f), xv[4 * i + 2], s0);
        s1 = fmaf(byte_f<3>(wv[i], 8388736.f), xv[4 * i + 3], s1);
      }
      acc[r][b] += d[r] * (s0 + s1);
    }
  }
}

__device__ __forceinline__ uint32_t spread4(uint32_t b) {  // 4 bits -> bit 4 of each byte
  return ((b & 1u) << 4) | ((b & 2u) << 11) | ((b & 4u) << 18) | ((b & 8u) << 25);
}

// Q5_0 unit = one block (32 weights).
template <int R, int BT>
__device__ __forceinline__ void unit_q50(const uint8_t* const* rowp, const uint8_t* const* auxp, int u, const float* x,
                                         uint32_t ldx, int ncols, float (&acc)[R][BT]) {
  uint4 q[R];
  uint32_t qh[R];
  float d[R];
#pragma unroll
  for (int r = 0; r < R; r++) {
    q[r] = ld_stream(rowp[r] + (size_t)u * 16);
    const uint2 a = __ldg(reinterpret_cast<const uint2*>(auxp[r]) + u);
    qh[r] = a.x;
    d[r] = fp16_ref(a.y & 0xFFFFu);
  }
  const int base = u * 32;
#pragma unroll
  for (int b = 0; b < BT; b++) {
    if (b >= ncols) break;
    const float* xb = x + (size_t)b * ldx + base;
    float xv[32];
#pragma unroll
    for (int i = 0; i < 8; i++) {
      float4 a = ldg4(xb + 4 * i);
      xv[4 * i] = a.x; xv[4 * i + 1] = a.y; xv[4 * i + 2] = a.z; xv[4 * i + 3] = a.w;
    }
#pragma unroll
    for (int r = 0; r < R; r++) {
      const uint32_t wv[4] = {q[r].x, q[r].y, q[r].z, q[r].w};
      float s0 = 0.f, s1 = 0.f;
#pragma unroll
      for (int i = 0; i < 4; i++) {
        const uint32_t lo = (wv[i] & 0x0F0F0F0Fu) | spread4((qh[r] >> (4 * i)) & 0xFu);
        const uint32_t hi = ((wv[i] >> 4) & 0x0F0F0F0Fu) | spread4((qh[r] >> (16 + 4 * i)) & 0xFu);
        s0 = fmaf(byte_f<0>(lo, 8388624.f), xv[4 * i + 0], s0);
        s1 = fmaf(byte_f<1>(lo, 8388624.f), xv[4 * i + 1], s1);
        s0 = fmaf(byte_f<2>(lo, 8388624.f), xv[4 * i + 2], s0);
        s1 = fmaf(byte_f<3>(lo, 8388624.f), xv[4 * i + 3], s1);
        s0 = fmaf(byte_f<0>(hi, 8388624.f), xv[16 + 4 * i + 0], s0);
        s1 = fmaf(byte_f<1>(hi, 8388624.f), xv[16 + 4 * i + 1], s1);
        s0 = fmaf(byte_f<2>(hi, 8388624.f), xv[16 + 4 * i + 2], s0);
        s1 = fmaf(byte_f<3>(hi, 8388624.f), xv[16 + 4 * i + 3], s1);
      }
      acc[r][b] += d[r] * (s0 + s1);
    }
  }
}

// Dot products of rows row0..row0+R-1 with columns col0..col0+ncols-1;
// returns the warp-reduced sums (every lane holds them).
template <int QT, int R, int BT>
__device__ __forceinline__ void gemv_rows(const GemvSeg& sg, const float* x, uint32_t ldx, int row0, int col0,
                                          int ncols, float (&acc)[R][BT]) {
  const DWDesc& w = sg.w;
  const int lane = threadIdx.x & 31;
  const uint8_t* rowp[R];
  const uint8_t* auxp[R];
#pragma unroll
  for (int r = 0; r < R; r++) {
    const uint32_t o = min((uint32_t)(row0 + r), w.n_out - 1);
    rowp[r] = w.body + (size_t)o * w.body_stride;
    auxp[r] = w.aux + (size_t)o * w.aux_stride;
  }
#pragma unroll
  for (int r = 0; r < R; r++)
#pragma unroll
    for (int b = 0; b < BT; b++) acc[r][b] = 0.f;
  const float* xc = x + (size_t)col0 * ldx;
  const uint32_t qt = QT ? (uint32_t)QT : w.type;
  if (qt == 12) {
    const int nu = (int)(w.n_in >> 8) * 8;
    for (int u = lane; u < nu; u += 32) unit_q4k<R, BT>(rowp, u, w.n_in >> 8, xc, ldx, ncols, acc);
  } else if (qt == 14) {
    const int nu = (int)(w.n_in >> 8) * 4;
    for (int u = lane; u < nu; u += 32) unit_q6k<R, BT>(rowp, u, w.n_in >> 8, xc, ldx, ncols, acc);
  } else if (qt == 8) {
    const int nu = (int)(w.n_in >> 5) * 2;
    for (int u = lane; u < nu; u += 32) unit_q80<R, BT>(rowp, auxp, u, xc, ldx, ncols, acc);
  } else {
    const int nu = (int)(w.n_in >> 5);
    for (int u = lane; u < nu; u += 32) unit_q50<R, BT>(rowp, auxp, u, xc, ldx, ncols, acc);
  }
#pragma unroll
  for (int r = 0; r < R; r++)
#pragma unroll
    for (int b = 0; b < BT; b++) acc[r][b] = warp_sum(acc[r][b]);
}

// ------------------------------------------------------------ epilogue ----
// Input RMSNorm scale of column col (1 when the input is not normalized):
// the sum of the producer's per-CTA partials in a fixed order (deterministic).
__device__ float input_scale(const GemvArgs& a, uint32_t col) {
  if (!a.in_parts) return 1.0f;
  const int lane = threadIdx.x & 31;
  float s = 0.f;
  for (uint32_t i = lane; i < a.in_np; i += 32) s += a.in_parts[(size_t)col * a.in_np + i];
  s = warp_sum(s);
  return 1.0f / sqrtf(s / (float)a.in_n + a.in_eps);
}

// Single-row epilogues; returns the new residual value for EPI_RESID, else 0.
__device__ __forceinline__ float epi_single(const GemvArgs& a, const GemvSeg& sg, uint32_t o, uint32_t col, float v) {
  if (sg.bias) v = v + sg.bias[o];
  float* y = sg.y + (size_t)col * sg.ldy + o;
  switch (sg.epi) {
    case EPI_STORE: *y = v; return 0.f;
    case EPI_ADD: *y = *y + v; return 0.f;
    case EPI_RESID: {  // x += v (qwen2.rs:536-538, 549-551)
      const float xn = *y + v;
      *y = xn;
      store_act(a.xn, a.ldxn, a.xn4, a.xn6, xperm_len(sg.w.n_out), col, o, xn * a.nw[o]);
      return xn;
    }
    case EPI_V: {  // v row into the cache at the row's position (qwen2.rs:498)
      const RowDesc rd = a.rows[col];
      const SeqDesc sd = a.seqs[rd.seq];
      sd.v[((size_t)a.layer * sd.cap + rd.pos) * a.kvd + o] = v;
      return 0.f;
    }
  }
  return 0.f;
}

// Pair epilogues on physical rows (o, o+1), o even.
__device__ __forceinline__ void epi_pair(const GemvArgs& a, const GemvSeg& sg, uint32_t o, uint32_t col, float v0,
                                         float v1) {
  if (sg.bias) { v0 = v0 + sg.bias[o]; v1 = v1 + sg.bias[o + 1]; }
  if (sg.epi == EPI_SILU) {  // gate = silu(gate) * up (qwen2.rs:546-548, 743-745)
    const uint32_t m = o >> 1;
    const float hv = __fmul_rn(__fdiv_rn(v0, __fadd_rn(1.0f, expf(-v0))), v1);
    store_act(a.h, a.ldh, a.h4, a.h6, xperm_len(sg.w.n_out >> 1), col, m, hv);
    return;
  }
  // NEOX RoPE of the pair (dim m, dim m + hd/2) at the row's position
  // (qwen2.rs:708-724); cos/sin from the host table.
  const uint32_t half = a.hd >> 1, h = o / a.hd, m = (o - h * a.hd) >> 1;
  const RowDesc rd = a.rows[col];
  const float c = a.cos_t[(size_t)rd.pos * half + m], s = a.sin_t[(size_t)rd.pos * half + m];
  const float r0 = __fsub_rn(__fmul_rn(v0, c), __fmul_rn(v1, s));
  const float r1 = __fadd_rn(__fmul_rn(v0, s), __fmul_rn(v1, c));
  if (sg.epi == EPI_ROPE_Q) {
    float* y = sg.y + (size_t)col * sg.ldy + h * a.hd + m;
    y[0] = r0;
    y[half] = r1;
  } else {  // EPI_ROPE_K: into the K cache (qwen2.rs:497)
    const SeqDesc sd = a.seqs[rd.seq];
    float* kc = sd.k + ((size_t)a.layer * sd.cap + rd.pos) * a.kvd + h * a.hd + m;
    kc[0] = r0;
    kc[half] = r1;
  }
}

// Applies the segment's epilogue to the CTA's results val[b * nrows + r]
// (rows row_base.., columns col0..). Called by all threads of the CTA.
__device__ void cta_epilogue(const GemvArgs& a, const GemvSeg& sg, const float* val, float* scratch, int row_base,
                             int nrows, int col0, int ncols, const float* inv) {
  const uint32_t n_out = sg.w.n_out;
  if (epi_is_pair(sg.epi)) {
    const int np = nrows >> 1;
    for (int t = threadIdx.x; t < np * ncols; t += blockDim.x) {
      const int b = t / np, pr = t - b * np;
      const uint32_t o = (uint32_t)(row_base + 2 * pr);
      if (o < n_out)
        epi_pair(a, sg, o, (uint32_t)(col0 + b), val[b * nrows + 2 * pr] * inv[b], val[b * nrows + 2 * pr + 1] * inv[b]);
    }
    return;
  }
  for (int t = threadIdx.x; t < nrows * ncols; t += blockDim.x) {
    const int b = t / nrows, r = t - b * nrows;
    const uint32_t o = (uint32_t)(row_base + r);
    float xn = 0.f;
    if (o < n_out) xn = epi_single(a, sg, o, (uint32_t)(col0 + b), val[t] * inv[b]);
    if (sg.epi == EPI_RESID) scratch[t] = xn * xn;
  }
  if (sg.epi != EPI_RESID) return;
  __syncthreads();
  if ((int)threadIdx.x < ncols) {  // per-column partial sum of x^2 over this CTA's rows, in row order
    const int b = threadIdx.x;
    float s2 = 0.f;
    for (int r = 0; r < nrows; r++) s2 += scratch[b * nrows + r];
    a.out_parts[(size_t)(col0 + b) * gridDim.y + blockIdx.y] = s2;
  }
}

// ------------------------------------------------------ batch-1 GEMV ----
// Batch 1 is the decode hot path. A lane owns 64 weights of one 256-weight
// block per row (Q4_K: the 32 qs bytes of one sub-block pair; Q6_K: one
// (half, 16-column) slice of all four 32-row groups) and the warp owns R rows
// that share the lane's 64 activations. Two weights at a time become exact
// f32 values with one LOP3 (two fields into the mantissas of a half2 of
// 1024 + q), one half2 subtract and two f16->f32 converts, and are multiplied
// into f32x2 accumulators with packed FMAs. The activations arrive
// pre-permuted (xperm_q4k / xperm_q6k) so every load is coalesced and each
// float4 holds the partners of bytes (0,2) and (1,3). The GGUF block header
// is decoded once per 64 weights per row.

// fp16 -> f32 with the reference's NaN -> +-Inf quirk (dequant.rs:25-26).
__device__ __forceinline__ float h2f_ref(uint32_t h) {
  const float v = __half2float(__ushort_as_half((unsigned short)h));
  return ((h & 0x7C00u) == 0x7C00u) ? __uint_as_float(((h & 0x8000u) << 16) | 0x7F800000u) : v;
}
__device__ __forceinline__ float2 f2(float a, float b) { return make_float2(a, b); }
// v = two halves (off + a, off + b), exact: returns (a, b) in f32.
__device__ __forceinline__ float2 hpair(uint32_t v, __half2 off) {
  __half2 h = *reinterpret_cast<__half2*>(&v);
  return __half22float2(__hsub2(h, off));
}
// acc01 += pair(bytes 0,2) * (x.x, x.y); acc23 += pair(bytes 1,3) * (x.z, x.w)
// where pair p02/p13 are half2 of (off + q) for the word's byte fields.
__device__ __forceinline__ void fma_pairs(uint32_t p02, uint32_t p13, const float4& xv, __half2 off, float2& a0,
                                          float2& a1) {
  a0 = __ffma2_rn(hpair(p02, off), f2(xv.x, xv.y), a0);
  a1 = __ffma2_rn(hpair(p13, off), f2(xv.z, xv.w), a1);
}
__device__ __forceinline__ float hsum(const float2& a, const float2& b) { return (a.x + a.y) + (b.x + b.y); }
__device__ __forceinline__ float sum4(const float4& v) { return (v.x + v.y) + (v.z + v.w); }

template <int R>
__device__ __forceinline__ void q4k_b1(const DWDesc& w, const float* __restrict__ x, int row0, int slice, int nslice,
                                       float (&acc)[R]) {
  const int lane = threadIdx.x & 31, bi = lane >> 2, j = lane & 3;
  const int nb = (int)(w.n_in >> 8);
  const uint8_t* rowp[R];
#pragma unroll
  for (int r = 0; r < R; r++) rowp[r] = w.body + (size_t)min((uint32_t)(row0 + r), w.n_out - 1) * w.body_stride;
  // scale/min bit positions of sub-blocks 2j and 2j+1 (get_scale_min_k4, dequant.rs:41-49)
  const int sh = 16 * (j & 1);
  const bool hi6 = j >= 2;
  const uint32_t lo_mask = hi6 ? 0x0Fu : 0x3Fu, hi_mask = hi6 ? 0x30u : 0u;
  const int m_off = hi6 ? 4 : 0;
  const __half2 off = __floats2half2_rn(1024.f, 1024.f);
  for (int b = bi + 8 * slice; b < nb; b += 8 * nslice) {
    const KqPos ps = kq_pos((uint32_t)b, (uint32_t)nb, q4k_group_bytes(8));
    const uint32_t ho = q4k_hdr_off(ps), q0 = q4k_qs_off(ps, (uint32_t)j, 0), q1 = q4k_qs_off(ps, (uint32_t)j, 1);
    uint4 hd[R], qa[R], qb[R];
#pragma unroll
    for (int r = 0; r < R; r++) {
      hd[r] = ld_stream(rowp[r] + ho);
      qa[r] = ld_stream(rowp[r] + q0);
      qb[r] = ld_stream(rowp[r] + q1);
    }
    const float* xs = x + (size_t)(b >> 3) * 2048 + 4 * lane;  // xperm_q4k layout
#pragma unroll
    for (int half = 0; half < 2; half++) {  // 0: low nibbles = sub-block 2j, 1: high nibbles (x16) = 2j+1
      float4 xv[8];
#pragma unroll
      for (int i = 0; i < 8; i++) xv[i] = ldg4(xs + (8 * half + i) * 128);
      float sx = 0.f;
#pragma unroll
      for (int i = 0; i < 8; i++) sx += sum4(xv[i]);
      const uint32_t nm = half ? 0x00F000F0u : 0x000F000Fu;
#pragma unroll
      for (int r = 0; r < R; r++) {
        const uint32_t wv[8] = {qa[r].x, qa[r].y, qa[r].z, qa[r].w, qb[r].x, qb[r].y, qb[r].z, qb[r].w};
        float2 a0 = f2(0.f, 0.f), a1 = a0;
#pragma unroll
        for (int i = 0; i < 8; i++)
          fma_pairs((wv[i] & nm) | 0x64006400u, ((wv[i] >> 8) & nm) | 0x64006400u, xv[i], off, a0, a1);
        const float d = h2f_ref(hd[r].x & 0xFFFFu), dmin = h2f_ref(hd[r].x >> 16);
        const uint32_t ss = hi6 ? hd[r].w : hd[r].y, sm = hi6 ? hd[r].w : hd[r].z;
        const int o8 = 8 * half;
        const uint32_t sc = ((ss >> (sh + o8)) & lo_mask) | ((hd[r].y >> (sh + 2 + o8)) & hi_mask);
        const uint32_t mn = ((sm >> (sh + o8 + m_off)) & lo_mask) | ((hd[r].z >> (sh + 2 + o8)) & hi_mask);
        const float ds = half ? d * 0.0625f : d;  // high nibbles were summed as 16*q
        acc[r] = fmaf(-(dmin * (float)mn), sx, fmaf(ds * (float)sc, hsum(a0, a1), acc[r]));
      }
    }
  }
}

template <int R>
__device__ __forceinline__ void q6k_b1(const DWDesc& w, const float* __restrict__ x, int row0, int slice, int nslice,
                                       float (&acc)[R]) {
  const int lane = threadIdx.x & 31, bi = lane >> 2, n = (lane >> 1) & 1, c = lane & 1;
  const int nb = (int)(w.n_in >> 8);
  const uint8_t* rowp[R];
#pragma unroll
  for (int r = 0; r < R; r++) rowp[r] = w.body + (size_t)min((uint32_t)(row0 + r), w.n_out - 1) * w.body_stride;
  const __half2 off = __floats2half2_rn(1056.f, 1056.f);  // 1024 + 32: yields q - 32
  for (int b = bi + 8 * slice; b < nb; b += 8 * nslice) {
    const KqPos ps = kq_pos((uint32_t)b, (uint32_t)nb, q6k_group_bytes(8));
    const uint32_t oa = q6k_q_off(ps, n, c, 0), ob = q6k_q_off(ps, n, c, 1), oh = q6k_q_off(ps, n, c, 2);
    const uint32_t os = q6k_sc_off(ps) + 8 * n, od = q6k_d_off(ps);
    uint4 qa[R], qb[R], qh[R];
    uint2 sc[R];
    uint32_t dh[R];
#pragma unroll
    for (int r = 0; r < R; r++) {
      qa[r] = ld_stream(rowp[r] + oa);
      qb[r] = ld_stream(rowp[r] + ob);
      qh[r] = ld_stream(rowp[r] + oh);
      sc[r] = __ldg(reinterpret_cast<const uint2*>(rowp[r] + os));
      dh[r] = __ldg(reinterpret_cast<const unsigned short*>(rowp[r] + od));
    }
    const float* xs = x + (size_t)(b >> 3) * 2048 + 4 * lane;  // xperm_q6k layout
#pragma unroll
    for (int g = 0; g < 4; g++) {  // group g: rows 32g.. of the slice, scale sc[n*8 + c + 2g]
      float4 xv[4];
#pragma unroll
      for (int i = 0; i < 4; i++) xv[i] = ldg4(xs + (4 * g + i) * 128);
#pragma unroll
      for (int r = 0; r < R; r++) {
        const uint32_t src[4] = {(g & 1) ? qb[r].x : qa[r].x, (g & 1) ? qb[r].y : qa[r].y,
                                 (g & 1) ? qb[r].z : qa[r].z, (g & 1) ? qb[r].w : qa[r].w};
        const uint32_t hv[4] = {qh[r].x, qh[r].y, qh[r].z, qh[r].w};
        float2 p0 = f2(0.f, 0.f), p1 = p0;
#pragma unroll
        for (int i = 0; i < 4; i++) {
          // 6-bit q per byte: nibble | 2 high bits << 4 (dequant.rs:195-198)
          const uint32_t nib = g < 2 ? (src[i] & 0x0F0F0F0Fu) : ((src[i] >> 4) & 0x0F0F0F0Fu);
          const int hs = 4 - 2 * g;  // qh bits 2g, 2g+1 -> bits 4, 5
          const uint32_t q = nib | ((hs >= 0 ? (hv[i] << hs) : (hv[i] >> -hs)) & 0x30303030u);
          fma_pairs((q & 0x003F003Fu) | 0x64006400u, ((q >> 8) & 0x003F003Fu) | 0x64006400u, xv[i], off, p0, p1);
        }
        float d = h2f_ref(dh[r]);
        if (!isfinite(d)) d = 0.f;  // the reference skips such a block (kernels/src/lib.rs:845)
        const uint32_t sw = (g < 2 ? sc[r].x : sc[r].y) >> (8 * c + 16 * (g & 1));
        acc[r] = fmaf(d * (float)(int8_t)(sw & 0xFF), hsum(p0, p1), acc[r]);
      }
    }
  }
}

constexpr int B1_R = 4;
constexpr int B1_WARPS = 8;

// CTA = 8 warps = (8/S) row groups of B1_R rows x S slices of each row's
// blocks (slice s takes blocks 8s.., stride 8S); partial sums meet in smem.
__global__ void __launch_bounds__(B1_WARPS * 32, 2) gemv1_kernel(const __grid_constant__ GemvArgs a, int nslice) {
  const uint32_t cta = blockIdx.y;
  GemvSeg sg = a.seg[0];
  if (a.nseg > 1 && cta >= a.seg[1].cta_begin) sg = a.seg[1];
  if (a.nseg > 2 && cta >= a.seg[2].cta_begin) sg = a.seg[2];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int groups = B1_WARPS / nslice, grp = warp / nslice, slice = warp - grp * nslice;
  const int row_base = (int)(cta - sg.cta_begin) * (groups * B1_R);
  const int row0 = row_base + grp * B1_R;
  __shared__ float red[B1_WARPS][B1_R];
  __shared__ float val[B1_WARPS * B1_R];
  __shared__ float scratch[B1_WARPS * B1_R];
  __shared__ float inv[1];
  float acc[B1_R];
#pragma unroll
  for (int r = 0; r < B1_R; r++) acc[r] = 0.f;
  if (row0 < (int)sg.w.n_out) {
    if (sg.w.type == 12) {
      q4k_b1<B1_R>(sg.w, a.xp4, row0, slice, nslice, acc);
    } else if (sg.w.type == 14) {
      q6k_b1<B1_R>(sg.w, a.xp6, row0, slice, nslice, acc);
    } else if (slice == 0) {  // Q8_0 / Q5_0: generic units, unsplit
      float acc2[B1_R][1];
      gemv_rows<0, B1_R, 1>(sg, a.x, a.ldx, row0, 0, 1, acc2);
#pragma unroll
      for (int r = 0; r < B1_R; r++) acc[r] = lane == 0 ? acc2[r][0] : 0.f;
    }
  }
#pragma unroll
  for (int r = 0; r < B1_R; r++) {
    const float v = warp_sum(acc[r]);
    if (lane == 0) red[warp][r] = v;
  }
  if (warp == 0) {
    const float sc = input_scale(a, 0);
    if (lane == 0) inv[0] = sc;
  }
  __syncthreads();
  const int nrows = groups * B1_R;
  if ((int)threadIdx.x < nrows) {
    const int g = threadIdx.x / B1_R, r = threadIdx.x - g * B1_R;
    float v = 0.f;
    for (int k = 0; k < nslice; k++) v += red[g * nslice + k][r];
    val[threadIdx.x] = v;
  }
  __syncthreads();
  cta_epilogue(a, sg, val, scratch, row_base, nrows, 0, 1, inv);
}

// grid.x = column tiles of BT (fastest, so CTAs sharing weights run together),
// grid.y = CTAs over the concatenated rows of all segments.
template <int R, int BT>
__global__ void __launch_bounds__(GEMV_WARPS * 32) gemv_kernel(const __grid_constant__ GemvArgs a) {
  const uint32_t cta = blockIdx.y;
  GemvSeg sg = a.seg[0];
  if (a.nseg > 1 && cta >= a.seg[1].cta_begin) sg = a.seg[1];
  if (a.nseg > 2 && cta >= a.seg[2].cta_begin) sg = a.seg[2];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int row_base = (int)(cta - sg.cta_begin) * (GEMV_WARPS * R);
  const int row0 = row_base + warp * R;
  const int col0 = blockIdx.x * BT;
  const int ncols = min(BT, (int)a.batch - col0);
  __shared__ float val[BT * GEMV_WARPS * R];
  __shared__ float scratch[BT * GEMV_WARPS * R];
  __shared__ float inv[BT];
  float acc[R][BT];
  if (row0 < (int)sg.w.n_out) {
    switch (sg.w.type) {
      case 12: gemv_rows<12, R, BT>(sg, a.x, a.ldx, row0, col0, ncols, acc); break;
      case 14: gemv_rows<14, R, BT>(sg, a.x, a.ldx, row0, col0, ncols, acc); break;
      case 8: gemv_rows<8, R, BT>(sg, a.x, a.ldx, row0, col0, ncols, acc); break;
      default: gemv_rows<6, R, BT>(sg, a.x, a.ldx, row0, col0, ncols, acc); break;
    }
  } else {
#pragma unroll
    for (int r = 0; r < R; r++)
#pragma unroll
      for (int b = 0; b < BT; b++) acc[r][b] = 0.f;
  }
  const int nrows = GEMV_WARPS * R;
  if (lane == 0) {
#pragma unroll
    for (int r = 0; r < R; r++)
#pragma unroll
      for (int b = 0; b < BT; b++) val[b * nrows + warp * R + r] = acc[r][b];
  }
  for (int b = warp; b < ncols; b += GEMV_WARPS) {
    const float sc = input_scale(a, (uint32_t)(col0 + b));
    if (lane == 0) inv[b] = sc;
  }
  __syncthreads();
  cta_epilogue(a, sg, val, scratch, row_base, nrows, col0, ncols, inv);
}

// Writes rows of natural-layout activations in both permuted layouts.
__global__ void xpack_kernel(const float* x, uint32_t ldx, uint32_t K, float* p4, float* p6, uint32_t ldp) {
  const uint32_t r = blockIdx.y;
  for (uint32_t e = blockIdx.x * blockDim.x + threadIdx.x; e < K; e += gridDim.x * blockDim.x)
    store_act(nullptr, 0, p4, p6, ldp, r, e, x[(size_t)r * ldx + e]);
}

// Embedding lookup (qwen2.rs:468-472) fused with the first layer's RMSNorm
// input: x = row tok of the table (exact dequant), xn = x * nw in the natural
// and permuted layouts, parts[r] = sum(x^2) (one partial per row).
__global__ void embed_norm_kernel(DWDesc w, const uint32_t* tokens, float* x, uint32_t ldx, const float* nw, float* xn,
                                  float* xn4, float* xn6, uint32_t ldxn, float* parts) {
  const uint32_t r = blockIdx.x, tok = tokens[r], n = w.n_in;
  float ss = 0.f;
  for (uint32_t e = threadIdx.x; e < n; e += blockDim.x) {
    const float v = dequant_elem(w, tok, e);
    x[(size_t)r * ldx + e] = v;
    store_act(xn, ldxn, xn4, xn6, xperm_len(n), r, e, v * nw[e]);
    ss += v * v;
  }
  __shared__ float red[32];
  ss = warp_sum(ss);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
  __syncthreads();
  if (threadIdx.x < 32) {
    float v = threadIdx.x < (blockDim.x >> 5) ? red[threadIdx.x] : 0.f;
    v = warp_sum(v);
    if (threadIdx.x == 0) parts[r] = v;
  }
}

// ------------------------------------------------------------ launch ----
// K-slices per row for batch 1: enough warps to cover every SM several times,
// at least one 8-block step per slice.
static int b1_slices(const GemvArgs& a) {
  uint32_t rows = 0;
  for (uint32_t i = 0; i < a.nseg; i++) rows += a.seg[i].w.n_out;
  const uint32_t nb = a.seg[0].w.n_in >> 8;
  int s = 1;
  while (s < B1_WARPS && (rows / B1_R) * s < 148u * 24u && nb >= 8u * (uint32_t)(2 * s)) s *= 2;
  for (uint32_t i = 0; i < a.nseg; i++)
    if (a.seg[i].w.type != 12 && a.seg[i].w.type != 14) s = 1;
  return s;
}

static int rows_per_cta(const GemvArgs& a) {
  if (a.batch <= 1) return (B1_WARPS / b1_slices(a)) * B1_R;
  return GEMV_WARPS * 2;
}

// Fills cta_begin of each segment; returns the total CTA count along y.
uint32_t gemv_plan(GemvArgs& a) {
  const int rpc = rows_per_cta(a);
  uint32_t c = 0;
  for (uint32_t i = 0; i < a.nseg; i++) {
    a.seg[i].cta_begin = c;
    c += (a.seg[i].w.n_out + rpc - 1) / rpc;
  }
  return c;
}

cudaError_t launch_gemv(GemvArgs a, cudaStream_t st, uint32_t* grid_y) {
  const uint32_t ny = gemv_plan(a);
  if (grid_y) *grid_y = ny;
  const dim3 blk(GEMV_WARPS * 32);
  if (a.batch == 1) gemv1_kernel<<<dim3(1, ny), B1_WARPS * 32, 0, st>>>(a, b1_slices(a));
  else if (a.batch == 2) gemv_kernel<2, 2><<<dim3(1, ny), blk, 0, st>>>(a);
  else if (a.batch <= 4) gemv_kernel<2, 4><<<dim3(1, ny), blk, 0, st>>>(a);
  else gemv_kernel<2, 8><<<dim3((a.batch + 7) / 8, ny), blk, 0, st>>>(a);
  return cudaGetLastError();
}

cudaError_t launch_xpack(const float* x, uint32_t ldx, uint32_t K, uint32_t rows, float* p4, float* p6, cudaStream_t st) {
  if (!rows) return cudaSuccess;
  xpack_kernel<<<dim3((K + 255) / 256, rows), 256, 0, st>>>(x, ldx, K, p4, p6, xperm_len(K));
  return cudaGetLastError();
}

cudaError_t launch_dequant(const DWDesc& w, float* out, cudaStream_t st) {
  size_t n = (size_t)w.n_out * w.n_in;
  if (!n) return cudaSuccess;
  dequant_kernel<<<(unsigned)((n + 255) / 256), 256, 0, st>>>(w, out);
  return cudaGetLastError();
}

cudaError_t launch_embed_norm(const DWDesc& w, const uint32_t* tokens, uint32_t rows, float* x, uint32_t ldx,
                              const float* nw, float* xn, float* xn4, float* xn6, uint32_t ldxn, float* parts,
                              cudaStream_t st) {
  if (!rows) return cudaSuccess;
  embed_norm_kernel<<<rows, 512, 0, st>>>(w, tokens, x, ldx, nw, xn, xn4, xn6, ldxn, parts);
  return cudaGetLastError();
}

cudaError_t launch_embed(const DWDesc& w, const uint32_t* tokens, uint32_t rows, float* x, uint32_t ldx, cudaStream_t st) {
  if (!rows) return cudaSuccess;
  embed_kernel<<<dim3((w.n_in + 255) / 256, rows), 256, 0, st>>>(w, tokens, x, ldx);
  return cudaGetLastError();
}

// ------------------------------------------------- no-allocation GEMV ----
// Scratch of sm_gemv_noalloc: the two permuted copies of one batch-1 input
// vector, in a fixed device array instead of memory the call allocates. Every
// call on a device shares it; the pack kernel of a call writes every entry its
// GEMV reads, so nothing needs clearing, and calls that overlap on the GPU
// race on it.
constexpr uint32_t NOALLOC_MAX_K = 32768;
static __device__ __align__(256) float g_noalloc_xp[2 * NOALLOC_MAX_K];

constexpr int NOALLOC_MAX_DEVICES = 64;
static std::mutex g_noalloc_mu;
static float* g_noalloc_ptr[NOALLOC_MAX_DEVICES] = {};

uint32_t gemv_noalloc_max_k() { return NOALLOC_MAX_K; }

// The scratch's device address on the current device, looked up once per
// device with that device current (host code cannot use the symbol itself).
static cudaError_t noalloc_scratch(float** out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  if (dev < 0 || dev >= NOALLOC_MAX_DEVICES) return cudaErrorInvalidDevice;
  std::lock_guard<std::mutex> lk(g_noalloc_mu);
  if (!g_noalloc_ptr[dev]) {
    float* p = nullptr;
    e = cudaGetSymbolAddress((void**)&p, g_noalloc_xp);
    if (e != cudaSuccess) return e;
    g_noalloc_ptr[dev] = p;
  }
  *out = g_noalloc_ptr[dev];
  return cudaSuccess;
}

// sm_gemv without any allocation: batch 1 packs x into the fixed scratch;
// larger batches read x directly and need no scratch. n_in must not exceed
// NOALLOC_MAX_K (checked by the caller).
cudaError_t launch_gemv_noalloc(GemvArgs a, cudaStream_t st) {
  if (a.batch == 1) {
    float* xp = nullptr;
    cudaError_t e = noalloc_scratch(&xp);
    if (e != cudaSuccess) return e;
    const uint32_t K = a.seg[0].w.n_in;
    a.xp4 = xp;
    a.xp6 = xp + NOALLOC_MAX_K;
    e = launch_xpack(a.x, a.ldx, K, 1, xp, xp + NOALLOC_MAX_K, st);
    if (e != cudaSuccess) return e;
  }
  return launch_gemv(a, st, nullptr);
}

}  // namespace sm
