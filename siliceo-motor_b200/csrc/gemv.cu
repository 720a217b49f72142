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
#include "gemv_common.cuh"

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
      const uint32_t blk = e >> 8, l = e & 255, rr = o & 15, sb = l >> 5, within = l & 31;
      const uint8_t* u = w.body + (size_t)(o >> 4) * w.body_stride + (size_t)blk * Q4T_UNIT;
      const uint8_t* h = u + 16 * rr;
      float d = fp16_ref(rd16(h)), dmin = fp16_ref(rd16(h + 2));
      uint32_t sc, m;
      scale_min_k4((int)sb, h + 4, &sc, &m);
      uint32_t qb = u[q4t_qs_off(rr, 32 * (sb >> 1) + within)];
      uint32_t q = (sb & 1) ? (qb >> 4) : (qb & 0x0F);
      float d1 = __fmul_rn(d, (float)sc), m1 = __fmul_rn(dmin, (float)m);
      return __fsub_rn(__fmul_rn(d1, (float)q), m1);
    }
    case 14: {  // Q6_K, dequant.rs:178-206
      const uint32_t blk = e >> 8, l = e & 255, rr = o & 15, sb = l >> 4, t = (l >> 2) & 3, k = l & 3;
      const uint32_t i = sb & 7, nib = sb >> 3;
      const uint8_t* u = w.body + (size_t)(o >> 4) * w.body_stride + (size_t)blk * Q6T_UNIT;
      float d = fp16_ref(rd16(u + 256 + 2 * rr));
      if (!isfinite(d)) return 0.0f;
      const uint32_t lo = (u[q6t_w_off(rr, t, i) + k] >> (4 * nib)) & 0x0F;
      const uint32_t hw = *reinterpret_cast<const uint32_t*>(u + q6t_h_off(rr, t, i >> 1));
      const uint32_t hi = (hw >> ((q6t_field(k, nib) + 8 * (i & 1)) & 31)) & 3;
      int32_t q = (int32_t)(lo | (hi << 4)) - 32;
      float sc = (float)(int8_t)u[16 * rr + sb];
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

// Q4_K / Q6_K unit = lane t's 64 weights of one block of a row in the tile
// layout (device.cuh); tp[r] is the row's tile, rrs[r] its row in the tile.
// Q4_K: 8 weights of each of the 8 sub-blocks (offsets 8t .. 8t + 7).
template <int R, int BT>
__device__ __forceinline__ void unit_q4k(const uint8_t* const* tp, const uint32_t* rrs, int u, const float* x,
                                         uint32_t ldx, int ncols, float (&acc)[R][BT]) {
  const int blk = u >> 2, t = u & 3;
  uint4 hd[R], qa[R], qb[R];
#pragma unroll
  for (int r = 0; r < R; r++) {
    const uint8_t* ub = tp[r] + (size_t)blk * Q4T_UNIT;
    const uint32_t rr = rrs[r], q0 = 256u + 1024u * (rr >> 3) + 16u * (4u * (rr & 7u) + (uint32_t)t);
    hd[r] = ldg_u4(ub + 16 * rr);
    qa[r] = ld_stream(ub + q0);
    qb[r] = ld_stream(ub + q0 + 512);
  }
  float ds[R][8], dm[R][8];
#pragma unroll
  for (int r = 0; r < R; r++) {
    const float d = fp16_ref(hd[r].x & 0xFFFFu), dmin = fp16_ref(hd[r].x >> 16);
#pragma unroll
    for (int sb = 0; sb < 8; sb++) {  // get_scale_min_k4, dequant.rs:41-49
      uint32_t sc, m;
      if (sb < 4) {
        sc = (hd[r].y >> (8 * sb)) & 63u;
        m = (hd[r].z >> (8 * sb)) & 63u;
      } else {
        const int s0 = 8 * (sb - 4);
        sc = ((hd[r].w >> s0) & 0xFu) | (((hd[r].y >> (s0 + 6)) & 3u) << 4);
        m = ((hd[r].w >> (s0 + 4)) & 0xFu) | (((hd[r].z >> (s0 + 6)) & 3u) << 4);
      }
      ds[r][sb] = d * (float)sc;
      dm[r][sb] = dmin * (float)m;
    }
  }
#pragma unroll
  for (int b = 0; b < BT; b++) {
    if (b >= ncols) break;
    const float* xb = x + (size_t)b * ldx + blk * 256 + 8 * t;
#pragma unroll
    for (int sb = 0; sb < 8; sb++) {
      const float4 x0 = ldg4(xb + 32 * sb), x1 = ldg4(xb + 32 * sb + 4);
      const float xs = sum4(x0) + sum4(x1);
      const int j = sb >> 1, nib = sb & 1;
#pragma unroll
      for (int r = 0; r < R; r++) {
        const uint4 q = j < 2 ? qa[r] : qb[r];
        const uint32_t wa = (j & 1) ? q.z : q.x, wb = (j & 1) ? q.w : q.y;
        const uint32_t la = (wa >> (4 * nib)) & 0x0F0F0F0Fu, lb = (wb >> (4 * nib)) & 0x0F0F0F0Fu;
        float s0 = byte_f<0>(la, 8388608.f) * x0.x;
        float s1 = byte_f<1>(la, 8388608.f) * x0.y;
        s0 = fmaf(byte_f<2>(la, 8388608.f), x0.z, s0);
        s1 = fmaf(byte_f<3>(la, 8388608.f), x0.w, s1);
        s0 = fmaf(byte_f<0>(lb, 8388608.f), x1.x, s0);
        s1 = fmaf(byte_f<1>(lb, 8388608.f), x1.y, s1);
        s0 = fmaf(byte_f<2>(lb, 8388608.f), x1.z, s0);
        s1 = fmaf(byte_f<3>(lb, 8388608.f), x1.w, s1);
        acc[r][b] += ds[r][sb] * (s0 + s1) - dm[r][sb] * xs;
      }
    }
  }
}

// Q6_K: 4 weights of each of the 16 sub-blocks (offsets 4t .. 4t + 3).
template <int R, int BT>
__device__ __forceinline__ void unit_q6k(const uint8_t* const* tp, const uint32_t* rrs, int u, const float* x,
                                         uint32_t ldx, int ncols, float (&acc)[R][BT]) {
  const int blk = u >> 2, t = u & 3;
  uint4 w0[R], w1[R], hh[R];
  float ds[R][16];
#pragma unroll
  for (int r = 0; r < R; r++) {
    const uint8_t* ub = tp[r] + (size_t)blk * Q6T_UNIT;
    const uint32_t rr = rrs[r], q0 = q6t_w_off(rr, (uint32_t)t, 0);
    w0[r] = ld_stream(ub + q0);
    w1[r] = ld_stream(ub + q0 + 512);
    hh[r] = ld_stream(ub + q0 + 1024);
    const uint4 sc = ldg_u4(ub + 16 * rr);
    float d = fp16_ref(__ldg(reinterpret_cast<const unsigned short*>(ub + 256 + 2 * rr)));
    if (!isfinite(d)) d = 0.f;  // the reference skips such a block (kernels/src/lib.rs:845)
    const uint32_t scw[4] = {sc.x, sc.y, sc.z, sc.w};
#pragma unroll
    for (int sb = 0; sb < 16; sb++) ds[r][sb] = d * (float)(int8_t)((scw[sb >> 2] >> (8 * (sb & 3))) & 0xFFu);
  }
#pragma unroll
  for (int b = 0; b < BT; b++) {
    if (b >= ncols) break;
    const float* xb = x + (size_t)b * ldx + blk * 256 + 4 * t;
#pragma unroll
    for (int i = 0; i < 8; i++) {
      const float4 xa = ldg4(xb + 16 * i), xc = ldg4(xb + 16 * (i + 8));
#pragma unroll
      for (int r = 0; r < R; r++) {
        const uint32_t wv = (i < 4 ? (&w0[r].x)[i] : (&w1[r].x)[i - 4]);
        const uint32_t hw = (&hh[r].x)[i >> 1];
        const uint32_t hq = (i & 1) ? __funnelshift_r(hw, hw, 8) : hw;
        const uint32_t va = (wv & 0x0F0F0F0Fu) | (hq & 0x00300030u) | ((hq << 6) & 0x30003000u);
        const uint32_t vb = ((wv >> 4) & 0x0F0F0F0Fu) | ((hq >> 4) & 0x00300030u) | ((hq << 2) & 0x30003000u);
        float sa = byte_f<0>(va, 8388640.f) * xa.x;
        sa = fmaf(byte_f<1>(va, 8388640.f), xa.y, sa);
        sa = fmaf(byte_f<2>(va, 8388640.f), xa.z, sa);
        sa = fmaf(byte_f<3>(va, 8388640.f), xa.w, sa);
        float sb2 = byte_f<0>(vb, 8388640.f) * xc.x;
        sb2 = fmaf(byte_f<1>(vb, 8388640.f), xc.y, sb2);
        sb2 = fmaf(byte_f<2>(vb, 8388640.f), xc.z, sb2);
        sb2 = fmaf(byte_f<3>(vb, 8388640.f), xc.w, sb2);
        acc[r][b] += ds[r][i] * sa + ds[r][i + 8] * sb2;
      }
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
  uint32_t rrs[R];
  const bool tiled = tiled_type(QT ? (uint32_t)QT : w.type);
#pragma unroll
  for (int r = 0; r < R; r++) {
    const uint32_t o = min((uint32_t)(row0 + r), w.n_out - 1);
    rowp[r] = tiled ? w.body + (size_t)(o >> 4) * w.body_stride : w.body + (size_t)o * w.body_stride;
    rrs[r] = o & 15u;
    auxp[r] = w.aux + (size_t)o * w.aux_stride;
  }
#pragma unroll
  for (int r = 0; r < R; r++)
#pragma unroll
    for (int b = 0; b < BT; b++) acc[r][b] = 0.f;
  const float* xc = x + (size_t)col0 * ldx;
  const uint32_t qt = QT ? (uint32_t)QT : w.type;
  if (qt == 12) {
    const int nu = (int)(w.n_in >> 8) * 4;
    for (int u = lane; u < nu; u += 32) unit_q4k<R, BT>(rowp, rrs, u, xc, ldx, ncols, acc);
  } else if (qt == 14) {
    const int nu = (int)(w.n_in >> 8) * 4;
    for (int u = lane; u < nu; u += 32) unit_q6k<R, BT>(rowp, rrs, u, xc, ldx, ncols, acc);
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

// Embedding lookup (qwen2.rs:468-472) fused with the first layer's RMSNorm
// input: x = row tok of the table (exact dequant), xn = x * nw, parts[r] =
// sum(x^2) (one partial per row).
__global__ void embed_norm_kernel(DWDesc w, const uint32_t* tokens, float* x, uint32_t ldx, const float* nw, float* xn,
                                  uint32_t ldxn, float* parts) {
  const uint32_t r = blockIdx.x, tok = tokens[r], n = w.n_in;
  float ss = 0.f;
  for (uint32_t e = threadIdx.x; e < n; e += blockDim.x) {
    const float v = dequant_elem(w, tok, e);
    x[(size_t)r * ldx + e] = v;
    xn[(size_t)r * ldxn + e] = v * nw[e];
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
// Fills cta_begin of each segment; returns the total CTA count along y.
uint32_t gemv_plan(GemvArgs& a) {
  const uint32_t rpc = GEMV_WARPS * 2;
  uint32_t c = 0;
  for (uint32_t i = 0; i < a.nseg; i++) {
    a.seg[i].cta_begin = c;
    c += (a.seg[i].w.n_out + rpc - 1) / rpc;
  }
  return c;
}

bool gemv_tc_ok(const GemvArgs& a);
cudaError_t launch_gemv_tc(GemvArgs a, cudaStream_t st, uint32_t* n_parts);
bool gemv_tcb_ok(const GemvArgs& a);
cudaError_t launch_gemv_tcb(GemvArgs a, cudaStream_t st, uint32_t* n_parts);

// Segments of one launch regrouped by weight type (the batched tensor-core
// kernel takes one type per launch); false if any segment is not tiled.
static bool split_by_type(const GemvArgs& a, GemvArgs* out, uint32_t* n) {
  *n = 0;
  for (uint32_t i = 0; i < a.nseg; i++) {
    if (!tiled_type(a.seg[i].w.type)) return false;
    uint32_t k = 0;
    while (k < *n && out[k].seg[0].w.type != a.seg[i].w.type) k++;
    if (k == *n) {
      out[k] = a;
      out[k].nseg = 0;
      (*n)++;
    }
    out[k].seg[out[k].nseg++] = a.seg[i];
  }
  return true;
}

cudaError_t launch_gemv(GemvArgs a, cudaStream_t st, uint32_t* n_parts) {
  if (gemv_tc_ok(a)) {
    const cudaError_t e = launch_gemv_tc(a, st, n_parts);
    if (e != cudaErrorNotSupported) return e;
  }
  GemvArgs parts[3];
  uint32_t np = 0;
  if (a.batch >= 2 && split_by_type(a, parts, &np) && (np == 1 || !n_parts)) {
    bool ok = true;
    for (uint32_t i = 0; i < np && ok; i++) ok = gemv_tcb_ok(parts[i]);
    if (ok) {
      cudaError_t e = cudaSuccess;
      for (uint32_t i = 0; i < np && e == cudaSuccess; i++) e = launch_gemv_tcb(parts[i], st, n_parts);
      if (e != cudaErrorNotSupported) return e;
    }
  }
  const uint32_t ny = gemv_plan(a);
  if (n_parts) *n_parts = ny;
  const dim3 blk(GEMV_WARPS * 32);
  if (a.batch <= 2) gemv_kernel<2, 2><<<dim3(1, ny), blk, 0, st>>>(a);
  else if (a.batch <= 4) gemv_kernel<2, 4><<<dim3(1, ny), blk, 0, st>>>(a);
  else gemv_kernel<2, 8><<<dim3((a.batch + 7) / 8, ny), blk, 0, st>>>(a);
  return cudaGetLastError();
}

cudaError_t launch_dequant(const DWDesc& w, float* out, cudaStream_t st) {
  size_t n = (size_t)w.n_out * w.n_in;
  if (!n) return cudaSuccess;
  dequant_kernel<<<(unsigned)((n + 255) / 256), 256, 0, st>>>(w, out);
  return cudaGetLastError();
}

cudaError_t launch_embed_norm(const DWDesc& w, const uint32_t* tokens, uint32_t rows, float* x, uint32_t ldx,
                              const float* nw, float* xn, uint32_t ldxn, float* parts, cudaStream_t st) {
  if (!rows) return cudaSuccess;
  embed_norm_kernel<<<rows, 512, 0, st>>>(w, tokens, x, ldx, nw, xn, ldxn, parts);
  return cudaGetLastError();
}

cudaError_t launch_embed(const DWDesc& w, const uint32_t* tokens, uint32_t rows, float* x, uint32_t ldx, cudaStream_t st) {
  if (!rows) return cudaSuccess;
  embed_kernel<<<dim3((w.n_in + 255) / 256, rows), 256, 0, st>>>(w, tokens, x, ldx);
  return cudaGetLastError();
}

// ------------------------------------------------- no-allocation GEMV ----
// Scratch of sm_gemv_noalloc: the K-split partial sums and arrival counters of
// the batch-1 tensor-core GEMV, in fixed device arrays instead of memory the
// call allocates. Every call on a device shares them; a launch leaves the
// counters at zero (device globals start at zero), so nothing needs clearing,
// and calls that overlap on the GPU race on them. A launch whose split does
// not fit runs with K unsplit.
constexpr uint32_t NOALLOC_PART = 65536, NOALLOC_CNT = 1024;
static __device__ __align__(256) float g_noalloc_part[NOALLOC_PART];
static __device__ __align__(256) uint32_t g_noalloc_cnt[NOALLOC_CNT];

constexpr int NOALLOC_MAX_DEVICES = 64;
static std::mutex g_noalloc_mu;
struct NoallocPtrs {
  float* part;
  uint32_t* cnt;
};
static NoallocPtrs g_noalloc_ptr[NOALLOC_MAX_DEVICES] = {};

// The scratch's device addresses on the current device, looked up once per
// device with that device current (host code cannot use the symbols).
static cudaError_t noalloc_scratch(NoallocPtrs* out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  if (dev < 0 || dev >= NOALLOC_MAX_DEVICES) return cudaErrorInvalidDevice;
  std::lock_guard<std::mutex> lk(g_noalloc_mu);
  if (!g_noalloc_ptr[dev].part) {
    NoallocPtrs p{};
    e = cudaGetSymbolAddress((void**)&p.part, g_noalloc_part);
    if (e == cudaSuccess) e = cudaGetSymbolAddress((void**)&p.cnt, g_noalloc_cnt);
    if (e != cudaSuccess) return e;
    g_noalloc_ptr[dev] = p;
  }
  *out = g_noalloc_ptr[dev];
  return cudaSuccess;
}

// sm_gemv without any allocation.
cudaError_t launch_gemv_noalloc(GemvArgs a, cudaStream_t st) {
  NoallocPtrs p{};
  cudaError_t e = noalloc_scratch(&p);
  if (e != cudaSuccess) return e;
  a.ks_part = p.part;
  a.ks_cnt = p.cnt;
  a.ks_part_cap = NOALLOC_PART;
  a.ks_cnt_cap = NOALLOC_CNT;
  return launch_gemv(a, st, nullptr);
}

}  // namespace sm
