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
      const uint32_t blk = e >> 8, l = e & 255, rr = o & 15, sb = l >> 4;
      const uint8_t* u = w.body + (size_t)(o >> 4) * w.body_stride + (size_t)blk * Q6T_UNIT;
      float d = fp16_ref(rd16(u + 256 + 2 * rr));
      if (!isfinite(d)) return 0.0f;
      int32_t q = (int32_t)q6t_value(u, rr, l) - 32;
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
  if (qt == 8) {
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
// input: x = row tok of the table (exact dequant), xn = x * nw, and per chunk
// of EMB_CHUNK elements (blockIdx.y) the partial sum(x^2) at
// parts[r * gridDim.y + chunk] (summed by the next GEMV in chunk order).
constexpr uint32_t EMB_CHUNK = 512;
__global__ void embed_norm_kernel(DWDesc w, const uint32_t* tokens, float* x, uint32_t ldx, const float* nw, float* xn,
                                  uint32_t ldxn, float* parts) {
  const uint32_t r = blockIdx.x, tok = tokens[r], n = w.n_in;
  const uint32_t e = blockIdx.y * EMB_CHUNK + threadIdx.x;
  float v = 0.f;
  if (e < n) {
    v = dequant_elem(w, tok, e);
    x[(size_t)r * ldx + e] = v;
    xn[(size_t)r * ldxn + e] = v * nw[e];
  }
  float ss = warp_sum(v * v);
  __shared__ float red[EMB_CHUNK / 32];
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
  __syncthreads();
  if (threadIdx.x < 32) {
    float s = threadIdx.x < (blockDim.x >> 5) ? red[threadIdx.x] : 0.f;
    s = warp_sum(s);
    if (threadIdx.x == 0) parts[(size_t)r * gridDim.y + blockIdx.y] = s;
  }
}

uint32_t embed_norm_parts(uint32_t n) { return (n + EMB_CHUNK - 1) / EMB_CHUNK; }

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

cudaError_t launch_gemv_tc(GemvArgs a, cudaStream_t st, uint32_t* n_parts);
cudaError_t launch_gemv_tcb(GemvArgs a, cudaStream_t st, uint32_t* n_parts);
cudaError_t launch_gemv_umma(GemvArgs a, cudaStream_t st, uint32_t* n_parts);

// Batches of 2..32 columns of one tiled type: tcgen05 (gemv_umma.cu), else
// the mma.sync kernel of gemv_tcb.cu when no plan of the former fits.
static cudaError_t launch_batched(const GemvArgs& a, cudaStream_t st, uint32_t* n_parts) {
  const cudaError_t e = launch_gemv_umma(a, st, n_parts);
  return e == cudaErrorNotSupported ? launch_gemv_tcb(a, st, n_parts) : e;
}

// Q4_K / Q6_K segments run on the tensor-core kernels (batch 1: gemv_tc.cu,
// mixed types in one launch; batches: launch_batched, one launch per type), the
// Q5_0 / Q8_0 fallback types on gemv_kernel; a launch whose segments mix the
// two families is split. n_parts (EPI_RESID) needs a single-segment launch.
static cudaError_t launch_generic(const GemvArgs& a0, cudaStream_t st, uint32_t* n_parts) {
  GemvArgs a = a0;
  const uint32_t ny = gemv_plan(a);
  if (n_parts) *n_parts = ny;
  const dim3 blk(GEMV_WARPS * 32);
  if (a.batch <= 2) gemv_kernel<2, 2><<<dim3(1, ny), blk, 0, st>>>(a);
  else if (a.batch <= 4) gemv_kernel<2, 4><<<dim3(1, ny), blk, 0, st>>>(a);
  else gemv_kernel<2, 8><<<dim3((a.batch + 7) / 8, ny), blk, 0, st>>>(a);
  return cudaGetLastError();
}

cudaError_t launch_gemv(GemvArgs a, cudaStream_t st, uint32_t* n_parts) {
  // segments by family: tiled types grouped per type (QT_Q4K, QT_Q6K), the rest together
  GemvArgs q4 = a, q6 = a, other = a;
  q4.nseg = q6.nseg = other.nseg = 0;
  for (uint32_t i = 0; i < a.nseg; i++) {
    GemvArgs& d = a.seg[i].w.type == 12 ? q4 : a.seg[i].w.type == 14 ? q6 : other;
    d.seg[d.nseg++] = a.seg[i];
  }
  const uint32_t launches = (q4.nseg > 0) + (q6.nseg > 0) + (other.nseg > 0);
  if (n_parts && (launches != 1 || a.nseg != 1)) return cudaErrorInvalidValue;
  cudaError_t e = cudaSuccess;
  if (a.batch == 1 && q4.nseg && q6.nseg) {  // one batch-1 launch for both tiled types
    GemvArgs t = a;
    t.nseg = 0;
    for (uint32_t i = 0; i < a.nseg; i++)
      if (tiled_type(a.seg[i].w.type)) t.seg[t.nseg++] = a.seg[i];
    e = launch_gemv_tc(t, st, n_parts);
  } else {
    for (GemvArgs* g : {&q4, &q6}) {
      if (!g->nseg || e != cudaSuccess) continue;
      e = g->batch == 1 ? launch_gemv_tc(*g, st, n_parts) : launch_batched(*g, st, n_parts);
    }
  }
  if (e == cudaSuccess && other.nseg) e = launch_generic(other, st, n_parts);
  return e;
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
  embed_norm_kernel<<<dim3(rows, embed_norm_parts(w.n_in)), EMB_CHUNK, 0, st>>>(w, tokens, x, ldx, nw, xn, ldxn, parts);
  return cudaGetLastError();
}

cudaError_t launch_embed(const DWDesc& w, const uint32_t* tokens, uint32_t rows, float* x, uint32_t ldx, cudaStream_t st) {
  if (!rows) return cudaSuccess;
  embed_kernel<<<dim3((w.n_in + 255) / 256, rows), 256, 0, st>>>(w, tokens, x, ldx);
  return cudaGetLastError();
}

// ------------------------------------------------- no-allocation GEMV ----
// Scratch of sm_gemv_noalloc: the K-split partial sums and arrival counters of
// the batch-1 and batched tensor-core GEMVs, in fixed device arrays instead of
// memory the call allocates, and the error word of their bounded waits. Every
// call on a device shares them. The counters advance with wrapping increments,
// so each complete launch leaves them at zero (device globals start at zero)
// and nothing needs clearing; calls that overlap on the GPU race on the
// partial sums (their results are then wrong) but leave the counters at zero
// once all of them have completed. A shape whose smallest K-split does not
// fit NOALLOC_PART floats is refused (cudaErrorNotSupported, nothing runs).
constexpr uint32_t NOALLOC_PART = 65536, NOALLOC_CNT = 1024;
static __device__ __align__(256) float g_noalloc_part[NOALLOC_PART];
static __device__ __align__(256) uint32_t g_noalloc_cnt[NOALLOC_CNT];
static __device__ __align__(256) uint32_t g_noalloc_err[64];

constexpr int NOALLOC_MAX_DEVICES = 64;
static std::mutex g_noalloc_mu;
struct NoallocPtrs {
  float* part;
  uint32_t* cnt;
  uint32_t* err;
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
    if (e == cudaSuccess) e = cudaGetSymbolAddress((void**)&p.err, g_noalloc_err);
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
  a.err = p.err;
  return launch_gemv(a, st, nullptr);
}

// Reads (and clears) the error word of the no-allocation GEMVs of the current
// device after the work queued on `st` so far: *flag is non-zero if a bounded
// wait of one of them gave up since the last query.
cudaError_t gemv_noalloc_status(cudaStream_t st, uint32_t* flag) {
  NoallocPtrs p{};
  cudaError_t e = noalloc_scratch(&p);
  if (e != cudaSuccess) return e;
  uint32_t h = 0;
  e = cudaMemcpyAsync(&h, p.err, sizeof(h), cudaMemcpyDeviceToHost, st);
  if (e == cudaSuccess) e = cudaStreamSynchronize(st);
  if (e == cudaSuccess && h) e = cudaMemsetAsync(p.err, 0, sizeof(uint32_t), st);
  if (e == cudaSuccess && h) e = cudaStreamSynchronize(st);
  *flag = h;
  return e;
}

}  // namespace sm
