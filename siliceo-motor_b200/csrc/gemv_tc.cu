// Batch-1 GEMV of Q4_K / Q6_K weights on the tensor cores.
//
// A decode step is one matrix-vector product per weight, so the work is bound
// by HBM bandwidth only if turning a 4/6-bit weight into something that can be
// multiplied costs almost nothing. On the CUDA cores it does not (the f16->f32
// conversions run on the quarter-rate XU pipe), so here the weights go
// straight into mma.sync.m16n8k16 (f16 x f16 -> f32) as the A operand:
//   * a quantized value q (0..15, or -32..31 for Q6_K) is exact in f16 and is
//     made with one LOP3 (the nibble into the mantissa of 1024) and one HSUB2
//     or HFMA2, two weights at a time;
//   * x is split into hi + lo f16 halves after scaling each 256-wide block by
//     a power of two (hi = x rounded to 11 bits, lo = the exact remainder), so
//     the products carry ~22 bits of x, as much as the f32 reference keeps
//     within rounding of its own sum;
//   * the 8 columns of the MMA are (sub-block mod 4, hi/lo): each k16 chunk of
//     weights belongs to one sub-block and meets x only in that sub-block's
//     two columns, so the accumulators hold one dot product per (row,
//     sub-block) and the GGUF scales are applied once per block:
//       Q4_K: y += d*sc_s*sum_s(q*x) - dmin*m_s*sum_s(x)   (dequant.rs:98-124)
//       Q6_K: y += d*sc_s*sum_s((q-32)*x)                  (dequant.rs:178-206)
// The weights stream from HBM once (tile layout, device.cuh) with a one-block
// register prefetch and L2 prefetches further ahead; x is converted once per
// CTA into shared memory, already in each lane's B-fragment order.
//
// Work: a unit is (8 tiles of 16 rows, K-slice). Warp w of a CTA owns tile
// w of the unit. When there are too few tiles to fill the GPU, K is split and
// the CTA that finishes a group last sums the slices in order (deterministic)
// and runs the epilogue. Epilogues are the fused ones of gemv_common.cuh.
#include <cuda_fp16.h>

#include <algorithm>
#include <mutex>
#include <type_traits>

#include "device.cuh"
#include "gemv_common.cuh"

namespace sm {

constexpr int TC_WARPS = 8, TC_THREADS = TC_WARPS * 32;
constexpr uint32_t TC_FRAG = 4096;             // expanded B fragments of one block, one type
constexpr uint32_t TC_XS = 64;                 // per block: 4 lanes' (X_t, X_t+4, 1/scale, 0)
constexpr uint32_t TC_SMEM_MAX = 200u * 1024u;
constexpr uint32_t TC_PREFETCH = 4;            // L2 prefetch distance, in blocks

struct TcPlan {
  uint32_t tiles, groups, ksplit, slice, units, grid, smem, t4, t6;
};

__device__ __forceinline__ void mma16816(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                         uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}
__device__ __forceinline__ uint32_t h2u(__half2 h) { return *reinterpret_cast<uint32_t*>(&h); }
__device__ __forceinline__ __half2 u2h(uint32_t u) { return *reinterpret_cast<__half2*>(&u); }
__device__ __forceinline__ void prefetch_l2(const void* p) { asm volatile("prefetch.global.L2 [%0];" ::"l"(p)); }

// Low nibbles of bytes (0, 2) as the exact half2 (q0, q2).
__device__ __forceinline__ uint32_t nib_lo(uint32_t w) {
  return h2u(__hsub2(u2h((w & 0x000F000Fu) | 0x64006400u), __floats2half2_rn(1024.f, 1024.f)));
}
// High nibbles of bytes (0, 2): (1024 + 16q) / 16 - 64, exact.
__device__ __forceinline__ uint32_t nib_hi(uint32_t w) {
  return h2u(__hfma2(u2h((w & 0x00F000F0u) | 0x64006400u), __floats2half2_rn(0.0625f, 0.0625f),
                     __floats2half2_rn(-64.f, -64.f)));
}
// Q6_K: 6-bit values (low nibble + 2 bits of h at 4-5 / 20-21) minus 32.
__device__ __forceinline__ uint32_t q6_lo(uint32_t w, uint32_t h) {
  return h2u(__hsub2(u2h((w & 0x000F000Fu) | 0x64006400u | (h & 0x00300030u)), __floats2half2_rn(1056.f, 1056.f)));
}
// Q6_K: high nibble + 2 bits of h at 8-9 / 24-25, as (1024 + 16v) / 16 - 96.
__device__ __forceinline__ uint32_t q6_hi(uint32_t w, uint32_t h) {
  return h2u(__hfma2(u2h((w & 0x00F000F0u) | 0x64006400u | (h & 0x03000300u)), __floats2half2_rn(0.0625f, 0.0625f),
                     __floats2half2_rn(-96.f, -96.f)));
}

// x (already scaled) -> (hi, lo): hi keeps 11 significant bits (round half
// away from zero on the magnitude), lo = x - hi exactly.
__device__ __forceinline__ float hi11(float v) { return __uint_as_float((__float_as_uint(v) + 0x1000u) & 0xFFFFE000u); }
__device__ __forceinline__ uint32_t hl_pair(float a, float b, bool lo) {
  const float ah = hi11(a), bh = hi11(b);
  return lo ? h2u(__floats2half2_rn(a - ah, b - bh)) : h2u(__floats2half2_rn(ah, bh));
}

// Converts block bl (global block b) of x into shared memory: per type the
// expanded B fragments [8 chunk pairs][32 lanes][4 words] (zero where the
// chunk's sub-block is not the lane's column), and per lane t of the Q4_K
// epilogue (X_t, X_t+4, 1/scale). One warp per block.
__device__ __forceinline__ void tc_build_x(const float* __restrict__ xb, uint4* f4, uint4* f6, float4* xs, bool t4,
                                           bool t6) {
  const int lane = threadIdx.x & 31, g = lane >> 2, t = lane & 3, u = g >> 1;
  const bool lo = g & 1;
  float4 v4[4], v6[4];
  float mx = 0.f;
  if (t4) {
#pragma unroll
    for (int i = 0; i < 4; i++) {  // runs of sub-blocks u, u+4 (i >> 1), halves c = i & 1
      v4[i] = ldg4(xb + 32 * (u + 4 * (i >> 1)) + 8 * t + 4 * (i & 1));
      mx = fmaxf(mx, fmaxf(fmaxf(fabsf(v4[i].x), fabsf(v4[i].y)), fmaxf(fabsf(v4[i].z), fabsf(v4[i].w))));
    }
  }
  if (t6) {
#pragma unroll
    for (int i = 0; i < 4; i++) {  // sub-block u + 4i, offsets 4t..4t+3
      v6[i] = ldg4(xb + 16 * (u + 4 * i) + 4 * t);
      mx = fmaxf(mx, fmaxf(fmaxf(fabsf(v6[i].x), fabsf(v6[i].y)), fmaxf(fabsf(v6[i].z), fabsf(v6[i].w))));
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
  // scale = 2^(141 - E) puts max|x| in [2^14, 2^15): hi stays below the f16 maximum.
  const uint32_t E = (__float_as_uint(mx) >> 23) & 0xFFu;
  const float scl = E >= 15u ? __uint_as_float((268u - E) << 23) : 1.0f;
  const float inv = E >= 15u ? __uint_as_float((E - 14u) << 23) : 1.0f;
  if (t4) {
    uint4 w[2];
#pragma unroll
    for (int i = 0; i < 2; i++) {
      const float4 a = v4[2 * i], c = v4[2 * i + 1];
      w[i] = make_uint4(hl_pair(a.x * scl, a.z * scl, lo), hl_pair(a.y * scl, a.w * scl, lo),
                        hl_pair(c.x * scl, c.z * scl, lo), hl_pair(c.y * scl, c.w * scl, lo));
    }
    const uint4 z = make_uint4(0, 0, 0, 0);
#pragma unroll
    for (int p = 0; p < 8; p++) f4[p * 32 + lane] = p == u ? w[0] : (p == u + 4 ? w[1] : z);
    // sums of x over sub-blocks u and u + 4 (unscaled), over the 4 lanes t
    float s0 = sum4(v4[0]) + sum4(v4[1]), s1 = sum4(v4[2]) + sum4(v4[3]);
    s0 += __shfl_xor_sync(0xffffffffu, s0, 1);
    s1 += __shfl_xor_sync(0xffffffffu, s1, 1);
    s0 += __shfl_xor_sync(0xffffffffu, s0, 2);
    s1 += __shfl_xor_sync(0xffffffffu, s1, 2);
    if (!lo && t == 0) xs[u] = make_float4(s0, s1, inv, 0.f);
  } else if (lane < 4) {
    xs[lane] = make_float4(0.f, 0.f, inv, 0.f);
  }
  if (t6) {
    const uint4 z = make_uint4(0, 0, 0, 0);
    uint2 w[4];
#pragma unroll
    for (int i = 0; i < 4; i++) {
      const float4 a = v6[i];
      w[i] = make_uint2(hl_pair(a.x * scl, a.z * scl, lo), hl_pair(a.y * scl, a.w * scl, lo));
    }
    // chunk s = u + 4i sits in pair s >> 1, words 2*(s & 1) and 2*(s & 1) + 1
#pragma unroll
    for (int p = 0; p < 8; p++) {
      uint4 v = z;
#pragma unroll
      for (int i = 0; i < 4; i++)
        if (((u + 4 * i) >> 1) == p) v = (u & 1) ? make_uint4(0, 0, w[i].x, w[i].y) : make_uint4(w[i].x, w[i].y, 0, 0);
      f6[p * 32 + lane] = v;
    }
  }
}

// ------------------------------------------------------------- Q4_K ----
// The register pipeline carries the quant bytes; the small per-row headers are
// read when the block is computed (the L2 prefetch has brought them in).
struct Q4Buf {
  uint4 q[4];  // loads 0..3 of the lane (rows g, g+8)
};
__device__ __forceinline__ void q4_load(Q4Buf& B, const uint8_t* unit, int lane) {
  const uint8_t* qs = unit + 256 + 16 * lane;
#pragma unroll
  for (int L = 0; L < 4; L++) B.q[L] = ld_stream(qs + 512 * L);
}
__device__ __forceinline__ float q4_row(const uint4& hd, int t, float P0, float P1, const float4& xs) {
  const float d = h2f_ref(hd.x & 0xFFFFu) * xs.z, dmin = h2f_ref(hd.x >> 16);
  const int s0 = 8 * t;  // get_scale_min_k4 of sub-blocks t and t + 4 (dequant.rs:41-49)
  const uint32_t sa = (hd.y >> s0) & 63u, ma = (hd.z >> s0) & 63u;
  const uint32_t sb = ((hd.w >> s0) & 0xFu) | (((hd.y >> (s0 + 6)) & 3u) << 4);
  const uint32_t mb = ((hd.w >> (s0 + 4)) & 0xFu) | (((hd.z >> (s0 + 6)) & 3u) << 4);
  return d * ((float)sa * P0 + (float)sb * P1) - dmin * ((float)ma * xs.x + (float)mb * xs.y);
}
__device__ __forceinline__ void q4_block(const Q4Buf& B, const uint8_t* unit, const uint4* __restrict__ f4,
                                         const float4* __restrict__ xs, int lane, float& rg, float& rh) {
  const uint4 hg = ldg_u4(unit + 16 * (lane >> 2)), hh = ldg_u4(unit + 16 * ((lane >> 2) + 8));
  float acc[2][4] = {};
#pragma unroll
  for (int s = 0; s < 8; s++) {
    const uint4 bf = f4[s * 32 + lane];
    const int j = s >> 1;
    const uint4 Lg = j < 2 ? B.q[0] : B.q[1], Lh = j < 2 ? B.q[2] : B.q[3];
    const uint32_t ga = (j & 1) ? Lg.z : Lg.x, gb = (j & 1) ? Lg.w : Lg.y;
    const uint32_t ha = (j & 1) ? Lh.z : Lh.x, hb = (j & 1) ? Lh.w : Lh.y;
    if (s & 1) {
      mma16816(acc[s >> 2], nib_hi(ga), nib_hi(ha), nib_hi(ga >> 8), nib_hi(ha >> 8), bf.x, bf.y);
      mma16816(acc[s >> 2], nib_hi(gb), nib_hi(hb), nib_hi(gb >> 8), nib_hi(hb >> 8), bf.z, bf.w);
    } else {
      mma16816(acc[s >> 2], nib_lo(ga), nib_lo(ha), nib_lo(ga >> 8), nib_lo(ha >> 8), bf.x, bf.y);
      mma16816(acc[s >> 2], nib_lo(gb), nib_lo(hb), nib_lo(gb >> 8), nib_lo(hb >> 8), bf.z, bf.w);
    }
  }
  const int t = lane & 3;
  const float4 x4 = xs[t];
  rg += q4_row(hg, t, acc[0][0] + acc[0][1], acc[1][0] + acc[1][1], x4);
  rh += q4_row(hh, t, acc[0][2] + acc[0][3], acc[1][2] + acc[1][3], x4);
}

// ------------------------------------------------------------- Q6_K ----
struct Q6Buf {
  uint4 q[6];  // ql 0-3, ql 4-7, qh of row g; the same of row g + 8
};
__device__ __forceinline__ void q6_load(Q6Buf& B, const uint8_t* unit, int lane) {
  const uint8_t* q = unit + Q6T_QOFF + 16 * lane;
#pragma unroll
  for (int L = 0; L < 6; L++) B.q[L] = ld_stream(q + 512 * L);
}
// Scales of sub-blocks t + 4a (a = 0..3) of one row half: word w of the row's
// 16 scale bytes holds sub-blocks 4w .. 4w+3.
__device__ __forceinline__ float q6_half(uint32_t w0, uint32_t w1, int t, const float (&acc)[2][4], int c) {
  const int sh = 8 * t;
  const float s0 = (float)(int8_t)((w0 >> sh) & 0xFFu), s1 = (float)(int8_t)((w1 >> sh) & 0xFFu);
  return s0 * (acc[0][c] + acc[0][c + 1]) + s1 * (acc[1][c] + acc[1][c + 1]);
}
__device__ __forceinline__ float q6_d(uint32_t dbits, float inv) {
  const float d = h2f_ref(dbits);
  return isfinite(d) ? d * inv : 0.f;  // the reference skips such a block (kernels/src/lib.rs:845)
}
// Two passes: sub-blocks 0-7 (low nibbles of the 8 ql words), then 8-15 (high
// nibbles), each into two accumulators that are scaled before the next pass.
__device__ __forceinline__ void q6_block(const Q6Buf& B, const uint8_t* unit, const uint4* __restrict__ f6,
                                         const float4* __restrict__ xs, int lane, float& rg, float& rh) {
  const int g = lane >> 2, t = lane & 3;
  const uint32_t gw[8] = {B.q[0].x, B.q[0].y, B.q[0].z, B.q[0].w, B.q[1].x, B.q[1].y, B.q[1].z, B.q[1].w};
  const uint32_t hw[8] = {B.q[3].x, B.q[3].y, B.q[3].z, B.q[3].w, B.q[4].x, B.q[4].y, B.q[4].z, B.q[4].w};
  const uint32_t gq[4] = {B.q[2].x, B.q[2].y, B.q[2].z, B.q[2].w};
  const uint32_t hq[4] = {B.q[5].x, B.q[5].y, B.q[5].z, B.q[5].w};
  float pg = 0.f, ph = 0.f;
#pragma unroll
  for (int pass = 0; pass < 2; pass++) {
    float acc[2][4] = {};
#pragma unroll
    for (int i = 0; i < 8; i += 2) {
      const uint4 bf = f6[(4 * pass + (i >> 1)) * 32 + lane];  // chunks 8*pass + i, + 1
#pragma unroll
      for (int e = 0; e < 2; e++) {
        const int k = i + e;
        const uint32_t wg = gw[k], wh = hw[k];
        const uint32_t qg = e ? __funnelshift_r(gq[k >> 1], gq[k >> 1], 8) : gq[k >> 1];
        const uint32_t qh = e ? __funnelshift_r(hq[k >> 1], hq[k >> 1], 8) : hq[k >> 1];
        const uint32_t b0 = e ? bf.z : bf.x, b1 = e ? bf.w : bf.y;
        if (pass == 0)
          mma16816(acc[k >> 2], q6_lo(wg, qg), q6_lo(wh, qh), q6_lo(wg >> 8, qg >> 2), q6_lo(wh >> 8, qh >> 2), b0, b1);
        else
          mma16816(acc[k >> 2], q6_hi(wg, qg), q6_hi(wh, qh), q6_hi(wg >> 8, qg >> 2), q6_hi(wh >> 8, qh >> 2), b0, b1);
      }
    }
    const uint2 sg = __ldg(reinterpret_cast<const uint2*>(unit + 16 * g + 8 * pass));
    const uint2 sh = __ldg(reinterpret_cast<const uint2*>(unit + 16 * (g + 8) + 8 * pass));
    pg += q6_half(sg.x, sg.y, t, acc, 0);
    ph += q6_half(sh.x, sh.y, t, acc, 2);
  }
  const float inv = xs[t].z;
  rg += q6_d(__ldg(reinterpret_cast<const unsigned short*>(unit + 256) + g), inv) * pg;
  rh += q6_d(__ldg(reinterpret_cast<const unsigned short*>(unit + 256) + g + 8), inv) * ph;
}

// One warp: tile rows g, g+8 over blocks b0 .. b0+nblk-1 (x fragments of
// block b0 + i at slot i). Returns the partial dot products in rg, rh
// (summed over the lane's sub-blocks only).
template <int QT>
__device__ __forceinline__ void tc_tile(const uint8_t* tile, uint32_t b0, uint32_t nblk, uint32_t nb,
                                        const uint4* f, const float4* xs, float& rg, float& rh) {
  const int lane = threadIdx.x & 31;
  constexpr uint32_t UB = QT == 12 ? Q4T_UNIT : Q6T_UNIT;
  using Buf = typename std::conditional<QT == 12, Q4Buf, Q6Buf>::type;
  auto load = [&](Buf& B, uint32_t i) {
    const uint8_t* unit = tile + (size_t)(b0 + i) * UB;
    const uint32_t pf = b0 + i + TC_PREFETCH;
    if (pf < nb && (uint32_t)lane * 128u < UB) prefetch_l2(tile + (size_t)pf * UB + 128u * lane);
    if constexpr (QT == 12) q4_load(B, unit, lane);
    else q6_load(B, unit, lane);
  };
  auto run = [&](const Buf& B, uint32_t i) {
    const uint8_t* unit = tile + (size_t)(b0 + i) * UB;
    if constexpr (QT == 12) q4_block(B, unit, f + (size_t)i * 256, xs + 4 * i, lane, rg, rh);
    else q6_block(B, unit, f + (size_t)i * 256, xs + 4 * i, lane, rg, rh);
  };
  if (!nblk) return;
  // first TC_PREFETCH blocks go to L2 ahead of the register pipeline
  for (uint32_t i = 1; i < TC_PREFETCH && i < nblk; i++)
    if ((uint32_t)lane * 128u < UB) prefetch_l2(tile + (size_t)(b0 + i) * UB + 128u * lane);
  Buf A, B;
  load(A, 0);
  for (uint32_t i = 0; i < nblk; i += 2) {
    if (i + 1 < nblk) load(B, i + 1);
    run(A, i);
    if (i + 1 >= nblk) break;
    if (i + 2 < nblk) load(A, i + 2);
    run(B, i + 1);
  }
}

// Epilogue of one tile: vg / vh are the full dot products of rows g, g + 8
// (in every lane of the group).
__device__ __forceinline__ void tc_epilogue(const GemvArgs& a, uint32_t tile, float vg, float vh) {
  const int lane = threadIdx.x & 31, g = lane >> 2, t = lane & 3;
  uint32_t si = 0;
  if (a.nseg > 1 && tile >= a.seg[1].cta_begin) si = 1;
  if (a.nseg > 2 && tile >= a.seg[2].cta_begin) si = 2;
  const GemvSeg& sg = a.seg[si];
  const uint32_t row0 = (tile - sg.cta_begin) * 16u;
  if (epi_is_pair(sg.epi)) {
    const float ng = __shfl_down_sync(0xffffffffu, vg, 4), nh = __shfl_down_sync(0xffffffffu, vh, 4);
    if (!(g & 1) && t < 2) {
      const uint32_t o = row0 + (uint32_t)g + 8u * (uint32_t)t;
      if (o < sg.w.n_out) epi_pair(a, sg, o, 0, t ? vh : vg, t ? nh : ng);
    }
  } else {
    float xn = 0.f;
    if (t < 2) {
      const uint32_t o = row0 + (uint32_t)g + 8u * (uint32_t)t;
      if (o < sg.w.n_out) xn = epi_single(a, sg, o, 0, t ? vh : vg);
    }
    if (sg.epi == EPI_RESID) {  // partial sum of x^2 over the tile's rows
      const float s2 = warp_sum(xn * xn);
      if (lane == 0) a.out_parts[tile] = s2;
    }
  }
}

__global__ void __launch_bounds__(TC_THREADS, 1) gemv_tc_kernel(const __grid_constant__ GemvArgs a,
                                                                const __grid_constant__ TcPlan p) {
  extern __shared__ __align__(16) uint8_t tc_smem[];
  __shared__ float s_in;
  __shared__ uint32_t s_last;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  uint4* f4 = reinterpret_cast<uint4*>(tc_smem);
  uint4* f6 = f4 + (p.t4 ? p.slice * 256 : 0);
  float4* xs = reinterpret_cast<float4*>(f6 + (p.t6 ? p.slice * 256 : 0));
  const uint32_t nb = a.seg[0].w.n_in >> 8;
  if (warp == 0) {
    const float v = input_scale(a, 0);
    if (lane == 0) s_in = v;
  }
  for (uint32_t unit = blockIdx.x; unit < p.units; unit += gridDim.x) {
    const uint32_t rg = unit / p.ksplit, ks = unit - rg * p.ksplit;
    const uint32_t b0 = ks * p.slice, nblk = min(p.slice, nb - b0);
    __syncthreads();  // the previous unit is done with the x fragments
    for (uint32_t i = warp; i < nblk; i += TC_WARPS)
      tc_build_x(a.x + (size_t)(b0 + i) * 256, f4 + i * 256, f6 + i * 256, xs + 4 * i, p.t4, p.t6);
    __syncthreads();
    const uint32_t tile = rg * TC_WARPS + warp;
    float vg = 0.f, vh = 0.f;
    if (tile < p.tiles) {
      uint32_t si = 0;
      if (a.nseg > 1 && tile >= a.seg[1].cta_begin) si = 1;
      if (a.nseg > 2 && tile >= a.seg[2].cta_begin) si = 2;
      const DWDesc& w = a.seg[si].w;
      const uint8_t* tb = w.body + (size_t)(tile - a.seg[si].cta_begin) * w.body_stride;
      if (w.type == 12) tc_tile<12>(tb, b0, nblk, nb, f4, xs, vg, vh);
      else tc_tile<14>(tb, b0, nblk, nb, f6, xs, vg, vh);
    }
    vg += __shfl_xor_sync(0xffffffffu, vg, 1);
    vh += __shfl_xor_sync(0xffffffffu, vh, 1);
    vg += __shfl_xor_sync(0xffffffffu, vg, 2);
    vh += __shfl_xor_sync(0xffffffffu, vh, 2);
    if (p.ksplit == 1) {
      if (tile < p.tiles) tc_epilogue(a, tile, vg * s_in, vh * s_in);
      continue;
    }
    // K-split: publish this slice, the last CTA of the group sums the slices in order.
    const size_t stride = (size_t)p.tiles * 16u;
    const int g = lane >> 2, t = lane & 3;
    if (tile < p.tiles && t < 2) a.ks_part[ks * stride + tile * 16u + g + 8u * t] = t ? vh : vg;
    __threadfence();
    __syncthreads();
    if (threadIdx.x == 0) s_last = atomicAdd(&a.ks_cnt[rg], 1u) == p.ksplit - 1;
    __syncthreads();
    if (s_last) {
      __threadfence();
      if (tile < p.tiles) {
        float sg = 0.f, sh = 0.f;
        for (uint32_t k = 0; k < p.ksplit; k++) {
          sg += __ldcg(a.ks_part + k * stride + tile * 16u + g);
          sh += __ldcg(a.ks_part + k * stride + tile * 16u + g + 8u);
        }
        tc_epilogue(a, tile, sg * s_in, sh * s_in);
      }
      if (threadIdx.x == 0) a.ks_cnt[rg] = 0;  // ready for the next launch
    }
  }
}

// ------------------------------------------------------------- host ----
bool gemv_tc_ok(const GemvArgs& a) {
  if (a.batch != 1 || !a.nseg) return false;
  for (uint32_t i = 0; i < a.nseg; i++) {
    const DWDesc& w = a.seg[i].w;
    if (!tiled_type(w.type) || w.n_in != a.seg[0].w.n_in) return false;
  }
  return true;
}

constexpr int TC_MAX_DEVICES = 64;
static std::mutex g_tc_mu;
static int g_tc_sms[TC_MAX_DEVICES] = {};

static cudaError_t tc_setup(uint32_t* sms) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  if (dev < 0 || dev >= TC_MAX_DEVICES) return cudaErrorInvalidDevice;
  std::lock_guard<std::mutex> lk(g_tc_mu);
  if (!g_tc_sms[dev]) {
    int n = 0;
    e = cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
    if (e == cudaSuccess) e = cudaFuncSetAttribute(gemv_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, TC_SMEM_MAX);
    if (e != cudaSuccess) return e;
    g_tc_sms[dev] = n;
  }
  *sms = (uint32_t)g_tc_sms[dev];
  return cudaSuccess;
}

// Called at model load, so that no launch inside a graph capture does the set-up.
cudaError_t gemv_tc_prepare() {
  uint32_t sms = 0;
  return tc_setup(&sms);
}

// Tiles per segment (cta_begin = first tile), K-split and shared memory. The
// split is the smallest that gives every SM a unit, bounded by the scratch
// (a split that does not fit falls back to one slice when the x fragments of
// all of K fit in shared memory). Returns false when no plan fits.
static bool tc_plan(GemvArgs& a, uint32_t sms, TcPlan* p) {
  uint32_t tiles = 0;
  bool t4 = false, t6 = false;
  for (uint32_t i = 0; i < a.nseg; i++) {
    a.seg[i].cta_begin = tiles;
    tiles += (a.seg[i].w.n_out + 15) / 16;
    (a.seg[i].w.type == 12 ? t4 : t6) = true;
  }
  const uint32_t nb = a.seg[0].w.n_in >> 8;
  const uint32_t per_blk = (t4 ? TC_FRAG : 0) + (t6 ? TC_FRAG : 0) + TC_XS;
  const uint32_t slice_max = TC_SMEM_MAX / per_blk;
  const uint32_t groups = (tiles + TC_WARPS - 1) / TC_WARPS;
  uint32_t ks = std::max((nb + slice_max - 1) / slice_max, std::min(nb, std::max(1u, sms / groups)));
  auto fits = [&](uint32_t k) {
    return k == 1 || (a.ks_part && a.ks_cnt && (uint64_t)k * tiles * 16u <= a.ks_part_cap && groups <= a.ks_cnt_cap);
  };
  if (!fits(ks)) ks = 1;
  const uint32_t slice = (nb + ks - 1) / ks;
  if (slice > slice_max) return false;
  ks = (nb + slice - 1) / slice;
  if (!fits(ks)) return false;
  p->tiles = tiles;
  p->groups = groups;
  p->ksplit = ks;
  p->slice = slice;
  p->units = groups * ks;
  p->grid = std::min(p->units, sms);
  p->smem = slice * per_blk;
  p->t4 = t4;
  p->t6 = t6;
  return true;
}

// The number of per-tile partials an EPI_RESID launch writes (out_parts) is
// returned in n_parts. cudaErrorNotSupported: no plan fits (use another kernel).
cudaError_t launch_gemv_tc(GemvArgs a, cudaStream_t st, uint32_t* n_parts) {
  uint32_t sms = 0;
  cudaError_t e = tc_setup(&sms);
  if (e != cudaSuccess) return e;
  TcPlan p;
  if (!tc_plan(a, sms, &p)) return cudaErrorNotSupported;
  if (n_parts) *n_parts = p.tiles;
  gemv_tc_kernel<<<p.grid, TC_THREADS, p.smem, st>>>(a, p);
  return cudaGetLastError();
}

// Scratch a K-split of this launch shape may use (floats of partials, counters).
void gemv_tc_scratch_need(GemvArgs a, uint32_t sms, uint64_t* part, uint32_t* cnt) {
  a.ks_part = reinterpret_cast<float*>(16);  // any non-null: plan as if unbounded
  a.ks_cnt = reinterpret_cast<uint32_t*>(16);
  a.ks_part_cap = 0xFFFFFFFFu;
  a.ks_cnt_cap = 0xFFFFFFFFu;
  TcPlan p;
  *part = 0;
  *cnt = 0;
  if (!tc_plan(a, sms, &p) || p.ksplit == 1) return;
  *part = (uint64_t)p.ksplit * p.tiles * 16u;
  *cnt = p.groups;
}

}  // namespace sm
