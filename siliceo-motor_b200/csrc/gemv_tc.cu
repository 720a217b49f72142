// Batch-1 GEMV of Q4_K / Q6_K weights on the tensor cores.
//
// A decode step is one matrix-vector product per weight, so the work is bound
// by HBM bandwidth only if turning a 4/6-bit weight into something that can be
// multiplied costs almost nothing. On the CUDA cores it does not (the f16->f32
// conversions run on the quarter-rate XU pipe), so here the weights go
// straight into mma.sync.m16n8k16 (f16 x f16 -> f32) as the A operand:
//   * a quantized value q (0..15, or the 6-bit q + 32 of Q6_K) goes into the
//     mantissa of an f16 with a zero exponent field: a subnormal q * 2^-24
//     (or 16q * 2^-24 for a high nibble), exact, made with one AND (Q4_K) or
//     two LOP3s (Q6_K) per two weights; the power of two and Q6_K's -32
//     (as -32 * sum(x) over the sub-block) are applied with the scales;
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
// The weights stream from HBM once (tile layout, device.cuh): every warp runs
// its own ring of shared-memory slots filled by bulk asynchronous copies (one
// per 16-row block unit, completion on an mbarrier); x is converted once per
// unit into shared memory, already in each lane's B-fragment order.
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
#include "pdl.cuh"
#include "tc_common.cuh"

namespace sm {

constexpr int TC_WARPS = 16, TC_THREADS = TC_WARPS * 32;
constexpr uint32_t TC_FRAG = 1024;             // B fragments of one block, one type: [2][32 lanes][16 B]
// per block: [4 x (X32_t, X32_t+4, 1/scale, 0)][4 x (X16_t, X16_t+4, X16_t+8, X16_t+12)]
// (X32 / X16: sums of x over 32- / 16-wide sub-blocks, for lane t's epilogue)
constexpr uint32_t TC_XS = 128;
constexpr uint32_t TC_SMEM_MAX = 225u * 1024u;
// Ring slots per warp: 16 warps x 2-3 slots of one block unit each keep HBM
// saturated; deeper rings (more requests in flight) lose bandwidth, and so do
// L2 prefetches ahead of the ring (both measured on B200).
constexpr uint32_t TC_MAX_STAGES = 3;

struct TcPlan {
  uint32_t tiles, groups, ksplit, slice, units, grid, smem, t4, t6;
  uint32_t stages, stage_bytes;  // per-warp cp.async ring of weight units
};

// B operand of the chunks of sub-block s: the lane's fragment words when s is
// in its column (s & 3 == u), else zero. fb[k] is the shared address the lane
// reads for sub-blocks s with s & 3 == k: its fragment slot of the current
// block, or a zero page (the fragments of the lane's sub-blocks u + 4 sigma
// sit sigma * 512 bytes apart; the zero page is 1 KB).

// Converts block bl (global block b) of x into shared memory: per type the
// lane's B fragments [2][32 lanes][4 words] for the sub-blocks of its column
// (u = lane >> 3: u, u + 4 for Q4_K; u, u + 4, u + 8, u + 12 for Q6_K; the
// MMA loops zero them for the other sub-blocks), and the x sums and the
// block's 1/scale for the epilogues. One warp per block.
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
    f4[lane] = w[0];       // sub-block u: chunk halves c = 0 (x, y), 1 (z, w)
    f4[32 + lane] = w[1];  // sub-block u + 4
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
    float q[4];  // sums over the 16-wide sub-blocks u + 4i, over the 4 lanes t
#pragma unroll
    for (int i = 0; i < 4; i++) {
      q[i] = sum4(v6[i]);
      q[i] += __shfl_xor_sync(0xffffffffu, q[i], 1);
      q[i] += __shfl_xor_sync(0xffffffffu, q[i], 2);
    }
    if (!lo && t == 0) xs[4 + u] = make_float4(q[0], q[1], q[2], q[3]);
    uint2 w[4];
#pragma unroll
    for (int i = 0; i < 4; i++) {
      const float4 a = v6[i];
      w[i] = make_uint2(hl_pair(a.x * scl, a.z * scl, lo), hl_pair(a.y * scl, a.w * scl, lo));
    }
    f6[lane] = make_uint4(w[0].x, w[0].y, w[1].x, w[1].y);       // sub-blocks u, u + 4
    f6[32 + lane] = make_uint4(w[2].x, w[2].y, w[3].x, w[3].y);  // sub-blocks u + 8, u + 12
  }
}

// ------------------------------------------------------------- Q4_K ----
// A block of a tile is computed from its unit in shared memory (st).
struct Q4Buf {
  uint4 q[4];  // loads 0..3 of the lane (rows g, g+8)
};
__device__ __forceinline__ void q4_load(Q4Buf& B, const uint8_t* st, int lane) {
  const uint4* qs = reinterpret_cast<const uint4*>(st + 256) + lane;
#pragma unroll
  for (int L = 0; L < 4; L++) B.q[L] = qs[32 * L];
}
// P0 / P1: the MMA sums of sub-blocks t and t + 4, times 2^-24 (t even: low
// nibbles) or 2^-20 (t odd: high nibbles) and the block's x scale.
__device__ __forceinline__ float q4_row(const uint4& hd, int t, float P0, float P1, const float4& xs) {
  const float d = h2f_ref(hd.x & 0xFFFFu) * (xs.z * ((t & 1) ? 1048576.f : 16777216.f)), dmin = h2f_ref(hd.x >> 16);
  const int s0 = 8 * t;  // get_scale_min_k4 of sub-blocks t and t + 4 (dequant.rs:41-49)
  const uint32_t sa = (hd.y >> s0) & 63u, ma = (hd.z >> s0) & 63u;
  const uint32_t sb = ((hd.w >> s0) & 0xFu) | (((hd.y >> (s0 + 6)) & 3u) << 4);
  const uint32_t mb = ((hd.w >> (s0 + 4)) & 0xFu) | (((hd.z >> (s0 + 6)) & 3u) << 4);
  return d * ((float)sa * P0 + (float)sb * P1) - dmin * ((float)ma * xs.x + (float)mb * xs.y);
}
__device__ __forceinline__ void q4_block(const uint8_t* st, const uint32_t (&fb)[4], const float4* __restrict__ xs,
                                         int lane, float& rg, float& rh) {
  Q4Buf B;
  q4_load(B, st, lane);
  const uint4 hg = reinterpret_cast<const uint4*>(st)[lane >> 2], hh = reinterpret_cast<const uint4*>(st)[(lane >> 2) + 8];
  // acc[s >> 2]: sub-blocks 0-3 / 4-7, the two chains alternate
  float acc[2][4] = {};
#pragma unroll
  for (int s4 = 0; s4 < 4; s4++) {
#pragma unroll
    for (int hi = 0; hi < 2; hi++) {
      const int s = s4 + 4 * hi, j = s >> 1;
      const uint4 bf = hi ? lds128<512>(fb[s4]) : lds128<0>(fb[s4]);
      const uint4 Lg = j < 2 ? B.q[0] : B.q[1], Lh = j < 2 ? B.q[2] : B.q[3];
      const uint32_t ga = (j & 1) ? Lg.z : Lg.x, gb = (j & 1) ? Lg.w : Lg.y;
      const uint32_t ha = (j & 1) ? Lh.z : Lh.x, hb = (j & 1) ? Lh.w : Lh.y;
      const uint32_t b0 = bf.x, b1 = bf.y, b2 = bf.z, b3 = bf.w;
      if (s & 1) {
        mma16816(acc[hi], nib_hi(ga), nib_hi(ha), nib_hi(ga >> 8), nib_hi(ha >> 8), b0, b1);
        mma16816(acc[hi], nib_hi(gb), nib_hi(hb), nib_hi(gb >> 8), nib_hi(hb >> 8), b2, b3);
      } else {
        mma16816(acc[hi], nib_lo(ga), nib_lo(ha), nib_lo(ga >> 8), nib_lo(ha >> 8), b0, b1);
        mma16816(acc[hi], nib_lo(gb), nib_lo(hb), nib_lo(gb >> 8), nib_lo(hb >> 8), b2, b3);
      }
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
__device__ __forceinline__ void q6_load(Q6Buf& B, const uint8_t* st, int lane) {
  const uint4* q = reinterpret_cast<const uint4*>(st + Q6T_QOFF) + lane;
#pragma unroll
  for (int L = 0; L < 6; L++) B.q[L] = q[32 * L];
}
// Pass p of a Q6_K row: sub-blocks s = 8p + t and 8p + t + 4 (scale bytes t of
// words w0, w1), MMA sums D * 2^-24 (p = 0) or 2^-20 (p = 1) times the x
// scale (F undoes both), minus 32 * sum(x) for the +32 of the stored values.
__device__ __forceinline__ float q6_half(uint32_t w0, uint32_t w1, int t, const float (&acc)[2][4], int c, float F,
                                         float X0, float X1) {
  const int sh = 8 * t;
  const float s0 = (float)(int8_t)((w0 >> sh) & 0xFFu), s1 = (float)(int8_t)((w1 >> sh) & 0xFFu);
  return s0 * fmaf(F, acc[0][c] + acc[0][c + 1], -32.f * X0) + s1 * fmaf(F, acc[1][c] + acc[1][c + 1], -32.f * X1);
}
// Two passes: sub-blocks 0-7 (low nibbles of the 8 ql words), then 8-15 (high
// nibbles), each into two accumulators that are scaled before the next pass.
__device__ __forceinline__ void q6_block(const uint8_t* unit, const uint32_t (&fb)[4], const float4* __restrict__ xs,
                                         int lane, float& rg, float& rh) {
  const int g = lane >> 2, t = lane & 3;
  Q6Buf B;
  q6_load(B, unit, lane);
  const float4 x16 = xs[4 + t];
  const uint32_t gw[8] = {B.q[0].x, B.q[0].y, B.q[0].z, B.q[0].w, B.q[1].x, B.q[1].y, B.q[1].z, B.q[1].w};
  const uint32_t hw[8] = {B.q[3].x, B.q[3].y, B.q[3].z, B.q[3].w, B.q[4].x, B.q[4].y, B.q[4].z, B.q[4].w};
  const uint32_t gq[4] = {B.q[2].x, B.q[2].y, B.q[2].z, B.q[2].w};
  const uint32_t hq[4] = {B.q[5].x, B.q[5].y, B.q[5].z, B.q[5].w};
  float pg = 0.f, ph = 0.f;
#pragma unroll
  for (int pass = 0; pass < 2; pass++) {
    float acc[2][4] = {};
#pragma unroll
    for (int i = 0; i < 4; i += 2) {
#pragma unroll
      for (int e = 0; e < 4; e++) {  // words i, i + 4, i + 1, i + 5: the two accumulators alternate
        const int k = i + (e >> 1) + 4 * (e & 1);
        const int sb = 8 * pass + k, sig = sb >> 2;  // sub-block; its fragment: slot sig >> 1, words 2*(sig & 1) ..
        const uint2 bf = sig == 0 ? lds64<0>(fb[sb & 3]) : sig == 1 ? lds64<8>(fb[sb & 3])
                       : sig == 2 ? lds64<512>(fb[sb & 3]) : lds64<520>(fb[sb & 3]);
        const uint32_t wg = gw[k], wh = hw[k];
        const uint32_t qg = (k & 1) ? __funnelshift_r(gq[k >> 1], gq[k >> 1], 8) : gq[k >> 1];
        const uint32_t qh = (k & 1) ? __funnelshift_r(hq[k >> 1], hq[k >> 1], 8) : hq[k >> 1];
        const uint32_t b0 = bf.x, b1 = bf.y;
        if (pass == 0)
          mma16816(acc[k >> 2], q6_lo(wg, qg), q6_lo(wh, qh), q6_lo(wg >> 8, qg >> 2), q6_lo(wh >> 8, qh >> 2), b0, b1);
        else
          mma16816(acc[k >> 2], q6_hi(wg, qg), q6_hi(wh, qh), q6_hi(wg >> 8, qg >> 2), q6_hi(wh >> 8, qh >> 2), b0, b1);
      }
    }
    const uint2 sg = *reinterpret_cast<const uint2*>(unit + 16 * g + 8 * pass);
    const uint2 sh = *reinterpret_cast<const uint2*>(unit + 16 * (g + 8) + 8 * pass);
    const float F = xs[t].z * (pass ? 1048576.f : 16777216.f);
    const float X0 = pass ? x16.z : x16.x, X1 = pass ? x16.w : x16.y;
    pg += q6_half(sg.x, sg.y, t, acc, 0, F, X0, X1);
    ph += q6_half(sh.x, sh.y, t, acc, 2, F, X0, X1);
  }
  rg += q6_d(reinterpret_cast<const unsigned short*>(unit + 256)[g]) * pg;
  rh += q6_d(reinterpret_cast<const unsigned short*>(unit + 256)[g + 8]) * ph;
}

// One warp: tile rows g, g+8 over blocks b0 .. b0+nblk-1 (x fragments of
// block b0 + i at slot i). The block units stream through the warp's ring of
// S shared-memory slots: lane 0 starts one bulk copy per unit, S - 1 units
// ahead of the one being computed, each completing on the slot's mbarrier
// (use n of the ring waits for parity (n / S) & 1; nuse counts the warp's
// uses across units). Returns the partial dot products in rg, rh (summed
// over the lane's sub-blocks only).
// The first `pre` copies may have been started by the caller already (ahead
// of the previous kernel, pdl.cuh).
template <int QT, int S>
__device__ __forceinline__ void tc_tile(const uint8_t* tile, uint32_t b0, uint32_t nblk, uint32_t pre, uint8_t* ring,
                                        uint32_t stage_bytes, uint64_t* bars, uint32_t& nuse, uint32_t* err,
                                        const uint4* f, const float4* xs, uint32_t zero_page, float& rg, float& rh) {
  const int lane = threadIdx.x & 31;
  constexpr uint32_t UB = QT == 12 ? Q4T_UNIT : Q6T_UNIT;
  // ring slot of the next copy to start (ip) and of the next block to compute (cp, phase cph)
  uint32_t ip = nuse % S, cp = ip, cph = (nuse / S) & 1u;
  for (uint32_t k = 0; k < pre; k++) ip = ip + 1 == S ? 0 : ip + 1;
  auto issue = [&](uint32_t i) {
    if (i >= nblk) return;
    if (lane == 0) tc_issue(tile + (size_t)(b0 + i) * UB, UB, ring, stage_bytes, bars, ip);
    ip = ip + 1 == S ? 0 : ip + 1;
  };
  for (uint32_t k = pre; k + 1 < S; k++) issue(k);
  uint32_t fb[4], dk[4];
#pragma unroll
  for (int k = 0; k < 4; k++) {
    fb[k] = (lane >> 3) == k ? smem_u32(f + lane) : zero_page;
    dk[k] = (lane >> 3) == k ? 1024u : 0u;  // fragments of one block, one type
  }
  for (uint32_t i = 0; i < nblk; i++) {
    issue(i + S - 1);
    mbar_wait(bars + cp, cph, err);
    const uint8_t* sp = ring + cp * stage_bytes;
    if (++cp == S) { cp = 0; cph ^= 1u; }
    if constexpr (QT == 12) q4_block(sp, fb, xs + 8 * i, lane, rg, rh);
    else q6_block(sp, fb, xs + 8 * i, lane, rg, rh);
#pragma unroll
    for (int k = 0; k < 4; k++) fb[k] += dk[k];  // next block's fragment slot (the zero page stays)
    __syncwarp();  // every lane is done with the slot before it is refilled
  }
  nuse += nblk;
}

// Segment of a tile (cta_begin holds each segment's first tile).
__device__ __forceinline__ uint32_t tc_seg(const GemvArgs& a, uint32_t tile) {
  uint32_t si = 0;
  if (a.nseg > 1 && tile >= a.seg[1].cta_begin) si = 1;
  if (a.nseg > 2 && tile >= a.seg[2].cta_begin) si = 2;
  return si;
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
  __shared__ __align__(8) uint64_t s_bars[TC_WARPS * TC_MAX_STAGES];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  uint4* f4 = reinterpret_cast<uint4*>(tc_smem);
  uint4* f6 = f4 + (p.t4 ? p.slice * 64 : 0);
  float4* xs = reinterpret_cast<float4*>(f6 + (p.t6 ? p.slice * 64 : 0));
  uint8_t* ring = reinterpret_cast<uint8_t*>(xs + 8 * p.slice) + (size_t)warp * p.stages * p.stage_bytes;
  const uint32_t nb = a.seg[0].w.n_in >> 8;
  uint64_t* bars = s_bars + warp * TC_MAX_STAGES;
  if (lane == 0) {
    for (uint32_t k = 0; k < p.stages; k++) mbar_init(bars + k, 1);
    fence_mbar_init();
  }
  __syncwarp();
  uint32_t nuse = 0;
  __shared__ __align__(16) uint4 s_zero[64];  // 1 KB zero page for the B operands of other columns
  for (uint32_t i = threadIdx.x; i < 64; i += blockDim.x) s_zero[i] = make_uint4(0, 0, 0, 0);
  const uint32_t zero_page = smem_u32(s_zero);
  // The weights do not depend on the previous kernel: start the first unit's
  // copies before waiting for it.
  pdl_trigger();
  uint32_t pre = 0;
  if (blockIdx.x < p.units) {
    const uint32_t rg = blockIdx.x / p.ksplit, ks = blockIdx.x - rg * p.ksplit;
    const uint32_t b0 = ks * p.slice, nblk = min(p.slice, nb - b0), tile = rg * TC_WARPS + warp;
    if (tile < p.tiles) {
      const uint32_t si = tc_seg(a, tile);
      const DWDesc& w = a.seg[si].w;
      const uint32_t UB = tile_unit_bytes(w.type);
      const uint8_t* tb = w.body + (size_t)(tile - a.seg[si].cta_begin) * w.body_stride;
      pre = min(p.stages - 1, nblk);
      if (lane == 0)
        for (uint32_t k = 0; k < pre; k++) tc_issue(tb + (size_t)(b0 + k) * UB, UB, ring, p.stage_bytes, bars, k);
    }
  }
  pdl_wait();
  if (warp == 0) {
    const float v = input_scale(a, 0);
    if (lane == 0) s_in = v;
  }
  for (uint32_t unit = blockIdx.x; unit < p.units; unit += gridDim.x) {
    const uint32_t rg = unit / p.ksplit, ks = unit - rg * p.ksplit;
    const uint32_t b0 = ks * p.slice, nblk = min(p.slice, nb - b0);
    __syncthreads();  // the previous unit is done with the x fragments
    for (uint32_t i = warp; i < nblk; i += TC_WARPS)
      tc_build_x(a.x + (size_t)(b0 + i) * 256, f4 + i * 64, f6 + i * 64, xs + 8 * i, p.t4, p.t6);
    __syncthreads();
    const uint32_t tile = rg * TC_WARPS + warp;
    float vg = 0.f, vh = 0.f;
    if (tile < p.tiles) {
      uint32_t si = 0;
      if (a.nseg > 1 && tile >= a.seg[1].cta_begin) si = 1;
      if (a.nseg > 2 && tile >= a.seg[2].cta_begin) si = 2;
      const DWDesc& w = a.seg[si].w;
      const uint8_t* tb = w.body + (size_t)(tile - a.seg[si].cta_begin) * w.body_stride;
#define TC_TILE(QT, S, F) \
  tc_tile<QT, S>(tb, b0, nblk, pre, ring, p.stage_bytes, bars, nuse, a.err, F, xs, zero_page, vg, vh)
      if (w.type == 12) {
        if (p.stages == 3) TC_TILE(12, 3, f4);
        else TC_TILE(12, 2, f4);
      } else {
        if (p.stages == 3) TC_TILE(14, 3, f6);
        else TC_TILE(14, 2, f6);
      }
#undef TC_TILE
    }
    pre = 0;
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
  const uint32_t stage_bytes = t6 ? Q6T_UNIT : Q4T_UNIT;
  // x fragments of up to 32 blocks per slice; the rest of shared memory is ring
  const uint32_t slice_max = std::max(1u, std::min(32u, (TC_SMEM_MAX - TC_WARPS * 2 * stage_bytes) / per_blk));
  const uint32_t groups = (tiles + TC_WARPS - 1) / TC_WARPS;
  auto fits = [&](uint32_t k) {
    return k == 1 || (a.ks_part && a.ks_cnt && (uint64_t)k * tiles * 16u <= a.ks_part_cap && groups <= a.ks_cnt_cap);
  };
  // the split with the least work on the busiest SM: rounds of units x (blocks
  // per unit + about half a block of per-unit cost: x conversion, epilogue)
  uint32_t ks = 0;
  uint64_t best = ~0ull;
  for (uint32_t k = 1; k <= std::min(nb, 64u); k++) {
    const uint32_t sl = (nb + k - 1) / k;
    const uint32_t kk = (nb + sl - 1) / sl;
    if (sl > slice_max || !fits(kk)) continue;
    const uint64_t rounds = ((uint64_t)groups * kk + sms - 1) / sms;
    if (rounds * (2 * sl + 1) < best) {
      best = rounds * (2 * sl + 1);
      ks = kk;
    }
  }
  if (!ks) return false;
  const uint32_t slice = (nb + ks - 1) / ks;
  const uint32_t stages = std::min(TC_MAX_STAGES, (TC_SMEM_MAX - slice * per_blk) / (TC_WARPS * stage_bytes));
  if (stages < 2) return false;
  const uint32_t ring = TC_WARPS * stages * stage_bytes;
  p->tiles = tiles;
  p->groups = groups;
  p->ksplit = ks;
  p->slice = slice;
  p->units = groups * ks;
  p->grid = std::min(p->units, sms);
  p->smem = slice * per_blk + ring;
  p->stages = stages;
  p->stage_bytes = stage_bytes;
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
  return launch_pdl(gemv_tc_kernel, dim3(p.grid), dim3(TC_THREADS), p.smem, st, a, p);
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
