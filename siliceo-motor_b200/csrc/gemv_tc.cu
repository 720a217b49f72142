// Batch-1 GEMV of Q4_K / Q6_K weights on the tensor cores (int8 MMA).
//
// A decode step is one matrix-vector product per weight, so the work is bound
// by HBM bandwidth only if turning a 4/6-bit weight into something that can be
// multiplied costs almost nothing. Here the weights go into
// mma.sync.m16n8k32 (u8 x s8 -> s32) as the A operand with one AND per four
// weights (Q4_K: a low nibble is q, a high nibble 16q; Q6_K: two LOP3s and
// shifts join the 4-bit and 2-bit parts of q + 32), and products are exact:
//   * x is cut per 32- (Q4_K) or 16-wide (Q6_K) sub-block into a power-of-two
//     scaled integer of 22 bits and three signed 8-bit limbs (x~ = l0 2^16 +
//     l1 2^8 + l2), as precise as the f32 x of the reference;
//   * one MMA covers 8 weights of each of 4 sub-blocks (k = 8 sigma + i), and
//     its 8 columns are (sub-block sigma, limb l0 | l1) -- a second MMA with the
//     same A carries l2 -- so lane t's accumulators hold the integer sums of
//     sub-block sigma = t for its two rows; four (Q4_K) or two (Q6_K) MMAs
//     complete a sub-block group, and the GGUF scales are applied once per
//     (row, sub-block) in f32 (dequant.rs:98-126, 178-206):
//       Q4_K: y += d*sc_s*u_s*S_s - dmin*m_s*X_s
//       Q6_K: y += d*sc_s*(u_s*S_s - 32*X_s)
//     with S_s the limb-combined integer sum, u_s = 1 / (x's scale of the
//     sub-block) (/16 for a high nibble) and X_s = sum of x over s.
// The weights stream from HBM once (tile layout, device.cuh): every warp runs
// its own ring of shared-memory slots filled by bulk asynchronous copies (one
// per 16-row block unit, completion on an mbarrier); x is converted once per
// unit into shared memory, already in each lane's B-fragment order.
//
// Work: a unit is (8 tiles of 16 rows, K-slice). Warp w of a CTA owns tile
// w of the unit. When there are too few tiles to fill the GPU, K is split and
// the CTA that finishes a group last sums the slices in order (deterministic)
// and runs the epilogue. Epilogues are the fused ones of gemv_common.cuh. The
// grid has up to two CTAs an SM.
#include <cuda_fp16.h>

#include <algorithm>
#include <mutex>
#include <type_traits>

#include "device.cuh"
#include "gemv_common.cuh"
#include "pdl.cuh"
#include "tc_common.cuh"

namespace sm {

// A CTA is 8 warps (one 16-row tile each) with at most TC_SMEM_MAX bytes of
// shared memory, so that two CTAs fit on an SM (registers: 2 x 256 threads x
// 128; shared memory: 2 x (110 KB + static)): a CTA of the NEXT kernel in the
// stream (programmatic dependent launch) can then start on an SM while this
// kernel's CTA still runs there, and fetch its weights into shared memory
// before it waits for this kernel's output.
constexpr int TC_WARPS = 8, TC_THREADS = TC_WARPS * 32;
// B fragments of one block, one type: [8 MMA positions][32 lanes][4 words]
// (b0, b1 of the l0|l1 MMA, b0, b1 of the l2 MMA; one word of each pair is 0)
constexpr uint32_t TC_FRAG = 4096;
// per block: (u_s, X_s) of the 8 Q4_K sub-blocks, then of the 16 Q6_K ones
constexpr uint32_t TC_XS = 256;
constexpr uint32_t TC_SMEM_MAX = 110u * 1024u;
// Ring slots per warp: 2-4 slots of one block unit each (as many as shared
// memory holds).
constexpr uint32_t TC_MAX_STAGES = 4;

struct TcPlan {
  uint32_t tiles, groups, ksplit, slice, units, grid, smem, t4, t6, mixed;
  uint32_t stages, stage_bytes;  // per-warp cp.async ring of weight units
};

__device__ __forceinline__ void mma_u8s8(int (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3, uint32_t b0,
                                         uint32_t b1) {
  asm("mma.sync.aligned.m16n8k32.row.col.s32.u8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
      : "+r"(d[0]), "+r"(d[1]), "+r"(d[2]), "+r"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}
// d = A B (a zero accumulator, without zeroing registers first)
__device__ __forceinline__ void mma_u8s8_z(int (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3, uint32_t b0,
                                           uint32_t b1) {
  asm("mma.sync.aligned.m16n8k32.row.col.s32.u8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%10,%10,%10,%10};"
      : "=r"(d[0]), "=r"(d[1]), "=r"(d[2]), "=r"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1), "r"(0));
}
__device__ __forceinline__ uint32_t word_of(const uint4& v, int c) { return c == 0 ? v.x : c == 1 ? v.y : c == 2 ? v.z : v.w; }

// Power-of-two scale for a sub-block whose largest |x| is mx: the scaled
// integers stay below 2^22 (three 8-bit limbs); returns 2^e, and 2^-e in inv.
__device__ __forceinline__ float limb_scale(float mx, float& inv) {
  const int E = (int)((__float_as_uint(mx) >> 23) & 0xFFu) - 127;
  const int e = mx > 0.f ? max(-100, min(100, 21 - E)) : 0;
  inv = __uint_as_float((uint32_t)(127 - e) << 23);
  return __uint_as_float((uint32_t)(127 + e) << 23);
}
// Four x values (scaled by f) as limb words: byte b of l[k] is limb k of value b.
__device__ __forceinline__ void limbs4(const float4& v, float f, uint32_t (&l)[3]) {
  const float vv[4] = {v.x, v.y, v.z, v.w};
  l[0] = l[1] = l[2] = 0;
#pragma unroll
  for (int b = 0; b < 4; b++) {
    const int xi = __float2int_rn(vv[b] * f);  // |xi| < 2^22
    const int l2 = ((xi + 128) & 255) - 128, r = (xi - l2) >> 8;
    const int l1 = ((r + 128) & 255) - 128, l0 = (r - l1) >> 8;
    l[0] |= (uint32_t)(l0 & 255) << (8 * b);
    l[1] |= (uint32_t)(l1 & 255) << (8 * b);
    l[2] |= (uint32_t)(l2 & 255) << (8 * b);
  }
}

// Converts block blk of x (256 values) into shared memory, one warp per
// block: per type the B fragments of its 8 MMA positions (f4, f6: [position]
// [lane] uint4 = b0, b1 of the l0/l1 MMA, b0, b1 of the l2 MMA), and per
// sub-block (u_s, X_s) (xs: 8 for Q4_K, then 16 for Q6_K). Column n = g of
// lane (g, t) is (sub-block sigma = g >> 1, limb g & 1); its b0 (k = 4t ..
// 4t + 3) holds sub-block t >> 1 and b1 (k = 4t + 16 ..) sub-block 2 + (t >> 1),
// so a lane's word is non-zero only where that matches sigma.
// The attention output x[e0 .. e0 + 7] of head e0 / hd, merged from the
// attention split kernel's partials: sum_s o_s e_s / sum_s l_s e_s with
// e_s = exp(m_s - max m) (the merge of attn_combine_kernel, layers.cu).
__device__ __forceinline__ void att_merge8(const GemvArgs& a, uint32_t e0, float4& v0, float4& v1) {
  const uint32_t hd = a.hd, h = e0 / hd, d0 = e0 - h * hd;
  const uint32_t L = a.rows[0].pos + 1, tiles = (L + 31) / 32, np = a.att_slots - a.att_first;
  const uint32_t tps = (tiles + np - 1) / np, ns = (tiles + tps - 1) / tps;
  const float* ml = a.att_ml + ((size_t)h * a.att_slots + a.att_first) * 2;
  const float* po = a.att_o + ((size_t)h * a.att_slots + a.att_first) * hd + d0;
  float M = -INFINITY;
#pragma unroll 4
  for (uint32_t s = 0; s < ns; s++) M = fmaxf(M, ml[2 * s]);
  float den = 0.f;
  float4 acc0 = make_float4(0.f, 0.f, 0.f, 0.f), acc1 = acc0;
#pragma unroll 4
  for (uint32_t s = 0; s < ns; s++) {
    const float es = expf(ml[2 * s] - M);
    den = fmaf(ml[2 * s + 1], es, den);
    const float4 o0 = ldg4(po + (size_t)s * hd), o1 = ldg4(po + (size_t)s * hd + 4);
    acc0.x = fmaf(o0.x, es, acc0.x); acc0.y = fmaf(o0.y, es, acc0.y);
    acc0.z = fmaf(o0.z, es, acc0.z); acc0.w = fmaf(o0.w, es, acc0.w);
    acc1.x = fmaf(o1.x, es, acc1.x); acc1.y = fmaf(o1.y, es, acc1.y);
    acc1.z = fmaf(o1.z, es, acc1.z); acc1.w = fmaf(o1.w, es, acc1.w);
  }
  v0 = make_float4(acc0.x / den, acc0.y / den, acc0.z / den, acc0.w / den);
  v1 = make_float4(acc1.x / den, acc1.y / den, acc1.z / den, acc1.w / den);
}

// x[256 blk + 8 lane .. + 7] of the calling lane (or the merged attention
// output, att_merge8).
__device__ __forceinline__ void tc_load_x(const GemvArgs& a, uint32_t blk, float4& v0, float4& v1) {
  const int lane = threadIdx.x & 31;
  if (a.att_o) {
    att_merge8(a, blk * 256u + 8u * lane, v0, v1);
  } else {
    const float* xb = a.x + (size_t)blk * 256;
    v0 = ldg4(xb + 8 * lane);
    v1 = ldg4(xb + 8 * lane + 4);
  }
}

// The B fragments and scales of block blk from the lanes' x values (tc_load_x).
__device__ __forceinline__ void tc_build_x(float4 v0, float4 v1, uint4* f4, uint4* f6, float2* xs, bool t4, bool t6) {
  const int lane = threadIdx.x & 31, g = lane >> 2, t = lane & 3, sn = g >> 1, lim = g & 1;
  const bool active = (t >> 1) == (sn & 1);
  const float mx = fmaxf(fmaxf(fmaxf(fabsf(v0.x), fabsf(v0.y)), fmaxf(fabsf(v0.z), fabsf(v0.w))),
                         fmaxf(fmaxf(fabsf(v1.x), fabsf(v1.y)), fmaxf(fabsf(v1.z), fabsf(v1.w))));
  const float sm = sum4(v0) + sum4(v1);
  // Each lane cuts its own 8 values into limbs (with its sub-block's scale);
  // the fragment words are then fetched from the owning lanes by shuffles.
  auto frag = [&](uint4* f, int wsub, float scl_own) {
    uint32_t L0[3], L1[3];  // limbs of values 8 lane + 0..3 and + 4..7
    limbs4(v0, scl_own, L0);
    limbs4(v1, scl_own, L1);
    const int nc = wsub / 8, half = t & 1;
#pragma unroll
    for (int P = 0; P < 8; P++) {
      // positions P = (sub-block group G, chunk c): 8 weights of each of 4 sub-blocks
      const int G = P / nc, c = P % nc, src = (4 * G + sn) * wsub / 8 + c;
      const uint32_t a00 = __shfl_sync(0xffffffffu, L0[0], src), a01 = __shfl_sync(0xffffffffu, L0[1], src);
      const uint32_t a10 = __shfl_sync(0xffffffffu, L1[0], src), a11 = __shfl_sync(0xffffffffu, L1[1], src);
      const uint32_t b0 = __shfl_sync(0xffffffffu, L0[2], src), b1 = __shfl_sync(0xffffffffu, L1[2], src);
      const uint32_t A = active ? (half ? (lim ? a11 : a10) : (lim ? a01 : a00)) : 0u;
      const uint32_t B = (active && !lim) ? (half ? b1 : b0) : 0u;
      f[P * 32 + lane] = (sn >> 1) ? make_uint4(0, A, 0, B) : make_uint4(A, 0, B, 0);
    }
  };
  if (t4) {  // 32-wide sub-blocks: lanes 4s .. 4s + 3
    float m = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 1));
    m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, 2));
    float su = sm + __shfl_xor_sync(0xffffffffu, sm, 1);
    su += __shfl_xor_sync(0xffffffffu, su, 2);
    float inv;
    const float scl = limb_scale(m, inv);
    if ((lane & 3) == 0) xs[lane >> 2] = make_float2(inv * (((lane >> 2) & 1) ? 0.0625f : 1.f), su);
    frag(f4, 32, scl);
  }
  if (t6) {  // 16-wide sub-blocks: lanes 2s, 2s + 1
    const float m = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 1));
    const float su = sm + __shfl_xor_sync(0xffffffffu, sm, 1);
    float inv;
    const float scl = limb_scale(m, inv);
    if ((lane & 1) == 0) xs[8 + (lane >> 1)] = make_float2(inv, su);
    frag(f6, 16, scl);
  }
}

// Integer sums of lane t's sub-block for rows g (d0) and g + 8 (d1), as floats.
__device__ __forceinline__ void limb_sums(const int (&A)[4], const int (&B)[4], float& d0, float& d1) {
  d0 = fmaf((float)A[0], 65536.f, (float)(A[1] * 256 + B[0]));
  d1 = fmaf((float)A[2], 65536.f, (float)(A[3] * 256 + B[2]));
}

// ------------------------------------------------------------- Q4_K ----
// get_scale_min_k4 of sub-block s = 4G + t (dequant.rs:41-49) from a row header.
__device__ __forceinline__ void q4_sc_m(const uint4& h, int G, int t, float& sc, float& m) {
  const int sh = 8 * t;
  if (G == 0) {
    sc = (float)((h.y >> sh) & 63u);
    m = (float)((h.z >> sh) & 63u);
  } else {
    sc = (float)(((h.w >> sh) & 0xFu) | (((h.y >> (sh + 6)) & 3u) << 4));
    m = (float)(((h.w >> (sh + 4)) & 0xFu) | (((h.z >> (sh + 6)) & 3u) << 4));
  }
}
__device__ __forceinline__ void q4_block(const uint8_t* st, const uint4* f, const float2* xs, int lane, float& rg,
                                         float& rh) {
  const int g = lane >> 2, t = lane & 3, p = t & 1;
  const uint32_t M = (t >> 1) ? 0xF0F0F0F0u : 0x0F0F0F0Fu;  // nibble of sub-blocks t >> 1, 2 + (t >> 1)
  uint4 Wg[4], Wh[4];
#pragma unroll
  for (int j = 0; j < 4; j++) {
    Wg[j] = *reinterpret_cast<const uint4*>(st + q4t_word_off(g, j, 0, p));
    Wh[j] = *reinterpret_cast<const uint4*>(st + q4t_word_off(g + 8, j, 0, p));
  }
  const uint4 hg = reinterpret_cast<const uint4*>(st)[g], hh = reinterpret_cast<const uint4*>(st)[g + 8];
  // per row: sum over the lane's two sub-blocks of sc*u*S and of m*X; d and
  // dmin are applied once
  float sg_ = 0.f, sh_ = 0.f, mg_ = 0.f, mh_ = 0.f;
#pragma unroll
  for (int G = 0; G < 2; G++) {
    int A[4], B[4];
#pragma unroll
    for (int c = 0; c < 4; c++) {
      const uint4 bf = f[(4 * G + c) * 32 + lane];
      const uint32_t a0 = word_of(Wg[2 * G], c) & M, a2 = word_of(Wg[2 * G + 1], c) & M;
      const uint32_t a1 = word_of(Wh[2 * G], c) & M, a3 = word_of(Wh[2 * G + 1], c) & M;
      if (c == 0) {
        mma_u8s8_z(A, a0, a1, a2, a3, bf.x, bf.y);
        mma_u8s8_z(B, a0, a1, a2, a3, bf.z, bf.w);
      } else {
        mma_u8s8(A, a0, a1, a2, a3, bf.x, bf.y);
        mma_u8s8(B, a0, a1, a2, a3, bf.z, bf.w);
      }
    }
    float Sg, Sh;
    limb_sums(A, B, Sg, Sh);
    const float2 ux = xs[4 * G + t];
    float scg, mg, sch, mh;
    q4_sc_m(hg, G, t, scg, mg);
    q4_sc_m(hh, G, t, sch, mh);
    sg_ = fmaf(scg, ux.x * Sg, sg_);
    sh_ = fmaf(sch, ux.x * Sh, sh_);
    mg_ = fmaf(mg, ux.y, mg_);
    mh_ = fmaf(mh, ux.y, mh_);
  }
  const float dg = h2f_ref(hg.x & 0xFFFFu), dmg = h2f_ref(hg.x >> 16);
  const float dh = h2f_ref(hh.x & 0xFFFFu), dmh = h2f_ref(hh.x >> 16);
  rg += dg * sg_ - dmg * mg_;
  rh += dh * sh_ - dmh * mh_;
}

// ------------------------------------------------------------- Q6_K ----
// A operands of sub-blocks h and 2 + h (h = t >> 1) from words W_h and H.
__device__ __forceinline__ void q6_a(uint32_t w, uint32_t hbits, int h, uint32_t& lo, uint32_t& hi) {
  const uint32_t hs = hbits << (4 * h);
  lo = (w & 0x0F0F0F0Fu) | (hs & 0x30303030u);
  hi = ((w >> 4) & 0x0F0F0F0Fu) | ((hs >> 2) & 0x30303030u);
}
__device__ __forceinline__ void q6_block(const uint8_t* unit, const uint4* f, const float2* xs, int lane, float& rg,
                                         float& rh) {
  const int g = lane >> 2, t = lane & 3, p = t & 1, h = t >> 1;
  // per row: W_h words (G, c) and H words (G, c), G = 0..3, c = 0..1
  const uint4 wg0 = *reinterpret_cast<const uint4*>(unit + q6t_word_off(g, h, 0, 0, p));
  const uint4 wg1 = *reinterpret_cast<const uint4*>(unit + q6t_word_off(g, h, 2, 0, p));
  const uint4 hg0 = *reinterpret_cast<const uint4*>(unit + q6t_word_off(g, 2, 0, 0, p));
  const uint4 hg1 = *reinterpret_cast<const uint4*>(unit + q6t_word_off(g, 2, 2, 0, p));
  const uint4 wh0 = *reinterpret_cast<const uint4*>(unit + q6t_word_off(g + 8, h, 0, 0, p));
  const uint4 wh1 = *reinterpret_cast<const uint4*>(unit + q6t_word_off(g + 8, h, 2, 0, p));
  const uint4 hh0 = *reinterpret_cast<const uint4*>(unit + q6t_word_off(g + 8, 2, 0, 0, p));
  const uint4 hh1 = *reinterpret_cast<const uint4*>(unit + q6t_word_off(g + 8, 2, 2, 0, p));
  const uint4 scg = reinterpret_cast<const uint4*>(unit)[g], sch = reinterpret_cast<const uint4*>(unit)[g + 8];
  const float dg = q6_d(reinterpret_cast<const unsigned short*>(unit + 256)[g]);
  const float dh = q6_d(reinterpret_cast<const unsigned short*>(unit + 256)[g + 8]);
  // eight independent accumulator chains (groups x limb sets) hide the MMA latency
  int A[4][4], B[4][4];
#pragma unroll
  for (int c = 0; c < 2; c++)
#pragma unroll
    for (int G = 0; G < 4; G++) {
      const int wi = 2 * (G & 1) + c;
      const uint4 bf = f[(2 * G + c) * 32 + lane];
      uint32_t a0, a1, a2, a3;
      q6_a(word_of(G < 2 ? wg0 : wg1, wi), word_of(G < 2 ? hg0 : hg1, wi), h, a0, a2);
      q6_a(word_of(G < 2 ? wh0 : wh1, wi), word_of(G < 2 ? hh0 : hh1, wi), h, a1, a3);
      if (c == 0) {
        mma_u8s8_z(A[G], a0, a1, a2, a3, bf.x, bf.y);
        mma_u8s8_z(B[G], a0, a1, a2, a3, bf.z, bf.w);
      } else {
        mma_u8s8(A[G], a0, a1, a2, a3, bf.x, bf.y);
        mma_u8s8(B[G], a0, a1, a2, a3, bf.z, bf.w);
      }
    }
  float ag = 0.f, ah = 0.f;  // per row: sum over the lane's sub-blocks of sc*(u*S - 32*X); d applied once
#pragma unroll
  for (int G = 0; G < 4; G++) {
    float Sg, Sh;
    limb_sums(A[G], B[G], Sg, Sh);
    const float2 ux = xs[8 + 4 * G + t];
    const float sg = (float)(int8_t)((word_of(scg, G) >> (8 * t)) & 0xFFu);
    const float sh = (float)(int8_t)((word_of(sch, G) >> (8 * t)) & 0xFFu);
    ag = fmaf(sg, fmaf(ux.x, Sg, -32.f * ux.y), ag);
    ah = fmaf(sh, fmaf(ux.x, Sh, -32.f * ux.y), ah);
  }
  rg += dg * ag;
  rh += dh * ah;
}

// One warp: tile rows g, g+8 over blocks b0 .. b0+nblk-1 (x fragments of
// block b0 + i at slot i). The block units stream through the warp's ring of
// S shared-memory slots: lane 0 fills the whole ring first, then refills the
// slot of each computed unit with the unit S further on, each copy
// completing on the slot's mbarrier (use n of the ring waits for parity
// (n / S) & 1; nuse counts the warp's uses across units). Returns the partial
// dot products in rg, rh (summed over the lane's sub-blocks only).
// The first `pre` copies (up to S) may have been started by the caller
// already, ahead of the previous kernel (pdl.cuh): the whole ring lands while
// the kernel waits for its input and converts x.
template <int QT, int S>
__device__ __forceinline__ void tc_tile(const uint8_t* tile, uint32_t b0, uint32_t nblk, uint32_t pre, uint8_t* ring,
                                        uint32_t stage_bytes, uint64_t* bars, uint32_t& nuse, uint32_t* err,
                                        const uint4* f, const float2* xs, float& rg, float& rh) {
  const int lane = threadIdx.x & 31;
  constexpr uint32_t UB = QT == 12 ? Q4T_UNIT : Q6T_UNIT;
  auto next = [](uint32_t i) -> uint32_t { return (S & (S - 1)) == 0 ? (i + 1) & (S - 1) : (i + 1 == S ? 0 : i + 1); };
  // ring slot of the next copy to start (ip) and of the next block to compute (cp, phase cph)
  uint32_t ip = nuse % S, cp = ip, cph = (nuse / S) & 1u;
  for (uint32_t k = 0; k < pre; k++) ip = next(ip);
  const uint8_t* src = tile + (size_t)b0 * UB;
  const uint32_t npro = min((uint32_t)S, nblk);
  for (uint32_t k = pre; k < npro; k++) {  // the first S copies: the whole ring
    if (lane == 0) tc_issue(src + (size_t)k * UB, UB, ring, stage_bytes, bars, ip);
    ip = next(ip);
  }
  auto compute = [&](uint32_t i) {
    mbar_wait(bars + cp, cph, err);
    const uint8_t* sp = ring + cp * stage_bytes;
    cp = next(cp);
    cph ^= cp == 0 ? 1u : 0u;
    if constexpr (QT == 12) q4_block(sp, f + (size_t)i * (TC_FRAG / 16), xs + 32 * i, lane, rg, rh);
    else q6_block(sp, f + (size_t)i * (TC_FRAG / 16), xs + 32 * i, lane, rg, rh);
    __syncwarp();  // every lane is done with the slot before it is refilled
  };
  for (uint32_t i = 0; i < nblk; i++) {  // this block, then the copy S blocks ahead into its slot
    compute(i);
    if (i + S < nblk) {
      if (lane == 0) tc_issue(src + (size_t)(i + S) * UB, UB, ring, stage_bytes, bars, ip);
      ip = next(ip);
    }
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

// Whether launch tile `tile` holds rows (padding tiles of a mixed launch do
// not), and its segment.
__device__ __forceinline__ bool tc_tile_at(const GemvArgs& a, uint32_t tile, uint32_t tiles, uint32_t& si) {
  if (tile >= tiles) return false;
  si = tc_seg(a, tile);
  return tile - a.seg[si].cta_begin < (a.seg[si].w.n_out + 15) / 16;
}

// Operands of a tile's fused epilogue that do not depend on the dot
// products, for the calling lane's row o (lanes t < 2; for pairs the even
// rows): read at the start of the unit so that the loads overlap the weight
// stream. Read after the dot products they would be chains of dependent
// loads (row -> sequence -> page) on the launch's critical path.
struct TcEpiIn {
  float bias;    // bias[o] (0 without a bias)
  float res, nw;  // EPI_RESID: the residual x[o] and the next norm's weight
  float c, s;    // pair RoPE: cos / sin at the row's position (qwen2.rs:708-724)
  float* dst;    // pair RoPE: q or the K cache at (head, m); EPI_V: the V cache at o
};

__device__ __forceinline__ TcEpiIn tc_epi_in(const GemvArgs& a, uint32_t tile) {
  const int lane = threadIdx.x & 31, g = lane >> 2, t = lane & 3;
  TcEpiIn e{0.f, 0.f, 0.f, 0.f, 0.f, nullptr};
  const GemvSeg& sg = a.seg[tc_seg(a, tile)];
  const uint32_t o = (tile - sg.cta_begin) * 16u + (uint32_t)g + 8u * (uint32_t)t, epi = sg.epi;
  if (t >= 2 || o >= sg.w.n_out) return e;
  if (sg.bias) e.bias = sg.bias[o];
  if (epi == EPI_RESID) {
    e.res = sg.y[o];
    e.nw = a.nw[o];
  } else if ((epi == EPI_ROPE_Q || epi == EPI_ROPE_K) && !(g & 1)) {
    const RowDesc rd = a.rows[0];
    const uint32_t half = a.hd >> 1, h = o / a.hd, m = (o - h * a.hd) >> 1;
    e.c = a.cos_t[(size_t)rd.pos * half + m];
    e.s = a.sin_t[(size_t)rd.pos * half + m];
    if (epi == EPI_ROPE_Q) {
      e.dst = sg.y + h * a.hd + m;
    } else {
      const SeqDesc sd = a.seqs[rd.seq];
      e.dst = sd.pages[rd.pos / KV_PAGE] + kv_page_off(a.layer, rd.pos, a.kvd) + h * a.hd + m;
    }
  } else if (epi == EPI_V) {
    const RowDesc rd = a.rows[0];
    const SeqDesc sd = a.seqs[rd.seq];
    e.dst = sd.pages[rd.pos / KV_PAGE] + sd.voff + kv_page_off(a.layer, rd.pos, a.kvd) + o;
  }
  return e;
}

// Epilogue of one tile (column 0): vg / vh are the full dot products of rows
// g, g + 8 (in every lane of the group); `in` holds the lane's operands read
// ahead (tc_epi_in). The arithmetic of epi_single / epi_pair (gemv_common.cuh).
__device__ __forceinline__ void tc_epilogue(const GemvArgs& a, uint32_t tile, float vg, float vh, const TcEpiIn& in) {
  const int lane = threadIdx.x & 31, g = lane >> 2, t = lane & 3;
  uint32_t si = 0;
  if (a.nseg > 1 && tile >= a.seg[1].cta_begin) si = 1;
  if (a.nseg > 2 && tile >= a.seg[2].cta_begin) si = 2;
  // the segment by value: read through the parameter reference after a store
  // its fields are fetched again
  const GemvSeg sg = a.seg[si];
  const uint32_t row0 = (tile - sg.cta_begin) * 16u, epi = sg.epi;
  const uint32_t o = row0 + (uint32_t)g + 8u * (uint32_t)t;
  const bool mine = t < 2 && o < sg.w.n_out, has_bias = sg.bias != nullptr;
  const float raw = t ? vh : vg;              // this lane's row o
  const float v = has_bias ? raw + in.bias : raw;  // with its bias
  if (epi_is_pair(epi)) {
    const float nv = __shfl_down_sync(0xffffffffu, v, 4);  // row o + 1, bias included
    if (!(g & 1) && mine) {
      if (epi == EPI_SILU) {  // gate = silu(gate) * up (qwen2.rs:546-548, 743-745)
        a.h[o >> 1] = __fmul_rn(__fdiv_rn(v, __fadd_rn(1.0f, expf(-v))), nv);
      } else {  // NEOX RoPE of the pair into q (natural order) or the K cache (qwen2.rs:497, 708-724)
        const uint32_t half = a.hd >> 1;
        in.dst[0] = __fsub_rn(__fmul_rn(v, in.c), __fmul_rn(nv, in.s));
        in.dst[half] = __fadd_rn(__fmul_rn(v, in.s), __fmul_rn(nv, in.c));
      }
    }
    return;
  }
  float xn = 0.f, stored = 0.f;
  if (mine) {
    if (epi == EPI_RESID) {  // x += v, then the next RMSNorm's x * w (qwen2.rs:536-538, 549-551)
      xn = in.res + v;
      sg.y[o] = xn;
      a.xn[o] = xn * in.nw;
    } else if (epi == EPI_STORE) {
      sg.y[o] = v;
      stored = v;
    } else if (epi == EPI_V) {  // the V cache row (qwen2.rs:498)
      in.dst[0] = v;
    } else {
      xn = epi_single(a, sg, o, 0, raw);
    }
  }
  if (epi == EPI_RESID) {  // partial sum of x^2 over the tile's rows
    const float s2 = warp_sum(xn * xn);
    if (lane == 0) a.out_parts[tile] = s2;
  }
  if (a.amax) {  // the tile's greedy candidate (the stored values, bias included)
    uint64_t key = 0;
    if (mine) key = argmax_key(epi == EPI_STORE ? stored : sg.y[o], o);
#pragma unroll
    for (int of = 16; of > 0; of >>= 1) {
      const uint64_t k2 = __shfl_xor_sync(0xffffffffu, key, of);
      key = k2 > key ? k2 : key;
    }
    if (lane == 0) a.amax[tile] = key;
  }
}

__global__ void __launch_bounds__(TC_THREADS, 2) gemv_tc_kernel(const __grid_constant__ GemvArgs a,
                                                                const __grid_constant__ TcPlan p) {
  extern __shared__ __align__(16) uint8_t tc_smem[];
  __shared__ float s_in;
  __shared__ uint32_t s_last;
  __shared__ __align__(8) uint64_t s_bars[TC_WARPS * TC_MAX_STAGES];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  // x fragments per type (a mixed launch: one region, of the CTA's type)
  uint4* f4 = reinterpret_cast<uint4*>(tc_smem);
  uint4* f6 = f4 + ((p.t4 && !p.mixed) ? p.slice * (TC_FRAG / 16) : 0);
  float2* xs = reinterpret_cast<float2*>(f6 + (p.t6 ? p.slice * (TC_FRAG / 16) : 0));
  uint8_t* ring = reinterpret_cast<uint8_t*>(xs + 32 * p.slice) + (size_t)warp * p.stages * p.stage_bytes;
  const uint32_t nb = a.seg[0].w.n_in >> 8;
  uint64_t* bars = s_bars + warp * TC_MAX_STAGES;
  if (lane == 0) {
    for (uint32_t k = 0; k < p.stages; k++) mbar_init(bars + k, 1);
    fence_mbar_init();
  }
  __syncwarp();
  uint32_t nuse = 0;
  // The weights do not depend on the previous kernel: start the first unit's
  // copies before waiting for it.
  pdl_trigger();
  uint32_t pre = 0;
  if (blockIdx.x < p.units) {
    const uint32_t rg = blockIdx.x / p.ksplit, ks = blockIdx.x - rg * p.ksplit;
    const uint32_t b0 = ks * p.slice, nblk = min(p.slice, nb - b0), tile = rg * TC_WARPS + warp;
    uint32_t si = 0;
    if (tc_tile_at(a, tile, p.tiles, si)) {
      const DWDesc& w = a.seg[si].w;
      const uint32_t UB = tile_unit_bytes(w.type);
      const uint8_t* tb = w.body + (size_t)(tile - a.seg[si].cta_begin) * w.body_stride;
      pre = min(p.stages, nblk);
      if (lane == 0)
        for (uint32_t k = 0; k < pre; k++) tc_issue(tb + (size_t)(b0 + k) * UB, UB, ring, p.stage_bytes, bars, k);
    }
  }
  pdl_wait();
  for (uint32_t unit = blockIdx.x; unit < p.units; unit += gridDim.x) {
    const uint32_t rg = unit / p.ksplit, ks = unit - rg * p.ksplit;
    const uint32_t b0 = ks * p.slice, nblk = min(p.slice, nb - b0);
    __syncthreads();  // the previous unit is done with the x fragments
    // the types this CTA's tiles have (a mixed launch: the type of its group)
    bool b4 = p.t4, b6 = p.t6;
    if (p.mixed) {
      const bool q4 = a.seg[tc_seg(a, rg * TC_WARPS)].w.type == 12;
      b4 = q4;
      b6 = !q4;
    }
    if (unit == blockIdx.x && warp == TC_WARPS - 1) {  // the input-norm scale, beside the other warps' x
      const float v = input_scale(a, 0);
      if (lane == 0) s_in = v;
    }
    for (uint32_t i = warp; i < nblk; i += 2 * TC_WARPS) {  // two blocks' x loads in flight, then their fragments
      const uint32_t j = i + TC_WARPS;
      float4 u0, u1, w0 = make_float4(0.f, 0.f, 0.f, 0.f), w1 = w0;
      tc_load_x(a, b0 + i, u0, u1);
      if (j < nblk) tc_load_x(a, b0 + j, w0, w1);
      tc_build_x(u0, u1, f4 + i * (TC_FRAG / 16), f6 + i * (TC_FRAG / 16), xs + 32 * i, b4, b6);
      if (j < nblk) tc_build_x(w0, w1, f4 + j * (TC_FRAG / 16), f6 + j * (TC_FRAG / 16), xs + 32 * j, b4, b6);
    }
    __syncthreads();
    const uint32_t tile = rg * TC_WARPS + warp;
    float vg = 0.f, vh = 0.f;
    uint32_t si = 0;
    const bool valid = tc_tile_at(a, tile, p.tiles, si);
    // the epilogue's operands, read while the weights stream (only the
    // group's last CTA uses them when K is split)
    const TcEpiIn ein = valid ? tc_epi_in(a, tile) : TcEpiIn{0.f, 0.f, 0.f, 0.f, 0.f, nullptr};
    if (valid) {
      const DWDesc& w = a.seg[si].w;
      const uint8_t* tb = w.body + (size_t)(tile - a.seg[si].cta_begin) * w.body_stride;
#define TC_TILE(QT, S, F) \
  tc_tile<QT, S>(tb, b0, nblk, pre, ring, p.stage_bytes, bars, nuse, a.err, F, xs, vg, vh)
      if (w.type == 12) {
        if (p.stages == 4) TC_TILE(12, 4, f4);
        else if (p.stages == 3) TC_TILE(12, 3, f4);
        else TC_TILE(12, 2, f4);
      } else {
        if (p.stages == 4) TC_TILE(14, 4, f6);
        else if (p.stages == 3) TC_TILE(14, 3, f6);
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
      if (valid) tc_epilogue(a, tile, vg * s_in, vh * s_in, ein);
      continue;
    }
    // K-split: publish this slice, the last CTA of the group sums the slices in order.
    const size_t stride = (size_t)p.tiles * 16u;
    const int g = lane >> 2, t = lane & 3;
    if (tile < p.tiles && t < 2) a.ks_part[ks * stride + tile * 16u + g + 8u * t] = t ? vh : vg;
    __syncthreads();
    if (threadIdx.x == 0) s_last = ks_arrive(&a.ks_cnt[rg], p.ksplit - 1u) == p.ksplit - 1u;
    __syncthreads();
    if (s_last) {
      if (valid) {
        float sg = 0.f, sh = 0.f;
        for (uint32_t k0 = 0; k0 < p.ksplit; k0 += 8) {  // eight slices' loads in flight, added in order
          float lg[8], lh[8];
#pragma unroll
          for (uint32_t k = 0; k < 8; k++) {
            const bool in = k0 + k < p.ksplit;
            lg[k] = in ? __ldcg(a.ks_part + (k0 + k) * stride + tile * 16u + g) : 0.f;
            lh[k] = in ? __ldcg(a.ks_part + (k0 + k) * stride + tile * 16u + g + 8u) : 0.f;
          }
#pragma unroll
          for (uint32_t k = 0; k < 8; k++)
            if (k0 + k < p.ksplit) {
              sg += lg[k];
              sh += lh[k];
            }
        }
        tc_epilogue(a, tile, sg * s_in, sh * s_in, ein);
      }
    }
  }
}

// ------------------------------------------------------------- host ----

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
    if (e == cudaSuccess)
      e = cudaFuncSetAttribute(gemv_tc_kernel, cudaFuncAttributePreferredSharedMemoryCarveout,
                               cudaSharedmemCarveoutMaxShared);
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
  bool t4 = false, t6 = false;
  for (uint32_t i = 0; i < a.nseg; i++) (a.seg[i].w.type == 12 ? t4 : t6) = true;
  // A launch of both types starts every segment on a CTA's first tile, so
  // that a CTA converts x for one type only (padding tiles do nothing).
  const bool mixed = t4 && t6;
  uint32_t tiles = 0;
  for (uint32_t i = 0; i < a.nseg; i++) {
    if (mixed) tiles = (tiles + TC_WARPS - 1) / TC_WARPS * TC_WARPS;
    a.seg[i].cta_begin = tiles;
    tiles += (a.seg[i].w.n_out + 15) / 16;
  }
  const uint32_t nb = a.seg[0].w.n_in >> 8;
  const uint32_t per_blk = (mixed ? TC_FRAG : (t4 ? TC_FRAG : 0) + (t6 ? TC_FRAG : 0)) + TC_XS;
  const uint32_t stage_bytes = t6 ? Q6T_UNIT : Q4T_UNIT;
  // x fragments of up to 32 blocks per slice; the rest of shared memory is
  // ring (at least two slots a warp)
  const uint32_t slice_max = std::max(1u, std::min(32u, (TC_SMEM_MAX - TC_WARPS * 2 * stage_bytes) / per_blk));
  const uint32_t slots = 2 * sms;  // two CTAs an SM
  const uint32_t groups = (tiles + TC_WARPS - 1) / TC_WARPS;
  auto fits = [&](uint32_t k) {
    return k == 1 || (a.ks_part && a.ks_cnt && (uint64_t)k * tiles * 16u <= a.ks_part_cap && groups <= a.ks_cnt_cap);
  };
  // the split with the least work on the busiest SM: rounds of units x (blocks
  // per unit + about half a block of per-unit cost: x conversion, epilogue).
  // (Splitting further to deepen the copy rings measured slower in a chain of
  // launches: 23.8 against 18.1 us for the 7B gate/up shape.)
  uint32_t ks = 0;
  uint64_t best = ~0ull;
  for (uint32_t k = 1; k <= std::min(nb, 64u); k++) {
    const uint32_t sl = (nb + k - 1) / k;
    const uint32_t kk = (nb + sl - 1) / sl;
    if (sl > slice_max || !fits(kk)) continue;
    if ((TC_SMEM_MAX - sl * per_blk) / (TC_WARPS * stage_bytes) < 2) continue;  // at least two ring slots
    const uint64_t rounds = ((uint64_t)groups * kk + slots - 1) / slots;
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
  p->grid = std::min(p->units, slots);
  p->smem = slice * per_blk + ring;
  p->stages = stages;
  p->stage_bytes = stage_bytes;
  p->t4 = t4;
  p->t6 = t6;
  p->mixed = mixed;
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
