// Batched GEMV (2..32 columns: batched decode steps and prefill chunks) of
// Q4_K / Q6_K weights on the tensor cores.
//
// The batch-1 kernel (gemv_tc.cu) spends the 8 columns of its int8 MMAs on
// sub-blocks of one vector; here f16 MMAs (m16n8k16) hold four columns of x,
// each split into hi + lo f16 halves (MMA columns 2c / 2c+1 = hi / lo of
// column 4n + c of n-tile n, so a lane's two accumulators of a row are one
// product and simply add). The A operand is an exact f16 subnormal made from
// the weight nibbles with one AND (w & 0x000F000F is q * 2^-24 in both
// halves; a high nibble, w & 0x00F000F0, is 16 times that and takes a 1/16
// factor), read from the same 16-row tile units; every k16 chunk lies in one
// sub-block, so a sub-block's MMAs go into a fresh accumulator that is scaled
// by the row's sub-block scale on the CUDA cores (dequant.rs:98-126, 178-206):
//   Q4_K: y += d*F*sum_s(sc_s*acc_s) - dmin*sum_s(m_s*X_s)
//   Q6_K: y += d*F*sum_s(sc_s*acc_s) - 32*d*sum_s(sc_s*X_s)
// with X_s = sum of x over sub-block s and F = 2^24 / (the power of two x was
// scaled by in this 256-block, per column).
//
// A CTA owns a group of 16 tiles (256 rows; warp w: tile w) and a K-slice.
// Per 256-block the whole CTA (i) finds each column's scale and sub-block
// sums two blocks ahead, (ii) converts the next block of x into B fragments in
// shared memory, and (iii) multiplies the current block: one barrier per
// block. The weights stream through per-warp rings of bulk copies as in the
// batch-1 kernel. K-splits end in the same deterministic last-arriver fixup.
#include <cuda_fp16.h>

#include <algorithm>
#include <mutex>

#include "device.cuh"
#include "gemv_common.cuh"
#include "pdl.cuh"
#include "tc_common.cuh"

namespace sm {

constexpr int TB_WARPS = 16, TB_THREADS = TB_WARPS * 32;
constexpr uint32_t TB_SMEM_MAX = 225u * 1024u;
constexpr uint32_t TB_STAGES = 2;
constexpr uint32_t TB_MAXB = 32;  // columns

struct TbPlan {
  uint32_t tiles, groups, ksplit, slice, units, grid, smem, stage_bytes;
};

// Shared memory of a CTA (NT n-tiles = 4*NT columns).
template <int NT>
struct TbSmem {
  static constexpr uint32_t FRAG = 4096u * NT;  // B fragments of one 256-block
  // frag[2][FRAG] | sums[3][16 sub-blocks][4 lanes t][NT] f32 | fscale[3][4][NT] f32 | scl[3][32] f32 | ring
  static constexpr uint32_t SUMS = 16u * 4u * NT * 4u, FSC = 4u * NT * 4u, SCL = TB_MAXB * 4u;
  static constexpr uint32_t OFF_SUMS = 2 * FRAG, OFF_FSC = OFF_SUMS + 3 * SUMS, OFF_SCL = OFF_FSC + 3 * FSC;
  static constexpr uint32_t OFF_RING = (OFF_SCL + 3 * SCL + 127) / 128 * 128;
};

// (i) Column scales and sub-block sums of 256-block `blk` (K offset k0), one
// warp per column: scl = the power of two that puts max|x| in [2^14, 2^15),
// fscale = 2^24 / scl, sums of x over the 16-wide
// (Q6_K) or 32-wide (Q4_K) sub-blocks in [s][t][n] order for the lane that
// owns column 4n + t. Columns >= batch get zeros.
template <int NT, int QT>
__device__ __forceinline__ void tb_scales(const float* __restrict__ x, uint32_t ldx, uint32_t batch, uint32_t k0,
                                          float* sums, float* fsc, float* scl) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  for (int c = warp; c < 4 * NT; c += TB_WARPS) {
    const int n = c >> 2, t = c & 3;
    float4 a = make_float4(0.f, 0.f, 0.f, 0.f), b = a;
    if ((uint32_t)c < batch) {
      const float* xp = x + (size_t)c * ldx + k0 + 8 * lane;
      a = ldg4(xp);
      b = ldg4(xp + 4);
    }
    float mx = fmaxf(fmaxf(fmaxf(fabsf(a.x), fabsf(a.y)), fmaxf(fabsf(a.z), fabsf(a.w))),
                     fmaxf(fmaxf(fabsf(b.x), fabsf(b.y)), fmaxf(fabsf(b.z), fabsf(b.w))));
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    float s = sum4(a) + sum4(b);  // lane holds x[8*lane .. 8*lane + 7]
    s += __shfl_xor_sync(0xffffffffu, s, 1);
    if (QT == 12) s += __shfl_xor_sync(0xffffffffu, s, 2);
    if (QT == 12) {
      if ((lane & 3) == 0) sums[((lane >> 2) * 4 + t) * NT + n] = s;  // sub-block lane / 4
    } else {
      if ((lane & 1) == 0) sums[((lane >> 1) * 4 + t) * NT + n] = s;  // sub-block lane / 2
    }
    if (lane == 0) {
      const uint32_t E = (__float_as_uint(mx) >> 23) & 0xFFu;
      scl[c] = E >= 15u ? __uint_as_float((268u - E) << 23) : 1.0f;
      fsc[t * NT + n] = (E >= 15u ? __uint_as_float((E - 14u) << 23) : 1.0f) * 16777216.f;
    }
  }
}

// (ii) B fragments of 256-block k0: entry (s, n, lane (g, t)) holds column
// c = 4n + g/2, hi (g even) or lo (g odd) of the scaled x at the lane's
// positions of sub-block s in the A operand's k order (tb_q4_block,
// tb_q6_block): Q4_K: x[32s + 4t + {0,2},{1,3}] then x[32s + 16 + 4t + ...]
// (16 B, one pair of words per MMA); Q6_K: x[16s + 4t + {0,2},{1,3}] (8 B).
template <int NT, int QT>
__device__ __forceinline__ void tb_frags(const float* __restrict__ x, uint32_t ldx, uint32_t batch, uint32_t k0,
                                         const float* scl, uint8_t* frag) {
  constexpr int NS = QT == 12 ? 8 : 16, N = NS * NT * 32;
  for (int i = threadIdx.x; i < N; i += TB_THREADS) {
    const int lane = i & 31, sn = i >> 5, n = sn % NT, s = sn / NT;
    const int g = lane >> 2, t = lane & 3, c = 4 * n + (g >> 1);
    const bool lo = g & 1;
    if (QT == 12) {
      uint4 w = make_uint4(0, 0, 0, 0);
      if ((uint32_t)c < batch) {
        const float* xp = x + (size_t)c * ldx + k0 + 32 * s + 4 * t;
        const float4 a = ldg4(xp), b = ldg4(xp + 16);
        const float f = scl[c];
        w = make_uint4(hl_pair(a.x * f, a.z * f, lo), hl_pair(a.y * f, a.w * f, lo), hl_pair(b.x * f, b.z * f, lo),
                       hl_pair(b.y * f, b.w * f, lo));
      }
      reinterpret_cast<uint4*>(frag)[i] = w;
    } else {
      uint2 w = make_uint2(0, 0);
      if ((uint32_t)c < batch) {
        const float4 a = ldg4(x + (size_t)c * ldx + k0 + 16 * s + 4 * t);
        const float f = scl[c];
        w = make_uint2(hl_pair(a.x * f, a.z * f, lo), hl_pair(a.y * f, a.w * f, lo));
      }
      reinterpret_cast<uint2*>(frag)[i] = w;
    }
  }
}

// (iii) One Q4_K block of the warp's tile (unit in shared memory st) into the
// row results yg[n], yh[n] (rows g, g + 8; column 4n + t).
template <int NT>
__device__ __forceinline__ void tb_q4_block(const uint8_t* st, const uint8_t* frag, const float* sums,
                                            const float* fsc, float (&yg)[NT], float (&yh)[NT]) {
  const int lane = threadIdx.x & 31, g = lane >> 2, t = lane & 3;
  // qs words (j, c, p = t & 1) of rows g, g + 8; MMA m of a sub-block takes word c = 2m + (t >> 1)
  const uint32_t c0 = t >> 1;
  uint32_t Wg[4][2], Wh[4][2];
#pragma unroll
  for (int j = 0; j < 4; j++)
#pragma unroll
    for (int m = 0; m < 2; m++) {
      Wg[j][m] = *reinterpret_cast<const uint32_t*>(st + q4t_word_off(g, j, 2 * m + c0, t & 1));
      Wh[j][m] = *reinterpret_cast<const uint32_t*>(st + q4t_word_off(g + 8, j, 2 * m + c0, t & 1));
    }
  const uint4 hg = reinterpret_cast<const uint4*>(st)[g], hh = reinterpret_cast<const uint4*>(st)[g + 8];
  float pg[NT], ph[NT];
#pragma unroll
  for (int n = 0; n < NT; n++) pg[n] = ph[n] = 0.f;
  const float dming = h2f_ref(hg.x >> 16), dminh = h2f_ref(hh.x >> 16);
#pragma unroll
  for (int s = 0; s < 8; s++) {
    const int j = s >> 1;
    const uint32_t ga = Wg[j][0], gb = Wg[j][1], ha = Wh[j][0], hb = Wh[j][1];
    uint32_t a1[4], a2[4];
    if (s & 1) {
      a1[0] = nib_hi(ga); a1[1] = nib_hi(ha); a1[2] = nib_hi(ga >> 8); a1[3] = nib_hi(ha >> 8);
      a2[0] = nib_hi(gb); a2[1] = nib_hi(hb); a2[2] = nib_hi(gb >> 8); a2[3] = nib_hi(hb >> 8);
    } else {
      a1[0] = nib_lo(ga); a1[1] = nib_lo(ha); a1[2] = nib_lo(ga >> 8); a1[3] = nib_lo(ha >> 8);
      a2[0] = nib_lo(gb); a2[1] = nib_lo(hb); a2[2] = nib_lo(gb >> 8); a2[3] = nib_lo(hb >> 8);
    }
    // get_scale_min_k4 of sub-block s for rows g, g + 8 (dequant.rs:41-49);
    // a high nibble's operand is 16q * 2^-24, so its sums are scaled by 1/16
    auto scale_min = [&](const uint4& h, float& sc, float& mn) {
      uint32_t a, m;
      if (s < 4) {
        a = (h.y >> (8 * s)) & 63u;
        m = (h.z >> (8 * s)) & 63u;
      } else {
        const int s4 = 8 * (s - 4);
        a = ((h.w >> s4) & 0xFu) | (((h.y >> (s4 + 6)) & 3u) << 4);
        m = ((h.w >> (s4 + 4)) & 0xFu) | (((h.z >> (s4 + 6)) & 3u) << 4);
      }
      sc = (float)a * ((s & 1) ? 0.0625f : 1.f);
      mn = (float)m;
    };
    float scg, mg, sch, mh;
    scale_min(hg, scg, mg);
    scale_min(hh, sch, mh);
    const float nmg = -dming * mg, nmh = -dminh * mh;
#pragma unroll
    for (int n = 0; n < NT; n++) {
      const uint4 bf = *reinterpret_cast<const uint4*>(frag + ((s * NT + n) * 32 + lane) * 16);
      float acc[4] = {0.f, 0.f, 0.f, 0.f};
      mma16816(acc, a1[0], a1[1], a1[2], a1[3], bf.x, bf.y);
      mma16816(acc, a2[0], a2[1], a2[2], a2[3], bf.z, bf.w);
      pg[n] = fmaf(scg, acc[0] + acc[1], pg[n]);
      ph[n] = fmaf(sch, acc[2] + acc[3], ph[n]);
      const float X = sums[(s * 4 + t) * NT + n];
      yg[n] = fmaf(nmg, X, yg[n]);
      yh[n] = fmaf(nmh, X, yh[n]);
    }
  }
  const float dg = h2f_ref(hg.x & 0xFFFFu), dh = h2f_ref(hh.x & 0xFFFFu);
#pragma unroll
  for (int n = 0; n < NT; n++) {
    const float F = fsc[t * NT + n];
    yg[n] = fmaf(dg * F, pg[n], yg[n]);
    yh[n] = fmaf(dh * F, ph[n], yh[n]);
  }
}

// (iii) One Q6_K block: one k16 MMA per 16-weight sub-block.
template <int NT>
__device__ __forceinline__ void tb_q6_block(const uint8_t* unit, const uint8_t* frag, const float* sums,
                                            const float* fsc, float (&yg)[NT], float (&yh)[NT]) {
  const int lane = threadIdx.x & 31, g = lane >> 2, t = lane & 3;
  // words W0, W1, H (G, c = t >> 1, p = t & 1) of rows g, g + 8 (device.cuh): lane t
  // holds weights 4t .. 4t + 3 of every sub-block
  const uint32_t c = t >> 1, p = t & 1;
  uint32_t wg[3][4], wh[3][4];
#pragma unroll
  for (int arr = 0; arr < 3; arr++)
#pragma unroll
    for (int G = 0; G < 4; G++) {
      wg[arr][G] = *reinterpret_cast<const uint32_t*>(unit + q6t_word_off(g, arr, G, c, p));
      wh[arr][G] = *reinterpret_cast<const uint32_t*>(unit + q6t_word_off(g + 8, arr, G, c, p));
    }
  // the 6-bit values of sub-block 4G + sg as four bytes
  auto v6 = [](const uint32_t (&w)[3][4], int G, int sg) -> uint32_t {
    const uint32_t n = w[sg & 1][G], h = w[2][G];
    const uint32_t lo = (sg >> 1) ? (n >> 4) : n;
    const uint32_t hi = sg == 0 ? h : sg == 1 ? (h << 4) : sg == 2 ? (h >> 2) : (h << 2);
    return (lo & 0x0F0F0F0Fu) | (hi & 0x30303030u);
  };
  const uint4 scg4 = reinterpret_cast<const uint4*>(unit)[g], sch4 = reinterpret_cast<const uint4*>(unit)[g + 8];
  const uint32_t scgw[4] = {scg4.x, scg4.y, scg4.z, scg4.w}, schw[4] = {sch4.x, sch4.y, sch4.z, sch4.w};
  const float dg = q6_d(reinterpret_cast<const unsigned short*>(unit + 256)[g]);
  const float dh = q6_d(reinterpret_cast<const unsigned short*>(unit + 256)[g + 8]);
  float pg[NT], ph[NT];
#pragma unroll
  for (int n = 0; n < NT; n++) pg[n] = ph[n] = 0.f;
#pragma unroll
  for (int s = 0; s < 16; s++) {
    const uint32_t vg = v6(wg, s >> 2, s & 3), vh = v6(wh, s >> 2, s & 3);
    // bytes 0, 2 / 1, 3 as f16 subnormals v * 2^-24
    const uint32_t a[4] = {vg & 0x003F003Fu, vh & 0x003F003Fu, (vg >> 8) & 0x003F003Fu, (vh >> 8) & 0x003F003Fu};
    const float sg = (float)(int8_t)((scgw[s >> 2] >> (8 * (s & 3))) & 0xFFu);
    const float sh = (float)(int8_t)((schw[s >> 2] >> (8 * (s & 3))) & 0xFFu);
    const float sgp = sg, shp = sh;
    const float nqg = -32.f * dg * sg, nqh = -32.f * dh * sh;  // the stored values are q + 32
#pragma unroll
    for (int n = 0; n < NT; n++) {
      const uint2 bf = *reinterpret_cast<const uint2*>(frag + ((s * NT + n) * 32 + lane) * 8);
      float acc[4] = {0.f, 0.f, 0.f, 0.f};
      mma16816(acc, a[0], a[1], a[2], a[3], bf.x, bf.y);
      pg[n] = fmaf(sgp, acc[0] + acc[1], pg[n]);
      ph[n] = fmaf(shp, acc[2] + acc[3], ph[n]);
      const float X = sums[(s * 4 + t) * NT + n];
      yg[n] = fmaf(nqg, X, yg[n]);
      yh[n] = fmaf(nqh, X, yh[n]);
    }
  }
#pragma unroll
  for (int n = 0; n < NT; n++) {
    const float F = fsc[t * NT + n];
    yg[n] = fmaf(dg * F, pg[n], yg[n]);
    yh[n] = fmaf(dh * F, ph[n], yh[n]);
  }
}

// Epilogue of one tile: v[n] = the full dot product of row (g | g + 8) with
// column 4n + t, already times the input-norm scale of its column.
template <int NT>
__device__ __forceinline__ void tb_epilogue(const GemvArgs& a, uint32_t tile, uint32_t n_parts, const float (&vg)[NT],
                                            const float (&vh)[NT]) {
  const int lane = threadIdx.x & 31, g = lane >> 2, t = lane & 3;
  uint32_t si = 0;
  if (a.nseg > 1 && tile >= a.seg[1].cta_begin) si = 1;
  if (a.nseg > 2 && tile >= a.seg[2].cta_begin) si = 2;
  const GemvSeg& sg = a.seg[si];
  const uint32_t row0 = (tile - sg.cta_begin) * 16u;
#pragma unroll
  for (int n = 0; n < NT; n++) {
    const uint32_t col = 4u * n + t;
    if (epi_is_pair(sg.epi)) {
      const float ng = __shfl_down_sync(0xffffffffu, vg[n], 4), nh = __shfl_down_sync(0xffffffffu, vh[n], 4);
      if (!(g & 1) && col < a.batch) {
        const uint32_t o = row0 + (uint32_t)g;
        if (o < sg.w.n_out) epi_pair(a, sg, o, col, vg[n], ng);
        if (o + 8 < sg.w.n_out) epi_pair(a, sg, o + 8, col, vh[n], nh);
      }
    } else {
      float xg = 0.f, xh = 0.f;
      if (col < a.batch) {
        const uint32_t o = row0 + (uint32_t)g;
        if (o < sg.w.n_out) xg = epi_single(a, sg, o, col, vg[n]);
        if (o + 8 < sg.w.n_out) xh = epi_single(a, sg, o + 8, col, vh[n]);
      }
      if (sg.epi == EPI_RESID) {  // partial sum of x^2 over the tile's 16 rows, per column
        float s2 = xg * xg + xh * xh;
        s2 += __shfl_xor_sync(0xffffffffu, s2, 4);
        s2 += __shfl_xor_sync(0xffffffffu, s2, 8);
        s2 += __shfl_xor_sync(0xffffffffu, s2, 16);
        if (g == 0 && col < a.batch) a.out_parts[(size_t)col * n_parts + tile] = s2;
      }
    }
  }
}

template <int NT, int QT>
__global__ void __launch_bounds__(TB_THREADS, 1) gemv_tcb_kernel(const __grid_constant__ GemvArgs a,
                                                                 const __grid_constant__ TbPlan p) {
  using L = TbSmem<NT>;
  extern __shared__ __align__(128) uint8_t tb_smem[];
  __shared__ float s_in[TB_MAXB];
  __shared__ uint32_t s_last;
  __shared__ __align__(8) uint64_t s_bars[TB_WARPS * TB_STAGES];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  uint8_t* ring = tb_smem + L::OFF_RING + (size_t)warp * TB_STAGES * p.stage_bytes;
  float* sums = reinterpret_cast<float*>(tb_smem + L::OFF_SUMS);
  float* fsc = reinterpret_cast<float*>(tb_smem + L::OFF_FSC);
  float* scl = reinterpret_cast<float*>(tb_smem + L::OFF_SCL);
  constexpr uint32_t SUMF = L::SUMS / 4, FSCF = L::FSC / 4;
  constexpr uint32_t UB = QT == 12 ? Q4T_UNIT : Q6T_UNIT;
  const uint32_t nb = a.seg[0].w.n_in >> 8;
  uint64_t* bars = s_bars + warp * TB_STAGES;
  if (lane == 0) {
    for (uint32_t k = 0; k < TB_STAGES; k++) mbar_init(bars + k, 1);
    fence_mbar_init();
  }
  __syncwarp();
  uint32_t nuse = 0;
  pdl_trigger();
  pdl_wait();
  for (uint32_t c = warp; c < a.batch; c += TB_WARPS) {
    const float v = input_scale(a, c);
    if (lane == 0) s_in[c] = v;
  }
  for (uint32_t unit = blockIdx.x; unit < p.units; unit += gridDim.x) {
    const uint32_t rg = unit / p.ksplit, ks = unit - rg * p.ksplit;
    const uint32_t b0 = ks * p.slice, nblk = min(p.slice, nb - b0), tile = rg * TB_WARPS + warp;
    const uint8_t* tb = nullptr;
    if (tile < p.tiles) {
      uint32_t si = 0;
      if (a.nseg > 1 && tile >= a.seg[1].cta_begin) si = 1;
      if (a.nseg > 2 && tile >= a.seg[2].cta_begin) si = 2;
      const DWDesc& w = a.seg[si].w;
      tb = w.body + (size_t)(tile - a.seg[si].cta_begin) * w.body_stride;
    }
    // ring: slot of the next copy (ip) and of the next block (cp, phase cph)
    uint32_t ip = nuse % TB_STAGES, cp = ip, cph = (nuse / TB_STAGES) & 1u;
    auto issue = [&](uint32_t i) {
      if (i >= nblk || !tb) return;
      if (lane == 0) tc_issue(tb + (size_t)(b0 + i) * UB, UB, ring, p.stage_bytes, bars, ip);
      ip = ip + 1 == TB_STAGES ? 0 : ip + 1;
    };
    for (uint32_t k = 0; k + 1 < TB_STAGES; k++) issue(k);
    __syncthreads();  // the previous unit is done with the shared x data
    tb_scales<NT, QT>(a.x, a.ldx, a.batch, (b0 + 0) * 256, sums, fsc, scl);
    if (nblk > 1) tb_scales<NT, QT>(a.x, a.ldx, a.batch, (b0 + 1) * 256, sums + SUMF, fsc + FSCF, scl + TB_MAXB);
    __syncthreads();
    tb_frags<NT, QT>(a.x, a.ldx, a.batch, b0 * 256, scl, tb_smem);
    float yg[NT], yh[NT];
#pragma unroll
    for (int n = 0; n < NT; n++) yg[n] = yh[n] = 0.f;
    for (uint32_t i = 0; i < nblk; i++) {
      __syncthreads();  // block i's fragments and scales are complete; i - 1's buffers are free
      if (i + 2 < nblk) {
        const uint32_t r3 = (i + 2) % 3;
        tb_scales<NT, QT>(a.x, a.ldx, a.batch, (b0 + i + 2) * 256, sums + r3 * SUMF, fsc + r3 * FSCF,
                          scl + r3 * TB_MAXB);
      }
      if (i + 1 < nblk)
        tb_frags<NT, QT>(a.x, a.ldx, a.batch, (b0 + i + 1) * 256, scl + ((i + 1) % 3) * TB_MAXB,
                         tb_smem + ((i + 1) & 1) * L::FRAG);
      if (tb) {
        issue(i + TB_STAGES - 1);
        mbar_wait(bars + cp, cph, a.err);
        const uint8_t* sp = ring + cp * p.stage_bytes;
        if (++cp == TB_STAGES) { cp = 0; cph ^= 1u; }
        const uint32_t r3 = i % 3;
        if constexpr (QT == 12)
          tb_q4_block<NT>(sp, tb_smem + (i & 1) * L::FRAG, sums + r3 * SUMF, fsc + r3 * FSCF, yg, yh);
        else
          tb_q6_block<NT>(sp, tb_smem + (i & 1) * L::FRAG, sums + r3 * SUMF, fsc + r3 * FSCF, yg, yh);
        __syncwarp();  // every lane is done with the slot before it is refilled
      }
    }
    if (tb) nuse += nblk;
    const int t = lane & 3;
#pragma unroll
    for (int n = 0; n < NT; n++) {
      const float si = (4 * n + t) < (int)a.batch ? s_in[4 * n + t] : 0.f;
      yg[n] *= si;
      yh[n] *= si;
    }
    if (p.ksplit == 1) {
      if (tile < p.tiles) tb_epilogue<NT>(a, tile, p.tiles, yg, yh);
      continue;
    }
    // K-split: publish this slice; the last CTA of the group sums the slices in order.
    const int g = lane >> 2;
    const size_t stride = (size_t)p.tiles * 16u * a.batch;
    if (tile < p.tiles) {
#pragma unroll
      for (int n = 0; n < NT; n++) {
        const uint32_t col = 4u * n + t;
        if (col < a.batch) {
          a.ks_part[ks * stride + ((size_t)tile * 16u + g) * a.batch + col] = yg[n];
          a.ks_part[ks * stride + ((size_t)tile * 16u + g + 8) * a.batch + col] = yh[n];
        }
      }
    }
    __threadfence();
    __syncthreads();
    // a wrapping increment: the group's counter is back at zero once its last
    // slice arrives, so no later store resets it
    if (threadIdx.x == 0) s_last = atomicInc(&a.ks_cnt[rg], p.ksplit - 1u) == p.ksplit - 1u;
    __syncthreads();
    if (s_last) {
      __threadfence();
      if (tile < p.tiles) {
#pragma unroll
        for (int n = 0; n < NT; n++) {
          const uint32_t col = 4u * n + t;
          float sg = 0.f, sh = 0.f;
          if (col < a.batch)
            for (uint32_t k = 0; k < p.ksplit; k++) {
              sg += __ldcg(a.ks_part + k * stride + ((size_t)tile * 16u + g) * a.batch + col);
              sh += __ldcg(a.ks_part + k * stride + ((size_t)tile * 16u + g + 8) * a.batch + col);
            }
          yg[n] = sg;
          yh[n] = sh;
        }
        tb_epilogue<NT>(a, tile, p.tiles, yg, yh);
      }
    }
  }
}

// ------------------------------------------------------------- host ----
namespace {

using TbKernel = void (*)(GemvArgs, TbPlan);

template <int NT>
uint32_t tb_smem_bytes(uint32_t stage_bytes) {
  return TbSmem<NT>::OFF_RING + TB_WARPS * TB_STAGES * stage_bytes;
}

TbKernel tb_kernel(uint32_t nt, uint32_t qt) {
  switch (nt * 100 + qt) {
    case 112: return gemv_tcb_kernel<1, 12>;
    case 114: return gemv_tcb_kernel<1, 14>;
    case 212: return gemv_tcb_kernel<2, 12>;
    case 214: return gemv_tcb_kernel<2, 14>;
    case 412: return gemv_tcb_kernel<4, 12>;
    case 414: return gemv_tcb_kernel<4, 14>;
    case 812: return gemv_tcb_kernel<8, 12>;
    case 814: return gemv_tcb_kernel<8, 14>;
  }
  return nullptr;
}

uint32_t tb_nt(uint32_t batch) { return batch <= 4 ? 1 : batch <= 8 ? 2 : batch <= 16 ? 4 : 8; }

uint32_t tb_smem_for(uint32_t nt, uint32_t stage_bytes) {
  switch (nt) {
    case 1: return tb_smem_bytes<1>(stage_bytes);
    case 2: return tb_smem_bytes<2>(stage_bytes);
    case 4: return tb_smem_bytes<4>(stage_bytes);
    default: return tb_smem_bytes<8>(stage_bytes);
  }
}

constexpr int TB_MAX_DEVICES = 64;
std::mutex g_tb_mu;
int g_tb_sms[TB_MAX_DEVICES] = {};

cudaError_t tb_setup(uint32_t* sms) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  if (dev < 0 || dev >= TB_MAX_DEVICES) return cudaErrorInvalidDevice;
  std::lock_guard<std::mutex> lk(g_tb_mu);
  if (!g_tb_sms[dev]) {
    int n = 0;
    e = cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
    for (uint32_t nt : {1u, 2u, 4u, 8u})
      for (uint32_t qt : {12u, 14u})
        if (e == cudaSuccess)
          e = cudaFuncSetAttribute(tb_kernel(nt, qt), cudaFuncAttributeMaxDynamicSharedMemorySize, TB_SMEM_MAX);
    if (e != cudaSuccess) return e;
    g_tb_sms[dev] = n;
  }
  *sms = (uint32_t)g_tb_sms[dev];
  return cudaSuccess;
}

// One weight type for every segment, batch 2..32, whole 256-blocks.
bool tb_ok(const GemvArgs& a) {
  if (a.batch < 2 || a.batch > TB_MAXB || !a.nseg) return false;
  const uint32_t qt = a.seg[0].w.type;
  if (!tiled_type(qt)) return false;
  for (uint32_t i = 0; i < a.nseg; i++)
    if (a.seg[i].w.type != qt || a.seg[i].w.n_in != a.seg[0].w.n_in) return false;
  return (a.ldx & 3u) == 0;
}

// Tiles, K-split and shared memory; the split minimizes rounds of units x
// (blocks per unit + 2 blocks of per-unit cost), bounded by the scratch.
bool tb_plan(GemvArgs& a, uint32_t sms, TbPlan* p) {
  uint32_t tiles = 0;
  for (uint32_t i = 0; i < a.nseg; i++) {
    a.seg[i].cta_begin = tiles;
    tiles += (a.seg[i].w.n_out + 15) / 16;
  }
  const uint32_t nb = a.seg[0].w.n_in >> 8, groups = (tiles + TB_WARPS - 1) / TB_WARPS;
  const uint32_t stage_bytes = a.seg[0].w.type == 12 ? Q4T_UNIT : Q6T_UNIT;
  if (tb_smem_for(tb_nt(a.batch), stage_bytes) > TB_SMEM_MAX || nb == 0) return false;
  auto fits = [&](uint32_t k) {
    return k == 1 || (a.ks_part && a.ks_cnt && (uint64_t)k * tiles * 16u * a.batch <= a.ks_part_cap &&
                      groups <= a.ks_cnt_cap);
  };
  uint32_t ks = 0;
  uint64_t best = ~0ull;
  for (uint32_t k = 1; k <= std::min(nb, 64u); k++) {
    const uint32_t sl = (nb + k - 1) / k, kk = (nb + sl - 1) / sl;
    if (!fits(kk)) continue;
    const uint64_t rounds = ((uint64_t)groups * kk + sms - 1) / sms;
    if (rounds * (sl + 2) < best) {
      best = rounds * (sl + 2);
      ks = kk;
    }
  }
  if (!ks) return false;
  p->tiles = tiles;
  p->groups = groups;
  p->ksplit = ks;
  p->slice = (nb + ks - 1) / ks;
  p->units = groups * ks;
  p->grid = std::min(p->units, sms);
  p->stage_bytes = stage_bytes;
  p->smem = tb_smem_for(tb_nt(a.batch), stage_bytes);
  return true;
}

}  // namespace

cudaError_t gemv_tcb_prepare() {
  uint32_t sms = 0;
  return tb_setup(&sms);
}

bool gemv_tcb_ok(const GemvArgs& a) { return tb_ok(a); }

// cudaErrorNotSupported: no plan fits (use another kernel). n_parts: the
// per-column partials an EPI_RESID launch writes (one per tile).
cudaError_t launch_gemv_tcb(GemvArgs a, cudaStream_t st, uint32_t* n_parts) {
  if (!tb_ok(a)) return cudaErrorNotSupported;
  uint32_t sms = 0;
  cudaError_t e = tb_setup(&sms);
  if (e != cudaSuccess) return e;
  TbPlan p;
  if (!tb_plan(a, sms, &p)) return cudaErrorNotSupported;
  if (n_parts) *n_parts = p.tiles;
  return launch_pdl(tb_kernel(tb_nt(a.batch), a.seg[0].w.type), dim3(p.grid), dim3(TB_THREADS), p.smem, st, a, p);
}

void gemv_tcb_scratch_need(GemvArgs a, uint32_t sms, uint64_t* part, uint32_t* cnt) {
  a.ks_part = reinterpret_cast<float*>(16);
  a.ks_cnt = reinterpret_cast<uint32_t*>(16);
  a.ks_part_cap = 0xFFFFFFFFu;
  a.ks_cnt_cap = 0xFFFFFFFFu;
  *part = 0;
  *cnt = 0;
  TbPlan p;
  if (!tb_ok(a) || !tb_plan(a, sms, &p) || p.ksplit == 1) return;
  *part = (uint64_t)p.ksplit * p.tiles * 16u * a.batch;
  *cnt = p.groups;
}

}  // namespace sm
