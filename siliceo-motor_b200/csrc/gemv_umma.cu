// Batched GEMV (2..32 columns: batched decode steps and prefill chunks) of
// Q4_K / Q6_K weights on the 5th-generation tensor cores (tcgen05, sm_100a).
//
// A CTA tile is 128 output rows (eight 16-row weight tiles, device.cuh) and a
// K-slice, computed as D[128 x N] += A[128 x 16] B[N x 16] MMAs (M = 128,
// N = 2 x columns, K = 16) with f32 accumulators in tensor memory:
//   * a prep kernel converts x once per launch into the shared-memory image
//     of the B operand (per column and 256-block a power-of-two scale, each
//     value as hi + lo f16 rows: 22 bits), plus the per-sub-block sums of x
//     and the input-norm scales; a producer warp bulk-copies that image block
//     by block into a ring of shared-memory slots;
//   * a second producer warp streams the block units of the eight weight
//     tiles from HBM into a ring of stages;
//   * eight row warps (one row per thread, tensor-memory lane = row) turn
//     the quants into exact f16 integers and store them as the A operand:
//       Q4_K: sc_s * q                     (sc <= 63, q <= 15: at most 945)
//       Q6_K: sc_s * ql / 16 and sc_s * qh (two operands of one accumulator:
//             their sum is sc_s * v / 16 for the stored v = q + 32 = ql +
//             16 qh, and each stays exact in f16 where sc_s * v would not)
//     with one LOP3 (mask | 0x6400 exponent) and one HFMA2 per two weights;
//   * two MMA warps (one for Q6_K) take alternate blocks: one thread each
//     issues the block's MMAs, and one more with both operands in shared
//     memory for the per-sub-block term: A2 = the Q4_K mins m_s or the Q6_K
//     scales sc_s, B2 = sum of x over sub-block s (times 2^-6);
//   * four epilogue warps (one row per thread) read both accumulators after
//     each block and apply the block's d / dmin in f32 (dequant.rs:98-126,
//     178-206):
//       Q4_K: y += u * (d * D - 64 * dmin * D2)
//       Q6_K: y += u * d * (16 * D - 2048 * D2)
//     with u = 1 / (the block's x scale of the column), then run the K-split
//     fixup and the fused epilogue.
// K orders of A and B agree: item i of a block (weights 8i .. 8i + 7) is K
// step i / 2 (16 wide), core-matrix half i % 2, in the order 0 2 1 3 4 6 5 7
// that one mask of a 32-bit quant word yields (weights e, e + 2 per f16x2).
//
// Synchronization is by mbarriers, every wait bounded: a wait that gives up
// sets the launch's error word and a CTA-wide abort flag after which the
// other waits return at once; the CTA then waits (bounded) for its own MMAs
// and copies, frees its tensor memory and exits. K-splits end in the
// deterministic last-arriver fixup of the other GEMVs (slices summed in
// order); epilogues are the fused ones of gemv_common.cuh.
#include <cuda_fp16.h>

#include <algorithm>
#include <mutex>

#include "device.cuh"
#include "gemv_common.cuh"
#include "pdl.cuh"
#include "tc_common.cuh"
#include "umma.cuh"

namespace sm {

uint64_t gemv_umma_blob_bytes(uint32_t n_in, uint32_t batch);

constexpr int UM_RW = 8, UM_EW = 4;  // row warps (A operands), epilogue warps (accumulators)
// Two MMA warps take alternate blocks (one thread issues at ~50 cycles per
// MMA, two keep the tensor pipe busy at N = 64); the first also owns the
// tensor-memory allocation.
constexpr int UM_EW0 = UM_RW, UM_BPW = UM_RW + UM_EW, UM_PROD = UM_BPW + 1, UM_MMAW = UM_BPW + 2,
              UM_WARPS = UM_BPW + 4;
constexpr int UM_THREADS = UM_WARPS * 32;
constexpr uint32_t UM_MAXB = 32;                // columns
constexpr uint32_t UM_TILES = 8;                // 16-row weight tiles per CTA tile
constexpr uint32_t UM_SMEM_MIN = 116u * 1024u;  // one CTA per SM: it holds all of tensor memory
constexpr uint32_t UM_SMEM_MAX = 224u * 1024u;  // with the static part (2 KB), within the 227 KB opt-in
// tensor-memory columns: A operands of two half-blocks, D and D2 of two blocks
constexpr uint32_t UM_TA = 0, UM_TD = 256, UM_TD2 = 384, UM_TCOLS = 512;
constexpr uint32_t UM_XPREP_THREADS = 128;

struct UmPlan {
  uint32_t tiles, groups, ksplit, slice, units, grid, smem;
};

// Byte offset of row `row`, core-matrix half kc (K 8kc .. 8kc + 7) in a
// K-major 16-wide operand without swizzle (LBO 128 B, SBO 256 B).
SM_HD uint32_t um_core(uint32_t row, uint32_t kc) { return (row >> 3) * 256u + kc * 128u + (row & 7u) * 16u; }

// The B image of one 256-block (NB columns, padded to 8 / 16 / 32):
// [16 K steps x N rows x 16 K f16][B2: N rows x 16][u: 32 f32]; the whole
// launch's image is nb of them followed by the input-norm scales (32 f32).
template <int NB>
struct UmBlob {
  static constexpr uint32_t N = 2 * NB;  // MMA N: a hi and a lo row per column
  static constexpr uint32_t KSTEP = N * 32, B2 = N * 32;
  static constexpr uint32_t OFF_B2 = 16 * KSTEP, OFF_U = OFF_B2 + B2, BLK = OFF_U + UM_MAXB * 4;
};
// Weight stages in flight per type.
template <int QT>
struct UmW {
  static constexpr uint32_t UB = QT == 12 ? Q4T_UNIT : Q6T_UNIT, STAGES = QT == 12 ? 4 : 3;
  static constexpr uint32_t BYTES = STAGES * UM_TILES * UB;
};
// Shared memory: weight stages | B slots | A2[2] (128 rows x 16 K f16) |
// the rows' (d, dmin) of the last 4 blocks
template <int NB, int QT>
struct UmSmem {
  static constexpr uint32_t SLOTS = QT == 12 ? (NB == 32 ? 4 : NB == 16 ? 6 : 8) : (NB == 32 ? 3 : NB == 16 ? 5 : 8);
  static constexpr uint32_t OFF_B = (UmW<QT>::BYTES + 1023u) / 1024u * 1024u;
  static constexpr uint32_t OFF_A2 = OFF_B + SLOTS * UmBlob<NB>::BLK;
  static constexpr uint32_t A2 = 128 * 32;
  static constexpr uint32_t OFF_DD = OFF_A2 + 2 * A2;
  static constexpr uint32_t BYTES = OFF_DD + 4 * 128 * 8;
};

__device__ __forceinline__ void mbar_arrive(uint64_t* b) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(b)) : "memory");
}
__device__ __forceinline__ void named_bar(uint32_t id, uint32_t n) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(n) : "memory");
}
// Bounded wait that also gives up soon after the CTA has aborted (the flag is
// read every 32nd try: read on every try, it costs the waiting warps a
// shared-memory load per try, ~18% of a long launch).
__device__ __forceinline__ bool um_wait(uint64_t* b, uint32_t parity, uint32_t* err, volatile uint32_t* abort) {
  for (uint32_t n = 0; n < TC_SPIN_MAX; n++) {
    if (mbar_try(b, parity)) return true;
    if ((n & 31u) == 31u && *abort) return false;
  }
  *abort = 1u;
  if (err) atomicOr(err, 1u);
  return false;
}
// Bounded wait for teardown (ignores the abort flag).
__device__ __forceinline__ void um_drain(uint64_t* b, uint32_t parity, uint32_t* err) {
  for (uint32_t n = 0; n < TC_SPIN_MAX; n++)
    if (mbar_try(b, parity)) return;
  if (err) atomicOr(err, 1u);
}
// (w & mask) | 0x6400 in both halves: 1024 + the masked field, as f16.
__device__ __forceinline__ __half2 um_mag(uint32_t w, uint32_t mask) {
  uint32_t r;
  asm("lop3.b32 %0, %1, %2, %3, 0xEA;" : "=r"(r) : "r"(w), "r"(mask), "r"(0x64006400u));  // (a & b) | c
  return u2h(r);
}
__device__ __forceinline__ uint32_t um_fma(__half2 v, __half2 m, __half2 c) { return h2u(__hfma2(v, m, c)); }
template <int K>
__device__ __forceinline__ void tmem_ld(uint32_t t, uint32_t (&r)[K]) {
  if constexpr (K == 8) tmem_ld8(t, r);
  else if constexpr (K == 16) tmem_ld16(t, r);
  else tmem_ld32(t, r);
}

// Q4_K: get_scale_min_k4 (dequant.rs:41-49) of all eight sub-blocks.
__device__ __forceinline__ void um_q4_scales(const uint4& h, uint32_t (&sc)[8], uint32_t (&mn)[8]) {
#pragma unroll
  for (int s = 0; s < 8; s++) {
    if (s < 4) {
      sc[s] = (h.y >> (8 * s)) & 63u;
      mn[s] = (h.z >> (8 * s)) & 63u;
    } else {
      const int s4 = 8 * (s - 4);
      sc[s] = ((h.w >> s4) & 0xFu) | (((h.y >> (s4 + 6)) & 3u) << 4);
      mn[s] = ((h.w >> (s4 + 4)) & 0xFu) | (((h.z >> (s4 + 6)) & 3u) << 4);
    }
  }
}

// A operand of one half-block for the calling row: Q4_K sub-blocks 2j, 2j + 1
// (words W[p][c] = qs bytes 32j + 8c + 4p .. + 3). Column sigma*16 + 4c + 2p
// + b holds weights (8c + 4p + b, + 2) of sub-block 2j + sigma.
__device__ __forceinline__ void um_q4_a(const uint4 (&W)[2], uint32_t sc0, uint32_t sc1, uint32_t (&A)[32]) {
  const __half2 m0 = __float2half2_rn((float)sc0), c0 = __float2half2_rn(-1024.f * (float)sc0);
  const __half2 m1 = __float2half2_rn(0.0625f * (float)sc1), c1 = __float2half2_rn(-64.f * (float)sc1);
#pragma unroll
  for (int p = 0; p < 2; p++) {
    const uint32_t w4[4] = {W[p].x, W[p].y, W[p].z, W[p].w};
#pragma unroll
    for (int c = 0; c < 4; c++) {
      const uint32_t w = w4[c], w8 = w >> 8;
      A[4 * c + 2 * p + 0] = um_fma(um_mag(w, 0x000F000Fu), m0, c0);
      A[4 * c + 2 * p + 1] = um_fma(um_mag(w8, 0x000F000Fu), m0, c0);
      A[16 + 4 * c + 2 * p + 0] = um_fma(um_mag(w, 0x00F000F0u), m1, c1);
      A[16 + 4 * c + 2 * p + 1] = um_fma(um_mag(w8, 0x00F000F0u), m1, c1);
    }
  }
}

// Q6_K operands of one half-block for the calling row, sub-blocks 4G + sigma:
// w[a][p] = words (a, G, c = 0, 1, p) (a: W0, W1, H). Column sigma*8 + 4c +
// 2p + b holds weights (8c + 4p + b, + 2); Al = sc * ql / 16, Ah = sc * qh.
__device__ __forceinline__ void um_q6_al(const uint2 (&w)[3][2], const int32_t (&sc)[4], uint32_t (&A)[32]) {
  __half2 m[4], c[4];
#pragma unroll
  for (int s = 0; s < 4; s++) {
    const float f = (float)sc[s];
    // sigma 0, 1: low nibble (1024 + ql); sigma 2, 3: high nibble (1024 + 16 ql)
    m[s] = __float2half2_rn(s < 2 ? f * 0.0625f : f * 0.00390625f);
    c[s] = __float2half2_rn(s < 2 ? -64.f * f : -4.f * f);
  }
#pragma unroll
  for (int p = 0; p < 2; p++)
#pragma unroll
    for (int cc = 0; cc < 2; cc++) {
      const uint32_t w0 = cc ? w[0][p].y : w[0][p].x, w1 = cc ? w[1][p].y : w[1][p].x;
#pragma unroll
      for (int b = 0; b < 2; b++) {
        const uint32_t v0 = b ? w0 >> 8 : w0, v1 = b ? w1 >> 8 : w1;
        const int col = 4 * cc + 2 * p + b;
        A[0 * 8 + col] = um_fma(um_mag(v0, 0x000F000Fu), m[0], c[0]);
        A[1 * 8 + col] = um_fma(um_mag(v1, 0x000F000Fu), m[1], c[1]);
        A[2 * 8 + col] = um_fma(um_mag(v0, 0x00F000F0u), m[2], c[2]);
        A[3 * 8 + col] = um_fma(um_mag(v1, 0x00F000F0u), m[3], c[3]);
      }
    }
}
__device__ __forceinline__ void um_q6_ah(const uint2 (&w)[3][2], const int32_t (&sc)[4], uint32_t (&A)[32]) {
  // H: bits 0-1 sigma 1 (moved to 2-3), 2-3 sigma 3, 4-5 sigma 0, 6-7 sigma 2
  __half2 m[4], c[4];
  const float mul[4] = {0.0625f, 0.25f, 0.015625f, 0.25f}, add[4] = {-64.f, -256.f, -16.f, -256.f};
#pragma unroll
  for (int s = 0; s < 4; s++) {
    m[s] = __float2half2_rn(mul[s] * (float)sc[s]);
    c[s] = __float2half2_rn(add[s] * (float)sc[s]);
  }
#pragma unroll
  for (int p = 0; p < 2; p++)
#pragma unroll
    for (int cc = 0; cc < 2; cc++) {
      const uint32_t h = cc ? w[2][p].y : w[2][p].x;
#pragma unroll
      for (int b = 0; b < 2; b++) {
        const uint32_t v = b ? h >> 8 : h, v2 = v << 2;
        const int col = 4 * cc + 2 * p + b;
        A[0 * 8 + col] = um_fma(um_mag(v, 0x00300030u), m[0], c[0]);
        A[1 * 8 + col] = um_fma(um_mag(v2, 0x000C000Cu), m[1], c[1]);
        A[2 * 8 + col] = um_fma(um_mag(v, 0x00C000C0u), m[2], c[2]);
        A[3 * 8 + col] = um_fma(um_mag(v, 0x000C000Cu), m[3], c[3]);
      }
    }
}

// Per-column constants of a decode launch, read once per CTA into shared
// memory by the epilogue warps while the blocks stream: the RoPE rows at the
// column's position and its K / V cache rows for this layer. Read inside the
// column loop they would be chains of dependent loads (row -> sequence ->
// page) per column, and the loop's stores keep the compiler from overlapping
// the loads of one column with another's.
struct UmCol {
  const float* cs;
  const float* sn;
  float* kc;
  float* vc;
};

// Column t's entry (t < batch; called by one thread per column).
__device__ __forceinline__ void um_col_fill(const GemvArgs& a, uint32_t t, UmCol* cols) {
  UmCol c{nullptr, nullptr, nullptr, nullptr};
  bool rope = false, kv = false;
  for (uint32_t i = 0; i < a.nseg; i++) {
    const uint32_t e = a.seg[i].epi;
    rope |= e == EPI_ROPE_Q || e == EPI_ROPE_K;
    kv |= e == EPI_ROPE_K || e == EPI_V;
  }
  if (a.rows && (rope || kv)) {
    const RowDesc rd = a.rows[t];
    if (rope) {
      const size_t r = (size_t)rd.pos * (a.hd >> 1);
      c.cs = a.cos_t + r;
      c.sn = a.sin_t + r;
    }
    if (kv) {
      const SeqDesc sd = a.seqs[rd.seq];
      c.kc = sd.pages[rd.pos / KV_PAGE] + kv_page_off(a.layer, rd.pos, a.kvd);
      c.vc = c.kc + sd.voff;
    }
  }
  cols[t] = c;
}

// Partial sum of x^2 over the tile's 16 rows for one column (EPI_RESID
// launches); every lane of the warp calls it.
__device__ __forceinline__ void um_resid_part(const GemvArgs& a, float xv, bool write, uint32_t col,
                                              uint32_t n_parts, uint32_t tile) {
  const int lane = threadIdx.x & 31;
  float s2 = xv * xv;
  s2 += __shfl_xor_sync(0xffffffffu, s2, 1);
  s2 += __shfl_xor_sync(0xffffffffu, s2, 2);
  s2 += __shfl_xor_sync(0xffffffffu, s2, 4);
  s2 += __shfl_xor_sync(0xffffffffu, s2, 8);
  if ((lane & 15) == 0 && write) a.out_parts[(size_t)col * n_parts + tile] = s2;
}

// Epilogue of the calling row (y[i]: column c0 + i, already times the
// input-norm scale): the fused epilogues of gemv_common.cuh (epi_single,
// epi_pair) with the same arithmetic, organized for 32 columns a thread. The
// segment's and the row's constants are read once into registers (read
// through the parameter reference they would be reloaded after every output
// store); columns go in chunks of 8 whose loads (residuals, RoPE rows) are
// all issued before the chunk's stores. Every lane of the warp calls it.
template <int NC>
__device__ __forceinline__ void um_epilogue(const GemvArgs& a, const UmCol* cols, uint32_t tile, uint32_t n_parts,
                                            bool valid, uint32_t rr, uint32_t c0, const float (&y)[NC]) {
  const int lane = threadIdx.x & 31;
  uint32_t si = 0;
  if (a.nseg > 1 && tile >= a.seg[1].cta_begin) si = 1;
  if (a.nseg > 2 && tile >= a.seg[2].cta_begin) si = 2;
  const GemvSeg sg = a.seg[si];
  const uint32_t o = (tile - sg.cta_begin) * 16u + rr, batch = a.batch, epi = sg.epi;
  const bool row_ok = valid && o < sg.w.n_out;
  const bool any_resid = a.seg[0].epi == EPI_RESID || (a.nseg > 1 && a.seg[1].epi == EPI_RESID) ||
                         (a.nseg > 2 && a.seg[2].epi == EPI_RESID);
  const bool has_bias = sg.bias != nullptr;
  const float bo = (has_bias && row_ok) ? sg.bias[o] : 0.f;
  float* const yb = sg.y + o;
  const uint32_t ldy = sg.ldy;
  constexpr int CH = NC < 8 ? NC : 8;
  if (epi == EPI_STORE || epi == EPI_ADD || epi == EPI_RESID) {
    // y = v, y += v, or x = y += v; xn = x * nw (qwen2.rs:536-538, 549-551)
    float* const xnb = epi == EPI_RESID ? a.xn + o : nullptr;
    const uint32_t ldxn = a.ldxn;
    const float nwo = (epi == EPI_RESID && row_ok) ? a.nw[o] : 0.f;
    const bool reads = epi != EPI_STORE;
#pragma unroll
    for (int g = 0; g < NC; g += CH) {
      float old[CH];
#pragma unroll
      for (int i = 0; i < CH; i++) {
        const uint32_t col = c0 + g + i;
        old[i] = (reads && row_ok && col < batch) ? yb[(size_t)col * ldy] : 0.f;
      }
#pragma unroll
      for (int i = 0; i < CH; i++) {
        const uint32_t col = c0 + g + i;
        const bool ok = row_ok && col < batch;
        const float v = has_bias ? y[g + i] + bo : y[g + i];
        float xv = 0.f;
        if (ok) {
          float* yy = yb + (size_t)col * ldy;
          if (epi == EPI_STORE) {
            *yy = v;
          } else if (epi == EPI_ADD) {
            *yy = old[i] + v;
          } else {
            xv = old[i] + v;
            *yy = xv;
            xnb[(size_t)col * ldxn] = xv * nwo;
          }
        }
        if (any_resid) um_resid_part(a, xv, valid && col < batch && epi == EPI_RESID, col, n_parts, tile);
      }
    }
    return;
  }
  if (epi_is_pair(epi)) {
    // rows (o, o + 1), o even, on lanes (2j, 2j + 1): the even lane finishes the pair
    const bool even = !(lane & 1), rope = epi != EPI_SILU;
    uint32_t half = 0, hoff = 0, m = 0;
    if (rope) {  // NEOX RoPE of (dim m, dim m + hd/2) of head h (qwen2.rs:708-724)
      const uint32_t hd = a.hd, h = o / hd;
      half = hd >> 1;
      m = (o - h * hd) >> 1;
      hoff = h * hd + m;
    }
    float* const hb = a.h + (o >> 1);
    const uint32_t ldh = a.ldh;
#pragma unroll
    for (int g = 0; g < NC; g += CH) {
      float cc[CH], ss[CH];
#pragma unroll
      for (int i = 0; i < CH; i++) {
        const uint32_t col = c0 + g + i;
        const bool ld = rope && even && row_ok && col < batch;
        cc[i] = ld ? cols[col].cs[m] : 0.f;
        ss[i] = ld ? cols[col].sn[m] : 0.f;
      }
#pragma unroll
      for (int i = 0; i < CH; i++) {
        const uint32_t col = c0 + g + i;
        const bool ok = row_ok && col < batch;
        const float v = has_bias ? y[g + i] + bo : y[g + i];
        const float nv = __shfl_xor_sync(0xffffffffu, v, 1);  // row o + 1, bias included
        if (ok && even) {
          if (epi == EPI_SILU) {  // gate = silu(gate) * up (qwen2.rs:546-548, 743-745)
            hb[(size_t)col * ldh] = __fmul_rn(__fdiv_rn(v, __fadd_rn(1.0f, expf(-v))), nv);
          } else {
            const float r0 = __fsub_rn(__fmul_rn(v, cc[i]), __fmul_rn(nv, ss[i]));
            const float r1 = __fadd_rn(__fmul_rn(v, ss[i]), __fmul_rn(nv, cc[i]));
            // EPI_ROPE_Q: q (natural order); EPI_ROPE_K: the K cache (qwen2.rs:497)
            float* d = epi == EPI_ROPE_Q ? sg.y + (size_t)col * ldy + hoff : cols[col].kc + hoff;
            d[0] = r0;
            d[half] = r1;
          }
        }
        if (any_resid) um_resid_part(a, 0.f, false, col, n_parts, tile);
      }
    }
    return;
  }
  // EPI_V (the V cache row, qwen2.rs:498) and EPI_PUSH (tensor parallel: this
  // rank's partial to every rank's receive area, tp.cu; the row's epoch read once)
  uint32_t pe = 0;
  if (epi == EPI_PUSH && row_ok) pe = __ldcg(a.push.epoch + (a.push.base + o) / a.push.per) + 1u;
#pragma unroll
  for (int i = 0; i < NC; i++) {
    const uint32_t col = c0 + i;
    const bool ok = row_ok && col < batch;
    const float v = has_bias ? y[i] + bo : y[i];
    if (ok) {
      if (epi == EPI_V) {
        cols[col].vc[o] = v;
      } else if (epi == EPI_PUSH) {
        const TpPush& P = a.push;
        const uint64_t pk = ((uint64_t)pe << 32) | __float_as_uint(v);
        const uint64_t off = (pe & 1u) * P.parity_stride + P.rank * P.src_stride + (uint64_t)col * P.ld + o;
        for (uint32_t k = 0; k < P.world; k++)
          asm volatile("st.volatile.global.u64 [%0], %1;" ::"l"(P.dst[k] + off), "l"(pk) : "memory");
      } else {
        epi_single(a, sg, o, col, v);
      }
    }
    if (any_resid) um_resid_part(a, 0.f, false, col, n_parts, tile);
  }
}

// ------------------------------------------------------- x prep kernel ----
// One CTA per (256-block, 8 columns): the B image of x[c, 256 b .. 256 b +
// 255] for those padded columns (column c: lanes (c % 8) * LPC .. + LPC - 1,
// each IPL items of 8 consecutive values). The first CTAs of each column
// group also write its columns' input-norm scales, one warp a column.
constexpr uint32_t UM_XPREP_COLS = 8;
template <int NB, int QT>
__global__ void __launch_bounds__(UM_XPREP_THREADS) umma_xprep_kernel(const __grid_constant__ GemvArgs a, uint32_t nb) {
  using L = UmBlob<NB>;
  constexpr uint32_t LPC = UM_XPREP_THREADS / UM_XPREP_COLS, IPL = 32 / LPC;  // lanes per column, items per lane
  constexpr uint32_t IPS = QT == 12 ? 4 : 2;                                 // items per sub-block
  constexpr uint32_t NXS = IPL / IPS > 0 ? IPL / IPS : 1;
  pdl_trigger();
  pdl_wait();
  const uint32_t blk = blockIdx.x, xt = threadIdx.x, c = blockIdx.y * UM_XPREP_COLS + xt / LPC, u = xt % LPC;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  uint8_t* out = a.xblob + (size_t)blk * L::BLK;
  float v[IPL][8];
  const bool live = c < a.batch;
  const float* xp = a.x + (size_t)c * a.ldx + (size_t)blk * 256 + 8 * IPL * u;
  float mx = 0.f;
#pragma unroll
  for (uint32_t j = 0; j < IPL; j++) {
    float4 lo = make_float4(0.f, 0.f, 0.f, 0.f), hi = lo;
    if (live) {
      lo = ldg4(xp + 8 * j);
      hi = ldg4(xp + 8 * j + 4);
    }
    v[j][0] = lo.x; v[j][1] = lo.y; v[j][2] = lo.z; v[j][3] = lo.w;
    v[j][4] = hi.x; v[j][5] = hi.y; v[j][6] = hi.z; v[j][7] = hi.w;
  }
  {  // the input-norm scales of this CTA row's columns, one warp a column (after
     // the x loads are issued: both sets of loads are then in flight together)
    float* s_in = reinterpret_cast<float*>(a.xblob + (size_t)nb * L::BLK);
    constexpr uint32_t NW = UM_XPREP_THREADS / 32;
    for (uint32_t cc = blk * NW + warp; cc < UM_XPREP_COLS; cc += nb * NW) {
      const uint32_t col = blockIdx.y * UM_XPREP_COLS + cc;
      if (col < a.batch) {
        const float sc = input_scale(a, col);
        if (lane == 0) s_in[col] = sc;
      }
    }
  }
#pragma unroll
  for (uint32_t j = 0; j < IPL; j++)
#pragma unroll
    for (int k = 0; k < 8; k++) mx = fmaxf(mx, fabsf(v[j][k]));
#pragma unroll
  for (uint32_t o = 1; o < LPC; o <<= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
  // the power of two that puts max|x| in [2^14, 2^15)
  const uint32_t E = (__float_as_uint(mx) >> 23) & 0xFFu;
  const float scl = E >= 15u ? __uint_as_float((268u - E) << 23) : 1.f;
  const float inv = E >= 15u ? __uint_as_float((E - 14u) << 23) : 1.f;
  if (u == 0) reinterpret_cast<float*>(out + L::OFF_U)[c] = inv;
  float xsum[NXS];
#pragma unroll
  for (uint32_t s = 0; s < NXS; s++) xsum[s] = 0.f;
  float xpart = 0.f;
#pragma unroll
  for (uint32_t j = 0; j < IPL; j++) {
    const uint32_t it = IPL * u + j, T = it >> 1, kc = it & 1;
    const float w[8] = {v[j][0] * scl, v[j][2] * scl, v[j][1] * scl, v[j][3] * scl,
                        v[j][4] * scl, v[j][6] * scl, v[j][5] * scl, v[j][7] * scl};
    uint32_t hw[4], lw[4];
#pragma unroll
    for (int q = 0; q < 4; q++) {
      const float ah = hi11(w[2 * q]), bh = hi11(w[2 * q + 1]);
      hw[q] = h2u(__floats2half2_rn(ah, bh));
      lw[q] = h2u(__floats2half2_rn(w[2 * q] - ah, w[2 * q + 1] - bh));
    }
    *reinterpret_cast<uint4*>(out + T * L::KSTEP + um_core(2 * c, kc)) = make_uint4(hw[0], hw[1], hw[2], hw[3]);
    *reinterpret_cast<uint4*>(out + T * L::KSTEP + um_core(2 * c + 1, kc)) = make_uint4(lw[0], lw[1], lw[2], lw[3]);
    const float s8 = ((w[0] + w[1]) + (w[2] + w[3])) + ((w[4] + w[5]) + (w[6] + w[7]));
    if constexpr (IPL >= IPS) xsum[j / IPS] += s8;
    else xpart += s8;
  }
  // B2: sub-block sums of the scaled x times 2^-6, hi / lo rows, K position = sub-block
  uint8_t* b2 = out + L::OFF_B2;
  if (QT == 12 && u == 0) {  // Q4_K has 8 sub-blocks: K 8..15 are zero
    *reinterpret_cast<uint4*>(b2 + um_core(2 * c, 1)) = make_uint4(0, 0, 0, 0);
    *reinterpret_cast<uint4*>(b2 + um_core(2 * c + 1, 1)) = make_uint4(0, 0, 0, 0);
  }
  auto put_sum = [&](uint32_t s, float X) {
    X *= 0.015625f;
    const float Xh = hi11(X);
    const uint32_t off = (s & 7u) * 2u;
    *reinterpret_cast<__half*>(b2 + um_core(2 * c, s >> 3) + off) = __float2half_rn(Xh);
    *reinterpret_cast<__half*>(b2 + um_core(2 * c + 1, s >> 3) + off) = __float2half_rn(X - Xh);
  };
  if constexpr (IPL >= IPS) {
#pragma unroll
    for (uint32_t s = 0; s < NXS; s++) put_sum((IPL * u) / IPS + s, xsum[s]);
  } else {  // two lanes share a sub-block
    xpart += __shfl_xor_sync(0xffffffffu, xpart, 1);
    if (!(u & 1)) put_sum((IPL * u) / IPS, xpart);
  }
}

template <int NB, int QT>
__global__ void __launch_bounds__(UM_THREADS, 1) gemv_umma_kernel(const __grid_constant__ GemvArgs a,
                                                                  const __grid_constant__ UmPlan p) {
  using XB = UmBlob<NB>;
  using W = UmW<QT>;
  using L = UmSmem<NB, QT>;
  constexpr uint32_t N = XB::N, UB = W::UB, WS = W::STAGES, BS = L::SLOTS;
  constexpr uint32_t NA = QT == 12 ? 4 : 2, ACOLS = QT == 12 ? 64 : 128;  // A buffers (half-blocks), columns each
  extern __shared__ __align__(1024) uint8_t um_smem[];
  __shared__ __align__(8) uint64_t bar_wfull[WS], bar_wempty[WS], bar_bfull[BS], bar_bfree[BS], bar_afull[NA],
      bar_afree[NA], bar_dfull[2], bar_dfree[2], bar_hdr[4], bar_fin[2];
  __shared__ uint32_t s_tmem, s_last, s_fix;
  __shared__ UmCol s_cols[UM_MAXB];
  __shared__ float s_scale[UM_MAXB];
  __shared__ uint32_t s_abort_word;
  volatile uint32_t* abort = &s_abort_word;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  uint8_t* ring = um_smem;
  uint8_t* bring = um_smem + L::OFF_B;
  uint8_t* a2buf = um_smem + L::OFF_A2;
  float2* dd = reinterpret_cast<float2*>(um_smem + L::OFF_DD);  // [block & 3][row]
  const uint32_t nb = a.seg[0].w.n_in >> 8;

  if (threadIdx.x == 0) {
    for (uint32_t k = 0; k < WS; k++) {
      mbar_init(&bar_wfull[k], 1);
      mbar_init(&bar_wempty[k], UM_RW * 32);
    }
    for (uint32_t k = 0; k < 4; k++) mbar_init(&bar_hdr[k], 4 * 32);
    for (uint32_t k = 0; k < BS; k++) {
      mbar_init(&bar_bfull[k], 1);
      mbar_init(&bar_bfree[k], UM_EW * 32);
    }
    for (uint32_t k = 0; k < NA; k++) {
      mbar_init(&bar_afull[k], UM_RW * 32);
      mbar_init(&bar_afree[k], 1);
    }
    for (uint32_t k = 0; k < 2; k++) {
      mbar_init(&bar_dfull[k], 1);
      mbar_init(&bar_dfree[k], UM_EW * 32);
    }
    mbar_init(&bar_fin[0], 1);
    mbar_init(&bar_fin[1], 1);
    *abort = 0u;
    s_fix = 0u;
    fence_mbar_init();
  }
  if (warp == UM_MMAW) {
    tmem_alloc(&s_tmem, UM_TCOLS);
    tmem_relinquish();
  }
  if (warp < UM_RW) {  // A2 starts zero (Q4_K: K 8..15 stay zero)
    const uint4 z = make_uint4(0, 0, 0, 0);
    for (uint32_t i = threadIdx.x; i < 2 * L::A2 / 16; i += UM_RW * 32) reinterpret_cast<uint4*>(a2buf)[i] = z;
    fence_proxy_async();
  }
  pdl_trigger();
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tb = s_tmem;

  if (warp == UM_PROD || warp == UM_BPW) {
    // ---------------------- producers: weight units / B images (bulk copies)
    const bool wprod = warp == UM_PROD;
    if (!wprod) pdl_wait();  // the B images come from the prep kernel
    const uint32_t S = wprod ? WS : BS;
    uint64_t* full = wprod ? bar_wfull : bar_bfull;
    uint32_t cnt = 0;
    if (lane == 0) {
      for (uint32_t unit = blockIdx.x; unit < p.units && !*abort; unit += gridDim.x) {
        const uint32_t rg = unit / p.ksplit, ks = unit - rg * p.ksplit;
        const uint32_t b0 = ks * p.slice, nblk = min(p.slice, nb - b0);
        const uint8_t* src[UM_TILES];
        uint32_t bytes = 0;
#pragma unroll
        for (uint32_t tl = 0; tl < UM_TILES; tl++) {
          const uint32_t tile = rg * UM_TILES + tl;
          src[tl] = nullptr;
          if (wprod && tile < p.tiles) {
            uint32_t si = 0;
            if (a.nseg > 1 && tile >= a.seg[1].cta_begin) si = 1;
            if (a.nseg > 2 && tile >= a.seg[2].cta_begin) si = 2;
            const DWDesc& w = a.seg[si].w;
            src[tl] = w.body + (size_t)(tile - a.seg[si].cta_begin) * w.body_stride;
            bytes += UB;
          }
        }
        for (uint32_t i = 0; i < nblk && !*abort; i++, cnt++) {
          const uint32_t st = cnt % S, k = cnt / S;
          if (k >= 1) um_wait(wprod ? &bar_wempty[st] : &bar_bfree[st], (k - 1) & 1u, a.err, abort);
          fence_proxy_async();
          // row groups start their K walk at different blocks, so that the CTAs
          // read different B images at a time
          const uint32_t blk = b0 + (i + rg) % nblk;
          if (wprod) {
            mbar_expect_tx(&full[st], bytes);
#pragma unroll
            for (uint32_t tl = 0; tl < UM_TILES; tl++)
              if (src[tl]) bulk_g2s(ring + (st * UM_TILES + tl) * UB, src[tl] + (size_t)blk * UB, UB, &full[st]);
          } else {
            mbar_expect_tx(&full[st], XB::BLK);
            bulk_g2s(bring + st * XB::BLK, a.xblob + (size_t)blk * XB::BLK, XB::BLK, &full[st]);
          }
        }
      }
      // teardown: every copy issued has landed
      for (uint32_t st = 0; st < S && st < cnt; st++) um_drain(&full[st], ((cnt - st + S - 1) / S - 1) & 1u, a.err);
    }
  } else if (warp >= UM_MMAW) {
    // ---------------------- MMA issuers: blocks gb with gb % NIS == me.
    // Every barrier an issuer waits on must see each of its phases: with two
    // issuers (Q4_K) block parity selects the issuer's own A buffers, B slots
    // (an even number of them), D and D2. Q6_K's two A buffers are shared by
    // consecutive blocks, whose MMAs cannot overlap anyway: one issuer.
    constexpr uint32_t NIS = QT == 12 ? 2 : 1;
    static_assert(NIS == 1 || (NA % 4 == 0 && BS % 2 == 0), "per-issuer barriers");
    const uint32_t me = warp - UM_MMAW;
    if (lane == 0 && me < NIS) {
      const uint32_t idesc = umma_idesc_f16(128, N);
      uint32_t gb = 0;
      for (uint32_t unit = blockIdx.x; unit < p.units; unit += gridDim.x) {
        const uint32_t ks = unit % p.ksplit, nblk = min(p.slice, nb - ks * p.slice);
        for (uint32_t i = 0; i < nblk; i++, gb++) {
          if (gb % NIS != me) continue;
          const uint32_t db = gb & 1, slot = gb % BS, td = tb + UM_TD + 64u * db, td2 = tb + UM_TD2 + 64u * db;
#pragma unroll
          for (uint32_t h = 0; h < 2; h++) {
            const uint32_t hb = 2 * gb + h, ab = hb % NA;
            um_wait(&bar_afull[ab], (hb / NA) & 1u, a.err, abort);
            if (h == 0) {
              um_wait(&bar_bfull[slot], (gb / BS) & 1u, a.err, abort);
              if (gb >= 2) um_wait(&bar_dfree[db], ((gb >> 1) + 1) & 1u, a.err, abort);  // block gb - 2 read
            }
            if (*abort) continue;
            // operands first, then the MMAs back to back: K step t of the half-block
            // is A columns ta + 8t and a B descriptor KSTEP bytes further per step
            const uint32_t ta = tb + UM_TA + ACOLS * ab;
            const uint64_t bd = umma_desc_k(smem_u32(bring + slot * XB::BLK) + h * 8 * XB::KSTEP, 128, 256);
            uint64_t bds[8];
            uint32_t tas[8];
#pragma unroll
            for (uint32_t t = 0; t < 8; t++) {
              bds[t] = bd + t * (XB::KSTEP >> 4);
              tas[t] = ta + 8 * t;
            }
            uint64_t a2d = 0, b2d = 0;
            if (h == 0) {
              a2d = umma_desc_k(smem_u32(a2buf + db * L::A2), 128, 256);
              b2d = umma_desc_k(smem_u32(bring + slot * XB::BLK + XB::OFF_B2), 128, 256);
            }
            tc_fence_after();
#pragma unroll
            for (uint32_t t = 0; t < 8; t++) umma_ts(td, tas[t], bds[t], idesc, (h | t) != 0);
            if constexpr (QT == 14) {
#pragma unroll
              for (uint32_t t = 0; t < 8; t++) umma_ts(td, tas[t] + 64, bds[t], idesc, 1u);
            }
            if (h == 0) umma_ss(td2, a2d, b2d, idesc, 0u);
            umma_commit(&bar_afree[ab]);
            if (h == 1) umma_commit(&bar_dfull[db]);
          }
        }
      }
      // teardown: every MMA issued is complete
      umma_commit(&bar_fin[me]);
      um_drain(&bar_fin[me], 0, a.err);
    }
  } else if (warp < UM_RW) {
    // --------------------------------------------- row warps: A operands
    const uint32_t q = warp & 3, e = warp >> 2, m = 32 * q + lane, tl = m >> 4, rr = m & 15;
    const uint32_t tlane = (32u * q) << 16;
    uint32_t gb = 0, wc = 0;
    for (uint32_t unit = blockIdx.x; unit < p.units; unit += gridDim.x) {
      const uint32_t ks = unit % p.ksplit, nblk = min(p.slice, nb - ks * p.slice);
      for (uint32_t i = 0; i < nblk; i++, gb++, wc++) {
        const uint32_t st = wc % WS;
        um_wait(&bar_wfull[st], (wc / WS) & 1u, a.err, abort);
        const uint8_t* un = ring + (st * UM_TILES + tl) * UB;
        const uint4 hd = *reinterpret_cast<const uint4*>(un + 16 * rr);
        uint4 W4[2][2];     // Q4_K: [half][p]
        uint2 W6[2][3][2];  // Q6_K: [half][array][p]
        if constexpr (QT == 12) {
#pragma unroll
          for (int h = 0; h < 2; h++)
#pragma unroll
            for (int pp = 0; pp < 2; pp++)
              W4[h][pp] = *reinterpret_cast<const uint4*>(un + q4t_word_off(rr, 2 * h + e, 0, pp));
        } else {
#pragma unroll
          for (int h = 0; h < 2; h++)
#pragma unroll
            for (int ar = 0; ar < 3; ar++)
#pragma unroll
              for (int pp = 0; pp < 2; pp++)
                W6[h][ar][pp] = *reinterpret_cast<const uint2*>(un + q6t_word_off(rr, ar, 2 * h + e, 0, pp));
        }
        float2 dmn = make_float2(0.f, 0.f);  // this row's block scales for the epilogue warps
        if (e == 0) {
          if constexpr (QT == 12) dmn = make_float2(h2f_ref(hd.x & 0xFFFFu), h2f_ref(hd.x >> 16));
          else dmn.x = q6_d(*reinterpret_cast<const unsigned short*>(un + 256 + 2 * rr));
        }
        mbar_arrive(&bar_wempty[st]);  // the stage's bytes this row needs are in registers
        uint32_t s4[8], m4[8];
        int32_t s6[16];
        if constexpr (QT == 12) {
          um_q4_scales(hd, s4, m4);
        } else {
          const uint32_t hw[4] = {hd.x, hd.y, hd.z, hd.w};
#pragma unroll
          for (int s = 0; s < 16; s++) s6[s] = (int32_t)(int8_t)((hw[s >> 2] >> (8 * (s & 3))) & 0xFFu);
        }
        uint32_t A[2][32];
#pragma unroll
        for (uint32_t h = 0; h < 2; h++) {
          const uint32_t hb = 2 * gb + h, ab = hb % NA;
          // sub-block scales of this warp's part (j = 2h + e, G = 2h + e), selected
          // without a run-time array index
          int32_t sc[4];
          if constexpr (QT == 12) {
            const uint32_t sc0 = e ? s4[4 * h + 2] : s4[4 * h], sc1 = e ? s4[4 * h + 3] : s4[4 * h + 1];
            um_q4_a(W4[h], sc0, sc1, A[h]);
          } else {
#pragma unroll
            for (int k = 0; k < 4; k++) sc[k] = e ? s6[8 * h + 4 + k] : s6[8 * h + k];
            um_q6_al(W6[h], sc, A[h]);
          }
          if (h == 1) {  // half 0's stores have had the half-1 work to complete
            tmem_wait_st();
            tc_fence_before();
            mbar_arrive(&bar_afull[(hb - 1) % NA]);
          }
          if (hb >= NA) um_wait(&bar_afree[ab], ((hb / NA) + 1) & 1u, a.err, abort);  // its last MMAs are done
          const uint32_t ta = tb + tlane + UM_TA + ACOLS * ab + 32u * e;
          if (h == 0 && e == 0) {  // per-block term operand A2 (row m); its MMA of block gb - 2 is done
            // (d, dmin) for the epilogue warps: block gb - 4 has been read back (MMA gb - 2 waited for it)
            dd[(gb & 3) * 128 + m] = dmn;
            mbar_arrive(&bar_hdr[gb & 3]);
            uint8_t* a2 = a2buf + (gb & 1) * L::A2;
            if constexpr (QT == 12) {
              uint32_t pk[4];
#pragma unroll
              for (int k = 0; k < 4; k++) pk[k] = h2u(__floats2half2_rn((float)m4[2 * k], (float)m4[2 * k + 1]));
              *reinterpret_cast<uint4*>(a2 + um_core(m, 0)) = make_uint4(pk[0], pk[1], pk[2], pk[3]);
            } else {
              uint32_t pk[8];
#pragma unroll
              for (int k = 0; k < 8; k++) pk[k] = h2u(__floats2half2_rn((float)s6[2 * k], (float)s6[2 * k + 1]));
              *reinterpret_cast<uint4*>(a2 + um_core(m, 0)) = make_uint4(pk[0], pk[1], pk[2], pk[3]);
              *reinterpret_cast<uint4*>(a2 + um_core(m, 1)) = make_uint4(pk[4], pk[5], pk[6], pk[7]);
            }
            fence_proxy_async();
          }
          tmem_st32(ta, A[h]);
          if constexpr (QT == 14) {
            uint32_t Ah[32];
            um_q6_ah(W6[h], sc, Ah);
            tmem_st32(ta + 64, Ah);
          }
        }
        tmem_wait_st();
        tc_fence_before();
        mbar_arrive(&bar_afull[(2 * gb + 1) % NA]);
      }
    }
  } else {
    // ------------------------------ epilogue warps: accumulators, results
    const uint32_t q = warp & 3, m = 32 * q + lane, tl = m >> 4, rr = m & 15;
    const uint32_t tlane = (32u * q) << 16;
    pdl_wait();
    if (threadIdx.x - UM_EW0 * 32 < a.batch) {
      // the column's table entry and input-norm scale, read while the blocks stream
      const uint32_t t = threadIdx.x - UM_EW0 * 32;
      um_col_fill(a, t, s_cols);
      s_scale[t] = reinterpret_cast<const float*>(a.xblob + (size_t)nb * XB::BLK)[t];
    }
    named_bar(1, UM_EW * 32);
    const float* s_in = s_scale;
    uint32_t gb = 0;
    // the accumulators of block g into y; then its D and B slot are free
    auto drain = [&](uint32_t g, float (&y)[NB]) {
      um_wait(&bar_dfull[g & 1], (g >> 1) & 1u, a.err, abort);
      um_wait(&bar_bfull[g % BS], (g / BS) & 1u, a.err, abort);  // the slot's scales are visible
      um_wait(&bar_hdr[g & 3], (g >> 2) & 1u, a.err, abort);
      const float2 dmn = dd[(g & 3) * 128 + m];
      const float d = dmn.x, dm = dmn.y;
      tc_fence_after();
      const float* uu = reinterpret_cast<const float*>(bring + (g % BS) * XB::BLK + XB::OFF_U);
      constexpr uint32_t CH = NB < 16 ? NB : 16;  // columns per read-back chunk (2 CH accumulator columns)
#pragma unroll
      for (uint32_t c0 = 0; c0 < NB; c0 += CH) {
        uint32_t dr[2 * CH], d2r[2 * CH];
        tmem_ld<2 * CH>(tb + tlane + UM_TD + 64u * (g & 1) + 2 * c0, dr);
        tmem_ld<2 * CH>(tb + tlane + UM_TD2 + 64u * (g & 1) + 2 * c0, d2r);
        float us[CH];
#pragma unroll
        for (uint32_t i = 0; i < CH; i += 4) {  // 16-byte aligned (OFF_U and BLK are multiples of 16)
          const float4 u4 = *reinterpret_cast<const float4*>(uu + c0 + i);
          us[i] = u4.x;
          if (i + 1 < CH) us[i + 1] = u4.y;
          if (i + 2 < CH) us[i + 2] = u4.z;
          if (i + 3 < CH) us[i + 3] = u4.w;
        }
        tmem_wait_ld();
#pragma unroll
        for (uint32_t i = 0; i < CH; i++) {
          const float D = __uint_as_float(dr[2 * i]) + __uint_as_float(dr[2 * i + 1]);
          const float D2 = __uint_as_float(d2r[2 * i]) + __uint_as_float(d2r[2 * i + 1]);
          if constexpr (QT == 12) y[c0 + i] = fmaf(us[i], fmaf(d, D, -64.f * dm * D2), y[c0 + i]);
          else y[c0 + i] = fmaf(us[i] * d, fmaf(16.f, D, -2048.f * D2), y[c0 + i]);
        }
      }
      tc_fence_before();
      mbar_arrive(&bar_dfree[g & 1]);
      mbar_arrive(&bar_bfree[g % BS]);
    };
    for (uint32_t unit = blockIdx.x; unit < p.units; unit += gridDim.x) {
      const uint32_t rg = unit / p.ksplit, ks = unit - rg * p.ksplit;
      const uint32_t b0 = ks * p.slice, nblk = min(p.slice, nb - b0), tile = rg * UM_TILES + tl;
      float y[NB];
#pragma unroll
      for (uint32_t i = 0; i < NB; i++) y[i] = 0.f;
      for (uint32_t i = 0; i < nblk; i++, gb++) drain(gb, y);
      // input-norm scale of each column
#pragma unroll
      for (uint32_t i = 0; i < NB; i++) y[i] *= i < a.batch ? s_in[i] : 0.f;
      const bool valid = tile < p.tiles;
      if (p.ksplit == 1) {
        um_epilogue<NB>(a, s_cols, valid ? tile : 0u, p.tiles, valid, rr, 0u, y);
        continue;
      }
      // K-split: publish this slice ([slice][column][row]: a warp's rows are
      // consecutive); the last CTA of the group sums the slices in order
      const uint32_t R = p.tiles * 16u;
      const size_t stride = (size_t)R * a.batch;
      float* mine = a.ks_part + (size_t)tile * 16u + rr;
      if (valid) {
#pragma unroll
        for (uint32_t i = 0; i < NB; i++)
          if (i < a.batch) mine[ks * stride + (size_t)i * R] = y[i];
      }
      named_bar(1, UM_EW * 32);
      if (threadIdx.x == UM_EW0 * 32) s_last = ks_arrive(&a.ks_cnt[rg], p.ksplit - 1u) == p.ksplit - 1u;
      named_bar(1, UM_EW * 32);
      if (s_last) {
        if (p.units <= gridDim.x) {  // one unit per CTA: every warp joins the fixup after the CTA's last barrier
          if (threadIdx.x == UM_EW0 * 32) s_fix = 1u;
          continue;
        }
#pragma unroll
        for (uint32_t i = 0; i < NB; i++) y[i] = 0.f;
        if (valid)
          for (uint32_t k = 0; k < p.ksplit; k++) {  // in slice order; the columns' loads are independent
            float t[NB];
#pragma unroll
            for (uint32_t i = 0; i < NB; i++) t[i] = __ldcg(mine + k * stride + (size_t)min(i, a.batch - 1) * R);
#pragma unroll
            for (uint32_t i = 0; i < NB; i++) y[i] += i < a.batch ? t[i] : 0.f;
          }
        um_epilogue<NB>(a, s_cols, valid ? tile : 0u, p.tiles, valid, rr, 0u, y);
      }
    }
  }
  // ------------------------------------------------------------ teardown
  // (each warp reconverges first: the roles above leave lanes 1..31 of the
  // producer and MMA warps idle while lane 0 works, and the CTA barrier
  // must count whole warps that have all finished)
  __syncwarp();
  tc_fence_before();
  __syncthreads();
  if (warp == UM_MMAW) {
    __syncwarp();
    tc_fence_after();
    tmem_dealloc(tb, UM_TCOLS);
  }
  if (s_fix) {
    // The last CTA of a single-round K-split group: all UM_THREADS threads sum
    // the slices (in slice order, as the epilogue warps would) and run the
    // epilogue, as 128 rows x 4 groups of NB / 4 columns. A thread's loads and
    // stores are a quarter of one epilogue thread's.
    constexpr uint32_t CPG = NB / 4;
    static_assert(UM_THREADS == 4 * 128, "four column groups");
    const uint32_t m = threadIdx.x & 127u, g = threadIdx.x >> 7;
    const uint32_t tile = (blockIdx.x / p.ksplit) * UM_TILES + (m >> 4), rr = m & 15u;
    const bool valid = tile < p.tiles;
    const uint32_t R = p.tiles * 16u;
    const size_t stride = (size_t)R * a.batch;
    const float* mine = a.ks_part + (size_t)tile * 16u + rr;
    float y[CPG];
#pragma unroll
    for (uint32_t i = 0; i < CPG; i++) y[i] = 0.f;
    // (the other slices' stores are visible: ks_arrive acquired them, and the
    // CTA's barriers order these loads after it)
    if (valid)
      for (uint32_t k0 = 0; k0 < p.ksplit; k0 += 4) {  // four slices' loads in flight, added in slice order
        float t[4][CPG];
#pragma unroll
        for (uint32_t kk = 0; kk < 4; kk++)
#pragma unroll
          for (uint32_t i = 0; i < CPG; i++) {
            const uint32_t col = g * CPG + i;
            t[kk][i] = (k0 + kk < p.ksplit && col < a.batch) ? __ldcg(mine + (k0 + kk) * stride + (size_t)col * R) : 0.f;
          }
#pragma unroll
        for (uint32_t kk = 0; kk < 4; kk++)
#pragma unroll
          for (uint32_t i = 0; i < CPG; i++)
            if (k0 + kk < p.ksplit) y[i] += t[kk][i];
      }
    um_epilogue<CPG>(a, s_cols, valid ? tile : 0u, p.tiles, valid, rr, g * CPG, y);
  }
}

// ------------------------------------------------------------- host ----
namespace {

using UmKernel = void (*)(GemvArgs, UmPlan);
using XpKernel = void (*)(GemvArgs, uint32_t);

UmKernel um_kernel(uint32_t nb8, uint32_t qt) {
  switch (nb8 * 100 + qt) {
    case 812: return gemv_umma_kernel<8, 12>;
    case 814: return gemv_umma_kernel<8, 14>;
    case 1612: return gemv_umma_kernel<16, 12>;
    case 1614: return gemv_umma_kernel<16, 14>;
    case 3212: return gemv_umma_kernel<32, 12>;
    case 3214: return gemv_umma_kernel<32, 14>;
  }
  return nullptr;
}
XpKernel xp_kernel(uint32_t nb8, uint32_t qt) {
  switch (nb8 * 100 + qt) {
    case 812: return umma_xprep_kernel<8, 12>;
    case 814: return umma_xprep_kernel<8, 14>;
    case 1612: return umma_xprep_kernel<16, 12>;
    case 1614: return umma_xprep_kernel<16, 14>;
    case 3212: return umma_xprep_kernel<32, 12>;
    case 3214: return umma_xprep_kernel<32, 14>;
  }
  return nullptr;
}
uint32_t um_nb8(uint32_t batch) { return batch <= 8 ? 8 : batch <= 16 ? 16 : 32; }
uint32_t um_blob_blk(uint32_t nb8) {
  return nb8 == 8 ? UmBlob<8>::BLK : nb8 == 16 ? UmBlob<16>::BLK : UmBlob<32>::BLK;
}
uint32_t um_smem_for(uint32_t nb8, uint32_t qt) {
  uint32_t b = 0;
  switch (nb8 * 100 + qt) {
    case 812: b = UmSmem<8, 12>::BYTES; break;
    case 814: b = UmSmem<8, 14>::BYTES; break;
    case 1612: b = UmSmem<16, 12>::BYTES; break;
    case 1614: b = UmSmem<16, 14>::BYTES; break;
    case 3212: b = UmSmem<32, 12>::BYTES; break;
    default: b = UmSmem<32, 14>::BYTES; break;
  }
  return std::max(b, UM_SMEM_MIN);
}

constexpr int UM_MAX_DEVICES = 64;
std::mutex g_um_mu;
int g_um_sms[UM_MAX_DEVICES] = {};

cudaError_t um_setup(uint32_t* sms) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  if (dev < 0 || dev >= UM_MAX_DEVICES) return cudaErrorInvalidDevice;
  std::lock_guard<std::mutex> lk(g_um_mu);
  if (!g_um_sms[dev]) {
    int n = 0;
    e = cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
    for (uint32_t nb8 : {8u, 16u, 32u})
      for (uint32_t qt : {12u, 14u})
        if (e == cudaSuccess)
          e = cudaFuncSetAttribute(um_kernel(nb8, qt), cudaFuncAttributeMaxDynamicSharedMemorySize, UM_SMEM_MAX);
    if (e != cudaSuccess) return e;
    g_um_sms[dev] = n;
  }
  *sms = (uint32_t)g_um_sms[dev];
  return cudaSuccess;
}

// One weight type for every segment, batch 2..32, whole 256-blocks, and room
// for the B image.
bool um_ok(const GemvArgs& a) {
  if (a.batch < 2 || a.batch > UM_MAXB || !a.nseg) return false;
  const uint32_t qt = a.seg[0].w.type;
  if (!tiled_type(qt)) return false;
  for (uint32_t i = 0; i < a.nseg; i++)
    if (a.seg[i].w.type != qt || a.seg[i].w.n_in != a.seg[0].w.n_in) return false;
  if ((a.ldx & 3u) || (reinterpret_cast<uintptr_t>(a.x) & 15u)) return false;
  return a.xblob && (reinterpret_cast<uintptr_t>(a.xblob) & 15u) == 0 &&
         gemv_umma_blob_bytes(a.seg[0].w.n_in, a.batch) <= a.xblob_cap;
}

// CTA tiles of 128 rows and a K-split that minimizes rounds of units x
// (blocks per unit + 2 blocks of per-unit cost) plus the fixup's reads (a
// quarter block per slice), bounded by the scratch.
bool um_plan(GemvArgs& a, uint32_t sms, UmPlan* p) {
  uint32_t tiles = 0;
  for (uint32_t i = 0; i < a.nseg; i++) {
    a.seg[i].cta_begin = tiles;
    tiles += (a.seg[i].w.n_out + 15) / 16;
  }
  const uint32_t nb = a.seg[0].w.n_in >> 8, groups = (tiles + UM_TILES - 1) / UM_TILES;
  const uint32_t smem = um_smem_for(um_nb8(a.batch), a.seg[0].w.type);
  if (smem > UM_SMEM_MAX || nb == 0) return false;
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
    const uint64_t cost = rounds * (4 * sl + 8) + (kk > 1 ? kk : 0);  // quarter blocks; + the slices' fixup
    if (cost < best) {
      best = cost;
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
  p->smem = smem;
  return true;
}

}  // namespace

uint64_t gemv_umma_blob_bytes(uint32_t n_in, uint32_t batch) {
  return (uint64_t)(n_in >> 8) * um_blob_blk(um_nb8(batch)) + UM_MAXB * 4;
}

cudaError_t gemv_umma_prepare() {
  uint32_t sms = 0;
  return um_setup(&sms);
}

// cudaErrorNotSupported: no plan fits (use another kernel). n_parts: the
// per-column partials an EPI_RESID launch writes (one per 16-row tile).
cudaError_t launch_gemv_umma(GemvArgs a, cudaStream_t st, uint32_t* n_parts) {
  if (!um_ok(a)) return cudaErrorNotSupported;
  uint32_t sms = 0;
  cudaError_t e = um_setup(&sms);
  if (e != cudaSuccess) return e;
  if (a.grid_cap) sms = std::min(sms, a.grid_cap);
  UmPlan p;
  if (!um_plan(a, sms, &p)) return cudaErrorNotSupported;
  if (n_parts) *n_parts = p.tiles;
  const uint32_t nb8 = um_nb8(a.batch), qt = a.seg[0].w.type, nb = a.seg[0].w.n_in >> 8;
  e = launch_pdl(xp_kernel(nb8, qt), dim3(nb, nb8 / UM_XPREP_COLS), dim3(UM_XPREP_THREADS), 0, st, a, nb);
  if (e != cudaSuccess) return e;
  return launch_pdl(um_kernel(nb8, qt), dim3(p.grid), dim3(UM_THREADS), p.smem, st, a, p);
}

void gemv_umma_scratch_need(GemvArgs a, uint32_t sms, uint64_t* part, uint32_t* cnt) {
  a.ks_part = reinterpret_cast<float*>(16);
  a.ks_cnt = reinterpret_cast<uint32_t*>(16);
  a.ks_part_cap = 0xFFFFFFFFu;
  a.ks_cnt_cap = 0xFFFFFFFFu;
  *part = 0;
  *cnt = 0;
  if (a.grid_cap) sms = std::min(sms, a.grid_cap);
  UmPlan p;
  if (!tiled_type(a.seg[0].w.type) || !um_plan(a, sms, &p) || p.ksplit == 1) return;
  *part = (uint64_t)p.ksplit * p.tiles * 16u * a.batch;
  *cnt = p.groups;
}

}  // namespace sm
