// Device-side layouts and helpers of the B200 decode engine (sm_100a).
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>

namespace sm {

// ---------------------------------------------------------------------------
// HBM layout of one quantized weight [n_out x n_in] (a row = one output).
// Every byte of the GGUF encoding is kept; only its order changes.
//
// Q4_K / Q6_K are stored in tiles of 16 rows (the last tile zero-padded): a
// tile holds its 256-weight blocks in order, and block b of a tile is one
// contiguous unit of all 16 rows (one bulk copy into shared memory). Inside a
// unit the quants are regrouped so that lane (g, t) = (lane >> 2, lane & 3)
// of a warp that owns rows g and g + 8 finds the A operands of
// mma.m16n8k32 (u8) for its rows in a few 16-byte loads: every 32-bit word
// holds four consecutive weights of one sub-block (Q4_K: their nibbles;
// Q6_K: low nibbles and the 2-bit high parts split over words), and the
// 16-byte chunks are rotated per row so that the lanes' loads hit distinct
// shared-memory banks.
//   Q4_K unit, 2304 B:
//     [16 rows x 16 B header: d, dmin, 12 scale bytes]
//     [16 rows x 128 B of qs]: word (j, c, p) = qs bytes 32j + 8c + 4p .. + 3
//       (j, c = 0..3, p = 0..1) at q4t_word_off(rr, j, c, p).
//     (Byte q of qs holds weight 64j + (q & 31) in its low nibble and weight
//     64j + 32 + (q & 31) in its high nibble, j = q >> 5: dequant.rs:98-124.)
//   Q6_K unit, 3360 B:
//     [16 rows x 16 int8 scales][16 rows x fp16 d][16 rows x 192 B]
//     Weight 8c + 4p + b (b = 0..3) of sub-block s = 4G + sigma (16 weights
//     per sub-block, G = 0..3, c, p = 0..1) as the 6-bit value v = q + 32
//     (dequant.rs:178-206) is byte b of three words (G, c, p) of its row:
//       W0: low nibble of v(sigma = 0) | low nibble of v(sigma = 2) << 4
//       W1: low nibble of v(sigma = 1) | low nibble of v(sigma = 3) << 4
//       H:  high 2 bits of v(1) | v(3) << 2 | v(0) << 4 | v(2) << 6
//     at q6t_word_off(rr, array 0/1/2, G, c, p).
//   Q8_0: body = 32 B of qs per block, aux = fp16 d per block (row-major).
//   Q5_0: body = 16 B of qs per block, aux = 8 B per block (qh u32 | d fp16 | 0).
// ---------------------------------------------------------------------------
#ifdef __CUDACC__
#define SM_HD __host__ __device__ __forceinline__
#else
#define SM_HD inline
#endif
constexpr uint32_t Q4T_UNIT = 2304, Q6T_UNIT = 3360, Q6T_QOFF = 288;
SM_HD bool tiled_type(uint32_t t) { return t == 12 || t == 14; }
SM_HD uint32_t tile_unit_bytes(uint32_t t) { return t == 12 ? Q4T_UNIT : Q6T_UNIT; }
// Q4_K: byte offset in a unit of qs word (j, c, p) of tile row rr: row rr's
// 128 bytes are 8 chunks of 16 B, logical chunk 4p + j stored at position
// (4p + j) ^ (rr & 7), word c of the chunk.
SM_HD uint32_t q4t_word_off(uint32_t rr, uint32_t j, uint32_t c, uint32_t p) {
  return 256u + 128u * rr + 16u * ((4u * p + j) ^ (rr & 7u)) + 4u * c;
}
// Q4_K: byte offset of qs byte q (0..127) of tile row rr.
SM_HD uint32_t q4t_qs_off(uint32_t rr, uint32_t q) {
  const uint32_t w = q & 31u;
  return q4t_word_off(rr, q >> 5, w >> 3, (w >> 2) & 1u) + (w & 3u);
}
// Q6_K: byte offset in a unit of word (G, c) of array a (0: W0, 1: W1, 2: H)
// for parity p of tile row rr. A row's 192 bytes are 12 chunks of 16 B,
// logical chunk 6p + 2a + (G >> 1) (words 2(G & 1) + c of it), stored at
// position (logical + 3 * ((rr & 7) >> 1)) mod 12.
SM_HD uint32_t q6t_word_off(uint32_t rr, uint32_t a, uint32_t G, uint32_t c, uint32_t p) {
  const uint32_t chunk = (6u * p + 2u * a + (G >> 1) + 3u * ((rr & 7u) >> 1)) % 12u;
  return Q6T_QOFF + 192u * rr + 16u * chunk + 4u * (2u * (G & 1u) + c);
}
// Q6_K: the 6-bit value v = q + 32 of weight l (0..255) of tile row rr.
SM_HD uint32_t q6t_value(const uint8_t* unit, uint32_t rr, uint32_t l) {
  const uint32_t s = l >> 4, w = l & 15u, G = s >> 2, sg = s & 3u, c = w >> 3, p = (w >> 2) & 1u, b = w & 3u;
  const uint32_t wv = unit[q6t_word_off(rr, sg & 1u, G, c, p) + b];
  const uint32_t h = unit[q6t_word_off(rr, 2, G, c, p) + b];
  const uint32_t lo = (sg >> 1) ? (wv >> 4) : (wv & 15u);
  const uint32_t hs = sg == 0 ? 4u : sg == 1 ? 0u : sg == 2 ? 6u : 2u;
  return lo | (((h >> hs) & 3u) << 4);
}

struct DWDesc {
  const uint8_t* body;
  const uint8_t* aux;
  uint32_t type, n_out, n_in;
  uint32_t body_stride;  // bytes per row; Q4_K / Q6_K: bytes per 16-row tile
  uint32_t aux_stride;   // bytes per row
};

// One row of a forward pass (a token): which sequence it belongs to and its
// absolute position.
struct RowDesc {
  uint32_t seq;
  uint32_t pos;
};

// A sequence's KV storage, in pages of KV_PAGE positions (f32, the
// reference's SeqState precision): page t holds positions [KV_PAGE t,
// KV_PAGE (t + 1)) of every layer, K as [layer][KV_PAGE][kv_dim] and V the
// same voff floats further. Sequences that share a prefix share its pages.
constexpr uint32_t KV_PAGE = 32;
struct SeqDesc {
  float* const* pages;  // device array: the base of page t (t < cap / KV_PAGE, rounded up)
  uint32_t cap;         // capacity in positions
  uint32_t voff;        // floats from a page's K half to its V half: n_layers * KV_PAGE * kv_dim
};
// Offset of (layer, position) inside its page, in floats (K half).
SM_HD size_t kv_page_off(uint32_t layer, uint32_t pos, uint32_t kvd) {
  return ((size_t)layer * KV_PAGE + (pos % KV_PAGE)) * kvd;
}

// What a GEMV does with the dot product v of (physical row o, column b).
// Pair kinds act on physical rows (2m, 2m+1) together.
enum GemvEpi : uint32_t {
  EPI_STORE = 0,   // y = v (+ bias)
  EPI_ADD = 1,     // y += v
  EPI_RESID = 2,   // x = y += v; xn = x * nw (natural and permuted); per-CTA sum of x^2
  EPI_ROPE_Q = 3,  // pair (dim m, dim m + hd/2) of a head: RoPE, store q (natural order)
  EPI_ROPE_K = 4,  // same, store into the K cache
  EPI_V = 5,       // store into the V cache
  EPI_SILU = 6,    // pair (gate m, up m): h[m] = silu(gate) * up (natural and permuted)
  EPI_PUSH = 7,    // tensor parallel: send (v, epoch) to every rank's receive area (TpPush)
};
__host__ __device__ inline bool epi_is_pair(uint32_t e) { return e == EPI_ROPE_Q || e == EPI_ROPE_K || e == EPI_SILU; }

// One output segment of a (possibly fused) GEMV launch.
struct GemvSeg {
  DWDesc w;
  float* y;            // y[b * ldy + o]
  const float* bias;   // optional, physical-row order
  uint32_t ldy;
  uint32_t epi;        // GemvEpi
  uint32_t cta_begin;  // first CTA index of this segment
};

// Where an EPI_PUSH GEMV sends its outputs (tensor parallelism, tp.hpp):
// element o of column b goes, as the 8-byte packet (v bits | epoch << 32), to
// dst[k][parity * parity_stride + rank * src_stride + b * ld + o] of every
// rank k (mapped peer memory; k == rank is local). The epoch is that of the
// consumer block owning global element base + o: epoch[(base + o) / per] + 1,
// and parity = epoch & 1.
constexpr uint32_t TP_MAX_RANKS = 8;
struct TpPush {
  uint64_t* dst[TP_MAX_RANKS];
  uint64_t parity_stride, src_stride;
  const uint32_t* epoch;
  uint32_t world, rank, ld, per, base;
};

struct GemvArgs {
  GemvSeg seg[3];
  uint32_t nseg;
  const float* x;  // x[b * ldx + d]
  uint32_t ldx;
  uint32_t batch;
  // Input RMSNorm (qwen2.rs:647-660) folded into the GEMV: x holds x*w of the
  // un-normalized residual, and the dot products of column b are scaled by
  // 1/sqrt(sum(in_parts[b*in_np .. +in_np]) / in_n + in_eps) when in_parts is set.
  const float* in_parts;
  uint32_t in_np, in_n;
  float in_eps;
  // EPI_RESID outputs: xn = x * nw, and partial sums of x^2 over groups of
  // rows (out_parts[b * n_parts + group]; launch_gemv returns n_parts).
  const float* nw;
  float* xn;
  uint32_t ldxn;
  float* out_parts;
  // EPI_SILU output
  float* h;
  uint32_t ldh;
  // RoPE and KV-cache epilogues
  const RowDesc* rows;
  const SeqDesc* seqs;
  const float* cos_t;
  const float* sin_t;
  uint32_t layer, hd, kvd;
  // Scratch of the tensor-core batch-1 GEMV when it splits K: per-slice
  // partial dot products and per-group arrival counters. A counter advances
  // with a wrapping increment (atomicInc modulo the split), so it is zero
  // again after every complete launch without a reset.
  float* ks_part;
  uint32_t* ks_cnt;
  uint32_t ks_part_cap, ks_cnt_cap;
  // Scratch of the tcgen05 batched GEMV: x converted once per launch into
  // the shared-memory image of its B operand (may be null: another kernel runs).
  uint8_t* xblob;
  uint64_t xblob_cap;  // bytes
  // Host planning only: a tcgen05 batched launch uses at most this many CTAs
  // (0: up to one per SM), so that a launch on another stream can run beside it.
  uint32_t grid_cap;
  // Set non-zero by a kernel whose bounded wait gave up (the launch's results
  // are then not valid); may be null.
  uint32_t* err;
  // Batch-1 EPI_STORE launches (the output head): per 16-row tile, the key of
  // its largest value, lowest row first (argmax_key); may be null.
  uint64_t* amax;
  // Batch-1 launches whose input is the attention output (the O projection):
  // when att_o is set, x is merged from the attention kernel's per-split
  // partials (o, and (m, l) in att_ml; att_slots slots per head, the row's
  // own splits from slot att_first on) instead of being read from x.
  const float* att_o;
  const float* att_ml;
  uint32_t att_slots, att_first;
  TpPush push;  // EPI_PUSH
};

// Greedy-sampling key of logit v at index i: larger value first, then lower
// index (argmax, sampling.rs:147-155); a NaN never wins (key 0).
SM_HD uint64_t argmax_key(float v, uint32_t i) {
  union {
    float f;
    uint32_t u;
  } b;
  b.f = v;
  if (v != v) return 0;
  const uint32_t k = (b.u & 0x80000000u) ? ~b.u : (b.u | 0x80000000u);
  return ((uint64_t)k << 32) | (0xFFFFFFFFu - i);
}

#ifdef __CUDACC__
// fp16 bit pattern -> f32 as the reference decodes it (dequant.rs:12-33):
// IEEE half, except that a NaN half decodes to +-Inf.
__device__ __forceinline__ float fp16_ref(uint32_t h) {
  uint32_t sign = (h >> 15) & 1u, ex = (h >> 10) & 0x1Fu, fr = h & 0x3FFu;
  if (ex == 0) {
    float v = (float)fr * 5.9604645e-8f;  // exact: fr * 2^-24
    return sign ? -v : v;
  }
  uint32_t bits = ex == 0x1F ? ((sign << 31) | 0x7F800000u) : ((sign << 31) | ((ex + 112u) << 23) | (fr << 13));
  return __uint_as_float(bits);
}

// Byte k of v (a value < 256) as the exact float (byte - off): the byte is
// placed in the mantissa of 2^23 and 2^23 + off is subtracted (exact).
template <int K>
__device__ __forceinline__ float byte_f(uint32_t v, float magic_off) {
  return __uint_as_float(__byte_perm(v, 0x4B000000u, 0x7540u + K)) - magic_off;
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

__device__ __forceinline__ float4 ldg4(const float* p) { return __ldg(reinterpret_cast<const float4*>(p)); }
__device__ __forceinline__ uint4 ldg_u4(const uint8_t* p) { return __ldg(reinterpret_cast<const uint4*>(p)); }
// Streamed weights: read once per step, keep them out of L1.
__device__ __forceinline__ uint4 ld_stream(const uint8_t* p) {
  uint4 r;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
               : "l"(p));
  return r;
}
#endif

}  // namespace sm
