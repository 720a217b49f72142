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
// contiguous unit of all 16 rows. Inside a unit the bytes sit where lane
// (g, t) = (lane >> 2, lane & 3) of a warp wants them when it owns rows g and
// g + 8 of the tile as the A operand of mma.m16n8k16: every 16-byte load of
// the warp reads 512 contiguous bytes.
//   Q4_K unit, 2304 B:
//     [16 rows x 16 B header: d, dmin, 12 scale bytes]
//     [qs: 4 loads x 32 lanes x 16 B]  load L, lane (g, t): row g + 8*(L >> 1),
//       bytes 32j + 8t .. 32j + 8t + 7 of qs for j = 2*(L & 1) and j + 1.
//     (Byte q of qs holds weight 64j + (q & 31) in its low nibble and weight
//     64j + 32 + (q & 31) in its high nibble, j = q >> 5: dequant.rs:98-124.)
//   Q6_K unit, 3360 B:
//     [16 rows x 16 int8 scales][16 rows x fp16 d][q: 6 loads x 32 lanes x 16 B]
//     Lane (g, t) owns, per row, weight 16s + 4t + k of every 16-weight
//     sub-block s (k = 0..3) as the 6-bit value v = q + 32, in 12 words:
//     loads 0-1 (row g; 3-4 for row g + 8) = ql words i = 0..7, byte k of
//     word i = low 4 bits of v(s = i, k) | low 4 bits of v(s = i + 8, k) << 4;
//     load 2 (5) = qh words m = 0..3, holding the top 2 bits of the values of
//     ql words 2m and 2m + 1 at bit (q6t_field(k, nib) + 8 * (i & 1)) & 31.
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
// Byte offset, inside a Q4_K unit, of qs byte q (0..127) of tile row rr (0..15).
SM_HD uint32_t q4t_qs_off(uint32_t rr, uint32_t q) {
  const uint32_t j = q >> 5, t = (q >> 3) & 3u, e = q & 7u;
  const uint32_t L = 2u * (rr >> 3) + (j >> 1), lane = 4u * (rr & 7u) + t;
  return 256u + 512u * L + 16u * lane + 8u * (j & 1u) + e;
}
// Byte offsets, inside a Q6_K unit, of ql word i (0..7) and qh word m (0..3)
// of lane t for tile row rr.
SM_HD uint32_t q6t_w_off(uint32_t rr, uint32_t t, uint32_t i) {
  return Q6T_QOFF + 512u * (3u * (rr >> 3) + (i >> 2)) + 16u * (4u * (rr & 7u) + t) + 4u * (i & 3u);
}
SM_HD uint32_t q6t_h_off(uint32_t rr, uint32_t t, uint32_t m) {
  return Q6T_QOFF + 512u * (3u * (rr >> 3) + 2u) + 16u * (4u * (rr & 7u) + t) + 4u * m;
}
// Bit position of the top 2 bits of byte k, nibble nib of an even ql word in
// its qh word (odd words: the same positions in the qh word rotated right by 8).
SM_HD uint32_t q6t_field(uint32_t k, uint32_t nib) { return (nib ? 8u : 4u) + 2u * (k & 1u) + 16u * (k >> 1); }

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

// A sequence's KV storage: k/v are [n_layers][cap][kv_dim] f32.
struct SeqDesc {
  float* k;
  float* v;
  uint32_t cap;
  uint32_t pad;
};

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
  // partial dot products and per-group arrival counters (zero between launches).
  float* ks_part;
  uint32_t* ks_cnt;
  uint32_t ks_part_cap, ks_cnt_cap;
  // Set non-zero by a kernel whose bounded wait gave up (the launch's results
  // are then not valid); may be null.
  uint32_t* err;
  TpPush push;  // EPI_PUSH
};

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
