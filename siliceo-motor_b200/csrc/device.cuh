// Device-side layouts and helpers of the B200 decode engine (sm_100a).
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>

namespace sm {

// ---------------------------------------------------------------------------
// HBM layout of one quantized weight [n_out x n_in] (row-major, a row = one
// output). Every byte of the GGUF encoding is kept; only its order changes so
// that the 32 lanes of a warp read 512 contiguous bytes per load. A row is a
// sequence of groups of up to 8 consecutive 256-weight blocks (nbg blocks in
// the last group); lane L = 4*bi + u works on block bi of a group.
//   Q4_K group: [nbg headers x 16 B: d, dmin, 12 scale bytes]
//               [qs round 0: 4*nbg lanes x 16 B][qs round 1: 4*nbg lanes x 16 B]
//               lane 4bi+j holds qs bytes 32j..32j+15 (round 0) and
//               32j+16..32j+31 (round 1) of block bi.   1152 B per 8 blocks.
//   Q6_K group: [ql a: 4*nbg x 16 B][ql b: 4*nbg x 16 B][qh: 4*nbg x 16 B]
//               [scales: nbg x 16 B][d: nbg x 2 B, padded to 16 B]
//               lane 4bi+2n+c holds ql[64n+16c..] (a), ql[64n+32+16c..] (b) and
//               qh[32n+16c..] of block bi.                 1680 B per 8 blocks.
//   Q8_0: body = 32 B of qs per block, aux = fp16 d per block.
//   Q5_0: body = 16 B of qs per block, aux = 8 B per block (qh u32 | d fp16 | 0).
// The GGUF block formats are dequant.rs:66-206 (Q6_K keeps d last in GGUF).
// ---------------------------------------------------------------------------
#ifdef __CUDACC__
#define SM_HD __host__ __device__ __forceinline__
#else
#define SM_HD inline
#endif
SM_HD uint32_t q4k_group_bytes(uint32_t nbg) { return 144u * nbg; }
SM_HD uint32_t q6k_group_bytes(uint32_t nbg) { return 208u * nbg + (2u * nbg + 15u) / 16u * 16u; }
SM_HD uint32_t q4k_row_bytes(uint32_t nb) { return nb / 8u * q4k_group_bytes(8) + q4k_group_bytes(nb % 8u); }
SM_HD uint32_t q6k_row_bytes(uint32_t nb) {
  return nb / 8u * q6k_group_bytes(8) + (nb % 8u ? q6k_group_bytes(nb % 8u) : 0u);
}
// Byte offsets inside a row for block b (of nb).
struct KqPos {
  uint32_t base, nbg, bi;
};
SM_HD KqPos kq_pos(uint32_t b, uint32_t nb, uint32_t group_bytes8) {
  KqPos p;
  p.base = (b >> 3) * group_bytes8;
  p.nbg = nb - (b & ~7u) < 8u ? nb - (b & ~7u) : 8u;
  p.bi = b & 7u;
  return p;
}
SM_HD uint32_t q4k_hdr_off(const KqPos& p) { return p.base + 16u * p.bi; }
SM_HD uint32_t q4k_qs_off(const KqPos& p, uint32_t j, uint32_t round) {
  return p.base + 16u * p.nbg + 16u * (round * 4u * p.nbg + 4u * p.bi + j);
}
// part 0: ql a, 1: ql b, 2: qh
SM_HD uint32_t q6k_q_off(const KqPos& p, uint32_t n, uint32_t c, uint32_t part) {
  return p.base + 16u * (part * 4u * p.nbg + 4u * p.bi + 2u * n + c);
}
SM_HD uint32_t q6k_sc_off(const KqPos& p) { return p.base + 192u * p.nbg + 16u * p.bi; }
SM_HD uint32_t q6k_d_off(const KqPos& p) { return p.base + 208u * p.nbg + 2u * p.bi; }

struct DWDesc {
  const uint8_t* body;
  const uint8_t* aux;
  uint32_t type, n_out, n_in;
  uint32_t body_stride;  // bytes per row
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

struct GemvArgs {
  GemvSeg seg[3];
  uint32_t nseg;
  const float* x;  // x[b * ldx + d]
  uint32_t ldx;
  uint32_t batch;
  // Batch 1 reads the activations in the lane order of its K-quant kernels
  // (xperm_q4k / xperm_q6k below); both copies are written by the kernel
  // that produced x.
  const float* xp4;
  const float* xp6;
  // Input RMSNorm (qwen2.rs:647-660) folded into the GEMV: x holds x*w of the
  // un-normalized residual, and the dot products of column b are scaled by
  // 1/sqrt(sum(in_parts[b*in_np .. +in_np]) / in_n + in_eps) when in_parts is set.
  const float* in_parts;
  uint32_t in_np, in_n;
  float in_eps;
  // EPI_RESID outputs: xn = x * nw, and per-CTA partial sums of x^2
  // (out_parts[b * gridDim.y + cta]).
  const float* nw;
  float *xn, *xn4, *xn6;
  uint32_t ldxn;
  float* out_parts;
  // EPI_SILU outputs
  float *h, *h4, *h6;
  uint32_t ldh;
  // RoPE and KV-cache epilogues
  const RowDesc* rows;
  const SeqDesc* seqs;
  const float* cos_t;
  const float* sin_t;
  uint32_t layer, hd, kvd;
};

// ---------------------------------------------------------------------------
// Lane-interleaved activation layouts of the batch-1 GEMV. A warp step covers
// 8 consecutive 256-weight blocks (2048 activations); lane L = 4*bi + u owns 64
// activations of block bi and reads them as 16 float4 loads k = 0..15. The
// float4 of (step t, k, lane) is stored at t*2048 + k*128 + 4*lane, so every
// load instruction of the warp reads 512 contiguous bytes. Rows are padded to
// whole steps: xperm_len(K) floats.
//   Q4_K lane (bi, j):    float4 k = activations 64j + 4k .. +3 of the block
//   Q6_K lane (bi, n, c): float4 k = 4g + i -> 128n + 16c + 32g + 4i .. +3
// Inside each float4 the four activations e..e+3 are stored as (e, e+2, e+1,
// e+3): the kernels turn bytes (0, 2) and (1, 3) of a weight word into one
// half2 each, and the float4's halves are then their f32x2 partners.
// ---------------------------------------------------------------------------
#ifdef __CUDACC__
__host__ __device__ __forceinline__
#else
inline
#endif
uint32_t xperm_len(uint32_t K) { return (K + 2047u) / 2048u * 2048u; }

#ifdef __CUDACC__
__device__ __forceinline__ uint32_t xperm_q4k(uint32_t e) {
  const uint32_t b = e >> 8, o = e & 255, t = b >> 3, bi = b & 7;
  const uint32_t j = o >> 6, r = o & 63;
  return t * 2048u + (r >> 2) * 128u + (4u * bi + j) * 4u + (((r & 1u) << 1) | ((r >> 1) & 1u));
}
__device__ __forceinline__ uint32_t xperm_q6k(uint32_t e) {
  const uint32_t b = e >> 8, o = e & 255, t = b >> 3, bi = b & 7;
  const uint32_t n = o >> 7, r1 = o & 127, g = r1 >> 5, r2 = r1 & 31, c = r2 >> 4, i = (r2 & 15) >> 2;
  return t * 2048u + (4u * g + i) * 128u + (4u * bi + 2u * n + c) * 4u + (((r2 & 1u) << 1) | ((r2 >> 1) & 1u));
}
// Writes activation e of row `row` in the natural layout and both permuted ones.
__device__ __forceinline__ void store_act(float* nat, uint32_t ldn, float* p4, float* p6, uint32_t ldp, uint32_t row,
                                          uint32_t e, float v) {
  if (nat) nat[(size_t)row * ldn + e] = v;
  if (p4) p4[(size_t)row * ldp + xperm_q4k(e)] = v;
  if (p6) p6[(size_t)row * ldp + xperm_q6k(e)] = v;
}
#endif

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
