// Device-side layouts and helpers of the B200 decode engine (sm_100a).
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>

namespace sm {

// ---------------------------------------------------------------------------
// HBM layout of one quantized weight [n_out x n_in] (row-major, a row = one
// output). Rows of `body` start on 16-byte boundaries so every lane reads its
// share of a row with 128-bit loads:
//   Q4_K: body = the GGUF blocks unchanged (144 B = 9 x 16 B per 256 values).
//   Q6_K: body = 208 B per block (ql 128 | qh 64 | scales 16), aux = fp16 d per
//         block. The GGUF block is 210 B with d last (dequant.rs:178-182); the
//         split only moves d so that blocks stay 16-byte aligned.
//   Q8_0: body = 32 B of qs per block, aux = fp16 d per block.
//   Q5_0: body = 16 B of qs per block, aux = 8 B per block (qh u32 | d fp16 | 0).
// Every byte of the GGUF encoding is kept; dequantization reads exactly the
// reference's bytes.
// ---------------------------------------------------------------------------
struct DWDesc {
  const uint8_t* body;
  const uint8_t* aux;
  uint32_t type, n_out, n_in;
  uint32_t body_stride;  // bytes per row
  uint32_t aux_stride;   // bytes per row
};

// One output segment of a (possibly fused) GEMV launch.
struct GemvSeg {
  DWDesc w;
  float* y;            // y[b * ldy + o]
  const float* bias;   // optional, added to every column
  uint32_t ldy;
  uint32_t add;        // 1: y += result (residual), 0: y = result
  uint32_t cta_begin;  // first CTA index of this segment
};

struct GemvArgs {
  GemvSeg seg[3];
  uint32_t nseg;
  const float* x;  // x[b * ldx + d]
  uint32_t ldx;
  uint32_t batch;
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
