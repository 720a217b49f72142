// Device helpers shared by the GEMV kernels (gemv.cu, gemv_stream.cu):
// exact small-integer -> f32 conversion of weight pairs, and the epilogues
// that turn a row's dot product into the next tensor (residual + RMSNorm
// input, RoPE + KV append, SwiGLU).
#pragma once
#include <cuda_fp16.h>

#include "device.cuh"

namespace sm {

// fp16 -> f32 with the reference's NaN -> +-Inf quirk (dequant.rs:25-26).
__device__ __forceinline__ float h2f_ref(uint32_t h) {
  const float v = __half2float(__ushort_as_half((unsigned short)h));
  return ((h & 0x7C00u) == 0x7C00u) ? __uint_as_float(((h & 0x8000u) << 16) | 0x7F800000u) : v;
}
// Q6_K block scale: a non-finite d makes the block zero (dequant.rs:183-186;
// the reference GPU kernel skips such a block, kernels/src/lib.rs:845).
__device__ __forceinline__ float q6_d(uint32_t dbits) {
  const float d = h2f_ref(dbits);
  return isfinite(d) ? d : 0.f;
}
__device__ __forceinline__ float2 f2(float a, float b) { return make_float2(a, b); }
// v = two halves (off + a, off + b), exact: returns (a, b) in f32.
__device__ __forceinline__ float2 hpair(uint32_t v, __half2 off) {
  __half2 h = *reinterpret_cast<__half2*>(&v);
  return __half22float2(__hsub2(h, off));
}
// acc01 += pair(bytes 0,2) * (x.x, x.y); acc23 += pair(bytes 1,3) * (x.z, x.w)
// where pair p02/p13 are half2 of (off + q) for the word's byte fields.
__device__ __forceinline__ void fma_pairs(uint32_t p02, uint32_t p13, const float4& xv, __half2 off, float2& a0,
                                          float2& a1) {
  a0 = __ffma2_rn(hpair(p02, off), f2(xv.x, xv.y), a0);
  a1 = __ffma2_rn(hpair(p13, off), f2(xv.z, xv.w), a1);
}
__device__ __forceinline__ float hsum(const float2& a, const float2& b) { return (a.x + a.y) + (b.x + b.y); }
__device__ __forceinline__ float sum4(const float4& v) { return (v.x + v.y) + (v.z + v.w); }

// ------------------------------------------------------------ epilogue ----
// Input RMSNorm scale of column col (1 when the input is not normalized):
// the sum of the producer's per-CTA partials in a fixed order (deterministic).
__device__ __forceinline__ float input_scale(const GemvArgs& a, uint32_t col) {
  if (!a.in_parts) return 1.0f;
  const int lane = threadIdx.x & 31;
  float s = 0.f;
  for (uint32_t i = lane; i < a.in_np; i += 32) s += a.in_parts[(size_t)col * a.in_np + i];
  s = warp_sum(s);
  return 1.0f / sqrtf(s / (float)a.in_n + a.in_eps);
}

// Single-row epilogues; returns the new residual value for EPI_RESID, else 0.
__device__ __forceinline__ float epi_single(const GemvArgs& a, const GemvSeg& sg, uint32_t o, uint32_t col, float v) {
  if (sg.bias) v = v + sg.bias[o];
  float* y = sg.y + (size_t)col * sg.ldy + o;
  switch (sg.epi) {
    case EPI_STORE: *y = v; return 0.f;
    case EPI_ADD: *y = *y + v; return 0.f;
    case EPI_RESID: {  // x += v (qwen2.rs:536-538, 549-551)
      const float xn = *y + v;
      *y = xn;
      a.xn[(size_t)col * a.ldxn + o] = xn * a.nw[o];
      return xn;
    }
    case EPI_PUSH: {  // tensor parallel: this rank's partial sum to every rank (tp.cu)
      const TpPush& P = a.push;
      const uint32_t e = __ldcg(P.epoch + (P.base + o) / P.per) + 1u;
      const uint64_t pk = ((uint64_t)e << 32) | __float_as_uint(v);
      const uint64_t off = (e & 1u) * P.parity_stride + P.rank * P.src_stride + (uint64_t)col * P.ld + o;
      for (uint32_t k = 0; k < P.world; k++)
        asm volatile("st.volatile.global.u64 [%0], %1;" ::"l"(P.dst[k] + off), "l"(pk) : "memory");
      return 0.f;
    }
    case EPI_V: {  // v row into the cache at the row's position (qwen2.rs:498)
      const RowDesc rd = a.rows[col];
      const SeqDesc sd = a.seqs[rd.seq];
      sd.pages[rd.pos / KV_PAGE][sd.voff + kv_page_off(a.layer, rd.pos, a.kvd) + o] = v;
      return 0.f;
    }
  }
  return 0.f;
}

// Pair epilogues on physical rows (o, o+1), o even.
__device__ __forceinline__ void epi_pair(const GemvArgs& a, const GemvSeg& sg, uint32_t o, uint32_t col, float v0,
                                         float v1) {
  if (sg.bias) { v0 = v0 + sg.bias[o]; v1 = v1 + sg.bias[o + 1]; }
  if (sg.epi == EPI_SILU) {  // gate = silu(gate) * up (qwen2.rs:546-548, 743-745)
    const uint32_t m = o >> 1;
    const float hv = __fmul_rn(__fdiv_rn(v0, __fadd_rn(1.0f, expf(-v0))), v1);
    a.h[(size_t)col * a.ldh + m] = hv;
    return;
  }
  // NEOX RoPE of the pair (dim m, dim m + hd/2) at the row's position
  // (qwen2.rs:708-724); cos/sin from the host table.
  const uint32_t half = a.hd >> 1, h = o / a.hd, m = (o - h * a.hd) >> 1;
  const RowDesc rd = a.rows[col];
  const float c = a.cos_t[(size_t)rd.pos * half + m], s = a.sin_t[(size_t)rd.pos * half + m];
  const float r0 = __fsub_rn(__fmul_rn(v0, c), __fmul_rn(v1, s));
  const float r1 = __fadd_rn(__fmul_rn(v0, s), __fmul_rn(v1, c));
  if (sg.epi == EPI_ROPE_Q) {
    float* y = sg.y + (size_t)col * sg.ldy + h * a.hd + m;
    y[0] = r0;
    y[half] = r1;
  } else {  // EPI_ROPE_K: into the K cache (qwen2.rs:497)
    const SeqDesc sd = a.seqs[rd.seq];
    float* kc = sd.pages[rd.pos / KV_PAGE] + kv_page_off(a.layer, rd.pos, a.kvd) + h * a.hd + m;
    kc[0] = r0;
    kc[half] = r1;
  }
}

}  // namespace sm
