// Device helpers of the tensor-core GEMVs (gemv_tc.cu: batch 1; gemv_umma.cu
// and gemv_tcb.cu: batches of 2..32): mma.sync, shared-memory loads, the
// mbarrier-completed bulk copies of the weight rings (with bounded waits),
// the quantized-value -> f16 operand tricks, and the hi/lo f16 split of x.
#pragma once
#include <cuda_fp16.h>
#include <stdint.h>

namespace sm {

constexpr uint32_t TC_SPIN_MAX = 1u << 22;  // bound on every mbarrier wait (then: error flag)

__device__ __forceinline__ void mma16816(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                         uint32_t b0, uint32_t b1) {
  asm(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}
__device__ __forceinline__ uint32_t h2u(__half2 h) { return *reinterpret_cast<uint32_t*>(&h); }
__device__ __forceinline__ __half2 u2h(uint32_t u) { return *reinterpret_cast<__half2*>(&u); }
__device__ __forceinline__ uint32_t smem_u32(const void* p) { return (uint32_t)__cvta_generic_to_shared(p); }
template <int OFF>
__device__ __forceinline__ uint4 lds128(uint32_t a) {
  uint4 v;
  asm volatile("ld.shared.v4.u32 {%0,%1,%2,%3}, [%4+%5];" : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "r"(a), "n"(OFF));
  return v;
}
template <int OFF>
__device__ __forceinline__ uint2 lds64(uint32_t a) {
  uint2 v;
  asm volatile("ld.shared.v2.u32 {%0,%1}, [%2+%3];" : "=r"(v.x), "=r"(v.y) : "r"(a), "n"(OFF));
  return v;
}
__device__ __forceinline__ void fence_proxy_async() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }
__device__ __forceinline__ void fence_mbar_init() { asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory"); }
__device__ __forceinline__ void mbar_init(uint64_t* b, uint32_t n) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(b)), "r"(n) : "memory");
}
__device__ __forceinline__ void mbar_expect_tx(uint64_t* b, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(b)), "r"(bytes) : "memory");
}
// One bulk copy global -> shared (16-byte aligned, size a multiple of 16) that
// completes `bytes` of transaction count on mbarrier b.
__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, uint32_t bytes, uint64_t* b) {
  asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                   smem_u32(dst)),
               "l"(src), "r"(bytes), "r"(smem_u32(b))
               : "memory");
}
// One wait of at most ~TC_SUSPEND_NS: the warp is parked by the hardware
// (not spinning) until the phase completes or the time hint runs out.
constexpr uint32_t TC_SUSPEND_NS = 1000;
__device__ __forceinline__ bool mbar_try(uint64_t* b, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{ .reg .pred p; mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3; selp.u32 %0, 1, 0, p; }"
      : "=r"(ok)
      : "r"(smem_u32(b)), "r"(parity), "n"(TC_SUSPEND_NS)
      : "memory");
  return ok != 0;
}
// Waits for phase `parity` of b to complete, at most TC_SPIN_MAX tries (a few
// seconds); a wait that gives up records it in *err and returns (the data is
// then not used for a result the caller keeps: the host reads the flag).
__device__ __forceinline__ void mbar_wait(uint64_t* b, uint32_t parity, uint32_t* err) {
  for (uint32_t n = 0; n < TC_SPIN_MAX; n++)
    if (mbar_try(b, parity)) return;
  if (err) atomicOr(err, 1u);
}

// Low nibbles of bytes (0, 2) as the half2 (q0, q2) * 2^-24 (exact subnormals).
__device__ __forceinline__ uint32_t nib_lo(uint32_t w) { return w & 0x000F000Fu; }
// High nibbles of bytes (0, 2): (q0, q2) * 2^-20.
__device__ __forceinline__ uint32_t nib_hi(uint32_t w) { return w & 0x00F000F0u; }
// Q6_K: 6-bit values v = q + 32 (low nibble + 2 bits of h at 4-5 / 20-21) * 2^-24.
__device__ __forceinline__ uint32_t q6_lo(uint32_t w, uint32_t h) { return (w & 0x000F000Fu) | (h & 0x00300030u); }
// Q6_K: high nibble + 2 bits of h at 8-9 / 24-25: v * 2^-20.
__device__ __forceinline__ uint32_t q6_hi(uint32_t w, uint32_t h) { return (w & 0x00F000F0u) | (h & 0x03000300u); }

// x (already scaled) -> (hi, lo): hi keeps 11 significant bits (round half
// away from zero on the magnitude), lo = x - hi exactly.
__device__ __forceinline__ float hi11(float v) { return __uint_as_float((__float_as_uint(v) + 0x1000u) & 0xFFFFE000u); }
__device__ __forceinline__ uint32_t hl_pair(float a, float b, bool lo) {
  const float ah = hi11(a), bh = hi11(b);
  return lo ? h2u(__floats2half2_rn(a - ah, b - bh)) : h2u(__floats2half2_rn(ah, bh));
}

// The arrival of one K-split slice at its group's counter, by one thread of a
// CTA after a barrier that follows the slice's stores: a wrapping increment
// (the counter is back at zero once the group's last slice arrives, so no
// store ever resets it) with acquire-release semantics at GPU scope. The
// release publishes the CTA's stores made before the barrier (cumulativity
// through the barrier); for the last arriver the acquire makes the other
// slices visible to the loads its threads make after the next barrier. One
// GPU-scope ordering point a CTA instead of a fence in every thread. Returns
// the counter's old value.
__device__ __forceinline__ uint32_t ks_arrive(uint32_t* cnt, uint32_t wrap) {
  uint32_t old;
  asm volatile("atom.acq_rel.gpu.global.inc.u32 %0, [%1], %2;" : "=r"(old) : "l"(cnt), "r"(wrap) : "memory");
  return old;
}

// Lane 0: the bulk copy of one block unit (UB bytes) into ring slot st.
__device__ __forceinline__ void tc_issue(const uint8_t* unit, uint32_t UB, uint8_t* ring, uint32_t stage_bytes,
                                         uint64_t* bars, uint32_t st) {
  fence_proxy_async();  // this slot's previous reads (ordered by __syncwarp) before the async write
  mbar_expect_tx(bars + st, UB);
  bulk_g2s(ring + st * stage_bytes, unit, UB, bars + st);
}

}  // namespace sm
