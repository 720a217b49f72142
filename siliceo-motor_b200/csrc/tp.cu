// Consumer kernels of tensor-parallel decode (see tp.hpp): the all-reduce
// that follows the row-split O and down GEMVs, fused with the residual add
// and the next RMSNorm's input, and the all-gather of the vocab-split logits.
// The producing GEMVs push their outputs as packets (EPI_PUSH); these kernels
// wait for the packets in their own memory and combine them.
//
// Replaces, for the partitioned 70B configuration, the per-block NCCL
// all-reduce of a Megatron split: the reference runs one process on one
// device (crates/s-backend-cuda/src/model.rs:146-211) and adds the O / down
// outputs to the residual in place (crates/s-models/src/qwen2.rs:536-551).
#include "device.cuh"
#include "pdl.cuh"
#include "tp.hpp"

namespace sm {
namespace {

constexpr uint32_t TP_THREADS = 128;

__device__ __forceinline__ uint64_t global_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}
__device__ __forceinline__ uint64_t ld_packet(const uint64_t* p) {
  uint64_t v;
  asm volatile("ld.volatile.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}

// The value of packet *p once it carries epoch e. A sender is at most one
// exchange ahead (it waits for this rank's packets of the next exchange), and
// the two halves of an area alternate, so the packet holds epoch e, e - 2
// (not yet written) or 0 (never written). The wait is bounded; after one
// timed-out wait the group is broken and later waits give up at once.
__device__ __forceinline__ float tp_wait_packet(const uint64_t* p, uint32_t e, const TpRecv& r, bool& ok) {
  uint64_t v = ld_packet(p);
  if ((uint32_t)(v >> 32) == e) return __uint_as_float((uint32_t)v);
  const uint64_t t0 = global_ns();
  while (ok) {
    if (*reinterpret_cast<volatile uint32_t*>(r.err) & TP_ERR_WAIT) {
      ok = false;
      break;
    }
    __nanosleep(32);
    v = ld_packet(p);
    if ((uint32_t)(v >> 32) == e) return __uint_as_float((uint32_t)v);
    if (global_ns() - t0 > r.wait_ns) {
      atomicOr(r.err, TP_ERR_WAIT);
      ok = false;
    }
  }
  return 0.f;
}

// Deterministic block sum (fixed shuffle tree, then warps in order).
__device__ __forceinline__ float block_sum(float v, float* red) {
  v = warp_sum(v);
  const uint32_t w = threadIdx.x >> 5;
  if ((threadIdx.x & 31) == 0) red[w] = v;
  __syncthreads();
  float s = 0.f;
  if (threadIdx.x == 0) {
#pragma unroll
    for (uint32_t i = 0; i < TP_THREADS / 32; i++) s += red[i];
  }
  __syncthreads();
  return s;
}

// This block's epoch of the exchange (packets mode), and its update once the
// block is done.
__device__ __forceinline__ uint32_t tp_epoch(const TpRecv& r) {
  __shared__ uint32_t s_e;
  if (threadIdx.x == 0) s_e = r.pk ? r.epoch[blockIdx.x] + 1u : 0u;
  __syncthreads();
  return s_e;
}
__device__ __forceinline__ void tp_epoch_done(const TpRecv& r, uint32_t e) {
  __syncthreads();
  if (threadIdx.x == 0 && r.pk) r.epoch[blockIdx.x] = e;
}

__global__ void __launch_bounds__(TP_THREADS, 16)
    tp_reduce_resid_kernel(const __grid_constant__ TpRecv r, uint32_t rows, uint32_t n, float* x, uint32_t ldx,
                           const float* nw, float* xn, uint32_t ldxn, float* parts) {
  pdl_trigger();  // the next GEMV may start its weight copies
  pdl_wait();     // this rank's producer GEMV has finished (its pushes are out)
  const uint32_t e = tp_epoch(r);
  __shared__ float red[TP_THREADS / 32];
  bool ok = true;
  const uint32_t nsrc = r.pk ? r.world : 1u;
  const uint32_t o0 = blockIdx.x * r.per, o1 = min(n, o0 + r.per);
  const uint64_t* half = r.pk ? r.pk + (e & 1u) * r.parity_stride : nullptr;
  for (uint32_t row = 0; row < rows; row++) {
    float ss = 0.f;
    for (uint32_t o = o0 + threadIdx.x; o < o1; o += TP_THREADS) {
      const size_t off = (size_t)row * r.ld + o;
      float acc = 0.f;
      if (half) {
        float v[TP_MAX];
#pragma unroll
        for (uint32_t k = 0; k < TP_MAX; k++)
          if (k < nsrc) v[k] = tp_wait_packet(half + k * r.src_stride + off, e, r, ok);
        acc = v[0];
#pragma unroll
        for (uint32_t k = 1; k < TP_MAX; k++)
          if (k < nsrc) acc = __fadd_rn(acc, v[k]);  // rank order: the same bits on every rank
      } else {
        acc = r.plain[off];
      }
      float* xp = x + (size_t)row * ldx + o;
      const float xv = __fadd_rn(*xp, acc);
      *xp = xv;
      xn[(size_t)row * ldxn + o] = __fmul_rn(xv, nw[o]);
      ss = __fmaf_rn(xv, xv, ss);
    }
    const float t = block_sum(ss, red);
    if (threadIdx.x == 0) parts[(size_t)row * TP_BLOCKS + blockIdx.x] = t;
  }
  tp_epoch_done(r, e);
}

__global__ void __launch_bounds__(TP_THREADS, 16)
    tp_gather_kernel(const __grid_constant__ TpRecv r, uint32_t rows, uint32_t nl, uint32_t n_total, float* out,
                     uint32_t ldo) {
  pdl_trigger();
  pdl_wait();  // this rank's head GEMV has finished
  const uint32_t e = tp_epoch(r);
  bool ok = true;
  const uint32_t v0 = blockIdx.x * r.per, v1 = min(n_total, v0 + r.per);
  for (uint32_t row = 0; row < rows; row++)
    for (uint32_t v = v0 + threadIdx.x; v < v1; v += TP_THREADS) {
      const uint32_t k = v / nl, j = v - k * nl;
      const size_t off = k * r.src_stride + (size_t)row * r.ld + j;
      out[(size_t)row * ldo + v] = r.pk ? tp_wait_packet(r.pk + off, e, r, ok) : r.plain[off];
    }
  tp_epoch_done(r, e);
}

}  // namespace

cudaError_t launch_tp_reduce_resid(const TpRecv& rv, uint32_t rows, uint32_t n, float* x, uint32_t ldx, const float* nw,
                                   float* xn, uint32_t ldxn, float* parts, cudaStream_t st) {
  if (rv.world == 0 || rv.world > TP_MAX || !rv.err || (!rv.pk && !rv.plain) || !rv.per) return cudaErrorInvalidValue;
  return launch_pdl(tp_reduce_resid_kernel, dim3(TP_BLOCKS), dim3(TP_THREADS), 0, st, rv, rows, n, x, ldx, nw, xn,
                    ldxn, parts);
}

cudaError_t launch_tp_gather(const TpRecv& rv, uint32_t rows, uint32_t nl, uint32_t n_total, float* out, uint32_t ldo,
                             cudaStream_t st) {
  if (rv.world == 0 || rv.world > TP_MAX || !rv.err || (!rv.pk && !rv.plain) || nl == 0 || !rv.per)
    return cudaErrorInvalidValue;
  return launch_pdl(tp_gather_kernel, dim3(TP_BLOCKS), dim3(TP_THREADS), 0, st, rv, rows, nl, n_total, out, ldo);
}

}  // namespace sm
