// Exchange kernels of tensor-parallel decode (see tp.hpp): the all-reduce
// that follows the row-split O and down GEMVs, fused with the residual add
// and the next RMSNorm's input, and the all-gather of the vocab-split logits.
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

struct TpSrc {
  const float* p[TP_MAX];
};

__device__ __forceinline__ uint64_t global_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}
__device__ __forceinline__ void st_release_sys(uint32_t* p, uint32_t v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
// Peer data: never served from a stale L1 line of an earlier exchange.
__device__ __forceinline__ float4 ld_peer4(const float* p) { return __ldcv(reinterpret_cast<const float4*>(p)); }
__device__ __forceinline__ float ld_peer(const float* p) { return __ldcv(p); }

// Block-level barrier of one exchange. Thread r < world publishes this
// block's epoch into rank r's flag slot [block][rank] and waits (bounded)
// until rank r has published the same epoch into ours. All ranks run the
// same sequence of exchanges with the same grid, so a block's epoch is the
// same on every rank. Returns false (and sets the error word) if a peer did
// not arrive within wait_ns.
__device__ bool tp_block_sync(const TpPeers& p) {
  __shared__ uint32_t s_ep, s_ok;
  const uint32_t b = blockIdx.x;
  if (threadIdx.x == 0) {
    const uint32_t e = p.epoch[b] + 1u;
    p.epoch[b] = e;
    s_ep = e;
    s_ok = 1u;
  }
  __syncthreads();
  if (!p.sync) return true;
  const uint32_t ep = s_ep;
  // After one timed-out wait the group is broken: the exchanges that follow
  // in the same pass give up at once instead of each waiting out the bound.
  const bool broken = (*reinterpret_cast<volatile uint32_t*>(p.err) & TP_ERR_WAIT) != 0u;
  if (broken) {
    if (threadIdx.x == 0) s_ok = 0u;
  } else if (threadIdx.x < p.world) {
    const uint32_t r = threadIdx.x;
    __threadfence_system();  // this rank's send data before the signal
    st_release_sys(p.flag[r] + b * TP_MAX + p.rank, ep);
    const uint32_t* f = p.flag[p.rank] + b * TP_MAX + r;
    const uint64_t t0 = global_ns();
    // A peer is at most one exchange ahead (it waits for this rank's signal
    // of the next one), so "arrived" is epoch >= ep, compared modulo 2^32.
    while ((int32_t)(ld_acquire_sys(f) - ep) < 0) {
      if (global_ns() - t0 > p.wait_ns) {
        atomicOr(p.err, TP_ERR_WAIT);
        s_ok = 0u;
        break;
      }
      __nanosleep(100);
    }
  }
  __syncthreads();
  return s_ok != 0u;
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

__global__ void __launch_bounds__(TP_THREADS, 16)
    tp_reduce_resid_kernel(const __grid_constant__ TpPeers p, const __grid_constant__ TpSrc s, uint32_t nsrc,
                           uint32_t rows, uint32_t n, float* x, uint32_t ldx, const float* nw, float* xn,
                           uint32_t ldxn, float* parts) {
  pdl_trigger();  // the next GEMV may start its weight copies
  pdl_wait();     // the GEMV that wrote this rank's partial sums has finished
  if (!tp_block_sync(p)) return;
  __shared__ float red[TP_THREADS / 32];
  const uint32_t per = (n + TP_BLOCKS - 1) / TP_BLOCKS;
  const uint32_t e0 = blockIdx.x * per, e1 = min(n, e0 + per);
  for (uint32_t r = 0; r < rows; r++) {
    float ss = 0.f;
    for (uint32_t e = e0 + threadIdx.x; e < e1; e += TP_THREADS) {
      const size_t off = (size_t)r * n + e;
      float v[TP_MAX];
#pragma unroll
      for (uint32_t k = 0; k < TP_MAX; k++)
        if (k < nsrc) v[k] = ld_peer(s.p[k] + off);
      float acc = v[0];
#pragma unroll
      for (uint32_t k = 1; k < TP_MAX; k++)
        if (k < nsrc) acc = __fadd_rn(acc, v[k]);
      float* xp = x + (size_t)r * ldx + e;
      const float xv = __fadd_rn(*xp, acc);
      *xp = xv;
      xn[(size_t)r * ldxn + e] = __fmul_rn(xv, nw[e]);
      ss = __fmaf_rn(xv, xv, ss);
    }
    const float t = block_sum(ss, red);
    if (threadIdx.x == 0) parts[(size_t)r * TP_BLOCKS + blockIdx.x] = t;
  }
}

__global__ void __launch_bounds__(TP_THREADS, 16)
    tp_gather_kernel(const __grid_constant__ TpPeers p, const __grid_constant__ TpSrc s, uint32_t nsrc, uint32_t rows,
                     uint32_t nl, uint32_t n_total, float* out, uint32_t ldo) {
  pdl_trigger();
  pdl_wait();  // the head GEMV that wrote this rank's slice has finished
  if (!tp_block_sync(p)) return;
  // Groups of 4 consecutive elements of one (row, source) slice.
  const uint32_t g_per = (nl + 3) / 4, per_row = g_per * nsrc, total = rows * per_row;
  for (uint32_t i = blockIdx.x * TP_THREADS + threadIdx.x; i < total; i += TP_BLOCKS * TP_THREADS) {
    const uint32_t r = i / per_row, rem = i - r * per_row, k = rem / g_per, j0 = 4u * (rem - k * g_per);
    const uint32_t base = k * nl;
    if (base >= n_total) continue;
    const uint32_t cnt = min(nl, n_total - base);
    const float* src = s.p[k] + (size_t)r * nl;
    float* dst = out + (size_t)r * ldo + base;
    float v[4];
#pragma unroll
    for (uint32_t q = 0; q < 4; q++) v[q] = (j0 + q < cnt) ? ld_peer(src + j0 + q) : 0.f;
#pragma unroll
    for (uint32_t q = 0; q < 4; q++)
      if (j0 + q < cnt) dst[j0 + q] = v[q];
  }
}

TpSrc to_src(const float* const* src, uint32_t nsrc) {
  TpSrc s{};
  for (uint32_t k = 0; k < nsrc && k < TP_MAX; k++) s.p[k] = src[k];
  return s;
}

}  // namespace

cudaError_t launch_tp_reduce_resid(const TpPeers& p, const float* const* src, uint32_t nsrc, uint32_t rows, uint32_t n,
                                   float* x, uint32_t ldx, const float* nw, float* xn, uint32_t ldxn, float* parts,
                                   cudaStream_t st) {
  if (nsrc == 0 || nsrc > TP_MAX) return cudaErrorInvalidValue;
  return launch_pdl(tp_reduce_resid_kernel, dim3(TP_BLOCKS), dim3(TP_THREADS), 0, st, p, to_src(src, nsrc), nsrc, rows,
                    n, x, ldx, nw, xn, ldxn, parts);
}

cudaError_t launch_tp_gather(const TpPeers& p, const float* const* src, uint32_t nsrc, uint32_t rows, uint32_t nl,
                             uint32_t n_total, float* out, uint32_t ldo, cudaStream_t st) {
  if (nsrc == 0 || nsrc > TP_MAX) return cudaErrorInvalidValue;
  return launch_pdl(tp_gather_kernel, dim3(TP_BLOCKS), dim3(TP_THREADS), 0, st, p, to_src(src, nsrc), nsrc, rows, nl,
                    n_total, out, ldo);
}

}  // namespace sm
