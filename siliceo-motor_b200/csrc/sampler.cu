// On-device Sampler::sample (crates/s-models/src/sampling.rs:94-144), bit for
// bit: only the token id and the RNG state leave the GPU.
//
// The reference, for temperature T > 0:
//   p_i = l_i / T; probs_i = exp(p_i - max p) / sum, the sum taken left to
//   right in f32 (softmax, sampling.rs:157-172); indices sorted by probs
//   descending, lower index first on ties; top-k truncation; top-p cut over
//   the sorted cumulative f32 sum (the crossing token kept, at least one);
//   total = f32 sum of the kept probs in sorted order; r = next_f32() * total,
//   and the sorted walk subtracts probs until r <= 0 (else the last kept).
// Greedy (T <= 0) is argmax: the first maximum; a NaN logit never wins,
// except that a NaN at index 0 is returned (the comparison x[i] > x[0] is
// false for every i).
//
// Every value the reference rounds is rounded the same way here:
//   * exp is glibc's expf (Rust's f32::exp on x86-64 Linux) on x <= 0:
//     expf_ref below (expf_ref.cuh, with a build-time table of glibc's
//     misrounded inputs);
//   * the softmax denominator is the exact value of the reference's
//     left-to-right f32 sum, obtained in parallel (exact_seq_sum): every
//     thread summarizes its chunk of the terms for the few float binades the
//     running sum can be in while the chunk is added (the integer sum of the
//     terms rounded to that binade's grid, for either parity of the running
//     sum, because a term exactly halfway rounds to even), and one warp
//     composes the chunks, 32 at a time by a shuffle scan of the summaries,
//     adding a chunk term by term only where the running sum leaves its
//     binade inside it;
//   * probs = e / sum with IEEE division; the order is by the probs values,
//     so terms that round to equal probs are ordered by index as in the
//     reference, not by their logits;
//   * cumulative, total and walk run in sorted order with f32 adds.
// top_k in 1..1024 finds a threshold key from per-thread counters of the
// keys' distance below the largest key, gathers the keys at or above it and
// sorts them in shared memory (a radix select when ties overflow the
// candidate buffer); otherwise (None, or larger) the whole vocabulary is
// sorted with a stable least-significant-digit radix sort in the row's
// scratch (four 8-bit passes) and scanned in order.
#include <cfloat>

#include "device.cuh"
#include "expf_ref.cuh"
#include "layers.cuh"
#include "pdl.cuh"

namespace sm {

#define SM_EXPF_EXC_DECL static __device__ const uint32_t
#include "expf_exc.inc"

__constant__ double c_exp2_32[32] = SM_EXP2_32_TABLE;

// glibc's expf(x) for an input whose rounded double f may differ from it:
// the table's value for x, else f.
__device__ __forceinline__ float expf_lookup(float x, float f) {
  const uint32_t xb = __float_as_uint(x);
  int lo = 0, hi = SM_EXPF_EXC_N - 1;
  while (lo <= hi) {
    const int mid = (lo + hi) >> 1;
    const uint32_t v = sm_expf_exc[mid][0];
    if (v == xb) return __uint_as_float(sm_expf_exc[mid][1]);
    if (v < xb) lo = mid + 1;
    else hi = mid - 1;
  }
  return f;
}

// glibc's expf(x) for x <= 0 (NaN passes through; x > 0 is outside the
// sampler's domain and uses CUDA's expf). With `check`, an input that needs
// the table is not looked up: *check is set and the rounded double returned,
// for a later expf_lookup(x, it).
// t32: the 2^(j/32) table (c_exp2_32, or its copy in shared memory: the
// lanes of a warp index it with different j, which constant memory serves
// one address at a time).
__device__ __forceinline__ float expf_ref(float x, const double* t32, bool* check = nullptr) {
  if (check) *check = false;
  if (x != x) return x;
  if (x > 0.0f) return expf(x);
  if (x < -104.0f) return 0.0f;
  const ExpfEval ev = expf_eval(x, t32);
  if (!ev.check) return ev.f;
  if (check) {
    *check = true;
    return ev.f;
  }
  return expf_lookup(x, ev.f);
}

__global__ void expf_ref_kernel(const float* x, float* y, size_t n) {
  for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x)
    y[i] = expf_ref(x[i], c_exp2_32);
}

constexpr int SMP_THREADS = 1024;
constexpr int SMP_KMAX = 1024;

__device__ __forceinline__ uint64_t rng_next(uint64_t& s) {  // sampling.rs:28-34
  s += 0x9E3779B97F4A7C15ull;
  uint64_t z = s;
  z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
  z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
  return z ^ (z >> 31);
}
__device__ __forceinline__ float rng_f32(uint64_t& s) {  // sampling.rs:37-40
  return __double2float_rn(__ddiv_rn((double)(rng_next(s) >> 11), 9007199254740992.0));
}
// Order-preserving key of a float (larger value -> larger key) and back.
__device__ __forceinline__ uint32_t fkey(float f) {
  const uint32_t u = __float_as_uint(f);
  return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}
__device__ __forceinline__ float fkey_inv(uint32_t k) {
  return __uint_as_float((k & 0x80000000u) ? (k & 0x7FFFFFFFu) : ~k);
}

struct Best {
  float v;
  uint32_t i;
};
__device__ __forceinline__ Best better(Best a, Best b) {  // larger value, then lower index
  if (b.v > a.v || (b.v == a.v && b.i < a.i)) return b;
  return a;
}

// ------------------------------------------------ exact sequential sum ----
// Per-chunk summary for the running sum s in binade E (2^E <= s < 2^(E+1),
// grid u = 2^(E-23)): D[E][p] = the sum of the chunk's terms each rounded to
// the grid (halfway terms to the even multiple, which depends on the parity
// p of s / u before the term), or SUM_SAT when it reaches 2^24.
constexpr int SUM_NE = 4;  // candidate binades per chunk
constexpr uint32_t SUM_SAT = 0xFFFFFFFFu;
struct SumRec {
  int32_t e_lo;   // first candidate binade
  uint32_t ok;    // bit 0: summary valid (no NaN, window small enough)
  uint32_t d[SUM_NE][2];
};
constexpr uint32_t SMP_SORT_COUNTS = 32 * 256, SMP_SORT_BASES = 512;
constexpr uint32_t SMP_PATCH = 8192;  // terms whose exp is looked up after the terms pass
constexpr size_t SMP_BIG = sizeof(SumRec) * SMP_THREADS;
static_assert(SMP_BIG >= sizeof(unsigned long long) * SMP_KMAX, "candidates fit the shared buffer");
static_assert(SMP_BIG >= 4 * (SMP_SORT_COUNTS + SMP_SORT_BASES), "sort counters fit the shared buffer");
static_assert(SMP_BIG >= 4 * SMP_PATCH, "the exp patch list fits the shared buffer");
static_assert(SMP_BIG >= 8 * SMP_KMAX + 4 * 32 * 8, "candidates and the selection counts fit the shared buffer");

// The rounded increment of a non-negative finite float term (bits tb) on the
// grid 2^(E-23): q = floor(term / u), and whether the remainder is above /
// exactly half of u.
__device__ __forceinline__ void grid_term(uint32_t tb, int E, uint64_t& q, bool& up, bool& tie) {
  up = tie = false;
  q = 0;
  if (tb == 0) return;
  const uint32_t ex = tb >> 23, mant = tb & 0x7FFFFFu;
  const uint32_t m24 = ex ? (mant | 0x800000u) : mant;
  const int e2 = ex ? (int)ex - 150 : -149;  // term = m24 * 2^e2
  const int sh = E - 23 - e2;                // term / u = m24 * 2^-sh
  if (sh <= 0) {
    q = -sh >= 40 ? (uint64_t(1) << 40) : ((uint64_t)m24 << (-sh));
    return;
  }
  if (sh > 25) return;  // below half of u
  q = m24 >> sh;
  const uint32_t rem = m24 & ((1u << sh) - 1u), half = 1u << (sh - 1);
  up = rem > half;
  tie = rem == half;
}

// Increment from starting parity p of a run of chunks A (increment a from
// p) followed by a run B (b0 / b1 from parity 0 / 1), or SUM_SAT when either
// saturates or the total reaches 2^24.
__device__ __forceinline__ uint32_t sum_cat(uint32_t a, uint32_t b0, uint32_t b1, uint32_t p) {
  if (a == SUM_SAT) return SUM_SAT;
  const uint32_t b = ((p + a) & 1u) ? b1 : b0;
  if (b == SUM_SAT) return SUM_SAT;
  const uint32_t t = a + b;
  return t >= (1u << 24) ? SUM_SAT : t;
}

// v[i .. i + 8) with zeros past e: two 16-byte loads when v + i is 16-byte
// aligned and all eight are in range, else eight 4-byte loads.
__device__ __forceinline__ void load8(const float* v, uint32_t i, uint32_t e, float (&t)[8]) {
  if (i + 8 <= e && (reinterpret_cast<uintptr_t>(v + i) & 15u) == 0) {
    const float4 x = *reinterpret_cast<const float4*>(v + i), y = *reinterpret_cast<const float4*>(v + i + 4);
    t[0] = x.x; t[1] = x.y; t[2] = x.z; t[3] = x.w;
    t[4] = y.x; t[5] = y.y; t[6] = y.z; t[7] = y.w;
  } else {
#pragma unroll
    for (int q = 0; q < 8; q++) t[q] = i + q < e ? v[i + q] : 0.0f;
  }
}

// Sixteen 8-bit counters in four words (a thread counts at most 255 keys).
__device__ __forceinline__ void pc_add(uint32_t (&pc)[4], uint32_t bin) {
  const uint32_t inc = 1u << (8u * (bin & 3u)), w = bin >> 2;
  pc[0] += w == 0 ? inc : 0u;
  pc[1] += w == 1 ? inc : 0u;
  pc[2] += w == 2 ? inc : 0u;
  pc[3] += w == 3 ? inc : 0u;
}
// The CTA's sums of the sixteen counters: lane l < 16 of warp 0 gets bin l
// (other threads get 0). wcnt: 32 x 8 words of shared memory. Called by all.
__device__ __forceinline__ uint32_t pc_reduce(const uint32_t (&pc)[4], uint32_t* wcnt) {
  const uint32_t lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  uint32_t u[8];  // 16-bit fields: word j holds bins 2j, 2j + 1
#pragma unroll
  for (int w = 0; w < 4; w++) {
    u[2 * w] = (pc[w] & 0xFFu) | ((pc[w] & 0xFF00u) << 8);
    u[2 * w + 1] = ((pc[w] >> 16) & 0xFFu) | ((pc[w] >> 8) & 0xFF0000u);
  }
#pragma unroll
  for (int j = 0; j < 8; j++)
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) u[j] += __shfl_xor_sync(0xffffffffu, u[j], o);
  if (lane == 0)
#pragma unroll
    for (int j = 0; j < 8; j++) wcnt[warp * 8 + j] = u[j];
  __syncthreads();
  uint32_t c = 0;
  if (warp == 0 && lane < 16)
    for (uint32_t w = 0; w < SMP_THREADS / 32; w++) c += (wcnt[w * 8 + (lane >> 1)] >> (16 * (lane & 1))) & 0xFFFFu;
  __syncthreads();
  return c;
}

// The reference's left-to-right f32 sum of v[0..n) (non-negative terms or NaN)
// computed by the whole CTA (SMP_THREADS threads, chunk c = [c*C, (c+1)*C)).
// v was written by this CTA before the call; each thread walks its own chunk
// with ordinary (L1-cached) loads, which see those writes after the CTA's
// barrier.
// With stop >= 0, instead returns in *cut the first index i at which the
// running sum after v[i] is >= stop (n if none) and the sum up to it.
// Called by all threads; the result is valid in every thread.
__device__ float exact_seq_sum(const float* v, uint32_t n, float stop, uint32_t* cut, SumRec* recs, double* scan) {
  const uint32_t tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const uint32_t C = ((n + SMP_THREADS - 1) / SMP_THREADS + 3) & ~3u;
  const uint32_t b = min(n, tid * C), e = min(n, b + C);
  // 1. approximate chunk sums (double) and their exclusive prefix
  double d = 0.0;
  bool nan = false;
  for (uint32_t i = b; i < e; i += 8) {
    float t[8];
    load8(v, i, e, t);
#pragma unroll
    for (int q = 0; q < 8; q++) {
      nan |= t[q] != t[q];
      d += (double)t[q];
    }
  }
  double inc = d;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const double t = __shfl_up_sync(0xffffffffu, inc, o);
    if (lane >= (uint32_t)o) inc += t;
  }
  if (lane == 31) scan[warp] = inc;
  __syncthreads();
  if (warp == 0) {
    const double w = scan[lane];
    double wi = w;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const double t = __shfl_up_sync(0xffffffffu, wi, o);
      if (lane >= (uint32_t)o) wi += t;
    }
    scan[32 + lane] = wi - w;
  }
  __syncthreads();
  const double P = scan[32 + warp] + inc - d;  // exact sum before this chunk, approximately
  // 2. candidate binades: the f32 running sum is within (n * 2^-24) < 2^-5
  //    relative of the exact one
  SumRec r;
  r.ok = 0;
  r.e_lo = 0;
  if (!nan && e > b && P > 0.0) {
    const int lo = ilogb(P * (1.0 - 0x1p-5)), hi = ilogb((P + d) * (1.0 + 0x1p-5));
    if (hi - lo < SUM_NE) {
      r.e_lo = lo;
      r.ok = 1;
      // only the binades the running sum can reach in this chunk (usually 1-2)
#pragma unroll
      for (int k = 0; k < SUM_NE; k++) r.d[k][0] = r.d[k][1] = SUM_SAT;
      for (int k = 0; k <= hi - lo; k++) {
        uint64_t D0 = 0, D1 = 0;
        uint32_t par0 = 0, par1 = 1;
        const int E = lo + k;
        for (uint32_t i = b; i < e; i += 8) {
          float t[8];
          load8(v, i, e, t);  // zeros past e add nothing
#pragma unroll
          for (int j = 0; j < 8; j++) {
            uint64_t q;
            bool up, tie;
            grid_term(__float_as_uint(t[j]), E, q, up, tie);
            const uint64_t r0 = q + (tie ? ((par0 + (uint32_t)q) & 1u) : (uint32_t)up);
            const uint64_t r1 = q + (tie ? ((par1 + (uint32_t)q) & 1u) : (uint32_t)up);
            D0 += r0;
            D1 += r1;
            par0 = (par0 + (uint32_t)r0) & 1u;
            par1 = (par1 + (uint32_t)r1) & 1u;
          }
        }
        r.d[k][0] = D0 >= (1u << 24) ? SUM_SAT : (uint32_t)D0;
        r.d[k][1] = D1 >= (1u << 24) ? SUM_SAT : (uint32_t)D1;
      }
    }
  }
  recs[tid] = r;
  __syncthreads();
  // 3. warp 0 composes the chunks in order, 32 at a time. In the running
  //    sum's binade, chunk summaries compose (the increment of A then B from
  //    parity p is D_A[p] + D_B[(p + D_A[p]) & 1]), so a shuffle scan gives
  //    the sum after each of the next 32 chunks; the first chunk that leaves
  //    the binade, has no summary there, or reaches `stop` is added term by
  //    term (its terms loaded by the whole warp at once, the adds done in
  //    order by every lane alike).
  if (warp == 0) {
    const uint32_t nch = C ? (n + C - 1) / C : 0u;
    float s = 0.0f;
    uint32_t where = n, c = 0;
    while (c < nch) {
      const uint32_t sb = __float_as_uint(s), ex = sb >> 23;
      const uint32_t m0 = (sb & 0x7FFFFFu) | 0x800000u;
      const uint32_t cj = c + lane;
      uint32_t q0 = SUM_SAT, q1 = SUM_SAT;
      if (cj < nch && ex >= 1 && ex < 255) {
        const SumRec& rc = recs[cj];
        const int k = (int)ex - 127 - rc.e_lo;
        if ((rc.ok & 1u) && k >= 0 && k < SUM_NE) {
          q0 = rc.d[k][0];
          q1 = rc.d[k][1];
        }
      }
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {  // inclusive scan: chunks c .. cj, per starting parity
        const uint32_t a0 = __shfl_up_sync(0xffffffffu, q0, o), a1 = __shfl_up_sync(0xffffffffu, q1, o);
        if (lane >= (uint32_t)o) {
          const uint32_t n0 = sum_cat(a0, q0, q1, 0u), n1 = sum_cat(a1, q0, q1, 1u);
          q0 = n0;
          q1 = n1;
        }
      }
      const uint32_t D = (m0 & 1u) ? q1 : q0;
      const bool fits = D != SUM_SAT && m0 + D < (1u << 24);
      const float sj = __uint_as_float((ex << 23) | ((m0 + D) & 0x7FFFFFu));
      const bool okj = cj < nch && fits && !(stop >= 0.0f && sj >= stop);
      const uint32_t bad = __ballot_sync(0xffffffffu, !okj);
      const uint32_t f = bad ? (uint32_t)__ffs(bad) - 1u : 32u;
      if (f > 0) s = __shfl_sync(0xffffffffu, sj, f - 1);
      c += f;
      if (f == 32) continue;
      if (c >= nch) break;
      const uint32_t cb = c * C, ce = min(n, cb + C);
      bool hit = false;
      for (uint32_t g0 = cb; g0 < ce && !hit; g0 += 256) {  // 256 terms' loads issued at once
        float t[8];
#pragma unroll
        for (int q = 0; q < 8; q++) t[q] = g0 + 32 * q + lane < ce ? v[g0 + 32 * q + lane] : 0.0f;
#pragma unroll
        for (int q = 0; q < 8; q++) {
          const uint32_t i0 = g0 + 32 * q;
          if (hit || i0 >= ce) break;
          const uint32_t cnt = min(32u, ce - i0);
          for (uint32_t j = 0; j < cnt; j++) {
            s = __fadd_rn(s, __shfl_sync(0xffffffffu, t[q], j));
            if (stop >= 0.0f && s >= stop) {
              where = i0 + j;
              hit = true;
              break;
            }
          }
        }
      }
      if (hit) break;
      c += 1;
    }
    if (lane == 0) {
      scan[64] = (double)s;
      scan[65] = (double)where;
    }
  }
  __syncthreads();
  const float s = (float)scan[64];
  if (cut) *cut = (uint32_t)scan[65];
  __syncthreads();
  return s;
}

// ----------------------------------------------------- stable radix sort ----
// Sorts (key, idx) of n entries ascending by key, stably, keys in ka/ia, using
// kb/ib as the other buffer (four passes: the result ends in ka/ia). Tiles of
// SMP_THREADS entries in order; within a tile a thread's rank among equal
// digits comes from warp matching, warps in order.
__device__ void radix_sort_stable(uint32_t* ka, uint32_t* ia, uint32_t* kb, uint32_t* ib, uint32_t n,
                                  uint32_t* wcount /* [32][256] */, uint32_t* base /* [512] */) {
  const uint32_t tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  for (int pass = 0; pass < 4; pass++) {
    const int shift = 8 * pass;
    uint32_t* sk = pass & 1 ? kb : ka;
    uint32_t* si = pass & 1 ? ib : ia;
    uint32_t* dk = pass & 1 ? ka : kb;
    uint32_t* di = pass & 1 ? ia : ib;
    for (uint32_t i = tid; i < 256; i += SMP_THREADS) base[i] = 0;
    __syncthreads();
    for (uint32_t i0 = 0; i0 < n; i0 += SMP_THREADS) {  // lanes with the same digit add once
      const uint32_t i = i0 + tid;
      const uint32_t dg = i < n ? (__ldcg(sk + i) >> shift) & 255u : 256u + lane;
      const uint32_t peers = __match_any_sync(0xffffffffu, dg);
      if (i < n && __ffs(peers) - 1 == (int)lane) atomicAdd(&base[dg], (uint32_t)__popc(peers));
    }
    __syncthreads();
    if (tid == 0) {  // exclusive prefix of the digit counts
      uint32_t run = 0;
      for (int dg = 0; dg < 256; dg++) {
        const uint32_t c = base[dg];
        base[dg] = run;
        run += c;
      }
    }
    __syncthreads();
    for (uint32_t t0 = 0; t0 < n; t0 += SMP_THREADS) {
      const uint32_t i = t0 + tid;
      const bool have = i < n;
      const uint32_t key = have ? __ldcg(sk + i) : 0u, idx = have ? __ldcg(si + i) : 0u;
      const uint32_t dg = have ? (key >> shift) & 255u : 256u + lane;  // absent entries match nobody
      for (uint32_t k = tid; k < 32 * 256; k += SMP_THREADS) wcount[k] = 0;
      __syncthreads();
      const uint32_t peers = __match_any_sync(0xffffffffu, dg);
      const uint32_t rank = __popc(peers & ((1u << lane) - 1u));
      if (have && rank == 0) wcount[warp * 256 + dg] = __popc(peers);
      __syncthreads();
      if (tid < 256) {  // per digit: exclusive prefix over the warps, and the tile's count
        uint32_t run = 0;
        for (int w = 0; w < 32; w++) {
          const uint32_t c = wcount[w * 256 + tid];
          wcount[w * 256 + tid] = run;
          run += c;
        }
        base[256 + tid] = run;
      }
      __syncthreads();
      if (have) {
        const uint32_t dst = base[dg] + wcount[warp * 256 + dg] + rank;
        dk[dst] = key;
        di[dst] = idx;
      }
      __syncthreads();
      if (tid < 256) base[tid] += base[256 + tid];
      __syncthreads();
    }
  }
}

// --------------------------------------------------------------- kernel ----
// scratch: per row sample_scratch_words(V) words: [0, V) the terms, then the
// probs keys; [V, 5V) the sort's key / index buffers.
__global__ void __launch_bounds__(SMP_THREADS) sample_kernel(const float* logits, uint32_t V, const uint8_t* mask,
                                                             const SampleParams* params, uint64_t* rng,
                                                             uint32_t* out_tok, uint32_t* next_tok, RowDesc* advance,
                                                             uint32_t* scratch, uint64_t scratch_words, uint64_t ldl,
                                                             const uint64_t* amax, uint32_t n_amax) {
  pdl_trigger();
  pdl_wait();  // the logits come from the output-head GEMV
  const uint32_t r = blockIdx.x, tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const float* lr = logits + (size_t)r * ldl;
  const uint8_t* mr = mask ? mask + (size_t)r * ldl : nullptr;
  const SampleParams P = params[r];
  __shared__ Best wb[32];
  __shared__ float red[32];
  __shared__ uint32_t hist[256];
  __shared__ uint32_t s_u[4];
  __shared__ uint32_t s_choice;
  __shared__ double scan[72];
  __shared__ double s_t32[32];
  if (tid < 32) s_t32[tid] = c_exp2_32[tid];  // read after the barriers below
  // one buffer, used in turn by: the exact sum's chunk records, the top-k
  // candidates, the radix sort's per-warp digit counts and digit bases
  __shared__ __align__(16) uint8_t big[SMP_BIG];
  SumRec* recs = reinterpret_cast<SumRec*>(big);
  unsigned long long* cand = reinterpret_cast<unsigned long long*>(big);
  auto logit = [&](uint32_t i) -> float { return (mr && !mr[i]) ? -INFINITY : lr[i]; };

  if (P.temperature <= 0.0f && amax && !mr && r == 0) {
    // greedy from the output head's per-tile candidates (argmax_key)
    unsigned long long best = 0;
    for (uint32_t i = tid; i < n_amax; i += SMP_THREADS) best = max(best, (unsigned long long)amax[i]);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) best = max(best, __shfl_xor_sync(0xffffffffu, best, o));
    __shared__ unsigned long long wk[32];
    if (lane == 0) wk[warp] = best;
    __syncthreads();
    if (warp == 0) {
      best = wk[lane];
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) best = max(best, __shfl_xor_sync(0xffffffffu, best, o));
      if (lane == 0) {
        const float l0 = lr[0];
        // x[i] > NaN is false for every i: a NaN at index 0 is the answer
        s_choice = (l0 != l0 || best == 0) ? 0u : 0xFFFFFFFFu - (uint32_t)(best & 0xFFFFFFFFu);
      }
    }
    __syncthreads();
  } else if (P.temperature <= 0.0f) {  // greedy (sampling.rs:96-98, 147-155); a NaN temperature samples
    Best b{-INFINITY, 0xFFFFFFFFu};
    for (uint32_t i = tid; i < V; i += SMP_THREADS) b = better(b, Best{logit(i), i});
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      Best c{__shfl_xor_sync(0xffffffffu, b.v, o), __shfl_xor_sync(0xffffffffu, b.i, o)};
      b = better(b, c);
    }
    if (lane == 0) wb[warp] = b;
    __syncthreads();
    if (warp == 0) {
      b = wb[lane];
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) {
        Best c{__shfl_xor_sync(0xffffffffu, b.v, o), __shfl_xor_sync(0xffffffffu, b.i, o)};
        b = better(b, c);
      }
      if (lane == 0) {
        const float l0 = logit(0);
        s_choice = (l0 != l0 || b.i == 0xFFFFFFFFu) ? 0u : b.i;  // x[i] > NaN is false for all i
      }
    }
    __syncthreads();
  } else {
    const float T = P.temperature;
    float* term = reinterpret_cast<float*>(scratch + (size_t)r * scratch_words);
    uint32_t* key = reinterpret_cast<uint32_t*>(term);
    // 1. max of p = l/T (a NaN never replaces the running max)
    float m = -INFINITY;
    for (uint32_t i0 = tid; i0 < V; i0 += 8 * SMP_THREADS) {  // eight loads in flight a thread
      float l[8];
#pragma unroll
      for (int q = 0; q < 8; q++) l[q] = i0 + q * SMP_THREADS < V ? logit(i0 + q * SMP_THREADS) : -INFINITY;
#pragma unroll
      for (int q = 0; q < 8; q++) m = fmaxf(m, __fdiv_rn(l[q], T));
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    if (lane == 0) red[warp] = m;
    __syncthreads();
    if (warp == 0) {
      float v = red[lane];
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
      if (lane == 0) red[0] = v;
    }
    __syncthreads();
    m = red[0];
    // 2. terms exp(p - max) and their exact left-to-right f32 sum
    //    (inputs that need glibc's exception table are listed and looked up
    //    after the pass by the whole CTA at once: a lookup is a chain of
    //    dependent loads that would stall its warp inside the pass)
    uint32_t* patch = reinterpret_cast<uint32_t*>(big);
    if (tid == 0) s_u[3] = 0;
    __syncthreads();
    for (uint32_t i0 = tid; i0 < V; i0 += 4 * SMP_THREADS) {
      float l[4];
#pragma unroll
      for (int q = 0; q < 4; q++) l[q] = i0 + q * SMP_THREADS < V ? logit(i0 + q * SMP_THREADS) : 0.0f;
#pragma unroll
      for (int q = 0; q < 4; q++) {
        const uint32_t i = i0 + q * SMP_THREADS;
        if (i < V) {
          const float x = __fsub_rn(__fdiv_rn(l[q], T), m);
          bool chk;
          float t = expf_ref(x, s_t32, &chk);
          if (chk) {
            const uint32_t slot = atomicAdd(&s_u[3], 1u);
            if (slot < SMP_PATCH) patch[slot] = i;
            else t = expf_lookup(x, t);  // list full: in place
          }
          term[i] = t;
        }
      }
    }
    __syncthreads();
    const uint32_t npatch = min(s_u[3], SMP_PATCH);
    for (uint32_t j = tid; j < npatch; j += SMP_THREADS) {
      const uint32_t i = patch[j];
      term[i] = expf_lookup(__fsub_rn(__fdiv_rn(logit(i), T), m), term[i]);
    }
    __syncthreads();
    const float S = exact_seq_sum(term, V, -1.0f, nullptr, recs, scan);
    // 3. probs, as order-preserving keys (in place of the terms)
    for (uint32_t i0 = tid; i0 < V; i0 += 4 * SMP_THREADS) {
      float t[4];
#pragma unroll
      for (int q = 0; q < 4; q++) t[q] = i0 + q * SMP_THREADS < V ? term[i0 + q * SMP_THREADS] : 0.0f;
#pragma unroll
      for (int q = 0; q < 4; q++)
        if (i0 + q * SMP_THREADS < V) key[i0 + q * SMP_THREADS] = fkey(__fdiv_rn(t[q], S));
    }
    __syncthreads();
    const int64_t k64 = P.top_k < 0 ? (int64_t)V : min((int64_t)V, max((int64_t)P.top_k, (int64_t)1));
    const uint32_t k = (uint32_t)k64;
    if (k <= (uint32_t)SMP_KMAX) {
      uint32_t nc = 0xFFFFFFFFu;  // candidates gathered; above SMP_KMAX: radix select
      // 4a. a threshold with at least k and at most SMP_KMAX keys at or above
      //     it, found without atomics: per-thread counts of the keys by their
      //     distance below the largest key kmax = key(1 / S) (the largest term
      //     is exp(0) = 1) in 16 bins of width 2^W (W = 23, a binade; the last
      //     bin takes everything further), refined 16-fold inside the boundary
      //     bin while too many keys remain. Those keys are then gathered.
      if (m == m && fabsf(m) != INFINITY && S > 0.0f && S < INFINITY && V <= 255u * SMP_THREADS) {
        const uint32_t kmax = fkey(__fdiv_rn(1.0f, S));
        uint32_t* wcnt = reinterpret_cast<uint32_t*>(big + SMP_KMAX * 8);  // after the candidates
        uint32_t hi = kmax, lo = 0, W = 23, above = 0;
        for (;;) {
          uint32_t pc[4] = {0u, 0u, 0u, 0u};
          for (uint32_t i0 = tid; i0 < V; i0 += 4 * SMP_THREADS) {
            uint32_t kk[4];
#pragma unroll
            for (int q = 0; q < 4; q++) kk[q] = i0 + q * SMP_THREADS < V ? key[i0 + q * SMP_THREADS] : 0u;
#pragma unroll
            for (int q = 0; q < 4; q++)
              if (i0 + q * SMP_THREADS < V && kk[q] >= lo && kk[q] <= hi) pc_add(pc, min((hi - kk[q]) >> W, 15u));
          }
          const uint32_t cnt = pc_reduce(pc, wcnt);
          if (warp == 0) {
            uint32_t cum = cnt;  // inclusive scan over the bins, nearest kmax first
#pragma unroll
            for (int o = 1; o < 32; o <<= 1) {
              const uint32_t t = __shfl_up_sync(0xffffffffu, cum, o);
              if (lane >= (uint32_t)o) cum += t;
            }
            const uint32_t hit = __ballot_sync(0xffffffffu, lane < 16 && above + cum >= k);
            const uint32_t l = hit ? (uint32_t)__ffs(hit) - 1u : 16u;
            const uint32_t cl = __shfl_sync(0xffffffffu, cum, l & 31u);
            const uint32_t cp = __shfl_sync(0xffffffffu, cum, (l - 1u) & 31u);
            if (lane == 0) {
              s_u[0] = l;
              s_u[1] = cl;
              s_u[2] = l ? cp : 0u;
            }
          }
          __syncthreads();
          const uint32_t l = s_u[0], cl = s_u[1], cp = s_u[2];
          __syncthreads();
          if (l >= 16 || (W == 23 && l == 15)) break;  // no threshold this way
          const uint32_t nhi = hi - (l << W), nlo = nhi - ((1u << W) - 1u);  // bin l: keys [nlo, nhi]
          if (above + cl <= (uint32_t)SMP_KMAX) {
            // 4b. gather every key >= nlo (warp-aggregated slots)
            if (tid == 0) s_u[3] = 0;
            __syncthreads();
            for (uint32_t i0 = 0; i0 < V; i0 += 4 * SMP_THREADS) {
              uint32_t kk[4];
#pragma unroll
              for (int q = 0; q < 4; q++) {
                const uint32_t i = i0 + q * SMP_THREADS + tid;
                kk[q] = i < V ? key[i] : 0u;
              }
#pragma unroll
              for (int q = 0; q < 4; q++) {
                const uint32_t i = i0 + q * SMP_THREADS + tid;
                const bool take = i < V && kk[q] >= nlo;
                const uint32_t bal = __ballot_sync(0xffffffffu, take);
                if (!bal) continue;
                const uint32_t lead = __ffs(bal) - 1;
                uint32_t base = 0;
                if (lane == lead) base = atomicAdd(&s_u[3], (uint32_t)__popc(bal));
                base = __shfl_sync(0xffffffffu, base, lead);
                if (take) cand[base + __popc(bal & ((1u << lane) - 1u))] = ((unsigned long long)kk[q] << 32) | (0xFFFFFFFFu - i);
              }
            }
            __syncthreads();
            nc = s_u[3];
            break;
          }
          if (W < 4) break;  // ties beyond the candidate buffer
          above += cp;
          hi = nhi;
          lo = nlo;
          W -= 4;
        }
      }
      if (nc > (uint32_t)SMP_KMAX) {
        // 4a'. otherwise the k largest keys (lowest indices among equal keys) by
        //      radix select
        uint32_t prefix = 0, need = k;
        for (int pass = 0; pass < 4; pass++) {
          const int shift = 24 - 8 * pass;
          const uint32_t hmask = pass == 0 ? 0u : (0xFFFFFFFFu << (32 - 8 * pass));
          for (uint32_t i = tid; i < 256; i += SMP_THREADS) hist[i] = 0;
          __syncthreads();
          // keys concentrate on a few bins: lanes with the same bin add once
          for (uint32_t i0 = 0; i0 < V; i0 += SMP_THREADS) {
            const uint32_t i = i0 + tid;
            const uint32_t kk = i < V ? key[i] : 0u;
            const bool in = i < V && (kk & hmask) == prefix;
            const uint32_t bin = in ? (kk >> shift) & 0xFF : 256u + lane;
            const uint32_t peers = __match_any_sync(0xffffffffu, bin);
            if (in && __ffs(peers) - 1 == (int)lane) atomicAdd(&hist[bin], (uint32_t)__popc(peers));
          }
          __syncthreads();
          if (tid == 0) {
            uint32_t acc = 0, bin = 0;
            for (int bb = 255; bb >= 0; bb--) {
              if (acc + hist[bb] >= need) { bin = (uint32_t)bb; break; }
              acc += hist[bb];
            }
            s_u[0] = prefix | (bin << shift);
            s_u[1] = need - acc;
          }
          __syncthreads();
          prefix = s_u[0];
          need = s_u[1];
          __syncthreads();
        }
        // every key > prefix, and the first `need` keys == prefix in index order
        const uint32_t per = (V + SMP_THREADS - 1) / SMP_THREADS;
        const uint32_t i0 = min(V, tid * per), i1 = min(V, i0 + per);
        uint32_t eq = 0;
        for (uint32_t i = i0; i < i1; i++) eq += key[i] == prefix;
        uint32_t incl = eq;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
          const uint32_t t = __shfl_up_sync(0xffffffffu, incl, o);
          if (lane >= (uint32_t)o) incl += t;
        }
        __shared__ uint32_t wsum[32];
        if (lane == 31) wsum[warp] = incl;
        if (tid == 0) s_u[2] = 0;
        __syncthreads();
        if (warp == 0) {
          uint32_t v = wsum[lane], iv = v;
#pragma unroll
          for (int o = 1; o < 32; o <<= 1) {
            const uint32_t t = __shfl_up_sync(0xffffffffu, iv, o);
            if (lane >= (uint32_t)o) iv += t;
          }
          wsum[lane] = iv - v;
        }
        __syncthreads();
        uint32_t rank = wsum[warp] + incl - eq;
        for (uint32_t i = i0; i < i1; i++) {
          const uint32_t kk = key[i];
          bool take = kk > prefix;
          if (kk == prefix) { take = rank < need; rank++; }
          if (take) {
            const uint32_t slot = atomicAdd(&s_u[2], 1u);
            if (slot < SMP_KMAX) cand[slot] = ((unsigned long long)kk << 32) | (0xFFFFFFFFu - i);
          }
        }
        __syncthreads();
        nc = min(s_u[2], (uint32_t)SMP_KMAX);
      }
      // bitonic sort of the candidates (padded to a power of two), descending
      // (key desc, index asc): the first k are the reference's sorted top-k
      uint32_t np2 = 1;
      while (np2 < nc) np2 <<= 1;
      for (uint32_t i = nc + tid; i < np2; i += SMP_THREADS) cand[i] = 0ull;
      __syncthreads();
      for (uint32_t size = 2; size <= np2; size <<= 1)
        for (uint32_t stride = size >> 1; stride > 0; stride >>= 1) {
          for (uint32_t i = tid; i < np2; i += SMP_THREADS) {
            const uint32_t j = i ^ stride;
            if (j > i) {
              const bool desc = (i & size) == 0;
              const unsigned long long a = cand[i], bb = cand[j];
              if (desc ? (a < bb) : (a > bb)) { cand[i] = bb; cand[j] = a; }
            }
          }
          __syncthreads();
        }
      // 5-6. top-p, total, multinomial walk (one thread, the reference's order)
      if (tid == 0) {
        uint64_t st = rng[r];
        uint32_t kept = k;
        auto prob = [&](uint32_t c) -> float { return fkey_inv((uint32_t)(cand[c] >> 32)); };
        auto index = [&](uint32_t c) -> uint32_t { return 0xFFFFFFFFu - (uint32_t)(cand[c] & 0xFFFFFFFFu); };
        if (P.top_p >= 0.0f) {
          float cum = 0.f;
          uint32_t cut = kept;
          for (uint32_t c = 0; c < kept; c++) {
            cum = __fadd_rn(cum, prob(c));
            if (cum >= P.top_p) { cut = c + 1; break; }
          }
          kept = max(cut, 1u);
        }
        float total = 0.f;
        for (uint32_t c = 0; c < kept; c++) total = __fadd_rn(total, prob(c));
        float rv = __fmul_rn(rng_f32(st), total);
        uint32_t choice = index(kept - 1);
        for (uint32_t c = 0; c < kept; c++) {
          rv = __fsub_rn(rv, prob(c));
          if (rv <= 0.0f) { choice = index(c); break; }
        }
        rng[r] = st;
        s_choice = choice;
      }
      __syncthreads();
    } else {
      // 4b. the whole vocabulary sorted (probs desc, index asc): ascending ~key, stable
      uint32_t* ka = key + V;
      uint32_t* ia = ka + V;
      uint32_t* kb = ia + V;
      uint32_t* ib = kb + V;
      for (uint32_t i = tid; i < V; i += SMP_THREADS) {
        ka[i] = ~key[i];
        ia[i] = i;
      }
      __syncthreads();
      radix_sort_stable(ka, ia, kb, ib, V, reinterpret_cast<uint32_t*>(big),
                        reinterpret_cast<uint32_t*>(big) + SMP_SORT_COUNTS);
      // sorted probs, in place of the keys
      float* sp = reinterpret_cast<float*>(kb);
      for (uint32_t i = tid; i < V; i += SMP_THREADS) sp[i] = fkey_inv(~ka[i]);
      __syncthreads();
      uint32_t kept = k;
      if (P.top_p >= 0.0f) {  // first position where the cumulative sum reaches top_p
        uint32_t cut = V;
        exact_seq_sum(sp, kept, P.top_p, &cut, recs, scan);
        kept = cut < kept ? cut + 1 : kept;
        kept = max(kept, 1u);
      }
      const float total = exact_seq_sum(sp, kept, -1.0f, nullptr, recs, scan);
      if (tid == 0) {
        uint64_t st = rng[r];
        float rv = __fmul_rn(rng_f32(st), total);
        uint32_t at = kept - 1;
        for (uint32_t c = 0; c < kept; c += 8) {  // terms fetched 8 at a time, subtracted in order
          float t[8];
#pragma unroll
          for (int q = 0; q < 8; q++) t[q] = c + q < kept ? __ldcg(sp + c + q) : 0.0f;
          bool hit = false;
#pragma unroll
          for (int q = 0; q < 8; q++) {
            if (hit || c + q >= kept) continue;
            rv = __fsub_rn(rv, t[q]);
            if (rv <= 0.0f) { at = c + q; hit = true; }
          }
          if (hit) break;
        }
        rng[r] = st;
        s_choice = __ldcg(ia + at);
      }
      __syncthreads();
    }
  }
  if (tid == 0) {
    out_tok[r] = s_choice;
    if (next_tok) next_tok[r] = s_choice;
    if (advance) advance[r].pos += 1;
  }
}

// softmax (sampling.rs:157-172) of rows of n values, one CTA per row: the
// reference's probs bit for bit (max, glibc exp, left-to-right f32 sum, IEEE
// division). out may alias nothing else; it holds the terms before the probs.
__global__ void __launch_bounds__(SMP_THREADS) softmax_kernel(const float* x, uint32_t n, float* out) {
  const uint32_t r = blockIdx.x, tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const float* xr = x + (size_t)r * n;
  float* o = out + (size_t)r * n;
  __shared__ float red[32];
  __shared__ double scan[72];
  __shared__ double s_t32[32];
  if (tid < 32) s_t32[tid] = c_exp2_32[tid];  // read after the max's barriers
  __shared__ __align__(16) uint8_t big[SMP_BIG];
  SumRec* recs = reinterpret_cast<SumRec*>(big);
  float m = -INFINITY;
  for (uint32_t i = tid; i < n; i += SMP_THREADS) m = fmaxf(m, xr[i]);
#pragma unroll
  for (int of = 16; of > 0; of >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, of));
  if (lane == 0) red[warp] = m;
  __syncthreads();
  if (warp == 0) {
    float v = red[lane];
#pragma unroll
    for (int of = 16; of > 0; of >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, of));
    if (lane == 0) red[0] = v;
  }
  __syncthreads();
  m = red[0];
  for (uint32_t i = tid; i < n; i += SMP_THREADS) o[i] = expf_ref(__fsub_rn(xr[i], m), s_t32);
  __syncthreads();
  const float S = exact_seq_sum(o, n, -1.0f, nullptr, recs, scan);
  for (uint32_t i = tid; i < n; i += SMP_THREADS) o[i] = __fdiv_rn(o[i], S);
}

cudaError_t launch_softmax(const float* x, uint32_t rows, uint32_t n, float* out, cudaStream_t st) {
  if (!rows || !n) return cudaSuccess;
  softmax_kernel<<<rows, SMP_THREADS, 0, st>>>(x, n, out);
  return cudaGetLastError();
}

uint64_t sample_scratch_words(uint32_t V) { return 5ull * V + 64; }

cudaError_t launch_sample(const float* logits, uint32_t V, uint32_t rows, const uint8_t* mask,
                          const SampleParams* params, uint64_t* rng, uint32_t* out_tok, uint32_t* next_tok,
                          RowDesc* advance, uint32_t* scratch, cudaStream_t st, uint64_t ldl, const uint64_t* amax,
                          uint32_t n_amax) {
  if (!rows) return cudaSuccess;
  return launch_pdl(sample_kernel, dim3(rows), dim3(SMP_THREADS), 0, st, logits, V, mask, params, rng, out_tok,
                    next_tok, advance, scratch, sample_scratch_words(V), ldl == ~0ull ? (uint64_t)V : ldl, amax,
                    n_amax);
}

cudaError_t launch_expf_ref(const float* x, float* y, size_t n, cudaStream_t st) {
  if (!n) return cudaSuccess;
  expf_ref_kernel<<<(unsigned)std::min<size_t>((n + 255) / 256, 148 * 64), 256, 0, st>>>(x, y, n);
  return cudaGetLastError();
}

}  // namespace sm
