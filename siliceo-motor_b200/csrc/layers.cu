// Per-layer kernels of the decode step: RMSNorm, bias+RoPE+KV append, split-K
// GQA attention, SwiGLU, and the on-device sampler.
#include <cfloat>

#include "device.cuh"
#include "layers.cuh"
#include "pdl.cuh"

namespace sm {

// ------------------------------------------------------------- RMSNorm ----
// out = x * (1/sqrt(sum(x^2)/n + eps)) * w  (qwen2.rs:647-660, 748-756).
// rows: optional row selection (row r of out reads row rows[r] of x).
__global__ void rmsnorm_kernel(const float* x, uint32_t ldx, const uint32_t* sel, const float* w, float* out,
                               uint32_t ldo, uint32_t n, float eps) {
  const uint32_t r = blockIdx.x;
  const float* xr = x + (size_t)(sel ? sel[r] : r) * ldx;
  float ss = 0.f;
  for (uint32_t i = threadIdx.x; i < n; i += blockDim.x) ss += xr[i] * xr[i];
  __shared__ float red[32];
  ss = warp_sum(ss);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
  __syncthreads();
  if (threadIdx.x < 32) {
    float v = threadIdx.x < (blockDim.x >> 5) ? red[threadIdx.x] : 0.f;
    v = warp_sum(v);
    if (threadIdx.x == 0) red[0] = v;
  }
  __syncthreads();
  const float inv = 1.0f / sqrtf(red[0] / (float)n + eps);
  for (uint32_t i = threadIdx.x; i < n; i += blockDim.x)
    out[(size_t)r * ldo + i] = __fmul_rn(__fmul_rn(xr[i], inv), w[i]);
}

// ------------------------------------------------------------ attention ----
// Split-K decode attention with GQA (qwen2.rs:502-533). CTA (row r, kv head
// g, split sp) covers a run of 32-position tiles of the row's context
// [0, pos]; the G = Hq/Hkv query heads of the group share each K/V tile.
// Both tiles of a step are staged with cp.async at once (V arrives while the
// scores are computed); rows are padded to hd+4 floats so that the float4
// shared-memory reads of 8 lanes hit distinct banks. Online softmax inside
// the CTA; splits are merged by attn_combine_kernel. A tile is one KV page.
constexpr int ATT_T = 32;     // positions per tile
static_assert(ATT_T == (int)KV_PAGE, "an attention tile is one KV page");
constexpr int ATT_THREADS = 128;

__device__ __forceinline__ void cp_async16(void* smem, const void* gmem) {
  const uint32_t s = (uint32_t)__cvta_generic_to_shared(smem);
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(s), "l"(gmem));
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() { asm volatile("cp.async.wait_group %0;" ::"n"(N)); }

__global__ void __launch_bounds__(ATT_THREADS) attn_split_kernel(const float* q, uint32_t ldq, const RowDesc* rows,
                                                                 const SeqDesc* seqs, uint32_t layer, uint32_t Hq,
                                                                 uint32_t Hkv, uint32_t hd, float scale, float* part_o,
                                                                 float* part_ml, uint32_t max_splits) {
  extern __shared__ __align__(16) float smem[];
  pdl_trigger();
  const uint32_t r = blockIdx.x / Hkv, g = blockIdx.x - r * Hkv, sp = blockIdx.y;
  const RowDesc rd = rows[r];
  const uint32_t L = rd.pos + 1;
  const uint32_t tiles = (L + ATT_T - 1) / ATT_T;
  const uint32_t tps = (tiles + max_splits - 1) / max_splits;
  const uint32_t tb = sp * tps;
  if (tb >= tiles) return;
  const uint32_t te = min(tiles, tb + tps);
  const uint32_t G = Hq / Hkv, kvd = Hkv * hd, hs = hd + 4, hd4 = hd / 4;
  const SeqDesc sd = seqs[rd.seq];
  {  // positions before rd.pos were written by earlier steps: start them towards L2
    const uint32_t p_end = min(te * ATT_T, rd.pos), lines = (hd * 4 + 127) / 128;
    const uint32_t nrow = p_end > tb * ATT_T ? p_end - tb * ATT_T : 0;
    for (uint32_t i = threadIdx.x; i < nrow * lines; i += blockDim.x) {
      const uint32_t pos = tb * ATT_T + i / lines;
      const float* kp = sd.pages[pos / KV_PAGE] + kv_page_off(layer, pos, kvd) + (size_t)g * hd + (i % lines) * 32;
      asm volatile("prefetch.global.L2 [%0];" ::"l"(kp));
      asm volatile("prefetch.global.L2 [%0];" ::"l"(kp + sd.voff));
    }
  }
  pdl_wait();  // q and this position's K / V come from the QKV GEMV
  float* qs = smem;                  // [G][hd]
  float* kt = qs + G * hd;           // [ATT_T][hd+4]
  float* vt = kt + ATT_T * hs;       // [ATT_T][hd+4]
  float* ps = vt + ATT_T * hs;       // [G][ATT_T]
  float* mrun = ps + G * ATT_T;      // [G] running max
  float* lrun = mrun + G;            // [G] running sum
  float* alpha = lrun + G;           // [G] rescale of this tile
  const float* qr = q + (size_t)r * ldq + (size_t)g * G * hd;
  for (uint32_t i = threadIdx.x; i < G * hd4; i += blockDim.x)
    reinterpret_cast<float4*>(qs)[i] = reinterpret_cast<const float4*>(qr)[i];
  if (threadIdx.x < G) { mrun[threadIdx.x] = -INFINITY; lrun[threadIdx.x] = 0.f; }
  constexpr int MAXO = 2;  // (G*hd/4) / ATT_THREADS <= 2 (G <= 8, hd <= 128)
  float4 o[MAXO];
#pragma unroll
  for (int i = 0; i < MAXO; i++) o[i] = make_float4(0.f, 0.f, 0.f, 0.f);
  const uint32_t warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  for (uint32_t t = tb; t < te; t++) {
    const uint32_t p0 = t * ATT_T, n = min((uint32_t)ATT_T, L - p0);
    // page t: rows (layer, p0 + pp) of K at kb + pp * kvd, of V voff floats further
    const float* kb = sd.pages[t] + (size_t)layer * KV_PAGE * kvd + (size_t)g * hd;
    __syncthreads();  // previous tile fully consumed
    for (uint32_t i = threadIdx.x; i < n * hd4; i += blockDim.x) {
      const uint32_t pp = i / hd4, d4 = i - pp * hd4;
      cp_async16(kt + pp * hs + 4 * d4, kb + (size_t)pp * kvd + 4 * d4);
    }
    cp_async_commit();
    for (uint32_t i = threadIdx.x; i < n * hd4; i += blockDim.x) {
      const uint32_t pp = i / hd4, d4 = i - pp * hd4;
      cp_async16(vt + pp * hs + 4 * d4, kb + sd.voff + (size_t)pp * kvd + 4 * d4);
    }
    cp_async_commit();
    cp_async_wait<1>();  // K landed
    __syncthreads();
    // scores: (head j, position pp) pairs
    for (uint32_t i = threadIdx.x; i < G * ATT_T; i += blockDim.x) {
      const uint32_t j = i / ATT_T, pp = i - j * ATT_T;
      float sc = -INFINITY;
      if (pp < n) {
        const float4* qj = reinterpret_cast<const float4*>(qs + j * hd);
        const float4* kr = reinterpret_cast<const float4*>(kt + pp * hs);
        float a0 = 0.f, a1 = 0.f;
        for (uint32_t d = 0; d < hd4; d++) {
          const float4 qa = qj[d], ka = kr[d];
          a0 = fmaf(qa.x, ka.x, a0);
          a1 = fmaf(qa.y, ka.y, a1);
          a0 = fmaf(qa.z, ka.z, a0);
          a1 = fmaf(qa.w, ka.w, a1);
        }
        sc = (a0 + a1) * scale;
      }
      ps[i] = sc;
    }
    __syncthreads();
    for (uint32_t j = warp; j < G; j += ATT_THREADS / 32) {
      const float s0 = ps[j * ATT_T + lane];
      float m = s0;
#pragma unroll
      for (int of = 16; of > 0; of >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, of));
      const float mold = mrun[j], mnew = fmaxf(mold, m);
      const float e0 = expf(s0 - mnew);
      ps[j * ATT_T + lane] = e0;
      const float sum = warp_sum(e0);
      if (lane == 0) {
        const float a = expf(mold - mnew);  // 0 on the first tile (mold = -inf)
        alpha[j] = a;
        lrun[j] = lrun[j] * a + sum;
        mrun[j] = mnew;
      }
    }
    cp_async_wait<0>();  // V landed
    __syncthreads();
#pragma unroll
    for (int k = 0; k < MAXO; k++) {
      const uint32_t i = threadIdx.x + k * ATT_THREADS;
      if (i < G * hd4) {
        const uint32_t j = i / hd4, d4 = i - j * hd4;
        const float* pj = ps + j * ATT_T;
        const float a = alpha[j];
        float4 acc = make_float4(o[k].x * a, o[k].y * a, o[k].z * a, o[k].w * a);
        for (uint32_t pp = 0; pp < n; pp++) {
          const float p = pj[pp];
          const float4 v = reinterpret_cast<const float4*>(vt + pp * hs)[d4];
          acc.x = fmaf(p, v.x, acc.x);
          acc.y = fmaf(p, v.y, acc.y);
          acc.z = fmaf(p, v.z, acc.z);
          acc.w = fmaf(p, v.w, acc.w);
        }
        o[k] = acc;
      }
    }
  }
  __syncthreads();
#pragma unroll
  for (int k = 0; k < MAXO; k++) {
    const uint32_t i = threadIdx.x + k * ATT_THREADS;
    if (i < G * hd4) {
      const uint32_t j = i / hd4, d4 = i - j * hd4, h = g * G + j;
      reinterpret_cast<float4*>(part_o + (((size_t)r * Hq + h) * max_splits + sp) * hd)[d4] = o[k];
    }
  }
  if (threadIdx.x < G) {
    const uint32_t h = g * G + threadIdx.x;
    float* ml = part_ml + (((size_t)r * Hq + h) * max_splits + sp) * 2;
    ml[0] = mrun[threadIdx.x];
    ml[1] = lrun[threadIdx.x];
  }
}

// Merges the splits of (row r, head h): out = sum_s o_s e_s / sum_s l_s e_s with
// e_s = exp(m_s - max m), sums in split order. The (m, l) pairs are staged in
// shared memory by one parallel load; the partial outputs are read eight
// splits at a time.
__global__ void attn_combine_kernel(const float* part_o, const float* part_ml, const RowDesc* rows, uint32_t Hq,
                                    uint32_t hd, uint32_t max_splits, float* out, uint32_t ldo) {
  __shared__ float sm_m[64], sm_e[64];
  pdl_trigger();
  const uint32_t r = blockIdx.x / Hq, h = blockIdx.x - r * Hq;
  const uint32_t L = rows[r].pos + 1;  // rows are set before the step's first kernel
  const uint32_t tiles = (L + ATT_T - 1) / ATT_T;
  const uint32_t tps = (tiles + max_splits - 1) / max_splits;
  const uint32_t ns = (tiles + tps - 1) / tps;  // <= max_splits <= 64
  pdl_wait();  // the partials come from attn_split_kernel
  const float* ml = part_ml + ((size_t)r * Hq + h) * max_splits * 2;
  for (uint32_t s = threadIdx.x; s < ns; s += blockDim.x) {
    sm_m[s] = ml[2 * s];
    sm_e[s] = ml[2 * s + 1];
  }
  __syncthreads();
  float M = -INFINITY;
  for (uint32_t s = 0; s < ns; s++) M = fmaxf(M, sm_m[s]);
  float den = 0.f;
  for (uint32_t s = 0; s < ns; s++) den += sm_e[s] * expf(sm_m[s] - M);
  __syncthreads();
  for (uint32_t s = threadIdx.x; s < ns; s += blockDim.x) sm_e[s] = expf(sm_m[s] - M);
  __syncthreads();
  const float* po = part_o + ((size_t)r * Hq + h) * max_splits * hd;
  for (uint32_t d = threadIdx.x; d < hd; d += blockDim.x) {
    float acc = 0.f;
    uint32_t s = 0;
    for (; s + 8 <= ns; s += 8) {
      float v[8];
#pragma unroll
      for (int u = 0; u < 8; u++) v[u] = po[(size_t)(s + u) * hd + d];
#pragma unroll
      for (int u = 0; u < 8; u++) acc = fmaf(v[u], sm_e[s + u], acc);
    }
    float v[8];
#pragma unroll
    for (int u = 0; u < 8; u++)
      if (s + u < ns) v[u] = po[(size_t)(s + u) * hd + d];
#pragma unroll
    for (int u = 0; u < 8; u++)
      if (s + u < ns) acc = fmaf(v[u], sm_e[s + u], acc);
    out[(size_t)r * ldo + h * hd + d] = acc / den;
  }
}

// -------------------------------------------------------------- SwiGLU ----
// gate = silu(gate) * up, silu(x) = x / (1 + exp(-x)) (qwen2.rs:743-745, 546-548).
__global__ void silu_mul_kernel(float* gate, const float* up, uint32_t F, size_t n) {
  for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x) {
    const float gv = gate[i];
    const uint32_t r = (uint32_t)(i / F), e = (uint32_t)(i - (size_t)r * F);
    gate[(size_t)r * F + e] = __fmul_rn(__fdiv_rn(gv, __fadd_rn(1.0f, expf(-gv))), up[i]);
  }
}

// ------------------------------------------------------------- sampler ----
// Sampler::sample (sampling.rs:94-144) per row, one CTA of 1024 threads.
// Greedy: first index of the maximum. Otherwise: p = l/T; softmax over the
// vocabulary; candidates = the top_k largest p (ties: lower index first);
// top-p cut over their sorted cumulative sum (crossing token kept); then
// r = next_f32() * sum(kept) and the sorted walk subtracts until r <= 0.
// Sums over the kept candidates run in the reference's sequential order; the
// softmax denominator is a tree sum over the vocabulary.
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
__device__ __forceinline__ uint32_t fkey(float f) {  // order-preserving (larger f -> larger key)
  uint32_t u = __float_as_uint(f);
  return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}

struct Best {
  float v;
  uint32_t i;
};
__device__ __forceinline__ Best better(Best a, Best b) {  // larger value, then lower index
  if (b.v > a.v || (b.v == a.v && b.i < a.i)) return b;
  return a;
}

__global__ void __launch_bounds__(SMP_THREADS) sample_kernel(const float* logits, uint32_t V, const uint8_t* mask,
                                                             const SampleParams* params, uint64_t* rng,
                                                             uint32_t* out_tok, uint32_t* next_tok, RowDesc* advance) {
  pdl_trigger();
  pdl_wait();  // the logits come from the output-head GEMV
  const uint32_t r = blockIdx.x, tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const float* lr = logits + (size_t)r * V;
  const uint8_t* mr = mask ? mask + (size_t)r * V : nullptr;
  const SampleParams P = params[r];
  __shared__ Best wb[32];
  __shared__ float red[32];
  __shared__ uint32_t hist[256];
  __shared__ uint32_t s_u[4];
  __shared__ unsigned long long cand[SMP_KMAX];
  __shared__ uint32_t s_choice;
  auto logit = [&](uint32_t i) -> float { return (mr && !mr[i]) ? -INFINITY : lr[i]; };

  if (!(P.temperature > 0.0f)) {  // greedy (sampling.rs:96-98, 147-155)
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
      if (lane == 0) s_choice = b.i == 0xFFFFFFFFu ? 0u : b.i;  // all -inf/NaN: index 0 like the reference
    }
    __syncthreads();
  } else {
    const float T = P.temperature;
    // 1. max of p = l/T
    float m = -INFINITY;
    for (uint32_t i = tid; i < V; i += SMP_THREADS) m = fmaxf(m, __fdiv_rn(logit(i), T));
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
    __syncthreads();
    // 2. softmax denominator
    float s = 0.f;
    for (uint32_t i = tid; i < V; i += SMP_THREADS) s += expf(__fdiv_rn(logit(i), T) - m);
    s = warp_sum(s);
    if (lane == 0) red[warp] = s;
    __syncthreads();
    if (warp == 0) {
      float v = red[lane];
      v = warp_sum(v);
      if (lane == 0) red[0] = v;
    }
    __syncthreads();
    const float S = red[0];
    // 3. k = min(top_k, V) candidates by radix select on the p keys (top_k is
    //    clamped to SMP_KMAX by the host).
    const uint32_t k = (uint32_t)min((int64_t)V, (int64_t)max(P.top_k, 1));
    uint32_t prefix = 0, need = k;  // select keys with the high bits = prefix
    for (int pass = 0; pass < 4; pass++) {
      const int shift = 24 - 8 * pass;
      const uint32_t hmask = pass == 0 ? 0u : (0xFFFFFFFFu << (32 - 8 * pass));
      for (uint32_t i = tid; i < 256; i += SMP_THREADS) hist[i] = 0;
      __syncthreads();
      for (uint32_t i = tid; i < V; i += SMP_THREADS) {
        const uint32_t key = fkey(__fdiv_rn(logit(i), T));
        if ((key & hmask) == prefix) atomicAdd(&hist[(key >> shift) & 0xFF], 1u);
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
    // prefix = key of the k-th largest; take every key > prefix and the first
    // `need` keys == prefix in index order (contiguous index ranges per thread).
    const uint32_t per = (V + SMP_THREADS - 1) / SMP_THREADS;
    const uint32_t i0 = min(V, tid * per), i1 = min(V, i0 + per);
    uint32_t eq = 0;
    for (uint32_t i = i0; i < i1; i++) eq += fkey(__fdiv_rn(logit(i), T)) == prefix;
    // exclusive scan of eq over threads
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
      const uint32_t key = fkey(__fdiv_rn(logit(i), T));
      bool take = key > prefix;
      if (key == prefix) { take = rank < need; rank++; }
      if (take) {
        const uint32_t slot = atomicAdd(&s_u[2], 1u);
        if (slot < SMP_KMAX) cand[slot] = ((unsigned long long)key << 32) | (0xFFFFFFFFu - i);
      }
    }
    __syncthreads();
    const uint32_t nc = min(s_u[2], (uint32_t)SMP_KMAX);
    // 4. bitonic sort, descending (key desc, index asc)
    for (uint32_t i = nc + tid; i < SMP_KMAX; i += SMP_THREADS) cand[i] = 0ull;
    __syncthreads();
    for (uint32_t size = 2; size <= SMP_KMAX; size <<= 1)
      for (uint32_t stride = size >> 1; stride > 0; stride >>= 1) {
        for (uint32_t i = tid; i < SMP_KMAX; i += SMP_THREADS) {
          const uint32_t j = i ^ stride;
          if (j > i) {
            const bool desc = (i & size) == 0;
            const unsigned long long a = cand[i], b = cand[j];
            if (desc ? (a < b) : (a > b)) { cand[i] = b; cand[j] = a; }
          }
        }
        __syncthreads();
      }
    // 5-6. top-p, total, multinomial walk (single thread, reference order)
    if (tid == 0) {
      uint64_t st = rng[r];
      uint32_t kept = nc;
      auto prob = [&](uint32_t c) -> float {
        const uint32_t idx = 0xFFFFFFFFu - (uint32_t)(cand[c] & 0xFFFFFFFFu);
        return __fdiv_rn(expf(__fdiv_rn(logit(idx), T) - m), S);
      };
      if (P.top_p >= 0.0f) {
        float cum = 0.f;
        uint32_t cut = kept;
        for (uint32_t c = 0; c < kept; c++) {
          cum += prob(c);
          if (cum >= P.top_p) { cut = c + 1; break; }
        }
        kept = max(cut, 1u);
      }
      float total = 0.f;
      for (uint32_t c = 0; c < kept; c++) total += prob(c);
      float rv = rng_f32(st) * total;
      uint32_t choice = 0xFFFFFFFFu - (uint32_t)(cand[kept - 1] & 0xFFFFFFFFu);
      for (uint32_t c = 0; c < kept; c++) {
        rv -= prob(c);
        if (rv <= 0.0f) { choice = 0xFFFFFFFFu - (uint32_t)(cand[c] & 0xFFFFFFFFu); break; }
      }
      rng[r] = st;
      s_choice = choice;
    }
    __syncthreads();
  }
  if (tid == 0) {
    out_tok[r] = s_choice;
    if (next_tok) next_tok[r] = s_choice;
    if (advance) advance[r].pos += 1;
  }
}

// Appends this step's tokens to a device history: hist[(*ctr) * rows + r].
__global__ void record_tokens_kernel(const uint32_t* tok, uint32_t rows, uint32_t* hist, uint32_t* ctr,
                                     uint32_t cap_steps) {
  const uint32_t step = *ctr;
  if (step < cap_steps)
    for (uint32_t r = threadIdx.x; r < rows; r += blockDim.x) hist[(size_t)step * rows + r] = tok[r];
  __syncthreads();
  if (threadIdx.x == 0) *ctr = step + 1;
}

// --------------------------------------------------------------- launch ----
cudaError_t launch_rmsnorm(const float* x, uint32_t ldx, const uint32_t* sel, const float* w, float* out, uint32_t ldo,
                           uint32_t rows, uint32_t n, float eps, cudaStream_t st) {
  if (!rows) return cudaSuccess;
  rmsnorm_kernel<<<rows, n >= 4096 ? 1024 : 512, 0, st>>>(x, ldx, sel, w, out, ldo, n, eps);
  return cudaGetLastError();
}

size_t attn_smem_bytes(uint32_t G, uint32_t hd) {
  return sizeof(float) * ((size_t)G * hd + 2 * (size_t)ATT_T * (hd + 4) + (size_t)G * ATT_T + 3 * G);
}

cudaError_t launch_attention(const float* q, uint32_t ldq, const RowDesc* rows, const SeqDesc* seqs, uint32_t nrows,
                             uint32_t layer, uint32_t Hq, uint32_t Hkv, uint32_t hd, float* part_o, float* part_ml,
                             uint32_t max_splits, float* out, uint32_t ldo, cudaStream_t st) {
  if (!nrows) return cudaSuccess;
  const uint32_t G = Hq / Hkv;
  const size_t sm = attn_smem_bytes(G, hd);
  const float scale = 1.0f / sqrtf((float)hd);  // qwen2.rs:505
  cudaError_t e = launch_pdl(attn_split_kernel, dim3(nrows * Hkv, max_splits), dim3(ATT_THREADS), sm, st, q, ldq,
                             rows, seqs, layer, Hq, Hkv, hd, scale, part_o, part_ml, max_splits);
  if (e != cudaSuccess) return e;
  return launch_pdl(attn_combine_kernel, dim3(nrows * Hq), dim3(hd), 0, st, part_o, part_ml, rows, Hq, hd, max_splits,
                    out, ldo);
}

cudaError_t launch_silu_mul(float* gate, const float* up, uint32_t F, size_t n, cudaStream_t st) {
  if (!n) return cudaSuccess;
  const unsigned blocks = (unsigned)std::min<size_t>((n + 255) / 256, 148 * 16);
  silu_mul_kernel<<<blocks, 256, 0, st>>>(gate, up, F, n);
  return cudaGetLastError();
}

cudaError_t launch_sample(const float* logits, uint32_t V, uint32_t rows, const uint8_t* mask,
                          const SampleParams* params, uint64_t* rng, uint32_t* out_tok, uint32_t* next_tok,
                          RowDesc* advance, cudaStream_t st) {
  if (!rows) return cudaSuccess;
  return launch_pdl(sample_kernel, dim3(rows), dim3(SMP_THREADS), 0, st, logits, V, mask, params, rng, out_tok, next_tok,
                    advance);
}

cudaError_t launch_record_tokens(const uint32_t* tok, uint32_t rows, uint32_t* hist, uint32_t* ctr,
                                 uint32_t cap_steps, cudaStream_t st) {
  record_tokens_kernel<<<1, 128, 0, st>>>(tok, rows, hist, ctr, cap_steps);
  return cudaGetLastError();
}

}  // namespace sm
