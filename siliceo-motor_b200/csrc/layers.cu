// Per-layer kernels of the decode step: RMSNorm, bias+RoPE+KV append, split-K
// GQA attention, SwiGLU (the on-device sampler is in sampler.cu).
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
// K and V of a tile are staged with cp.async (rows padded to hd+4 floats so
// that the float4 shared-memory reads of 8 lanes hit distinct banks); the
// first tile's rows of earlier positions are copied before the kernel waits
// for the QKV GEMV (programmatic dependent launch), so only q and the newest
// row are fetched after it. Online softmax inside the CTA; splits are merged
// by attn_combine_kernel. A tile is one KV page.
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
                                                                 float* part_ml, uint32_t max_splits,
                                                                 uint32_t one_seq, const uint32_t* shared_tiles) {
  extern __shared__ __align__(16) float smem[];
  pdl_trigger();
  const uint32_t r = blockIdx.x / Hkv, g = blockIdx.x - r * Hkv, sp = blockIdx.y;
  const RowDesc rd = rows[r];
  const uint32_t L = rd.pos + 1;
  const uint32_t tiles = (L + ATT_T - 1) / ATT_T;
  // tiles below ts are read once for all rows by attn_shared_kernel
  const uint32_t ts = shared_tiles ? min(*shared_tiles, tiles) : 0u;
  const uint32_t tps = (tiles - ts + gridDim.y - 1) / gridDim.y;
  const uint32_t tb = ts + sp * tps;
  if (tb >= tiles) return;
  const uint32_t slot = ATT_SHARED_SPLITS + sp;
  const uint32_t te = min(tiles, tb + tps);
  const uint32_t G = Hq / Hkv, kvd = Hkv * hd, hs = hd + 4, hd4 = hd / 4;
  const SeqDesc sd = seqs[rd.seq];
  float* qs = smem;                  // [G][hd]
  float* kt = qs + G * hd;           // [ATT_T][hd+4]
  float* vt = kt + ATT_T * hs;       // [ATT_T][hd+4]
  float* ps = vt + ATT_T * hs;       // [G][ATT_T]
  float* mrun = ps + G * ATT_T;      // [G] running max
  float* lrun = mrun + G;            // [G] running sum
  float* alpha = lrun + G;           // [G] rescale of this tile
  // Positions below `fresh` were written before this launch's QKV GEMV: the
  // row's own position, or with one_seq (the rows are consecutive positions
  // of one sequence: a prefill chunk) the first row's.
  const uint32_t fresh = one_seq ? rows[0].pos : rd.pos;
  // K and V rows [lo, hi) of tile t (positions, clipped to the tile) into
  // shared memory.
  auto stage = [&](uint32_t t, uint32_t lo, uint32_t hi) {
    const uint32_t p0 = t * ATT_T, n = min((uint32_t)ATT_T, L - p0);
    const uint32_t a = min(max(lo, p0), p0 + n) - p0, b = min(max(hi, p0), p0 + n) - p0;  // rows [a, b) of the tile
    const float* kb = sd.pages[t] + (size_t)layer * KV_PAGE * kvd + (size_t)g * hd;
    for (uint32_t i = threadIdx.x + a * hd4; i < b * hd4; i += blockDim.x) {
      const uint32_t pp = i / hd4, d4 = i - pp * hd4;
      cp_async16(kt + pp * hs + 4 * d4, kb + (size_t)pp * kvd + 4 * d4);
      cp_async16(vt + pp * hs + 4 * d4, kb + sd.voff + (size_t)pp * kvd + 4 * d4);
    }
    cp_async_commit();
  };
  // The first tile's rows of earlier positions were written by earlier
  // launches: start copying them before waiting for the QKV GEMV.
  stage(tb, 0, fresh);
  pdl_wait();  // q and the K / V rows from `fresh` on come from the QKV GEMV
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
    if (t == tb) {
      stage(t, fresh, L);  // the rows this launch's QKV GEMV wrote (if in this tile)
    } else {
      __syncthreads();  // previous tile fully consumed
      stage(t, 0, L);
    }
    cp_async_wait<0>();
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
      reinterpret_cast<float4*>(part_o + (((size_t)r * Hq + h) * max_splits + slot) * hd)[d4] = o[k];
    }
  }
  if (threadIdx.x < G) {
    const uint32_t h = g * G + threadIdx.x;
    float* ml = part_ml + (((size_t)r * Hq + h) * max_splits + slot) * 2;
    ml[0] = mrun[threadIdx.x];
    ml[1] = lrun[threadIdx.x];
  }
}

// Attention over the shared prefix of a batch (the prefix cache,
// crates/s-server/src/prefix.rs:59-109, whose pages every sequence of the
// batch holds): tiles [0, ts) are the same physical KV pages for every row,
// so CTA (kv head g, query group qg, split sp) reads each of its tiles once
// and scores it against the queries of all rows (row r, head g*G + j): up to
// ASH_Q of them, a query group. Its partial (o, m, l) per query goes to split
// slot sp of that (row, head), merged by attn_combine_kernel with the row's
// own tiles. Scores and P.V in f32 (4 queries x 4 positions and 4 queries x
// hd/8 dims per thread; a quarter-warp's lanes read consecutive K rows and
// consecutive V float4s, so their shared-memory loads hit distinct banks),
// online softmax per query across the CTA's tiles.
constexpr int ASH_THREADS = 256, ASH_Q = 128;

size_t attn_shared_smem_bytes(uint32_t hd) {
  return sizeof(float) * ((size_t)ASH_Q * (hd + 4) + 2 * (size_t)ATT_T * (hd + 4) + (size_t)ASH_Q * (ATT_T + 1) +
                          3 * ASH_Q);
}

__global__ void __launch_bounds__(ASH_THREADS) attn_shared_kernel(const float* q, uint32_t ldq, const SeqDesc* seqs,
                                                                  const uint32_t* shared_tiles, uint32_t nrows,
                                                                  uint32_t layer, uint32_t Hq, uint32_t Hkv,
                                                                  uint32_t hd, float scale, float* part_o,
                                                                  float* part_ml, uint32_t max_splits) {
  extern __shared__ __align__(16) float smem[];
  pdl_trigger();
  const uint32_t G = Hq / Hkv, Q = nrows * G, nqg = (Q + ASH_Q - 1) / ASH_Q;
  const uint32_t g = blockIdx.x / nqg, qg = blockIdx.x - g * nqg, sp = blockIdx.y;
  const uint32_t ts = *shared_tiles;  // the step's input block: written before the step's first kernel
  if (!ts) return;
  const uint32_t tps = (ts + gridDim.y - 1) / gridDim.y, tb = sp * tps;
  if (tb >= ts) return;
  const uint32_t te = min(ts, tb + tps), q0 = qg * ASH_Q, nq = min((uint32_t)ASH_Q, Q - q0);
  const uint32_t kvd = Hkv * hd, hs = hd + 4, hd4 = hd / 4, tid = threadIdx.x;
  float* qs = smem;                     // [ASH_Q][hd+4]
  float* kt = qs + ASH_Q * hs;          // [ATT_T][hd+4]
  float* vt = kt + ATT_T * hs;          // [ATT_T][hd+4]
  float* ps = vt + ATT_T * hs;          // [ASH_Q][ATT_T+1]
  float* mrun = ps + ASH_Q * (ATT_T + 1);
  float* lrun = mrun + ASH_Q;
  float* alpha = lrun + ASH_Q;
  const SeqDesc sd = seqs[0];  // tiles below ts are the same pages in every row
  auto stage = [&](uint32_t t) {
    const float* kb = sd.pages[t] + (size_t)layer * KV_PAGE * kvd + (size_t)g * hd;
    for (uint32_t i = tid; i < ATT_T * hd4; i += ASH_THREADS) {
      const uint32_t pp = i / hd4, d4 = i - pp * hd4;
      cp_async16(kt + pp * hs + 4 * d4, kb + (size_t)pp * kvd + 4 * d4);
      cp_async16(vt + pp * hs + 4 * d4, kb + sd.voff + (size_t)pp * kvd + 4 * d4);
    }
    cp_async_commit();
  };
  stage(tb);  // shared positions are older than every row's: not written by this step
  pdl_wait();  // the queries come from the QKV GEMV
  for (uint32_t i = tid; i < ASH_Q * hd4; i += ASH_THREADS) {
    const uint32_t qi = i / hd4, d4 = i - qi * hd4;
    float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
    if (qi < nq) {
      const uint32_t gq = q0 + qi, r = gq / G, j = gq - r * G;
      v = reinterpret_cast<const float4*>(q + (size_t)r * ldq + (size_t)(g * G + j) * hd)[d4];
    }
    reinterpret_cast<float4*>(qs + qi * hs)[d4] = v;
  }
  for (uint32_t i = tid; i < ASH_Q; i += ASH_THREADS) { mrun[i] = -INFINITY; lrun[i] = 0.f; }
  // thread -> 4 queries (i0 .. i0+3) x 4 positions (scores) / x hd/8 dims (output)
  const uint32_t i0 = (tid >> 3) * 4, c8 = tid & 7, dpt = hd / 8;  // dims per thread: a multiple of 4
  float4 acc[4][4];
#pragma unroll
  for (int a = 0; a < 4; a++)
#pragma unroll
    for (int b = 0; b < 4; b++) acc[a][b] = make_float4(0.f, 0.f, 0.f, 0.f);
  const uint32_t warp = tid >> 5, lane = tid & 31;
  for (uint32_t t = tb; t < te; t++) {
    if (t != tb) {
      __syncthreads();  // the previous tile is consumed
      stage(t);
    }
    cp_async_wait<0>();
    __syncthreads();
    {  // scores of queries i0..i0+3 at positions c8 + 8b (consecutive lanes read
       // consecutive K rows: distinct banks)
      float sc[4][4] = {};
      for (uint32_t d4 = 0; d4 < hd4; d4++) {
        float4 qv[4], kv[4];
#pragma unroll
        for (int a = 0; a < 4; a++) qv[a] = reinterpret_cast<const float4*>(qs + (i0 + a) * hs)[d4];
#pragma unroll
        for (int b = 0; b < 4; b++) kv[b] = reinterpret_cast<const float4*>(kt + (c8 + 8 * b) * hs)[d4];
#pragma unroll
        for (int a = 0; a < 4; a++)
#pragma unroll
          for (int b = 0; b < 4; b++) {
            sc[a][b] = fmaf(qv[a].x, kv[b].x, sc[a][b]);
            sc[a][b] = fmaf(qv[a].y, kv[b].y, sc[a][b]);
            sc[a][b] = fmaf(qv[a].z, kv[b].z, sc[a][b]);
            sc[a][b] = fmaf(qv[a].w, kv[b].w, sc[a][b]);
          }
      }
#pragma unroll
      for (int a = 0; a < 4; a++)
#pragma unroll
        for (int b = 0; b < 4; b++) ps[(i0 + a) * (ATT_T + 1) + c8 + 8 * b] = sc[a][b] * scale;
    }
    __syncthreads();
    for (uint32_t i = warp; i < nq; i += ASH_THREADS / 32) {  // online softmax, one warp per query
      const float s0 = ps[i * (ATT_T + 1) + lane];
      float mx = s0;
#pragma unroll
      for (int of = 16; of > 0; of >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, of));
      const float mold = mrun[i], mnew = fmaxf(mold, mx);
      const float e0 = expf(s0 - mnew);
      ps[i * (ATT_T + 1) + lane] = e0;
      const float sum = warp_sum(e0);
      if (lane == 0) {
        const float al = expf(mold - mnew);
        alpha[i] = al;
        lrun[i] = lrun[i] * al + sum;
        mrun[i] = mnew;
      }
    }
    __syncthreads();
    {  // acc[a][b] (dims 4 (c8 + 8b) ..: consecutive lanes, consecutive float4s)
       //   = acc * alpha + sum_p P[i0+a][p] V[p]
      float al[4];
#pragma unroll
      for (int a = 0; a < 4; a++) al[a] = alpha[i0 + a];
#pragma unroll
      for (int a = 0; a < 4; a++)
#pragma unroll
        for (int b = 0; b < 4; b++) {
          acc[a][b].x *= al[a]; acc[a][b].y *= al[a]; acc[a][b].z *= al[a]; acc[a][b].w *= al[a];
        }
      for (uint32_t pp = 0; pp < ATT_T; pp++) {
        float pw[4];
#pragma unroll
        for (int a = 0; a < 4; a++) pw[a] = ps[(i0 + a) * (ATT_T + 1) + pp];
#pragma unroll
        for (int b = 0; b < 4; b++) {
          if (4 * b >= (int)dpt) break;
          const float4 v = reinterpret_cast<const float4*>(vt + pp * hs)[c8 + 8 * b];
#pragma unroll
          for (int a = 0; a < 4; a++) {
            acc[a][b].x = fmaf(pw[a], v.x, acc[a][b].x);
            acc[a][b].y = fmaf(pw[a], v.y, acc[a][b].y);
            acc[a][b].z = fmaf(pw[a], v.z, acc[a][b].z);
            acc[a][b].w = fmaf(pw[a], v.w, acc[a][b].w);
          }
        }
      }
    }
  }
#pragma unroll
  for (int a = 0; a < 4; a++) {
    const uint32_t qi = i0 + a;
    if (qi >= nq) continue;
    const uint32_t gq = q0 + qi, r = gq / G, h = g * G + (gq - r * G);
    float* po = part_o + (((size_t)r * Hq + h) * max_splits + sp) * hd;
#pragma unroll
    for (int b = 0; b < 4; b++)
      if (4 * b < (int)dpt) reinterpret_cast<float4*>(po)[c8 + 8 * b] = acc[a][b];
    if (c8 == 0) {
      float* ml = part_ml + (((size_t)r * Hq + h) * max_splits + sp) * 2;
      ml[0] = mrun[qi];
      ml[1] = lrun[qi];
    }
  }
}

// Merges the splits of (row r, head h): out = sum_s o_s e_s / sum_s l_s e_s with
// e_s = exp(m_s - max m), sums in split order (the shared splits first). The (m, l) pairs are staged in
// shared memory by one parallel load; the partial outputs are read eight
// splits at a time.
__global__ void attn_combine_kernel(const float* part_o, const float* part_ml, const RowDesc* rows, uint32_t Hq,
                                    uint32_t hd, uint32_t max_splits, uint32_t np, float* out, uint32_t ldo,
                                    const uint32_t* shared_tiles) {
  __shared__ float sm_m[64], sm_e[64];
  pdl_trigger();
  const uint32_t r = blockIdx.x / Hq, h = blockIdx.x - r * Hq;
  const uint32_t L = rows[r].pos + 1;  // rows are set before the step's first kernel
  const uint32_t tiles = (L + ATT_T - 1) / ATT_T;
  const uint32_t ts = shared_tiles ? min(*shared_tiles, tiles) : 0u;
  // splits with work: shared ones (slots 0..) and the row's own (slots ATT_SHARED_SPLITS..)
  const uint32_t tss = ts ? (ts + ATT_SHARED_SPLITS - 1) / ATT_SHARED_SPLITS : 1u;
  const uint32_t nsh = ts ? (ts + tss - 1) / tss : 0u;
  const uint32_t tps = (tiles - ts + np - 1) / np;  // np: the split kernel's private splits (its grid's y)
  const uint32_t npr = tiles > ts ? (tiles - ts + tps - 1) / tps : 0u;
  const uint32_t ns = nsh + npr;  // <= max_splits <= 64
  pdl_wait();  // the partials come from attn_split_kernel / attn_shared_kernel
  const float* ml = part_ml + ((size_t)r * Hq + h) * max_splits * 2;
  auto slot = [&](uint32_t s) { return s < nsh ? s : ATT_SHARED_SPLITS + (s - nsh); };
  for (uint32_t s = threadIdx.x; s < ns; s += blockDim.x) {
    sm_m[s] = ml[2 * slot(s)];
    sm_e[s] = ml[2 * slot(s) + 1];
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
      for (int u = 0; u < 8; u++) v[u] = po[(size_t)slot(s + u) * hd + d];
#pragma unroll
      for (int u = 0; u < 8; u++) acc = fmaf(v[u], sm_e[s + u], acc);
    }
    float v[8];
#pragma unroll
    for (int u = 0; u < 8; u++)
      if (s + u < ns) v[u] = po[(size_t)slot(s + u) * hd + d];
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
                             uint32_t max_splits, float* out, uint32_t ldo, cudaStream_t st, uint32_t one_seq,
                             const uint32_t* shared_tiles, SideStream side) {
  if (!nrows) return cudaSuccess;
  const uint32_t G = Hq / Hkv;
  const size_t sm = attn_smem_bytes(G, hd);
  const float scale = 1.0f / sqrtf((float)hd);  // qwen2.rs:505
  cudaError_t e;
  const bool fork = shared_tiles && side.st;
  // the rows' own tiles in np splits: fewer for many rows (more tiles a CTA,
  // fewer partials to merge), all of them for one row (its only parallelism)
  const uint32_t np = nrows > 1 ? std::min(ATT_BATCH_SPLITS, max_splits - ATT_SHARED_SPLITS)
                                : max_splits - ATT_SHARED_SPLITS;
  if (shared_tiles) {  // the batch's shared prefix, once for all rows
    const uint32_t nqg = (nrows * G + ASH_Q - 1) / ASH_Q;
    const dim3 grid(Hkv * nqg, ATT_SHARED_SPLITS), blk(ASH_THREADS);
    if (fork) {  // on the side stream, concurrent with the split kernel: both need only the QKV GEMV
      if ((e = cudaEventRecord(side.fork, st)) != cudaSuccess || (e = cudaStreamWaitEvent(side.st, side.fork, 0)))
        return e;
      attn_shared_kernel<<<grid, blk, attn_shared_smem_bytes(hd), side.st>>>(
          q, ldq, seqs, shared_tiles, nrows, layer, Hq, Hkv, hd, scale, part_o, part_ml, max_splits);
      if ((e = cudaGetLastError()) != cudaSuccess || (e = cudaEventRecord(side.join, side.st)) != cudaSuccess)
        return e;
    } else {
      e = launch_pdl(attn_shared_kernel, grid, blk, attn_shared_smem_bytes(hd), st, q, ldq, seqs, shared_tiles, nrows,
                     layer, Hq, Hkv, hd, scale, part_o, part_ml, max_splits);
      if (e != cudaSuccess) return e;
    }
  }
  e = launch_pdl(attn_split_kernel, dim3(nrows * Hkv, np), dim3(ATT_THREADS), sm, st, q,
                 ldq, rows, seqs, layer, Hq, Hkv, hd, scale, part_o, part_ml, max_splits, one_seq, shared_tiles);
  if (e != cudaSuccess || !out) return e;  // no out: the consumer merges the partials itself
  if (fork) {  // the merge needs both passes: an ordinary launch after the join
    if ((e = cudaStreamWaitEvent(st, side.join, 0)) != cudaSuccess) return e;
    attn_combine_kernel<<<nrows * Hq, hd, 0, st>>>(part_o, part_ml, rows, Hq, hd, max_splits, np, out, ldo,
                                                   shared_tiles);
    return cudaGetLastError();
  }
  return launch_pdl(attn_combine_kernel, dim3(nrows * Hq), dim3(hd), 0, st, part_o, part_ml, rows, Hq, hd, max_splits,
                    np, out, ldo, shared_tiles);
}

// Per-device set-up of the attention kernels (shared memory above 48 KB).
cudaError_t attention_prepare() {
  return cudaFuncSetAttribute(attn_shared_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                              (int)attn_shared_smem_bytes(128));
}

cudaError_t launch_silu_mul(float* gate, const float* up, uint32_t F, size_t n, cudaStream_t st) {
  if (!n) return cudaSuccess;
  const unsigned blocks = (unsigned)std::min<size_t>((n + 255) / 256, 148 * 16);
  silu_mul_kernel<<<blocks, 256, 0, st>>>(gate, up, F, n);
  return cudaGetLastError();
}

cudaError_t launch_record_tokens(const uint32_t* tok, uint32_t rows, uint32_t* hist, uint32_t* ctr,
                                 uint32_t cap_steps, cudaStream_t st) {
  record_tokens_kernel<<<1, 128, 0, st>>>(tok, rows, hist, ctr, cap_steps);
  return cudaGetLastError();
}

}  // namespace sm
