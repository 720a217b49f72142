// Host-visible declarations of the engine's kernels and their launchers.
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>

#include <algorithm>

#include "device.cuh"

namespace sm {

struct SampleParams {
  float temperature;
  int32_t top_k;  // < 0: None
  float top_p;    // < 0: None
  int32_t pad;
};


uint32_t gemv_plan(GemvArgs& a);
// n_parts: the number of out_parts entries per column an EPI_RESID launch writes.
cudaError_t launch_gemv(GemvArgs a, cudaStream_t st, uint32_t* n_parts = nullptr);
cudaError_t launch_dequant(const DWDesc& w, float* out, cudaStream_t st);
// Writes embed_norm_parts(n_in) partial sums of x^2 per row into parts.
cudaError_t launch_embed_norm(const DWDesc& w, const uint32_t* tokens, uint32_t rows, float* x, uint32_t ldx,
                              const float* nw, float* xn, uint32_t ldxn, float* parts, cudaStream_t st);
uint32_t embed_norm_parts(uint32_t n);
cudaError_t launch_embed(const DWDesc& w, const uint32_t* tokens, uint32_t rows, float* x, uint32_t ldx,
                         cudaStream_t st);
cudaError_t launch_rmsnorm(const float* x, uint32_t ldx, const uint32_t* sel, const float* w, float* out, uint32_t ldo,
                           uint32_t rows, uint32_t n, float eps, cudaStream_t st);
size_t attn_smem_bytes(uint32_t G, uint32_t hd);
// one_seq: the rows are consecutive positions of one sequence (a prefill
// chunk), so every row's K/V from rows[0].pos on is written by this pass.
// shared_tiles (device, may be null): the number of leading KV pages that
// every row holds as the same physical page (all their positions older than
// every row's): attn_shared_kernel reads them once for all rows. Partials:
// max_splits slots per (row, head), the first ATT_SHARED_SPLITS for the
// shared tiles. out = null: only the partials are written (a batch-1 O GEMV
// merges them as it reads its input: GemvArgs::att_o).
// side.st (optional): a second stream on which the shared pass runs
// concurrently with the split kernel (fork and join through the two events;
// they become graph edges when the launches are captured).
constexpr uint32_t ATT_SHARED_SPLITS = 16;
// Splits of the rows' own tiles in a step of several rows (one row: all the
// remaining max_splits - ATT_SHARED_SPLITS slots).
constexpr uint32_t ATT_BATCH_SPLITS = 16;
struct SideStream {
  cudaStream_t st;
  cudaEvent_t fork, join;
};
cudaError_t launch_attention(const float* q, uint32_t ldq, const RowDesc* rows, const SeqDesc* seqs, uint32_t nrows,
                             uint32_t layer, uint32_t Hq, uint32_t Hkv, uint32_t hd, float* part_o, float* part_ml,
                             uint32_t max_splits, float* out, uint32_t ldo, cudaStream_t st, uint32_t one_seq,
                             const uint32_t* shared_tiles, SideStream side = SideStream{nullptr, nullptr, nullptr});
size_t attn_shared_smem_bytes(uint32_t hd);
cudaError_t attention_prepare();
cudaError_t launch_silu_mul(float* gate, const float* up, uint32_t F, size_t n, cudaStream_t st);
// The on-device sampler (sampler.cu): rows CTAs, row r's logits at
// logits + r * ldl (ldl = ~0: V), scratch of sample_scratch_words(V) words per
// row (used when the row's temperature is > 0). amax (may be null): n_amax
// per-tile argmax keys of row 0's logits written by the output head's
// epilogue; a greedy row 0 without a mask reduces those instead.
uint64_t sample_scratch_words(uint32_t V);
cudaError_t launch_sample(const float* logits, uint32_t V, uint32_t rows, const uint8_t* mask,
                          const SampleParams* params, uint64_t* rng, uint32_t* out_tok, uint32_t* next_tok,
                          RowDesc* advance, uint32_t* scratch, cudaStream_t st, uint64_t ldl = ~0ull,
                          const uint64_t* amax = nullptr, uint32_t n_amax = 0);
// softmax (sampling.rs:157-172) of `rows` rows of n values, bit for bit.
cudaError_t launch_softmax(const float* x, uint32_t rows, uint32_t n, float* out, cudaStream_t st);
// The sampler's exp (glibc's expf on x <= 0) applied to n values.
cudaError_t launch_expf_ref(const float* x, float* y, size_t n, cudaStream_t st);

// sm_gemv_noalloc: scratch in fixed device arrays; cudaErrorNotSupported when
// the shape's smallest K-split does not fit them (nothing is launched).
cudaError_t launch_gemv_noalloc(GemvArgs a, cudaStream_t st);
cudaError_t gemv_noalloc_status(cudaStream_t st, uint32_t* flag);
// Batch-1 Q4_K/Q6_K GEMVs run on the tensor cores (gemv_tc.cu); launch_gemv
// dispatches to that kernel. Per-device set-up, and the K-split scratch
// (floats, counters) a launch of this shape may use on a GPU with `sms` SMs:
cudaError_t gemv_tc_prepare();
void gemv_tc_scratch_need(GemvArgs a, uint32_t sms, uint64_t* part, uint32_t* cnt);
// The same for the batched (2..32 columns, one weight type) tensor-core GEMV
// of gemv_tcb.cu (a.batch columns).
cudaError_t gemv_tcb_prepare();
void gemv_tcb_scratch_need(GemvArgs a, uint32_t sms, uint64_t* part, uint32_t* cnt);
// The same for the tcgen05 batched GEMV of gemv_umma.cu, which launch_gemv
// uses for batches of 2..32 (gemv_tcb.cu when no plan of it fits).
cudaError_t gemv_umma_prepare();
void gemv_umma_scratch_need(GemvArgs a, uint32_t sms, uint64_t* part, uint32_t* cnt);
// Bytes of the x image (GemvArgs::xblob) a launch of n_in inputs and `batch`
// columns needs; without it launch_gemv runs the gemv_tcb.cu kernel.
uint64_t gemv_umma_blob_bytes(uint32_t n_in, uint32_t batch);
cudaError_t launch_record_tokens(const uint32_t* tok, uint32_t rows, uint32_t* hist, uint32_t* ctr,
                                 uint32_t cap_steps, cudaStream_t st);

}  // namespace sm
