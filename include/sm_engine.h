/*
 * siliceo-motor B200 decode engine — C ABI.
 *
 * Drop-in boundary for the qwen2/llama decode path of PROGETTO-SILICEO/
 * siliceo-motor. Each group below names the reference interface it replaces
 * (paths relative to the reference repository). All functions return an
 * sm_status (0 = ok); on error, sm_last_error() gives a message for the
 * calling thread. Nothing aborts or throws across this boundary. Pointers
 * named *_dev are CUDA device pointers; everything else is host memory.
 */
#ifndef SM_ENGINE_H
#define SM_ENGINE_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef enum {
  SM_OK = 0,
  SM_ERR_ARG = 1,         /* invalid argument */
  SM_ERR_IO = 2,          /* file could not be read or written */
  SM_ERR_FORMAT = 3,      /* malformed GGUF / missing tensor or key */
  SM_ERR_UNSUPPORTED = 4, /* architecture, type or shape not supported */
  SM_ERR_CUDA = 5,        /* CUDA runtime error (message has the CUDA text) */
  SM_ERR_OOM = 6,         /* device or host allocation failed */
  SM_ERR_CAPACITY = 7,    /* sequence would exceed the cache capacity */
  SM_ERR_STATE = 8,       /* operation not valid for the object's state */
  SM_ERR_PEER = 9         /* a tensor-parallel peer failed or did not arrive in time;
                             the model's group is unusable from then on */
} sm_status;

/* Message of the last failed call on this thread ("" if none). */
const char* sm_last_error(void);
/* ABI version: increments on any incompatible change (2: tensor-parallel
 * fields of sm_load_opts). */
int sm_abi_version(void);

/* ------------------------------------------------------------------------
 * Model. Replaces `s_models::qwen2::Model` / `s_backend_cuda::model::GpuQwen2`
 * as the `impl Device` for qwen2/llama (crates/s-models/src/device.rs:20-34,
 * crates/s-models/src/qwen2.rs:99-150, crates/s-backend-cuda/src/model.rs:146-211).
 * Quantized weights stay quantized in HBM.
 * ---------------------------------------------------------------------- */
typedef struct sm_model sm_model;
typedef struct sm_cache sm_cache;

/* Mirrors qwen2::Config (crates/s-models/src/qwen2.rs:16-26). */
typedef struct {
  uint64_t n_layers, n_embd, n_ff, n_heads, n_kv_heads, head_dim;
  float rope_theta, rms_eps;
  uint64_t vocab_size;
} sm_config;

typedef struct {
  int32_t device;        /* CUDA device ordinal */
  uint32_t max_batch;    /* largest decode batch: 0 (= 32) .. 32 */
  uint32_t max_context;  /* largest position + 1 any cache may reach (default 32768) */
  uint32_t tp_rank;      /* tensor-parallel rank, below tp_size */
  uint32_t tp_size;      /* tensor-parallel size: 0 or 1 = none, else 2..8 (one process per GPU) */
  uint32_t tp_flags;     /* SM_TP_* */
  uint32_t tp_wait_ms;   /* bound on one wait for a peer (0 = 10000); group formation waits 6x this */
  const void* tp_group;  /* SM_TP_ID_BYTES from sm_tp_group_id (made once, on one rank) */
} sm_load_opts;

/* Tensor parallelism (Megatron split; one process per GPU of one node).
 * Every rank loads the same GGUF with its own tp_rank, the same tp_size and
 * the same group id, and then makes the same calls with the same arguments
 * (tokens, samplers, RNG states) in the same order. Each rank keeps the
 * attention heads [rank*Hq/N, (rank+1)*Hq/N) (and their KV heads), FFN
 * columns [rank*F/N, ...), the matching input columns of attn_output and
 * ffn_down, and a 1/N slice of the output head's rows. After the O and down
 * projections the partial sums are all-reduced in rank order (every rank
 * gets bit-identical activations), and the logit slices are all-gathered
 * before sampling, so every rank returns the same tokens and logits.
 * Exchanges run over peer memory (CUDA IPC over NVLink) with kernels of the
 * engine; SM_TP_NCCL uses NCCL all-reduce / all-gather instead. A peer that
 * does not arrive within tp_wait_ms fails the call with SM_ERR_PEER.
 * Per-rank views: sm_model_weight_bytes counts this rank's shard,
 * sm_cache_read_kv returns this rank's KV heads. */
#define SM_TP_ID_BYTES 128
#define SM_TP_NCCL 1u
/* Makes a group id (an NCCL unique id) to share with every rank. */
int sm_tp_group_id(void* id_out);
/* Which part of a model rank `rank` of `size` holds (no device needed). The
 * loader additionally needs the split inputs of attn_output (q_heads x
 * head_dim) and ffn_down (ff) to be whole quant blocks. */
typedef struct {
  uint64_t q_head0, q_heads;   /* query heads [q_head0, q_head0 + q_heads) */
  uint64_t kv_head0, kv_heads; /* KV heads */
  uint64_t ff0, ff;            /* FFN columns (ffn_gate/ffn_up rows, ffn_down inputs) */
  uint64_t vocab0, vocab;      /* output-head rows */
} sm_tp_shard;
int sm_tp_plan(const sm_config* cfg, uint32_t rank, uint32_t size, sm_tp_shard* out);
/* Marks the model's group failed without touching the GPU: for a host that
 * learned (from its own heartbeat or store) that a peer left. Later compute
 * calls return SM_ERR_PEER at once, and sm_model_free skips its final
 * barrier with the peers. No effect on a model without tensor parallelism. */
int sm_model_tp_abort(sm_model* m);

/* Model::load / GpuQwen2::load. opts may be NULL (defaults). */
int sm_model_load(const char* gguf_path, const sm_load_opts* opts, sm_model** out);
/* Same, from a GGUF image in host memory (the buffer may be freed after). */
int sm_model_load_memory(const void* gguf, uint64_t len, const sm_load_opts* opts, sm_model** out);
/* Releases the handle (the model lives on while caches of it exist). With
 * tensor parallelism every rank frees its handle at the same point of its
 * program: the call waits (bounded by tp_wait_ms) for the other ranks, and
 * the model makes no exchanges afterwards. */
int sm_model_free(sm_model* m);
/* Device::config */
int sm_model_config(const sm_model* m, sm_config* out);
/* Quantized weight bytes one decode step streams from HBM (all 2-D weights,
 * output head included, embedding table excluded: one row is gathered). */
int sm_model_weight_bytes(const sm_model* m, uint64_t* out);
/* The CUDA stream the model's work is issued on (a cudaStream_t). */
int sm_model_stream(const sm_model* m, void** stream);
/* Bytes one decode step copies host->device (token, position, RNG and
 * sampler state of every row, one pinned block) and device->host (tokens,
 * RNG states). */
int sm_model_step_io_bytes(const sm_model* m, uint64_t* h2d, uint64_t* d2h);
/* Kernels one sm_decode_run step of n_rows sequences launches (the kernel
 * nodes of its CUDA graph; available after such a run). No reference
 * counterpart. */
int sm_model_step_launches(const sm_model* m, uint64_t n_rows, uint64_t* out);

/* ------------------------------------------------------------------------
 * Sequence state. Replaces `s_models::state::SeqState` for dense models
 * (crates/s-models/src/state.rs:202-361) and the position counter GpuCache
 * (crates/s-backend-cuda/src/model.rs:97-105): K/V live in HBM, f32, in
 * pages of 32 positions ([layer][32][kv_dim] of K, then the same of V) drawn
 * from a pool of the model. A clone shares its source's pages; a page is
 * copied before one of its holders writes it, so clones behave as the
 * reference's deep copies while a shared prefix sits in HBM once. Positions
 * never written read as zeros.
 * ---------------------------------------------------------------------- */
int sm_cache_new(sm_model* m, uint64_t max_seq, sm_cache** out); /* Device::new_cache (qwen2.rs:633-637) */
int sm_cache_free(sm_cache* c);
int sm_cache_len(const sm_cache* c, uint64_t* out);          /* SeqState.len */
int sm_cache_capacity(const sm_cache* c, uint64_t* out);     /* state.rs:309-318 */
int sm_cache_advance(sm_cache* c, uint64_t n);               /* state.rs:289-291 (len += n, within capacity) */
int sm_cache_reset(sm_cache* c);                             /* state.rs:297-304 */
int sm_cache_truncate(sm_cache* c, uint64_t len);            /* state.rs:341-360: error if len > current len */
int sm_cache_ensure_capacity(sm_cache* c, uint64_t min_cap); /* state.rs:323-329: keeps positions 0..len */
int sm_cache_clone(const sm_cache* c, sm_cache** out);       /* SeqState: Clone (state.rs:64-69) */
/* Host copy of the K and V rows (kv_dim floats each) of one position. */
int sm_cache_read_kv(const sm_cache* c, uint64_t layer, uint64_t pos, float* k_out, float* v_out);
/* Pages of the model's KV pool held by caches, and pages allocated in all
 * (held + free), each of kv_page_bytes bytes. No reference counterpart: the
 * reference's SeqState owns contiguous vectors. */
int sm_model_kv_pages(const sm_model* m, uint64_t* held, uint64_t* allocated, uint64_t* kv_page_bytes);

/* Row `token` of the embedding table (n_embd floats, host) as the forward's
 * first kernel gathers it: the exact dequantized row (qwen2.rs:468-472). */
int sm_model_embedding(sm_model* m, uint32_t token, float* out);

/* ------------------------------------------------------------------------
 * Forward. Device::forward_cached (crates/s-models/src/device.rs:33,
 * crates/s-models/src/qwen2.rs:460-561): processes `n` tokens at absolute
 * position sm_cache_len(), appends their K/V, and writes the last token's
 * logits [vocab] to logits_out (host) unless it is NULL.
 * ---------------------------------------------------------------------- */
int sm_forward_cached(sm_model* m, sm_cache* c, const uint32_t* tokens, uint64_t n, float* logits_out);

/* Sampler (crates/s-models/src/sampling.rs:43-60, 94-144). temperature <= 0
 * is greedy (lowest index wins ties); top_k < 0 and top_p < 0 mean None;
 * every combination is sampled on the device.
 * The splitmix64 state (sampling.rs:12-41) is passed in and returned. */
typedef struct {
  float temperature;
  int64_t top_k;
  float top_p;
} sm_sampler;

/* Sampler::sample / sample_masked (crates/s-models/src/sampling.rs:66-144)
 * on the device, for logits in host memory: row i (i < n_rows) samples the
 * `vocab` logits at logits + i * ld with samplers[i] and rng_states[i]
 * (updated); ld = 0: every row samples the same logits. mask (may be NULL)
 * has the same layout, 0 = forbidden. The kernel the decode steps run, bit
 * for bit the reference's result (the reference's f32 rounding at every step,
 * glibc's expf). Uses the current device; allocates its buffers per call. */
int sm_sample(const float* logits, uint64_t n_rows, uint64_t ld, uint64_t vocab, const uint8_t* mask,
              const sm_sampler* samplers, uint64_t* rng_states, uint32_t* out_tokens);
/* softmax (crates/s-models/src/sampling.rs:157-172) of `rows` rows of n
 * device floats into probs_dev (device, not aliasing x_dev): the sampler's
 * probabilities, bit for bit the reference's (max, glibc expf, the
 * left-to-right f32 sum, IEEE division). */
int sm_softmax(const float* x_dev, uint64_t rows, uint64_t n, float* probs_dev, void* stream);
/* The sampler's exp on n floats in device memory: glibc's expf (Rust's
 * f32::exp on x86-64 Linux) for x <= 0 and NaN, bit for bit. No reference
 * counterpart; exposed so its exactness can be checked. */
int sm_expf_ref(const float* x_dev, float* y_dev, uint64_t n, void* stream);

/* Initial splitmix64 state for Rng::new(seed). */
uint64_t sm_rng_seed(uint64_t seed);

/* Forward `n` tokens and sample the next one on the device: only the token
 * id (and the RNG state) cross PCIe. mask (host, vocab bytes, 0 = forbidden)
 * may be NULL (sampling.rs:66-88). */
int sm_forward_sample(sm_model* m, sm_cache* c, const uint32_t* tokens, uint64_t n, const sm_sampler* s,
                      uint64_t* rng_state, const uint8_t* mask, uint32_t* out_token);
/* One decode step for each of n sequences, batched (one token each; each
 * cache advances by one). samplers and rng_states have n entries. */
int sm_decode_batch(sm_model* m, sm_cache* const* caches, uint64_t n, const uint32_t* tokens,
                    const sm_sampler* samplers, uint64_t* rng_states, uint32_t* out_tokens);
/* sm_decode_batch that also copies the logits its sampler drew from to
 * logits_out (host, n x vocab floats): forward_cached's return value for each
 * sequence of the batch (device.rs:33) next to the on-device sample. */
int sm_decode_batch_logits(sm_model* m, sm_cache* const* caches, uint64_t n, const uint32_t* tokens,
                           const sm_sampler* samplers, uint64_t* rng_states, uint32_t* out_tokens, float* logits_out);

/* n_steps decode steps for each of n sequences entirely on the device: the
 * token sampled at step i is the input of step i+1 (no stop checks; the
 * caller truncates a cache past an EOS). out_tokens[step * n + i]. If
 * ev_begin / ev_end (cudaEvent_t) are given they are recorded on the model's
 * stream around the steps. The loop of generate.rs:204-238 without its
 * per-token callbacks. */
int sm_decode_run(sm_model* m, sm_cache* const* caches, uint64_t n, const uint32_t* tokens,
                  const sm_sampler* samplers, uint64_t* rng_states, uint64_t n_steps, uint32_t* out_tokens,
                  void* ev_begin, void* ev_end);

/* ------------------------------------------------------------------------
 * Generation loop. generate_tokens_seeded (crates/s-models/src/generate.rs:149-250)
 * over any device given as a vtable (the `Device` trait), and over the
 * engine itself. Stop strings need a detokenizer: stop_cb receives the
 * generated ids and reports a hit.
 * ---------------------------------------------------------------------- */
typedef int (*sm_on_token_fn)(void* ud, uint32_t token);                 /* 0 = abort ("stop") */
typedef int (*sm_masker_fn)(void* ud, uint8_t* mask, uint64_t vocab);    /* 1 = mask written */
typedef int (*sm_stop_fn)(void* ud, const uint32_t* ids, uint64_t n);    /* 1 = stop-string hit */
typedef void (*sm_on_prefill_fn)(void* ud, void* cache);                 /* once, after prefill */

typedef struct {
  uint64_t max_tokens;
  float temperature;
  int64_t top_k;  /* < 0: None */
  float top_p;    /* < 0: None */
  int32_t has_seed;
  uint64_t seed;
} sm_gen_params;

typedef struct {
  uint64_t n_ids;
  int32_t finish_stop; /* 1 = "stop", 0 = "length" */
  uint64_t prompt_tokens;
  uint64_t prefix_reused;
  double elapsed_secs;
} sm_gen_result;

/* The Device trait as a vtable: new_cache / free_cache, and forward+sample
 * (forward_cached followed by Sampler::sample[_masked]). */
typedef struct {
  int (*new_cache)(void* dev, uint64_t max_seq, void** cache);
  int (*free_cache)(void* dev, void* cache);
  int (*forward_sample)(void* dev, void* cache, const uint32_t* tokens, uint64_t n, const sm_sampler* s,
                        uint64_t* rng_state, const uint8_t* mask, uint32_t* out_token);
} sm_device_vtbl;

/* out_ids must hold params->max_tokens entries. seed_cache (may be NULL) is
 * used, not consumed, when 0 < seed_n < n_prompt; its length must be seed_n. */
int sm_generate_with(const sm_device_vtbl* vt, void* dev, uint64_t vocab, const uint32_t* prompt, uint64_t n_prompt,
                     const sm_gen_params* params, const uint32_t* eos, uint64_t n_eos, sm_on_token_fn on_token,
                     sm_masker_fn masker, sm_stop_fn stop, sm_on_prefill_fn on_prefill, void* ud, void* seed_cache,
                     uint64_t seed_n, uint32_t* out_ids, sm_gen_result* res);
/* sm_generate_with over the engine (caches are sm_cache*). */
int sm_generate(sm_model* m, const uint32_t* prompt, uint64_t n_prompt, const sm_gen_params* params,
                const uint32_t* eos, uint64_t n_eos, sm_on_token_fn on_token, sm_masker_fn masker, sm_stop_fn stop,
                sm_on_prefill_fn on_prefill, void* ud, sm_cache* seed_cache, uint64_t seed_n, uint32_t* out_ids,
                sm_gen_result* res);

/* ------------------------------------------------------------------------
 * Kernel-level entry points (the reference's per-kernel GPU tests drive its
 * kernels the same way: crates/s-backend-cuda/src/runtime.rs:120-899).
 * A device weight holds one GGUF tensor [n_out x n_in] in the engine's HBM
 * layout. Types: Q4_K (12), Q6_K (14), Q5_0 (6), Q8_0 (8).
 * ---------------------------------------------------------------------- */
typedef struct sm_dweight sm_dweight;
/* Uploads GGUF bytes (host) of a row-major [n_out x n_in] tensor. */
int sm_dweight_upload(uint32_t ggml_type, const void* gguf_bytes, uint64_t n_out, uint64_t n_in, sm_dweight** out);
int sm_dweight_free(sm_dweight* w);
/* Bytes of the encoded tensor (what one GEMV must read from HBM). */
int sm_dweight_bytes(const sm_dweight* w, uint64_t* out);
/* Bit-exact dequantization of all rows into out_dev[n_out x n_in]
 * (crates/s-gguf/src/dequant.rs:66-206). stream may be NULL. */
int sm_dequant(const sm_dweight* w, float* out_dev, void* stream);
/* Dequant-fused GEMV: y_dev[b][o] = sum_d W[o][d] * x_dev[b][d] for b < batch
 * (batch 1..32; qwen2.rs:663-674, kernels/src/lib.rs:709-876). */
int sm_gemv(const sm_dweight* w, const float* x_dev, float* y_dev, uint64_t batch, void* stream);
/* Reports whether a bounded wait inside an sm_gemv on this weight gave up
 * (a weight copy into shared memory did not complete) since the last call:
 * waits for `stream`, then returns SM_ERR_CUDA (that output is invalid) and
 * clears the flag, or SM_OK. No reference counterpart: the reference's
 * kernels have no bounded waits. */
int sm_gemv_status(const sm_dweight* w, void* stream);
/* sm_gemv for callers that cannot allocate device memory: hosts that hand out
 * all device memory from their own pool, and latency-critical paths that may
 * not call cudaMalloc (it can synchronize the device). No counterpart in the
 * reference. It allocates nothing: the K-split of the tensor-core kernels
 * keeps its partial sums and arrival counters in a fixed 260 KB device array
 * of the library instead of the scratch sm_dweight_upload allocates for
 * sm_gemv. A Q4_K/Q6_K shape whose smallest K-split does not fit the array is
 * refused with SM_ERR_ARG (roughly: ceil(n_in / 8192) * n_out floats, n_out
 * rounded up to 16, at most 65536; 7168 instead of 8192 for Q6_K; rows of at
 * most 8192 (Q4_K) or 7168 (Q6_K) inputs always fit). Every call on a device
 * shares that array, so calls that overlap on the GPU race and their outputs
 * are wrong; the arrival counters advance by wrapping increments, so every
 * completed call (overlapping ones and ones whose bounded wait gave up
 * included) leaves them at zero and later calls are unaffected; nothing
 * needs clearing. The first call on a device looks the array's address up
 * (once per device, with the weight's device current); make that first call
 * before any stream capture. */
int sm_gemv_noalloc(const sm_dweight* w, const float* x_dev, float* y_dev, uint64_t batch, void* stream);
/* sm_gemv_status for the sm_gemv_noalloc calls of the current device (one
 * error word in fixed device memory, shared by those calls). */
int sm_gemv_noalloc_status(void* stream);

/* ------------------------------------------------------------------------
 * Synthetic GGUF models (the stand-in for real model files). Shapes and
 * metadata keys follow qwen2.rs:30-63; values are seeded N(0, weight_std).
 * ---------------------------------------------------------------------- */
typedef struct {
  int32_t arch; /* 0 = "qwen2", 1 = "llama" */
  uint32_t n_embd, n_layers, n_heads, n_kv_heads, n_ff, vocab;
  float rope_theta, rms_eps;
  int32_t qkv_bias;      /* attn_{q,k,v}.bias present */
  int32_t tied;          /* no output.weight (tied embeddings) */
  uint64_t seed;
  float weight_std;      /* 0.02 */
  int32_t type_override; /* -1: Q4_K_M mix; else ggml type for every 2-D weight */
} sm_synth_spec;

/* Presets for the benchmark configurations 0 (Qwen2.5-0.5B), 2 (Qwen2.5-7B),
 * 3 (Llama-3-8B) and 4 (Llama-3-70B). */
int sm_synth_preset(int config_index, sm_synth_spec* out);
int sm_synth_size(const sm_synth_spec* s, uint64_t* len);
int sm_synth_write(const sm_synth_spec* s, const char* path, int threads);
int sm_synth_memory(const sm_synth_spec* s, int threads, void** buf, uint64_t* len);
void sm_synth_free(void* buf);
/* Encodes n f32 values (whole blocks) as ggml type `type` into out. */
int sm_quantize(uint32_t type, const float* x, uint64_t n, void* out);

#ifdef __cplusplus
}
#endif
#endif /* SM_ENGINE_H */
