// CPU ORACLE — test infrastructure only.
//
// A C++ restatement of the reference's CPU f32 path for the qwen2/llama
// decode loop (PROGETTO-SILICEO/siliceo-motor, Rust):
//   crates/s-gguf/src/{lib,dequant,types,value}.rs   GGUF parser + dequant
//   crates/s-models/src/qwen2.rs                     Config, load, forward_cached
//   crates/s-models/src/state.rs                     SeqState (KV) semantics
//   crates/s-models/src/sampling.rs                  Rng (splitmix64), Sampler
//   crates/s-models/src/generate.rs                  generate_tokens_seeded
//
// Every f32 operation is done in the reference's order, without FMA
// contraction (built with -ffp-contract=off), with glibc expf/powf/sinf/cosf
// as Rust's std uses on x86-64 Linux. Work is split across threads only over
// independent output elements, so every f32 result is the one the
// single-threaded reference computes.
//
// Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg may
// load this library. The engine never links or calls it.
#pragma once
#include <cstddef>
#include <cstdint>
#include <memory>
#include <string>
#include <vector>

namespace orc {

// ---- ggml types (crates/s-gguf/src/types.rs:33-61, 103-127) ----
enum GgmlType : uint32_t {
  T_F32 = 0, T_F16 = 1, T_Q4_0 = 2, T_Q4_1 = 3, T_Q5_0 = 6, T_Q5_1 = 7,
  T_Q8_0 = 8, T_Q8_1 = 9, T_Q2K = 10, T_Q3K = 11, T_Q4K = 12, T_Q5K = 13,
  T_Q6K = 14, T_Q8K = 15, T_BF16 = 30,
};
bool is_quantized(uint32_t t);
// (elements per block, bytes per block)  types.rs:103-127
void block_layout(uint32_t t, uint32_t* bs, uint32_t* tb);
uint32_t type_size(uint32_t t);  // types.rs:93-99

// ---- dequant (crates/s-gguf/src/dequant.rs) ----
float fp16_to_f32(uint16_t h);                                 // :12-33
float bf16_to_f32(uint16_t h);                                 // :36-38
void get_scale_min_k4(int j, const uint8_t* s, uint8_t* d, uint8_t* m);  // :41-49
void dequant_q4_0(const uint8_t* b, float* out);               // :54-63
void dequant_q8_0(const uint8_t* b, float* out);               // :66-71
void dequant_q5_0(const uint8_t* b, float* out);               // :79-94
void dequant_q4_k(const uint8_t* b, float* out);               // :98-124
void dequant_q4_1(const uint8_t* b, float* out);               // :128-136
void dequant_q6_k(const uint8_t* b, float* out);               // :178-206
// dequantize(): dequant.rs:209-310. Returns 0, or -1 on a truncated/unsupported tensor.
int dequantize(uint32_t type, uint64_t n_elements, const uint8_t* raw, uint64_t raw_len,
               float* out, std::string* err);

// ---- GGUF (crates/s-gguf/src/lib.rs, value.rs) ----
struct Value {
  uint32_t type = 0;  // value.rs:3-5 codes
  uint64_t u = 0;
  int64_t i = 0;
  double f = 0;
  bool b = false;
  std::string s;
  uint32_t elem_type = 0;
  std::vector<Value> arr;
  bool as_u64(uint64_t* out) const;  // value.rs:61-73
  bool as_f32(float* out) const;     // value.rs:82-88
};
struct TensorInfo {
  std::string name;
  std::vector<uint64_t> dims;
  uint32_t type = 0;
  uint64_t offset = 0;
  uint64_t n_elements() const;  // lib.rs:81-83
  uint64_t n_bytes() const;     // lib.rs:85-93
};
struct Gguf {
  uint32_t version = 0;
  uint64_t tensor_count = 0, kv_count = 0;
  uint64_t alignment = 32, data_start = 0;
  std::vector<std::pair<std::string, Value>> metadata;
  std::vector<TensorInfo> tensors;
  // whole file mapped read-only
  const uint8_t* map = nullptr;
  size_t map_len = 0;
  ~Gguf();
  const TensorInfo* tensor(const std::string& name) const;  // lib.rs:182-187
  const Value* meta(const std::string& key) const;
  // tensor_data_raw (lib.rs:190-197): pointer into the mapping, bounds-checked.
  const uint8_t* raw(const TensorInfo& t, std::string* err) const;
};
// GgufFile::open (lib.rs:114-179). Returns nullptr and sets *err on failure.
std::unique_ptr<Gguf> gguf_open(const std::string& path, std::string* err);

// ---- model (crates/s-models/src/qwen2.rs) ----
struct Config {  // qwen2.rs:16-26
  size_t n_layers, n_embd, n_ff, n_heads, n_kv_heads, head_dim;
  float rope_theta, rms_eps;
  size_t vocab_size;
};

// A weight kept in its GGUF encoding; rows are dequantized on demand with
// exactly the values dequantize() gives for the whole tensor.
struct QWeight {
  const uint8_t* raw = nullptr;
  uint32_t type = 0;
  size_t n_out = 0, n_in = 0;
  std::vector<float> dense;  // used when rows do not fall on block boundaries
  void row(size_t o, float* out) const;
  void row_range(size_t o, size_t d0, size_t n, float* out) const;  // whole blocks
  size_t tile_width() const;  // a multiple of the block size, about 256
};

struct LayerW {
  std::vector<float> attn_norm, ffn_norm;
  QWeight wq, wk, wv, wo, w_gate, w_up, w_down;
  bool has_bq = false, has_bk = false, has_bv = false;
  std::vector<float> bq, bk, bv;
};

// SeqState restricted to the all-KV case of dense qwen2/llama
// (state.rs:32-120, 202-361).
struct SeqState {
  size_t n_layers = 0, dim = 0, cap = 0, len = 0;
  std::vector<std::vector<float>> k, v;  // per layer [cap × dim]
  static SeqState all_kv(size_t n_layers, size_t kv_dim, size_t max_seq);  // :212-214
  void advance(size_t n) { len += n; }                                    // :289-291
  void reset() { len = 0; }                                               // :297-304
  size_t capacity() const { return cap; }                                 // :309-318
  void ensure_capacity(size_t min_capacity);                              // :323-329
  int truncate(size_t new_len, std::string* err);                         // :341-360
};

struct Model {
  Config c;
  std::unique_ptr<Gguf> g;
  QWeight tok_embd, output;
  std::vector<float> output_norm;
  std::vector<LayerW> layers;
  int threads = 1;
};
std::unique_ptr<Model> model_load(const std::string& path, int threads, std::string* err);
// forward_cached (qwen2.rs:460-561): returns 0 and fills logits[vocab], or -1.
int forward_cached(const Model& m, const uint32_t* tokens, size_t n, SeqState& cache,
                   float* logits, std::string* err);
// logits_from_hidden (qwen2.rs:425-446)
void logits_from_hidden(const Model& m, const float* last_hidden, float* logits);

// ---- sampling (crates/s-models/src/sampling.rs) ----
struct Rng {  // :12-41
  uint64_t s;
  explicit Rng(uint64_t seed) : s(seed + 0x9E3779B97F4A7C15ull) {}
  uint64_t next_u64();
  float next_f32();
};
struct Sampler {  // :43-60
  float temperature = 0.f;
  long top_k = -1;   // <0: None
  float top_p = -1;  // <0: None
  size_t sample(const float* logits, size_t n, Rng& rng) const;                       // :94-144
  size_t sample_masked(const float* logits, const uint8_t* mask, size_t n, Rng& rng) const;  // :66-88
};
size_t argmax(const float* x, size_t n);  // :147-155
void softmax_row_ref(float* x, size_t n);  // :157-172

}  // namespace orc
