// CPU ORACLE — test infrastructure only. C entry points over oracle.cpp for
// the Python tests and the CPU-baseline leg of bench.py (ctypes).
#include <chrono>
#include <cmath>
#include <cstdio>
#include <cstring>
#include <string>
#include <vector>

#include "oracle.hpp"

#include <algorithm>
#include <cmath>
#include <thread>
#include <vector>

using namespace orc;

namespace {
void set_err(char* buf, size_t len, const std::string& s) {
  if (!buf || !len) return;
  size_t n = std::min(len - 1, s.size());
  std::memcpy(buf, s.data(), n);
  buf[n] = 0;
}
std::string json_escape(const std::string& s) {
  std::string o;
  for (char ch : s) {
    if (ch == '"' || ch == '\\') { o += '\\'; o += ch; }
    else if ((unsigned char)ch < 0x20) { char b[8]; snprintf(b, sizeof b, "\\u%04x", ch); o += b; }
    else o += ch;
  }
  return o;
}
std::string value_json(const Value& v) {
  char b[64];
  switch (v.type) {
    case 0: case 2: case 4: case 10: snprintf(b, sizeof b, "%llu", (unsigned long long)v.u); return b;
    case 1: case 3: case 5: case 11: snprintf(b, sizeof b, "%lld", (long long)v.i); return b;
    case 6: case 12:
      if (!std::isfinite(v.f)) return "null";
      snprintf(b, sizeof b, "%.17g", v.f);
      return b;
    case 7: return v.b ? "true" : "false";
    case 8: return "\"" + json_escape(v.s) + "\"";
    case 9: {
      std::string o = "[";
      for (size_t i = 0; i < v.arr.size(); i++) o += (i ? "," : "") + value_json(v.arr[i]);
      return o + "]";
    }
  }
  return "null";
}
}  // namespace

extern "C" {

typedef struct {
  uint64_t n_layers, n_embd, n_ff, n_heads, n_kv_heads, head_dim;
  float rope_theta, rms_eps;
  uint64_t vocab_size;
} orc_config;

float orc_fp16_to_f32(uint16_t h) { return fp16_to_f32(h); }

int orc_dequantize(uint32_t type, uint64_t n, const uint8_t* raw, uint64_t raw_len, float* out) {
  return dequantize(type, n, raw, raw_len, out, nullptr);
}

// GGUF header, metadata and tensor index as JSON. Returns the full length
// (write again with a larger buffer if it exceeds len), or -1 with the error in buf.
long orc_gguf_info_json(const char* path, char* buf, size_t len) {
  std::string err;
  auto g = gguf_open(path, &err);
  if (!g) { set_err(buf, len, err); return -1; }
  std::string o = "{\"version\":" + std::to_string(g->version) +
                  ",\"tensor_count\":" + std::to_string(g->tensor_count) +
                  ",\"kv_count\":" + std::to_string(g->kv_count) +
                  ",\"alignment\":" + std::to_string(g->alignment) +
                  ",\"data_start\":" + std::to_string(g->data_start) + ",\"metadata\":{";
  for (size_t i = 0; i < g->metadata.size(); i++)
    o += (i ? ",\"" : "\"") + json_escape(g->metadata[i].first) + "\":{\"type\":" +
         std::to_string(g->metadata[i].second.type) + ",\"value\":" + value_json(g->metadata[i].second) + "}";
  o += "},\"tensors\":[";
  for (size_t i = 0; i < g->tensors.size(); i++) {
    auto& t = g->tensors[i];
    o += (i ? ",{" : "{") + std::string("\"name\":\"") + json_escape(t.name) + "\",\"type\":" +
         std::to_string(t.type) + ",\"offset\":" + std::to_string(t.offset) +
         ",\"n_bytes\":" + std::to_string(t.n_bytes()) + ",\"dims\":[";
    for (size_t d = 0; d < t.dims.size(); d++) o += (d ? "," : "") + std::to_string(t.dims[d]);
    o += "]}";
  }
  o += "]}";
  if (o.size() + 1 <= len) std::memcpy(buf, o.c_str(), o.size() + 1);
  return (long)o.size();
}

// tensor_data_f32 (lib.rs:200-204): dequantized tensor into out[n_elements].
int orc_gguf_tensor_f32(const char* path, const char* name, float* out, uint64_t n, char* err, size_t errlen) {
  std::string e;
  auto g = gguf_open(path, &e);
  if (!g) { set_err(err, errlen, e); return -1; }
  const TensorInfo* t = g->tensor(name);
  if (!t) { set_err(err, errlen, std::string("tensor not found: ") + name); return -1; }
  if (t->n_elements() != n) { set_err(err, errlen, "size mismatch"); return -1; }
  const uint8_t* raw = g->raw(*t, &e);
  if (!raw) { set_err(err, errlen, e); return -1; }
  if (dequantize(t->type, n, raw, t->n_bytes(), out, &e) != 0) { set_err(err, errlen, e); return -1; }
  return 0;
}

void* orc_model_load(const char* path, int threads, char* err, size_t errlen) {
  std::string e;
  auto m = model_load(path, threads, &e);
  if (!m) { set_err(err, errlen, e); return nullptr; }
  return m.release();
}
void orc_model_free(void* m) { delete (Model*)m; }
void orc_model_set_threads(void* m, int threads) { ((Model*)m)->threads = threads < 1 ? 1 : threads; }
void orc_model_config(void* m, orc_config* out) {
  const Config& c = ((Model*)m)->c;
  out->n_layers = c.n_layers; out->n_embd = c.n_embd; out->n_ff = c.n_ff;
  out->n_heads = c.n_heads; out->n_kv_heads = c.n_kv_heads; out->head_dim = c.head_dim;
  out->rope_theta = c.rope_theta; out->rms_eps = c.rms_eps; out->vocab_size = c.vocab_size;
}
// The embedding row of a token exactly as the forward copies it.
void orc_model_embedding(void* m, uint32_t tok, float* out) { ((Model*)m)->tok_embd.row(tok, out); }

// Device::new_cache for qwen2 (qwen2.rs:633-637)
void* orc_cache_new(void* m, size_t max_seq) {
  const Config& c = ((Model*)m)->c;
  return new SeqState(SeqState::all_kv(c.n_layers, c.n_kv_heads * c.head_dim, max_seq));
}
void orc_cache_free(void* s) { delete (SeqState*)s; }
void* orc_cache_clone(void* s) { return new SeqState(*(SeqState*)s); }
size_t orc_cache_len(void* s) { return ((SeqState*)s)->len; }
size_t orc_cache_capacity(void* s) { return ((SeqState*)s)->capacity(); }
void orc_cache_advance(void* s, size_t n) { ((SeqState*)s)->advance(n); }
void orc_cache_reset(void* s) { ((SeqState*)s)->reset(); }
void orc_cache_ensure_capacity(void* s, size_t n) { ((SeqState*)s)->ensure_capacity(n); }
int orc_cache_truncate(void* s, size_t n, char* err, size_t errlen) {
  std::string e;
  int rc = ((SeqState*)s)->truncate(n, &e);
  if (rc) set_err(err, errlen, e);
  return rc;
}
// K and V rows of one position of one layer (kv_dim floats each).
int orc_cache_read_kv(void* s, size_t layer, size_t pos, float* k, float* v) {
  SeqState* st = (SeqState*)s;
  if (layer >= st->n_layers || pos >= st->cap) return -1;
  std::memcpy(k, st->k[layer].data() + pos * st->dim, st->dim * 4);
  std::memcpy(v, st->v[layer].data() + pos * st->dim, st->dim * 4);
  return 0;
}

int orc_forward_cached(void* m, void* s, const uint32_t* toks, size_t n, float* logits, char* err,
                       size_t errlen) {
  std::string e;
  int rc = forward_cached(*(Model*)m, toks, n, *(SeqState*)s, logits, &e);
  if (rc) set_err(err, errlen, e);
  return rc;
}

// Rng (sampling.rs:12-41): the state word after Rng::new(seed).
uint64_t orc_rng_new(uint64_t seed) { return Rng(seed).s; }
uint64_t orc_rng_next_u64(uint64_t* st) { Rng r(0); r.s = *st; uint64_t v = r.next_u64(); *st = r.s; return v; }
float orc_rng_next_f32(uint64_t* st) { Rng r(0); r.s = *st; float v = r.next_f32(); *st = r.s; return v; }

// Sampler::sample / sample_masked. top_k < 0 and top_p < 0 mean None.
size_t orc_sample(const float* logits, const uint8_t* mask, size_t n, float temperature, long top_k,
                  float top_p, uint64_t* rng_state) {
  Sampler smp;
  smp.temperature = temperature;
  smp.top_k = top_k;
  smp.top_p = top_p;
  Rng r(0);
  r.s = *rng_state;
  size_t out = mask ? smp.sample_masked(logits, mask, n, r) : smp.sample(logits, n, r);
  *rng_state = r.s;
  return out;
}

// Many Sampler::sample[_masked] draws, threaded over rows (each draw is the
// single-threaded reference computation): row i samples logits + i * ld
// (ld = 0: every row the same logits) with its own sampler and RNG state.
void orc_sample_batch(const float* logits, size_t ld, size_t n, const uint8_t* mask, size_t rows,
                      const float* temperature, const long* top_k, const float* top_p, uint64_t* rng_state,
                      uint64_t* out, int threads) {
  std::vector<std::thread> pool;
  const size_t nt = std::max<size_t>(1, std::min<size_t>((size_t)std::max(threads, 1), rows));
  for (size_t t = 0; t < nt; t++)
    pool.emplace_back([&, t] {
      for (size_t i = t; i < rows; i += nt) {
        Sampler smp;
        smp.temperature = temperature[i];
        smp.top_k = top_k[i];
        smp.top_p = top_p[i];
        Rng r(0);
        r.s = rng_state[i];
        const float* lg = logits + i * ld;
        out[i] = mask ? smp.sample_masked(lg, mask + i * ld, n, r) : smp.sample(lg, n, r);
        rng_state[i] = r.s;
      }
    });
  for (auto& th : pool) th.join();
}

// The sampler's softmax (sampling.rs:157-172) of one row, in place.
void orc_softmax(float* x, size_t n) { softmax_row_ref(x, n); }

// glibc's expf (Rust's f32::exp on x86-64 Linux) on n values, threaded.
void orc_expf_block(const float* x, float* y, size_t n, int threads) {
  std::vector<std::thread> pool;
  const size_t nt = std::max<size_t>(1, std::min<size_t>((size_t)std::max(threads, 1), n / 4096 + 1));
  for (size_t t = 0; t < nt; t++)
    pool.emplace_back([&, t] {
      for (size_t i = n * t / nt; i < n * (t + 1) / nt; i++) y[i] = expf(x[i]);
    });
  for (auto& th : pool) th.join();
}

// generate_tokens_seeded (generate.rs:149-250) over the oracle model.
typedef int (*orc_on_token_fn)(void* ud, uint32_t tok);
typedef int (*orc_masker_fn)(void* ud, uint8_t* mask, size_t n);
typedef int (*orc_stop_fn)(void* ud, const uint32_t* ids, size_t n);
typedef void (*orc_on_prefill_fn)(void* ud, void* cache);
typedef struct {
  uint64_t max_tokens;
  float temperature;
  int64_t top_k;  // <0: None
  float top_p;    // <0: None
  int32_t has_seed;
  uint64_t seed;
} orc_gen_params;
typedef struct {
  uint64_t n_ids;
  int32_t finish_stop;  // 1 "stop", 0 "length"
  uint64_t prompt_tokens;
  uint64_t prefix_reused;
  double elapsed_secs;
} orc_gen_result;

int orc_generate(void* model, const uint32_t* prompt, size_t n_prompt, const orc_gen_params* p,
                 const uint32_t* eos, size_t n_eos, orc_on_token_fn on_token, orc_masker_fn masker,
                 orc_stop_fn stop, orc_on_prefill_fn on_prefill, void* ud, void* seed_cache,
                 size_t seed_n, uint32_t* out_ids, orc_gen_result* res, char* err, size_t errlen) {
  Model& m = *(Model*)model;
  auto t0 = std::chrono::steady_clock::now();
  Sampler smp;
  smp.temperature = p->temperature;
  smp.top_k = p->top_k;
  smp.top_p = p->top_p;
  uint64_t seed = p->has_seed ? p->seed
                              : (uint64_t)std::chrono::duration_cast<std::chrono::nanoseconds>(
                                    std::chrono::system_clock::now().time_since_epoch()).count();
  Rng rng(seed);
  size_t max_seq = n_prompt + p->max_tokens;
  const size_t V = m.c.vocab_size;
  std::vector<float> logits(V);
  std::vector<uint8_t> mask(V);
  std::string e;
  SeqState owned;
  SeqState* cache;
  size_t prefix_reused = 0;
  uint32_t last;
  bool usable = seed_cache && n_prompt > 0 && seed_n > 0 && seed_n < n_prompt;
  if (usable) {
    cache = (SeqState*)seed_cache;
    if (forward_cached(m, prompt + seed_n, n_prompt - seed_n, *cache, logits.data(), &e)) {
      set_err(err, errlen, e);
      return -1;
    }
    if (on_prefill) on_prefill(ud, cache);
    prefix_reused = seed_n;
    last = prompt[n_prompt - 1];
  } else {
    owned = SeqState::all_kv(m.c.n_layers, m.c.n_kv_heads * m.c.head_dim, max_seq);
    cache = &owned;
    if (forward_cached(m, prompt, n_prompt, *cache, logits.data(), &e)) {
      set_err(err, errlen, e);
      return -1;
    }
    if (on_prefill) on_prefill(ud, cache);
    last = n_prompt ? prompt[n_prompt - 1] : 0;
  }
  (void)last;
  int stop_reason = 0;
  size_t n = 0;
  for (size_t step = 0; step < p->max_tokens; step++) {
    if (step > 0) {
      if (forward_cached(m, &last, 1, *cache, logits.data(), &e)) {
        set_err(err, errlen, e);
        return -1;
      }
    }
    bool has_mask = masker && masker(ud, mask.data(), V);
    Rng r = rng;
    uint32_t next = (uint32_t)(has_mask ? smp.sample_masked(logits.data(), mask.data(), V, r)
                                        : smp.sample(logits.data(), V, r));
    rng = r;
    out_ids[n++] = next;
    last = next;
    if (on_token && !on_token(ud, next)) { stop_reason = 1; break; }
    bool is_eos = false;
    for (size_t i = 0; i < n_eos; i++) is_eos |= eos[i] == next;
    if (is_eos) { stop_reason = 1; break; }
    if (stop && stop(ud, out_ids, n)) { stop_reason = 1; break; }
  }
  res->n_ids = n;
  res->finish_stop = stop_reason;
  res->prompt_tokens = n_prompt;
  res->prefix_reused = prefix_reused;
  res->elapsed_secs = std::chrono::duration<double>(std::chrono::steady_clock::now() - t0).count();
  return 0;
}

}  // extern "C"
