// Seeded synthetic qwen2/llama GGUF models (the stand-in for real model
// files, which are not available on the build or GPU machines).
//
// Tensor names, shapes and metadata keys are the ones the reference loader
// reads (crates/s-models/src/qwen2.rs:30-63, 99-150). Weight values are
// N(0, std) from a counter-based generator: element e of tensor t is a
// Box-Muller draw from splitmix64(key_t + e/2), so any row range can be
// produced independently and in parallel, with the same bytes every time.
// Quant types follow llama.cpp's Q4_K_M mix: Q6_K for attn_v, every other
// ffn_down (even layers), output and token_embd; Q4_K elsewhere; rows whose
// length is not a multiple of 256 fall back to Q5_0 (for Q4_K) or Q8_0 (for
// Q6_K). Norm weights are 1.0; qkv biases are N(0, std).
#include <fcntl.h>
#include <unistd.h>

#include <algorithm>
#include <cmath>
#include <cstdlib>
#include <thread>

#include "../../include/sm_engine.h"
#include "common.hpp"
#include "gguf.hpp"

namespace sm {
bool quantize_row(uint32_t t, const float* x, uint64_t n, uint8_t* out);
void normal_fill(uint64_t key, uint64_t e0, uint64_t n, float stdv, float* x);  // synth_normal.cpp

namespace {

inline uint64_t mix64(uint64_t z) {
  z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
  z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
  return z ^ (z >> 31);
}

enum Kind { K_NORMAL, K_ONES };

struct TSpec {
  std::string name;
  uint64_t n_in, n_out;  // GGUF dims [n_in, n_out]; 1-D tensors have n_out = 1
  uint32_t type;
  Kind kind;
  bool one_dim;
};

uint32_t pick(uint32_t want, uint64_t n_in, int32_t override_type) {
  if (override_type >= 0) want = (uint32_t)override_type;
  uint32_t bs, tb;
  if (!qtype_layout(want, &bs, &tb)) return QT_F32;
  if (n_in % bs == 0) return want;
  if (want == QT_Q4K) return n_in % 32 == 0 ? QT_Q5_0 : QT_F32;
  if (want == QT_Q6K) return n_in % 32 == 0 ? QT_Q8_0 : QT_F32;
  return QT_F32;
}

std::vector<TSpec> layout(const sm_synth_spec& s) {
  std::vector<TSpec> v;
  const uint64_t H = s.n_embd, F = s.n_ff, hd = s.n_embd / s.n_heads, kvd = hd * s.n_kv_heads;
  const int32_t ov = s.type_override;
  v.push_back({"token_embd.weight", H, s.vocab, pick(QT_Q6K, H, ov), K_NORMAL, false});
  v.push_back({"output_norm.weight", H, 1, QT_F32, K_ONES, true});
  if (!s.tied) v.push_back({"output.weight", H, s.vocab, pick(QT_Q6K, H, ov), K_NORMAL, false});
  for (uint32_t i = 0; i < s.n_layers; i++) {
    std::string p = "blk." + std::to_string(i) + ".";
    v.push_back({p + "attn_norm.weight", H, 1, QT_F32, K_ONES, true});
    v.push_back({p + "attn_q.weight", H, H, pick(QT_Q4K, H, ov), K_NORMAL, false});
    if (s.qkv_bias) v.push_back({p + "attn_q.bias", H, 1, QT_F32, K_NORMAL, true});
    v.push_back({p + "attn_k.weight", H, kvd, pick(QT_Q4K, H, ov), K_NORMAL, false});
    if (s.qkv_bias) v.push_back({p + "attn_k.bias", kvd, 1, QT_F32, K_NORMAL, true});
    v.push_back({p + "attn_v.weight", H, kvd, pick(QT_Q6K, H, ov), K_NORMAL, false});
    if (s.qkv_bias) v.push_back({p + "attn_v.bias", kvd, 1, QT_F32, K_NORMAL, true});
    v.push_back({p + "attn_output.weight", H, H, pick(QT_Q4K, H, ov), K_NORMAL, false});
    v.push_back({p + "ffn_norm.weight", H, 1, QT_F32, K_ONES, true});
    v.push_back({p + "ffn_gate.weight", H, F, pick(QT_Q4K, H, ov), K_NORMAL, false});
    v.push_back({p + "ffn_up.weight", H, F, pick(QT_Q4K, H, ov), K_NORMAL, false});
    v.push_back({p + "ffn_down.weight", F, H, pick(i % 2 == 0 ? QT_Q6K : QT_Q4K, F, ov), K_NORMAL, false});
  }
  return v;
}

struct Sink {
  uint8_t* mem = nullptr;  // memory mode
  int fd = -1;             // file mode
  bool write(uint64_t off, const uint8_t* p, uint64_t n) {
    if (mem) { std::memcpy(mem + off, p, n); return true; }
    while (n) {
      ssize_t w = pwrite(fd, p, n, (off_t)off);
      if (w <= 0) return false;
      p += w; off += (uint64_t)w; n -= (uint64_t)w;
    }
    return true;
  }
};

bool produce(const sm_synth_spec& s, Sink& sink, int threads, uint64_t* total_len) {
  auto specs = layout(s);
  GgufWriter w;
  const char* arch = s.arch == 0 ? "qwen2" : "llama";
  w.kv_str("general.architecture", arch);
  w.kv_str("general.name", std::string("synthetic-") + arch);
  w.kv_u32("general.alignment", 32);
  w.kv_u32("general.file_type", 15);  // MOSTLY_Q4_K_M
  std::string a = arch;
  w.kv_u32(a + ".block_count", s.n_layers);
  w.kv_u32(a + ".context_length", 32768);
  w.kv_u32(a + ".embedding_length", s.n_embd);
  w.kv_u32(a + ".feed_forward_length", s.n_ff);
  w.kv_u32(a + ".attention.head_count", s.n_heads);
  w.kv_u32(a + ".attention.head_count_kv", s.n_kv_heads);
  w.kv_f32(a + ".rope.freq_base", s.rope_theta);
  w.kv_f32(a + ".attention.layer_norm_rms_epsilon", s.rms_eps);
  for (auto& t : specs)
    w.add_tensor(t.name, t.one_dim ? std::vector<uint64_t>{t.n_in} : std::vector<uint64_t>{t.n_in, t.n_out}, t.type);
  auto hdr = w.header();
  *total_len = hdr.size() + w.data_bytes();
  if (sink.mem == nullptr && sink.fd < 0) return true;  // size query only
  if (!sink.write(0, hdr.data(), hdr.size())) return false;
  const uint64_t base = hdr.size();
  if (threads < 1) threads = 1;
  bool ok = true;
  for (size_t ti = 0; ti < specs.size() && ok; ti++) {
    const TSpec& t = specs[ti];
    const uint64_t key = mix64(s.seed ^ (0xA24BAED4963EE407ull * (ti + 1)));
    const uint64_t rb = qtype_row_bytes(t.type, t.n_in);
    const uint64_t off = base + w.tensor_offset(ti);
    const uint64_t rows = t.n_out;
    const int nt = (int)std::min<uint64_t>((uint64_t)threads, std::max<uint64_t>(1, rows / 16));
    std::vector<std::thread> pool;
    std::vector<int> res(nt, 1);
    for (int k = 0; k < nt; k++) {
      pool.emplace_back([&, k] {
        uint64_t r0 = rows * k / nt, r1 = rows * (k + 1) / nt;
        const uint64_t chunk = std::max<uint64_t>(1, (8u << 20) / std::max<uint64_t>(rb, 1));
        std::vector<float> x;
        std::vector<uint8_t> q;
        for (uint64_t r = r0; r < r1; r += chunk) {
          uint64_t nr = std::min(chunk, r1 - r);
          x.resize(nr * t.n_in);
          q.resize(nr * rb);
          if (t.kind == K_ONES) std::fill(x.begin(), x.end(), 1.0f);
          else normal_fill(key, r * t.n_in, nr * t.n_in, s.weight_std, x.data());
          for (uint64_t i = 0; i < nr; i++)
            if (!quantize_row(t.type, x.data() + i * t.n_in, t.n_in, q.data() + i * rb)) { res[k] = 0; return; }
          if (!sink.write(off + r * rb, q.data(), nr * rb)) { res[k] = 0; return; }
        }
      });
    }
    for (auto& th : pool) th.join();
    for (int r : res) ok &= r == 1;
    // alignment padding after the tensor
    uint64_t pad = (t.n_in * t.n_out == 0) ? 0 : ((rows * rb + 31) / 32 * 32 - rows * rb);
    if (ok && pad) {
      uint8_t z[32] = {0};
      ok = sink.write(off + rows * rb, z, pad);
    }
  }
  return ok;
}

bool valid(const sm_synth_spec* s) {
  return s && s->n_embd && s->n_layers && s->n_heads && s->n_kv_heads && s->n_ff && s->vocab &&
         s->n_embd % s->n_heads == 0 && s->n_heads % s->n_kv_heads == 0 && (s->n_embd / s->n_heads) % 2 == 0 &&
         (s->arch == 0 || s->arch == 1);
}

}  // namespace
}  // namespace sm

using namespace sm;

extern "C" {

int sm_synth_preset(int config_index, sm_synth_spec* o) {
  if (!o) { set_error("sm_synth_preset: null spec"); return SM_ERR_ARG; }
  std::memset(o, 0, sizeof *o);
  o->seed = 0;
  o->weight_std = 0.02f;
  o->type_override = -1;
  switch (config_index) {
    case 0:  // Qwen2.5-0.5B shape
      *o = {0, 896, 24, 14, 2, 4864, 151936, 1e6f, 1e-6f, 1, 1, 0, 0.02f, -1};
      return SM_OK;
    case 2:  // Qwen2.5-7B shape
      *o = {0, 3584, 28, 28, 4, 18944, 152064, 1e6f, 1e-6f, 1, 0, 0, 0.02f, -1};
      return SM_OK;
    case 3:  // Llama-3-8B shape
      *o = {1, 4096, 32, 32, 8, 14336, 128256, 5e5f, 1e-5f, 0, 0, 0, 0.02f, -1};
      return SM_OK;
    case 4:  // Llama-3-70B shape
      *o = {1, 8192, 80, 64, 8, 28672, 128256, 5e5f, 1e-5f, 0, 0, 0, 0.02f, -1};
      return SM_OK;
    default:
      set_error("sm_synth_preset: configs are 0, 2, 3 and 4");
      return SM_ERR_ARG;
  }
}

int sm_synth_size(const sm_synth_spec* s, uint64_t* len) {
  if (!valid(s) || !len) { set_error("sm_synth_size: invalid spec"); return SM_ERR_ARG; }
  Sink sink;
  sink.fd = -1;
  return produce(*s, sink, 1, len) ? SM_OK : SM_ERR_ARG;
}

int sm_synth_write(const sm_synth_spec* s, const char* path, int threads) {
  if (!valid(s) || !path) { set_error("sm_synth_write: invalid spec"); return SM_ERR_ARG; }
  uint64_t len = 0;
  if (sm_synth_size(s, &len) != SM_OK) return SM_ERR_ARG;
  std::string tmp = std::string(path) + ".partial";
  int fd = ::open(tmp.c_str(), O_CREAT | O_TRUNC | O_WRONLY, 0644);
  if (fd < 0) { set_error(std::string("io: cannot create ") + tmp); return SM_ERR_IO; }
  Sink sink;
  sink.fd = fd;
  bool ok = ftruncate(fd, (off_t)len) == 0 && produce(*s, sink, threads, &len);
  ok = (::close(fd) == 0) && ok;
  if (!ok || rename(tmp.c_str(), path) != 0) {
    unlink(tmp.c_str());
    set_error(std::string("io: writing ") + path + " failed");
    return SM_ERR_IO;
  }
  return SM_OK;
}

int sm_synth_memory(const sm_synth_spec* s, int threads, void** buf, uint64_t* len) {
  if (!valid(s) || !buf || !len) { set_error("sm_synth_memory: invalid spec"); return SM_ERR_ARG; }
  if (sm_synth_size(s, len) != SM_OK) return SM_ERR_ARG;
  uint8_t* mem = (uint8_t*)std::calloc(1, *len);
  if (!mem) { set_error("sm_synth_memory: out of host memory"); return SM_ERR_OOM; }
  Sink sink;
  sink.mem = mem;
  if (!produce(*s, sink, threads, len)) { std::free(mem); set_error("sm_synth_memory: failed"); return SM_ERR_ARG; }
  *buf = mem;
  return SM_OK;
}

void sm_synth_free(void* buf) { std::free(buf); }

// Quantizes n f32 values (a whole number of blocks) into ggml type `type`.
int sm_quantize(uint32_t type, const float* x, uint64_t n, void* out) {
  if (!x || !out) { set_error("sm_quantize: null pointer"); return SM_ERR_ARG; }
  if (!quantize_row(type, x, n, (uint8_t*)out)) { set_error("sm_quantize: unsupported type or size"); return SM_ERR_ARG; }
  return SM_OK;
}

}  // extern "C"
