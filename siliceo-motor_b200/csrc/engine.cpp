// Engine runtime: model load into HBM, sequence caches, forward passes,
// batched decode steps captured in CUDA graphs, and the C ABI over them.
//
// Replaces, for qwen2/llama: s_models::qwen2::Model as `impl Device`
// (crates/s-models/src/qwen2.rs:625-642), s_backend_cuda::model::GpuQwen2
// (crates/s-backend-cuda/src/model.rs:107-629) and SeqState
// (crates/s-models/src/state.rs:202-361).
#include <cuda_runtime.h>

#include <atomic>
#include <chrono>
#include <cmath>
#include <unordered_map>
#include <initializer_list>
#include <map>
#include <memory>
#include <mutex>
#include <string>
#include <thread>
#include <vector>

#include "../../include/sm_engine.h"
#include "common.hpp"
#include "gguf.hpp"
#include "layers.cuh"
#include "tp.hpp"

using namespace sm;

namespace {

#define CK(expr)                                                                         \
  do {                                                                                   \
    cudaError_t e_ = (expr);                                                             \
    if (e_ != cudaSuccess) {                                                             \
      set_error(std::string("cuda: ") + cudaGetErrorString(e_) + " at " #expr);         \
      return SM_ERR_CUDA;                                                                \
    }                                                                                    \
  } while (0)

// ------------------------------------------------------ device weights ----
struct DW {
  DWDesc d{};
  void* mem = nullptr;
  uint64_t enc_bytes = 0;  // bytes of the GGUF encoding
};

bool engine_type(uint32_t t) { return t == QT_Q4K || t == QT_Q6K || t == QT_Q8_0 || t == QT_Q5_0; }

// GGUF rows -> engine HBM layout (see device.cuh). Returns the status.
int upload_weight(uint32_t type, const uint8_t* src, uint64_t n_out, uint64_t n_in, DW* out) {
  if (!engine_type(type)) {
    set_error("unsupported weight type " + std::to_string(type) + " (engine handles Q4_K, Q6_K, Q5_0, Q8_0)");
    return SM_ERR_UNSUPPORTED;
  }
  uint32_t bs = 1, tb = 4;
  qtype_layout(type, &bs, &tb);
  if (n_in % bs != 0 || n_out == 0 || n_out > 0xFFFFFFFFull || n_in > 0xFFFFFFFFull) {
    set_error("weight shape not supported: n_in must be a multiple of " + std::to_string(bs));
    return SM_ERR_UNSUPPORTED;
  }
  const uint64_t nb = n_in / bs, row_src = nb * tb;
  const bool tiled = tiled_type(type);
  const uint64_t n_tiles = (n_out + 15) / 16;
  uint64_t body_stride = 0, aux_stride = 0;
  switch (type) {
    case QT_Q4K: body_stride = nb * Q4T_UNIT; break;  // per 16-row tile
    case QT_Q6K: body_stride = nb * Q6T_UNIT; break;
    case QT_Q8_0: body_stride = nb * 32; aux_stride = nb * 2; break;
    case QT_Q5_0: body_stride = nb * 16; aux_stride = nb * 8; break;
  }
  if (body_stride > 0xFFFFFFFFull) {
    set_error("weight row too long");
    return SM_ERR_UNSUPPORTED;
  }
  aux_stride = (aux_stride + 15) / 16 * 16;
  const uint64_t body_bytes = tiled ? body_stride * n_tiles : body_stride * n_out, aux_bytes = aux_stride * n_out;
  std::vector<uint8_t> body(body_bytes, 0), aux(aux_bytes, 0);
  // Rows are repacked independently (a tile's rows write disjoint bytes), in
  // parallel over ranges of whole tiles; padding rows of the last tile stay
  // zero (d = 0).
  auto repack = [&](uint64_t o_begin, uint64_t o_end) {
    uint8_t v6[256];
    for (uint64_t o = o_begin; o < o_end; o++) {
      const uint8_t* r = src + o * row_src;
      const uint32_t rr = (uint32_t)(o & 15);
      uint8_t* tile = body.data() + (o >> 4) * body_stride;
      uint8_t* bd = body.data() + o * body_stride;
      uint8_t* ax = aux.data() + o * aux_stride;
      switch (type) {
        case QT_Q4K:  // 16-row tiles (device.cuh)
          for (uint32_t b = 0; b < nb; b++) {
            const uint8_t* blk = r + (size_t)b * 144;  // d | dmin | scales 12 | qs 128
            uint8_t* u = tile + (size_t)b * Q4T_UNIT;
            std::memcpy(u + 16 * rr, blk, 16);
            for (uint32_t q = 0; q < 128; q++) u[q4t_qs_off(rr, q)] = blk[16 + q];
          }
          break;
        case QT_Q6K:
          for (uint32_t b = 0; b < nb; b++) {
            const uint8_t* blk = r + (size_t)b * 210;  // ql 128 | qh 64 | scales 16 | d 2 (dequant.rs:178-206)
            uint8_t* u = tile + (size_t)b * Q6T_UNIT;
            for (uint32_t l = 0; l < 256; l++) {  // 6-bit value q + 32 of weight l
              const uint32_t n = l >> 7, k = (l & 127) >> 5, ll = l & 31;
              const uint32_t qlb = blk[64 * n + ll + 32 * (k & 1)];
              const uint32_t lo = (k >> 1) ? (qlb >> 4) : (qlb & 0x0F);
              const uint32_t hi = (blk[128 + 32 * n + ll] >> (2 * k)) & 3;
              v6[l] = (uint8_t)(lo | (hi << 4));
            }
            for (uint32_t l = 0; l < 256; l++) {  // into the words of device.cuh (the unit starts zeroed)
              const uint32_t sb = l >> 4, w = l & 15, G = sb >> 2, sg = sb & 3, c = w >> 3, pp = (w >> 2) & 1,
                             bb = w & 3, v = v6[l];
              u[q6t_word_off(rr, sg & 1, G, c, pp) + bb] |= (uint8_t)((v & 15) << (4 * (sg >> 1)));
              const uint32_t hs = sg == 0 ? 4 : sg == 1 ? 0 : sg == 2 ? 6 : 2;
              u[q6t_word_off(rr, 2, G, c, pp) + bb] |= (uint8_t)((v >> 4) << hs);
            }
            std::memcpy(u + 16 * rr, blk + 192, 16);
            std::memcpy(u + 256 + 2 * rr, blk + 208, 2);
          }
          break;
        case QT_Q8_0:
          for (uint64_t b = 0; b < nb; b++) {
            std::memcpy(ax + b * 2, r + b * 34, 2);
            std::memcpy(bd + b * 32, r + b * 34 + 2, 32);
          }
          break;
        case QT_Q5_0:
          for (uint64_t b = 0; b < nb; b++) {
            std::memcpy(ax + b * 8 + 4, r + b * 22, 2);  // d
            std::memcpy(ax + b * 8, r + b * 22 + 2, 4);  // qh
            std::memcpy(bd + b * 16, r + b * 22 + 6, 16);
          }
          break;
      }
    }
  };
  {
    const uint64_t work = n_out * nb;
    const unsigned hw = std::max(1u, std::thread::hardware_concurrency());
    const uint64_t nt = std::min<uint64_t>(hw, std::max<uint64_t>(1, work / (1u << 16)));
    std::vector<std::thread> pool;
    for (uint64_t k = 1; k < nt; k++)
      pool.emplace_back(repack, std::min(n_out, 16 * (n_tiles * k / nt)), std::min(n_out, 16 * (n_tiles * (k + 1) / nt)));
    repack(0, std::min(n_out, 16 * (n_tiles / nt)));
    for (auto& t : pool) t.join();
  }
  void* mem = nullptr;
  const uint64_t total = body_bytes + aux_bytes + 256;
  if (cudaMalloc(&mem, total) != cudaSuccess) {
    cudaGetLastError();
    set_error("cudaMalloc failed for a weight of " + std::to_string(total) + " bytes");
    return SM_ERR_OOM;
  }
  uint8_t* base = (uint8_t*)mem;
  uint8_t* auxp = base + (body_bytes + 255) / 256 * 256;
  CK(cudaMemcpy(base, body.data(), body_bytes, cudaMemcpyHostToDevice));
  if (aux_bytes) CK(cudaMemcpy(auxp, aux.data(), aux_bytes, cudaMemcpyHostToDevice));
  out->mem = mem;
  out->enc_bytes = row_src * n_out;
  out->d.body = base;
  out->d.aux = aux_bytes ? auxp : base;
  out->d.type = type;
  out->d.n_out = (uint32_t)n_out;
  out->d.n_in = (uint32_t)n_in;
  out->d.body_stride = (uint32_t)body_stride;
  out->d.aux_stride = (uint32_t)aux_stride;
  return SM_OK;
}

GemvSeg seg(const DW& w, float* y, uint32_t ldy, const float* bias, uint32_t epi) {
  GemvSeg s{};
  s.w = w.d;
  s.y = y;
  s.ldy = ldy;
  s.bias = bias;
  s.epi = epi;
  return s;
}

void free_weight(DW& w) {
  if (w.mem) cudaFree(w.mem);
  w.mem = nullptr;
}

// Per-layer weights. wq / wk (and bq / bk) hold their rows in RoPE-pair
// order: physical row h*hd + 2m + s is logical row h*hd + m + s*hd/2, so one
// warp sees both halves of every rotated pair. wgu interleaves ffn_gate and
// ffn_up: physical row 2m is gate row m, 2m+1 is up row m.
struct Layer {
  float* attn_norm = nullptr;
  float* ffn_norm = nullptr;
  float* bq = nullptr;
  float* bk = nullptr;
  float* bv = nullptr;
  DW wq, wk, wv, wo, wgu, wdown;
};

// Per-step host->device state, one pinned block copied with one memcpy.
struct StepIn {
  uint32_t* tok;        // [rows]
  RowDesc* rows;        // [rows]
  SeqDesc* seqs;        // [rows]
  SampleParams* sp;     // [rows]
  uint64_t* rng;        // [rows]
  uint32_t* sel;        // [rows]
  uint32_t* shared;     // [1]: leading KV pages all rows of a batched step share (attention reads them once)
};
struct StepOut {
  uint32_t* tok;  // [rows]
  uint64_t* rng;  // [rows]
  uint32_t* err;  // error word of the bounded waits (GEMV copy rings, tensor-parallel peers)
};

}  // namespace

// A sequence state (SeqState): its KV pages (device.cuh) in position order.
// Pages are shared between clones (reference counted by the model) and
// copied before a shared page is written; a page that was never written is
// absent and reads as zeros.
struct sm_cache {
  sm_model* m = nullptr;
  std::vector<float*> pages;    // page t's base or nullptr, t < ceil(cap / KV_PAGE)
  float** pages_dev = nullptr;  // the same array on the device, for the kernels
  uint64_t cap = 0, len = 0;
  bool dirty = true;            // pages_dev is behind pages
};

struct sm_model {
  int device = 0;
  cudaStream_t stream = nullptr;
  SideStream side{nullptr, nullptr, nullptr};  // the shared-prefix attention pass of batched steps
  sm_config c{};
  uint32_t kvd = 0;  // this rank's KV width (kv heads x head_dim)
  // Tensor parallelism (sh.world == 1: none): the shard plan, the group, and
  // this rank's attention width (q heads x head_dim) and FFN width.
  TpShard sh;
  TpGroup* tp = nullptr;
  uint32_t qd = 0, fl = 0;
  bool failed = false;  // a bounded wait gave up: results are invalid from then on
  DW tok_embd, output;
  bool tied = false;
  float* output_norm = nullptr;
  std::vector<Layer> layers;
  float* cos_t = nullptr;
  float* sin_t = nullptr;
  uint32_t max_ctx = 0;
  uint32_t rows_max = 0, max_splits = 32 + ATT_SHARED_SPLITS;  // attention partial slots per (row, head)
  // workspace
  float *x = nullptr, *xn = nullptr, *q = nullptr, *k = nullptr, *v = nullptr, *att = nullptr, *g = nullptr,
        *u = nullptr, *logits = nullptr, *part_o = nullptr, *part_ml = nullptr;
  // K-split scratch of the batch-1 tensor-core GEMVs (counters zeroed at load)
  float* ks_part = nullptr;
  uint32_t* ks_cnt = nullptr;
  uint32_t ks_part_cap = 0, ks_cnt_cap = 0;
  // x images of the tcgen05 batched GEMV (one launch at a time, stream order)
  uint8_t* xblob = nullptr;
  uint64_t xblob_cap = 0;
  // Batched steps whose V weight has another type than Q and K run the V
  // GEMV on the side stream beside the Q+K one (each launch's time is mostly
  // its fixed latency): its own scratch, and how many CTAs each may use.
  bool qkv_side = false;
  uint32_t qk_cap = 0, v_cap = 0;
  float* ks_part2 = nullptr;
  uint32_t* ks_cnt2 = nullptr;
  uint32_t ks_part2_cap = 0, ks_cnt2_cap = 0;
  uint8_t* xblob2 = nullptr;
  uint64_t xblob2_cap = 0;
  cudaEvent_t qkv_join = nullptr;
  // partial sums of x^2 written by residual GEMVs, read by the next GEMV
  float *parts_a = nullptr, *parts_b = nullptr;
  uint32_t parts_cap = 0;
  uint8_t* mask_dev = nullptr;
  uint32_t* smp_scratch = nullptr;  // the sampler's per-row scratch (sample_scratch_words(V) words a row)
  uint64_t* amax = nullptr;         // the batch-1 output head's per-tile argmax keys
  uint32_t amax_n = 0;
  void* in_dev = nullptr;   // StepIn block on the device
  void* in_host = nullptr;  // pinned
  void* out_dev = nullptr;  // StepOut block on the device
  void* out_host = nullptr; // pinned
  size_t in_bytes = 0, out_bytes = 0;
  StepIn din{}, hin{};
  StepOut dout{}, hout{};
  std::vector<void*> allocs;
  // KV pages of all the model's caches: chunks of device memory cut into pages
  // of 2 * voff floats, a free list and reference counts.
  uint32_t kv_voff = 0;
  std::vector<void*> page_chunks;
  std::vector<float*> free_pages;
  std::unordered_map<float*, uint32_t> page_refs;
  std::map<uint32_t, cudaGraphExec_t> graphs;       // one step, state from the host
  std::map<uint32_t, cudaGraphExec_t> run_graphs;   // one step, state carried on the device
  std::map<uint32_t, uint64_t> run_graph_kernels;    // kernel launches in each of them
  uint32_t* hist = nullptr;  // [HIST_TOKENS] tokens recorded by decode runs
  uint32_t* hist_ctr = nullptr;
  std::mutex mu;
  uint64_t weight_bytes = 0;
  // The user's handle and every live cache hold a reference; the model (and
  // its device memory) is destroyed when the last one is released.
  std::atomic<int> refs{1};
};

namespace {

constexpr uint32_t HIST_TOKENS = 1u << 16;

template <class T>
void carve(uint8_t*& p, T*& out, size_t n) {
  out = reinterpret_cast<T*>(p);
  p += (n * sizeof(T) + 255) / 256 * 256;
}

size_t step_in_bytes(uint32_t R) {
  return 7 * 256 + (size_t)R * (sizeof(uint32_t) * 2 + sizeof(RowDesc) + sizeof(SeqDesc) + sizeof(SampleParams) +
                                sizeof(uint64_t));
}
void layout_in(void* base, uint32_t R, StepIn& s) {
  uint8_t* p = (uint8_t*)base;
  carve(p, s.tok, R);
  carve(p, s.rows, R);
  carve(p, s.seqs, R);
  carve(p, s.sp, R);
  carve(p, s.rng, R);
  carve(p, s.sel, R);
  carve(p, s.shared, 1);
}
size_t step_out_bytes(uint32_t R) { return 3 * 256 + (size_t)R * (sizeof(uint32_t) + sizeof(uint64_t)) + 4; }
void layout_out(void* base, uint32_t R, StepOut& s) {
  uint8_t* p = (uint8_t*)base;
  carve(p, s.tok, R);
  carve(p, s.rng, R);
  carve(p, s.err, 1);
}

int dev_alloc(sm_model* m, void** p, size_t bytes) {
  if (cudaMalloc(p, bytes) != cudaSuccess) {
    cudaGetLastError();
    set_error("cudaMalloc of " + std::to_string(bytes) + " bytes failed");
    return SM_ERR_OOM;
  }
  m->allocs.push_back(*p);
  return SM_OK;
}

int upload_f32(sm_model* m, const GgufReader& g, const std::string& name, size_t n, float** out) {
  const GgufTensor* t = g.tensor(name);
  if (!t) { set_error("tensor not found: " + name); return SM_ERR_FORMAT; }
  if (t->type != QT_F32 || t->n_elements() != n) {
    set_error(name + ": expected an F32 tensor of " + std::to_string(n) + " elements");
    return SM_ERR_UNSUPPORTED;
  }
  const uint8_t* src = g.data(*t);
  if (!src) { set_error(name + ": truncated tensor data"); return SM_ERR_FORMAT; }
  int rc = dev_alloc(m, (void**)out, n * 4);
  if (rc) return rc;
  CK(cudaMemcpy(*out, src, n * 4, cudaMemcpyHostToDevice));
  return SM_OK;
}

int upload_2d(const GgufReader& g, const std::string& name, uint64_t n_in, uint64_t n_out, DW* w) {
  const GgufTensor* t = g.tensor(name);
  if (!t) { set_error("tensor not found: " + name); return SM_ERR_FORMAT; }
  if (t->dims.size() != 2 || t->dims[0] != n_in || t->dims[1] != n_out) {
    set_error(name + ": unexpected shape");
    return SM_ERR_FORMAT;
  }
  const uint8_t* src = g.data(*t);
  if (!src) { set_error(name + ": truncated tensor data"); return SM_ERR_FORMAT; }
  int rc = upload_weight(t->type, src, n_out, n_in, w);
  if (rc) set_error(name + ": " + get_error());
  return rc;
}

// Uploads rows of a 2-D tensor [n_out x n_in], reordered and possibly a
// subset: physical row p is logical row map[p].
int upload_2d_rows(const GgufReader& g, const std::string& name, uint64_t n_in, uint64_t n_out,
                   const std::vector<uint32_t>& map, DW* w) {
  const GgufTensor* t = g.tensor(name);
  if (!t) { set_error("tensor not found: " + name); return SM_ERR_FORMAT; }
  if (t->dims.size() != 2 || t->dims[0] != n_in || t->dims[1] != n_out) { set_error(name + ": unexpected shape"); return SM_ERR_FORMAT; }
  const uint8_t* src = g.data(*t);
  if (!src) { set_error(name + ": truncated tensor data"); return SM_ERR_FORMAT; }
  const uint64_t rb = qtype_row_bytes(t->type, n_in), n_loc = map.size();
  std::vector<uint8_t> buf(rb * n_loc);
  for (uint64_t p = 0; p < n_loc; p++) std::memcpy(buf.data() + p * rb, src + (uint64_t)map[p] * rb, rb);
  int rc = upload_weight(t->type, buf.data(), n_loc, n_in, w);
  if (rc) set_error(name + ": " + get_error());
  return rc;
}

// RoPE-pair row order for heads [h0, h0 + n_heads) of a projection (see Layer).
std::vector<uint32_t> rope_pair_map(uint64_t n_heads, uint64_t hd, uint64_t h0 = 0) {
  std::vector<uint32_t> map(n_heads * hd);
  const uint64_t half = hd / 2;
  for (uint64_t h = 0; h < n_heads; h++)
    for (uint64_t mm = 0; mm < half; mm++)
      for (uint64_t sdx = 0; sdx < 2; sdx++)
        map[h * hd + 2 * mm + sdx] = (uint32_t)((h0 + h) * hd + mm + sdx * half);
  return map;
}

std::vector<uint32_t> range_map(uint64_t first, uint64_t n) {
  std::vector<uint32_t> map(n);
  for (uint64_t i = 0; i < n; i++) map[i] = (uint32_t)(first + i);
  return map;
}

// Uploads input columns [c0, c0 + nc) of every row of a 2-D tensor (the row
// split of tensor parallelism): whole quant blocks of each row.
int upload_2d_cols(const GgufReader& g, const std::string& name, uint64_t n_in, uint64_t n_out, uint64_t c0,
                   uint64_t nc, DW* w) {
  const GgufTensor* t = g.tensor(name);
  if (!t) { set_error("tensor not found: " + name); return SM_ERR_FORMAT; }
  if (t->dims.size() != 2 || t->dims[0] != n_in || t->dims[1] != n_out) { set_error(name + ": unexpected shape"); return SM_ERR_FORMAT; }
  const uint8_t* src = g.data(*t);
  if (!src) { set_error(name + ": truncated tensor data"); return SM_ERR_FORMAT; }
  uint32_t bs = 1, tb = 4;
  if (!qtype_layout(t->type, &bs, &tb) || c0 % bs || nc % bs || c0 + nc > n_in) {
    set_error(name + ": the tensor-parallel split of its " + std::to_string(n_in) +
              " input columns does not fall on quant block boundaries");
    return SM_ERR_UNSUPPORTED;
  }
  const uint64_t rb = qtype_row_bytes(t->type, n_in), lb = nc / bs * tb, o0 = c0 / bs * tb;
  std::vector<uint8_t> buf(lb * n_out);
  for (uint64_t r = 0; r < n_out; r++) std::memcpy(buf.data() + r * lb, src + r * rb + o0, lb);
  int rc = upload_weight(t->type, buf.data(), n_out, nc, w);
  if (rc) set_error(name + ": " + get_error());
  return rc;
}

// Rows [f0, f0 + fl) of ffn_gate and ffn_up interleaved row by row into one
// weight (see Layer).
int upload_gate_up(const GgufReader& g, const std::string& pg, const std::string& pu, uint64_t n_in, uint64_t n_ff,
                   uint64_t f0, uint64_t fl, DW* w) {
  const GgufTensor* tg = g.tensor(pg);
  const GgufTensor* tu = g.tensor(pu);
  if (!tg || !tu) { set_error("tensor not found: " + (tg ? pu : pg)); return SM_ERR_FORMAT; }
  for (const GgufTensor* t : {tg, tu})
    if (t->dims.size() != 2 || t->dims[0] != n_in || t->dims[1] != n_ff) { set_error(t->name + ": unexpected shape"); return SM_ERR_FORMAT; }
  if (tg->type != tu->type) { set_error(pg + " and " + pu + " have different types"); return SM_ERR_UNSUPPORTED; }
  const uint8_t* sg_ = g.data(*tg);
  const uint8_t* su = g.data(*tu);
  if (!sg_ || !su) { set_error(pg + ": truncated tensor data"); return SM_ERR_FORMAT; }
  const uint64_t rb = qtype_row_bytes(tg->type, n_in);
  std::vector<uint8_t> buf(rb * 2 * fl);
  for (uint64_t r = 0; r < fl; r++) {
    std::memcpy(buf.data() + (2 * r) * rb, sg_ + (f0 + r) * rb, rb);
    std::memcpy(buf.data() + (2 * r + 1) * rb, su + (f0 + r) * rb, rb);
  }
  int rc = upload_weight(tg->type, buf.data(), 2 * fl, n_in, w);
  if (rc) set_error(pg + ": " + get_error());
  return rc;
}

int load_model(const GgufReader& g, const sm_load_opts* opts, sm_model* m) {
  // Famiglia::detect (crates/s-models/src/registry.rs:38-60)
  const GgufValue* arch = g.meta("general.architecture");
  if (!arch || arch->type != 8) { set_error("missing metadata: general.architecture"); return SM_ERR_FORMAT; }
  if (arch->s != "qwen2" && arch->s != "llama") {
    set_error("architecture '" + arch->s + "' not supported (qwen2, llama)");
    return SM_ERR_UNSUPPORTED;
  }
  // Config::from_gguf (qwen2.rs:30-63): "qwen2." keys first, then "llama."
  auto get_u = [&](const char* suf, uint64_t* out) -> int {
    for (const char* pre : {"qwen2", "llama"}) {
      const GgufValue* v = g.meta(std::string(pre) + "." + suf);
      if (v) {
        if (!v->as_u64(out)) { set_error(std::string(pre) + "." + suf + ": unexpected type"); return SM_ERR_FORMAT; }
        return SM_OK;
      }
    }
    set_error(std::string("missing metadata: ") + suf);
    return SM_ERR_FORMAT;
  };
  auto get_f = [&](const char* suf, float* out) -> int {
    for (const char* pre : {"qwen2", "llama"}) {
      const GgufValue* v = g.meta(std::string(pre) + "." + suf);
      if (v) {
        if (!v->as_f32(out)) { set_error(std::string(pre) + "." + suf + ": unexpected type"); return SM_ERR_FORMAT; }
        return SM_OK;
      }
    }
    set_error(std::string("missing metadata: ") + suf);
    return SM_ERR_FORMAT;
  };
  sm_config& c = m->c;
  int rc;
  if ((rc = get_u("embedding_length", &c.n_embd)) || (rc = get_u("attention.head_count", &c.n_heads)) ||
      (rc = get_u("attention.head_count_kv", &c.n_kv_heads)) || (rc = get_u("block_count", &c.n_layers)) ||
      (rc = get_u("feed_forward_length", &c.n_ff)) || (rc = get_f("rope.freq_base", &c.rope_theta)) ||
      (rc = get_f("attention.layer_norm_rms_epsilon", &c.rms_eps)))
    return rc;
  if (!c.n_heads || !c.n_kv_heads || c.n_heads % c.n_kv_heads) { set_error("bad head counts"); return SM_ERR_FORMAT; }
  c.head_dim = c.n_embd / c.n_heads;
  const GgufTensor* te = g.tensor("token_embd.weight");
  if (!te || te->dims.size() != 2) { set_error("tensor not found: token_embd.weight"); return SM_ERR_FORMAT; }
  c.vocab_size = te->dims[1];
  const uint64_t H = c.n_embd, hd = c.head_dim, G = c.n_heads / c.n_kv_heads, kvd_full = c.n_kv_heads * hd;
  // Tensor-parallel shard of this rank (world 1: the whole model).
  const uint32_t world = opts && opts->tp_size > 1 ? opts->tp_size : 1, rank = world > 1 ? opts->tp_rank : 0;
  if (world > 1 && !opts->tp_group) { set_error("tensor parallelism needs the group id (tp_group)"); return SM_ERR_ARG; }
  if (world > 1 && rank >= world) { set_error("tp_rank must be below tp_size"); return SM_ERR_ARG; }
  {
    const std::string why = tp_plan(c.n_heads, c.n_kv_heads, hd, c.n_ff, c.vocab_size, 0, 0, rank, world, &m->sh);
    if (!why.empty()) { set_error(why); return SM_ERR_UNSUPPORTED; }
  }
  const TpShard& sh = m->sh;
  const uint64_t qd = sh.q_heads * hd, kvd = sh.kv_heads * hd, fl = sh.ff;
  m->kvd = (uint32_t)kvd;
  m->kv_voff = (uint32_t)(c.n_layers * KV_PAGE * kvd);
  m->qd = (uint32_t)qd;
  m->fl = (uint32_t)fl;
  if (c.n_heads * hd != H || hd % 4 || hd > 128 || G > 8 || (G * hd) > 1024 || H % 4 || c.n_ff % 4 || fl % 4) {
    set_error("shape not supported by the attention kernels (head_dim <= 128, heads/kv_heads <= 8)");
    return SM_ERR_UNSUPPORTED;
  }
  if ((rc = upload_2d(g, "token_embd.weight", H, c.vocab_size, &m->tok_embd))) return rc;
  const char* head_name = g.tensor("output.weight") ? "output.weight" : "token_embd.weight";  // tied: qwen2.rs:115-118
  if (world > 1) {  // this rank's rows of the vocab-split head
    if ((rc = upload_2d_rows(g, head_name, H, c.vocab_size, range_map(sh.vocab0, sh.vocab), &m->output))) return rc;
  } else if (g.tensor("output.weight")) {
    if ((rc = upload_2d(g, "output.weight", H, c.vocab_size, &m->output))) return rc;
  } else {
    m->output = m->tok_embd;
    m->tied = true;
  }
  if ((rc = upload_f32(m, g, "output_norm.weight", H, &m->output_norm))) return rc;
  m->weight_bytes = m->output.enc_bytes;
  // This rank's heads (q rows in RoPE-pair order), KV heads and FFN columns.
  const std::vector<uint32_t> qmap = rope_pair_map(sh.q_heads, hd, rank * sh.q_heads),
                              kmap = rope_pair_map(sh.kv_heads, hd, rank * sh.kv_heads),
                              vmap = range_map(rank * kvd, kvd);
  for (uint64_t i = 0; i < c.n_layers; i++) {
    Layer L;
    const std::string p = "blk." + std::to_string(i) + ".";
    auto opt_bias = [&](const char* n, uint64_t len, const std::vector<uint32_t>& map, float** out) -> int {
      if (!g.tensor(p + n)) return SM_OK;  // opt_bias (qwen2.rs:687-697)
      const GgufTensor* t = g.tensor(p + n);
      if (t->type != QT_F32 || t->n_elements() != len) { set_error(p + n + ": expected F32"); return SM_ERR_UNSUPPORTED; }
      const float* src = reinterpret_cast<const float*>(g.data(*t));
      if (!src) { set_error(p + n + ": truncated tensor data"); return SM_ERR_FORMAT; }
      std::vector<float> b(map.size());
      for (size_t k = 0; k < map.size(); k++) b[k] = src[map[k]];
      int rc2 = dev_alloc(m, (void**)out, b.size() * 4);
      if (rc2) return rc2;
      CK(cudaMemcpy(*out, b.data(), b.size() * 4, cudaMemcpyHostToDevice));
      return SM_OK;
    };
    const bool split = world > 1;
    if ((rc = opt_bias("attn_q.bias", H, qmap, &L.bq)) || (rc = opt_bias("attn_k.bias", kvd_full, kmap, &L.bk)) ||
        (rc = opt_bias("attn_v.bias", kvd_full, vmap, &L.bv)) ||
        (rc = upload_f32(m, g, p + "attn_norm.weight", H, &L.attn_norm)) ||
        (rc = upload_f32(m, g, p + "ffn_norm.weight", H, &L.ffn_norm)) ||
        (rc = upload_2d_rows(g, p + "attn_q.weight", H, H, qmap, &L.wq)) ||
        (rc = upload_2d_rows(g, p + "attn_k.weight", H, kvd_full, kmap, &L.wk)) ||
        (rc = split ? upload_2d_rows(g, p + "attn_v.weight", H, kvd_full, vmap, &L.wv)
                    : upload_2d(g, p + "attn_v.weight", H, kvd, &L.wv)) ||
        (rc = split ? upload_2d_cols(g, p + "attn_output.weight", H, H, rank * qd, qd, &L.wo)
                    : upload_2d(g, p + "attn_output.weight", H, H, &L.wo)) ||
        (rc = upload_gate_up(g, p + "ffn_gate.weight", p + "ffn_up.weight", H, c.n_ff, rank * fl, fl, &L.wgu)) ||
        (rc = split ? upload_2d_cols(g, p + "ffn_down.weight", c.n_ff, H, rank * fl, fl, &L.wdown)
                    : upload_2d(g, p + "ffn_down.weight", c.n_ff, H, &L.wdown))) {
      m->layers.push_back(L);  // so that free releases what was uploaded
      return rc;
    }
    m->weight_bytes += L.wq.enc_bytes + L.wk.enc_bytes + L.wv.enc_bytes + L.wo.enc_bytes + L.wgu.enc_bytes +
                       L.wdown.enc_bytes;
    m->layers.push_back(L);
  }
  // RoPE table with the reference's f32 formula (qwen2.rs:712-718).
  m->max_ctx = opts && opts->max_context ? opts->max_context : 32768;
  const uint64_t half = hd / 2;
  std::vector<float> ct(m->max_ctx * half), st(m->max_ctx * half);
  std::vector<float> freq(half);
  for (uint64_t i = 0; i < half; i++) freq[i] = powf(c.rope_theta, -(2.0f * (float)i) / (float)hd);
  for (uint64_t p = 0; p < m->max_ctx; p++)
    for (uint64_t i = 0; i < half; i++) {
      const float angle = (float)p * freq[i];
      ct[p * half + i] = cosf(angle);
      st[p * half + i] = sinf(angle);
    }
  if ((rc = dev_alloc(m, (void**)&m->cos_t, ct.size() * 4)) || (rc = dev_alloc(m, (void**)&m->sin_t, st.size() * 4)))
    return rc;
  CK(cudaMemcpy(m->cos_t, ct.data(), ct.size() * 4, cudaMemcpyHostToDevice));
  CK(cudaMemcpy(m->sin_t, st.data(), st.size() * 4, cudaMemcpyHostToDevice));
  // workspace
  // Rows of one pass (decode batch, prefill chunk): the batched GEMV takes up to 32 columns.
  if (opts && opts->max_batch > 32) {
    set_error("max_batch above 32 is not supported (the batched GEMV takes up to 32 columns)");
    return SM_ERR_UNSUPPORTED;
  }
  const uint32_t R = 32;
  m->rows_max = R;
  const size_t F = fl, V = c.vocab_size;
  if ((rc = dev_alloc(m, (void**)&m->x, R * H * 4)) || (rc = dev_alloc(m, (void**)&m->xn, R * H * 4)) ||
      (rc = dev_alloc(m, (void**)&m->q, R * qd * 4)) || (rc = dev_alloc(m, (void**)&m->k, R * kvd * 4)) ||
      (rc = dev_alloc(m, (void**)&m->v, R * kvd * 4)) || (rc = dev_alloc(m, (void**)&m->att, R * qd * 4)) ||
      (rc = dev_alloc(m, (void**)&m->g, R * F * 4)) || (rc = dev_alloc(m, (void**)&m->u, R * F * 4)) ||
      (rc = dev_alloc(m, (void**)&m->logits, R * V * 4)) ||
      (rc = dev_alloc(m, (void**)&m->part_o, (size_t)R * sh.q_heads * m->max_splits * hd * 4)) ||
      (rc = dev_alloc(m, (void**)&m->part_ml, (size_t)R * sh.q_heads * m->max_splits * 2 * 4)) ||
      (rc = dev_alloc(m, (void**)&m->mask_dev, R * V)) ||
      (rc = dev_alloc(m, (void**)&m->smp_scratch, R * sample_scratch_words((uint32_t)V) * 4)))
    return rc;
  if (!m->tp && tiled_type(m->output.d.type)) {  // batch-1 heads run on gemv_tc: one key per 16-row tile
    m->amax_n = (uint32_t)((V + 15) / 16);
    if ((rc = dev_alloc(m, (void**)&m->amax, (size_t)m->amax_n * 8))) return rc;
  }
  {
    // K-split scratch: the most any batch-1 GEMV of this model asks for
    int sms = 0;
    CK(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, m->device));
    uint64_t need_part = 0;
    uint32_t need_cnt = 0;
    // a launch of these segments: batch 1 (gemv_tc) and batches up to R
    // (gemv_umma, or gemv_tcb without its x image; one launch per weight type)
    auto need = [&](std::initializer_list<const DW*> ws) {
      GemvArgs a{};
      for (const DW* w : ws) a.seg[a.nseg++] = seg(*w, nullptr, 0, nullptr, EPI_STORE);
      uint64_t pp = 0;
      uint32_t pc = 0;
      a.batch = 1;
      gemv_tc_scratch_need(a, (uint32_t)sms, &pp, &pc);
      need_part = std::max(need_part, pp);
      need_cnt = std::max(need_cnt, pc);
      for (uint32_t qt : {(uint32_t)QT_Q4K, (uint32_t)QT_Q6K}) {
        GemvArgs b{};
        for (const DW* w : ws)
          if (w->d.type == qt) b.seg[b.nseg++] = seg(*w, nullptr, 0, nullptr, EPI_STORE);
        if (!b.nseg) continue;
        b.batch = R;
        b.ldx = b.seg[0].w.n_in;
        gemv_tcb_scratch_need(b, (uint32_t)sms, &pp, &pc);
        need_part = std::max(need_part, pp);
        need_cnt = std::max(need_cnt, pc);
        gemv_umma_scratch_need(b, (uint32_t)sms, &pp, &pc);
        need_part = std::max(need_part, pp);
        need_cnt = std::max(need_cnt, pc);
      }
    };
    for (const Layer& L : m->layers) {
      need({&L.wq, &L.wk, &L.wv});
      need({&L.wo});
      need({&L.wgu});
      need({&L.wdown});
    }
    need({&m->output});
    // Q+K and V side by side (see qkv_side): the SMs split by their weight
    // bytes (a Q6_K row streams 210 bytes a block, a Q4_K row 144)
    const Layer& L0 = m->layers[0];
    const auto mixed = [](const Layer& L) {
      return tiled_type(L.wq.d.type) && L.wk.d.type == L.wq.d.type && tiled_type(L.wv.d.type) &&
             L.wv.d.type != L.wq.d.type;
    };
    bool any_mixed = false;
    for (const Layer& L : m->layers) any_mixed |= mixed(L);
    uint64_t need_part2 = 0;
    uint32_t need_cnt2 = 0;
    if (R >= 2 && any_mixed) {
      const uint64_t qk_rows = (uint64_t)L0.wq.d.n_out + L0.wk.d.n_out, v_rows = L0.wv.d.n_out;
      const auto row_bytes = [](uint32_t type) -> uint64_t { return type == QT_Q6K ? 210 : 144; };
      const uint64_t vb = v_rows * row_bytes(L0.wv.d.type), qb = qk_rows * row_bytes(L0.wq.d.type);
      m->v_cap = (uint32_t)std::max<uint64_t>(8, ((uint64_t)sms * vb + qb + vb - 1) / (qb + vb));
      m->qk_cap = (uint32_t)sms > m->v_cap + 8 ? (uint32_t)sms - m->v_cap : 0u;
      m->qkv_side = m->qk_cap != 0;
    }
    if (m->qkv_side)
      for (const Layer& L : m->layers) {
        if (!mixed(L)) continue;
        GemvArgs b{};
        b.seg[b.nseg++] = seg(L.wq, nullptr, 0, nullptr, EPI_STORE);
        b.seg[b.nseg++] = seg(L.wk, nullptr, 0, nullptr, EPI_STORE);
        b.batch = R;
        b.ldx = b.seg[0].w.n_in;
        b.grid_cap = m->qk_cap;
        uint64_t pp = 0;
        uint32_t pc = 0;
        gemv_umma_scratch_need(b, (uint32_t)sms, &pp, &pc);
        need_part = std::max(need_part, pp);
        need_cnt = std::max(need_cnt, pc);
        GemvArgs v{};
        v.seg[v.nseg++] = seg(L.wv, nullptr, 0, nullptr, EPI_STORE);
        v.batch = R;
        v.ldx = v.seg[0].w.n_in;
        v.grid_cap = m->v_cap;
        gemv_umma_scratch_need(v, (uint32_t)sms, &pp, &pc);
        need_part2 = std::max(need_part2, pp);
        need_cnt2 = std::max(need_cnt2, pc);
      }
    m->ks_part_cap = (uint32_t)std::max<uint64_t>(need_part, 16);
    m->ks_cnt_cap = std::max<uint32_t>(need_cnt, 16);
    if ((rc = dev_alloc(m, (void**)&m->ks_part, (size_t)m->ks_part_cap * 4)) ||
        (rc = dev_alloc(m, (void**)&m->ks_cnt, (size_t)m->ks_cnt_cap * 4)))
      return rc;
    CK(cudaMemset(m->ks_cnt, 0, (size_t)m->ks_cnt_cap * 4));
    for (uint32_t n_in : {(uint32_t)H, m->qd, m->fl})
      m->xblob_cap = std::max(m->xblob_cap, gemv_umma_blob_bytes(n_in, R));
    if ((rc = dev_alloc(m, (void**)&m->xblob, (size_t)m->xblob_cap))) return rc;
    if (m->qkv_side) {
      m->ks_part2_cap = (uint32_t)std::max<uint64_t>(need_part2, 16);
      m->ks_cnt2_cap = std::max<uint32_t>(need_cnt2, 16);
      m->xblob2_cap = gemv_umma_blob_bytes((uint32_t)H, R);
      if ((rc = dev_alloc(m, (void**)&m->ks_part2, (size_t)m->ks_part2_cap * 4)) ||
          (rc = dev_alloc(m, (void**)&m->ks_cnt2, (size_t)m->ks_cnt2_cap * 4)) ||
          (rc = dev_alloc(m, (void**)&m->xblob2, (size_t)m->xblob2_cap)))
        return rc;
      CK(cudaMemset(m->ks_cnt2, 0, (size_t)m->ks_cnt2_cap * 4));
    }
    m->parts_cap = (uint32_t)(H / 4 + 64);
    if ((rc = dev_alloc(m, (void**)&m->parts_a, (size_t)R * m->parts_cap * 4)) ||
        (rc = dev_alloc(m, (void**)&m->parts_b, (size_t)R * m->parts_cap * 4)))
      return rc;
  }
  m->in_bytes = step_in_bytes(R);
  m->out_bytes = step_out_bytes(R);
  if ((rc = dev_alloc(m, &m->in_dev, m->in_bytes)) || (rc = dev_alloc(m, &m->out_dev, m->out_bytes)) ||
      (rc = dev_alloc(m, (void**)&m->hist, HIST_TOKENS * 4)) || (rc = dev_alloc(m, (void**)&m->hist_ctr, 256)))
    return rc;
  CK(cudaMallocHost(&m->in_host, m->in_bytes));
  CK(cudaMallocHost(&m->out_host, m->out_bytes));
  std::memset(m->in_host, 0, m->in_bytes);
  layout_in(m->in_dev, R, m->din);
  layout_in(m->in_host, R, m->hin);
  layout_out(m->out_dev, R, m->dout);
  layout_out(m->out_host, R, m->hout);
  for (uint32_t i = 0; i < R; i++) m->hin.sel[i] = i;
  CK(cudaMemset(m->out_dev, 0, m->out_bytes));
  if (world > 1) {
    // Formed last, so that ranks whose loading takes longer do not run
    // into the peers' wait bound: the group forms once every rank is ready.
    CK(cudaDeviceSynchronize());
    rc = tp_group_create(opts->tp_group, rank, world, opts->tp_flags, opts->tp_wait_ms, R, (uint32_t)H,
                         (uint32_t)sh.vocab_stride, &m->tp);
    if (rc) return rc;
  }
  return SM_OK;
}

void destroy_model(sm_model* m) {
  if (!m) return;
  cudaSetDevice(m->device);
  if (m->stream) cudaStreamSynchronize(m->stream);
  for (auto& kv : m->graphs) cudaGraphExecDestroy(kv.second);
  for (auto& kv : m->run_graphs) cudaGraphExecDestroy(kv.second);
  tp_group_destroy(m->tp);
  m->tp = nullptr;
  free_weight(m->tok_embd);
  if (!m->tied) free_weight(m->output);
  for (auto& L : m->layers) {
    free_weight(L.wq); free_weight(L.wk); free_weight(L.wv); free_weight(L.wo);
    free_weight(L.wgu); free_weight(L.wdown);
  }
  for (void* p : m->allocs) cudaFree(p);
  for (void* p : m->page_chunks) cudaFree(p);
  if (m->in_host) cudaFreeHost(m->in_host);
  if (m->out_host) cudaFreeHost(m->out_host);
  if (m->side.st) cudaStreamSynchronize(m->side.st);
  if (m->side.st) cudaStreamDestroy(m->side.st);
  if (m->side.fork) cudaEventDestroy(m->side.fork);
  if (m->side.join) cudaEventDestroy(m->side.join);
  if (m->qkv_join) cudaEventDestroy(m->qkv_join);
  if (m->stream) cudaStreamDestroy(m->stream);
  delete m;
}

// The layer stack for `nrows` rows described in din (tokens, rows, seqs),
// then final norm + output head for the nsel rows listed in din.sel.
// qwen2.rs:460-561 with the kernels of gemv.cu / layers.cu.
// The layer stack for `nrows` rows described in din (tokens, rows, seqs),
// then final norm + output head for the nsel rows listed in din.sel
// (qwen2.rs:460-561). Per layer: QKV GEMV (input RMSNorm, bias, RoPE, KV
// append in its epilogue), attention, O GEMV (+ residual, next norm's input),
// gate/up GEMV (+ SwiGLU), down GEMV (+ residual, next norm's input).
//
// With tensor parallelism the O and down GEMVs push this rank's partial sums
// to every rank (EPI_PUSH) and tp_reduce_resid_kernel adds the sum over ranks
// to the residual (and prepares the next norm's input); the output head
// pushes this rank's vocab slice and tp_gather_kernel assembles the logits.
// The batch-1 output head's per-tile argmax keys (the greedy sampler's fast
// path), or null. Not with tensor parallelism: there the head's epilogue
// sends each rank's vocab slice to the other ranks (it stores no logits to
// read a key from), and a rank's keys would cover its slice only.
static uint64_t* head_amax(const sm_model* m, uint32_t rows) { return rows == 1 && !m->tp ? m->amax : nullptr; }

cudaError_t run_rows(sm_model* m, uint32_t nrows, uint32_t nsel, cudaStream_t st) {
  const sm_config& c = m->c;
  const uint32_t H = (uint32_t)c.n_embd, F = m->fl, kvd = m->kvd, hd = (uint32_t)c.head_dim, qd = m->qd;
  const uint32_t Hq = (uint32_t)m->sh.q_heads, Hkv = (uint32_t)m->sh.kv_heads;
  TpGroup* tp = m->tp;
  // a batched decode step (one row per sequence) may share prefix pages
  const uint32_t* shared = nrows > 1 && nsel == nrows && hd % 32 == 0 ? m->din.shared : nullptr;
  cudaError_t e;
#define RK(x) do { if ((e = (x)) != cudaSuccess) return e; } while (0)
  // A row-split GEMV (O or down) whose rank partials are all-reduced into the
  // residual, which also yields the next norm's input.
  auto split_gemv = [&](GemvArgs g, const DW& w, const float* nw, float* parts, uint32_t* np) -> cudaError_t {
    const TpExchange ex = tp_allreduce(tp, m->dout.err);
    if (ex.send) {
      g.seg[0] = seg(w, ex.send, H, nullptr, EPI_STORE);
    } else {
      g.seg[0] = seg(w, nullptr, H, nullptr, EPI_PUSH);
      g.push = ex.push;
    }
    cudaError_t e2 = launch_gemv(g, st);
    if (e2 == cudaSuccess && ex.send) e2 = tp_allreduce_issue(tp, nrows, st);
    if (e2 == cudaSuccess) e2 = launch_tp_reduce_resid(ex.recv, nrows, H, m->x, H, nw, m->xn, H, parts, st);
    *np = TP_BLOCKS;
    return e2;
  };
  GemvArgs base{};
  base.batch = nrows;
  base.in_n = H;
  base.in_eps = c.rms_eps;
  base.rows = m->din.rows;
  base.seqs = m->din.seqs;
  base.cos_t = m->cos_t;
  base.sin_t = m->sin_t;
  base.hd = hd;
  base.kvd = kvd;
  base.ks_part = m->ks_part;
  base.ks_cnt = m->ks_cnt;
  base.ks_part_cap = m->ks_part_cap;
  base.ks_cnt_cap = m->ks_cnt_cap;
  base.xblob = m->xblob;
  base.xblob_cap = m->xblob_cap;
  base.err = m->dout.err;
  RK(launch_embed_norm(m->tok_embd.d, m->din.tok, nrows, m->x, H, m->layers[0].attn_norm, m->xn, H, m->parts_a, st));
  uint32_t np_a = embed_norm_parts(H), np_b = 0;
  for (uint32_t li = 0; li < c.n_layers; li++) {
    const Layer& L = m->layers[li];
    GemvArgs a = base;
    a.layer = li;
    a.x = m->xn; a.ldx = H;
    a.in_parts = m->parts_a; a.in_np = np_a;
    a.nseg = 3;
    a.seg[0] = seg(L.wq, m->q, qd, L.bq, EPI_ROPE_Q);
    a.seg[1] = seg(L.wk, nullptr, 0, L.bk, EPI_ROPE_K);
    a.seg[2] = seg(L.wv, nullptr, 0, L.bv, EPI_V);
    if (nrows > 1 && m->qkv_side && tiled_type(L.wq.d.type) && L.wk.d.type == L.wq.d.type &&
        tiled_type(L.wv.d.type) && L.wv.d.type != L.wq.d.type) {
      // V on the side stream (own scratch, v_cap CTAs) beside Q+K (qk_cap CTAs);
      // attention waits for both
      GemvArgs v = a;
      v.nseg = 1;
      v.seg[0] = a.seg[2];
      v.grid_cap = m->v_cap;
      v.ks_part = m->ks_part2;
      v.ks_cnt = m->ks_cnt2;
      v.ks_part_cap = m->ks_part2_cap;
      v.ks_cnt_cap = m->ks_cnt2_cap;
      v.xblob = m->xblob2;
      v.xblob_cap = m->xblob2_cap;
      a.nseg = 2;
      a.grid_cap = m->qk_cap;
      RK(cudaEventRecord(m->side.fork, st));
      RK(cudaStreamWaitEvent(m->side.st, m->side.fork, 0));
      RK(launch_gemv(v, m->side.st));
      RK(cudaEventRecord(m->qkv_join, m->side.st));
      RK(launch_gemv(a, st));
      RK(cudaStreamWaitEvent(st, m->qkv_join, 0));
    } else {
      RK(launch_gemv(a, st));
    }
    // one row whose O projection runs on gemv_tc: the O GEMV merges the attention partials itself
    const bool merge = nrows == 1 && tiled_type(L.wo.d.type);
    RK(launch_attention(m->q, qd, m->din.rows, m->din.seqs, nrows, li, Hq, Hkv, hd, m->part_o, m->part_ml,
                        m->max_splits, merge ? nullptr : m->att, qd, st, nsel != nrows ? 1u : 0u, shared, m->side));
    GemvArgs o = base;
    o.layer = li;
    o.x = m->att; o.ldx = qd;
    o.nseg = 1;
    if (merge) {
      o.att_o = m->part_o;
      o.att_ml = m->part_ml;
      o.att_slots = m->max_splits;
      o.att_first = ATT_SHARED_SPLITS;
    }
    if (tp) {
      RK(split_gemv(o, L.wo, L.ffn_norm, m->parts_b, &np_b));
    } else {
      o.seg[0] = seg(L.wo, m->x, H, nullptr, EPI_RESID);
      o.nw = L.ffn_norm; o.xn = m->xn; o.ldxn = H; o.out_parts = m->parts_b;
      RK(launch_gemv(o, st, &np_b));
    }
    GemvArgs gu = base;
    gu.layer = li;
    gu.x = m->xn; gu.ldx = H;
    gu.in_parts = m->parts_b; gu.in_np = np_b;
    gu.nseg = 1;
    gu.seg[0] = seg(L.wgu, nullptr, 0, nullptr, EPI_SILU);
    gu.h = m->g; gu.ldh = F;
    RK(launch_gemv(gu, st));
    GemvArgs dn = base;
    dn.layer = li;
    dn.x = m->g; dn.ldx = F;
    dn.nseg = 1;
    const float* next_norm = li + 1 < c.n_layers ? m->layers[li + 1].attn_norm : m->output_norm;
    if (tp) {
      RK(split_gemv(dn, L.wdown, next_norm, m->parts_a, &np_a));
    } else {
      dn.seg[0] = seg(L.wdown, m->x, H, nullptr, EPI_RESID);
      dn.nw = next_norm;
      dn.xn = m->xn; dn.ldxn = H; dn.out_parts = m->parts_a;
      RK(launch_gemv(dn, st, &np_a));
    }
  }
  if (nsel) {
    GemvArgs hd_ = base;
    hd_.batch = nsel;
    hd_.nseg = 1;
    const uint32_t vs = (uint32_t)m->sh.vocab_stride;
    TpExchange gx{};
    if (tp) {  // this rank's slice [vocab0, vocab0 + vocab) goes to every rank
      gx = tp_gather(tp, nsel, m->sh.vocab0, m->dout.err);
      if (gx.send) {
        hd_.seg[0] = seg(m->output, gx.send, vs, nullptr, EPI_STORE);
      } else {
        hd_.seg[0] = seg(m->output, nullptr, vs, nullptr, EPI_PUSH);
        hd_.push = gx.push;
      }
    } else {
      hd_.seg[0] = seg(m->output, m->logits, (uint32_t)c.vocab_size, nullptr, EPI_STORE);
    }
    hd_.x = m->xn; hd_.ldx = H;
    if (nsel == nrows) {  // every row: the last down GEMV prepared the final norm's input
      hd_.in_parts = m->parts_a;
      hd_.in_np = np_a;
    } else {  // a selection (prefill): normalize the selected rows here (qwen2.rs:555-560)
      RK(launch_rmsnorm(m->x, H, m->din.sel, m->output_norm, m->xn, H, nsel, H, c.rms_eps, st));
    }
    hd_.amax = head_amax(m, nsel);  // greedy candidates per tile (the sampler's fast path)
    RK(launch_gemv(hd_, st));
    if (tp) {  // the full logits on every rank
      if (gx.send) RK(tp_gather_issue(tp, nsel, st));
      RK(launch_tp_gather(gx.recv, nsel, vs, (uint32_t)c.vocab_size, m->logits, (uint32_t)c.vocab_size, st));
    }
  }
#undef RK
  return cudaSuccess;
}

// Every Sampler of the reference is accepted: any temperature, top_k None
// (< 0) or any k (0 acts as 1, as k.max(1) does), top_p None (< 0) or any p.
int check_sampler(const sm_sampler*) { return SM_OK; }

SampleParams to_params(const sm_sampler* s) {
  SampleParams p{};
  if (!s) { p.temperature = 0.f; p.top_k = -1; p.top_p = -1.f; return p; }
  p.temperature = s->temperature;
  p.top_k = (int32_t)std::max<int64_t>(-1, std::min<int64_t>(s->top_k, INT32_MAX));
  p.top_p = s->top_p;
  return p;
}

// Page management; the caller holds m->mu.
static int page_alloc(sm_model* m, float** out) {
  const size_t pbytes = (size_t)m->kv_voff * 2 * 4;
  if (m->free_pages.empty()) {
    const size_t per_chunk = std::max<size_t>(1, (size_t(256) << 20) / pbytes);
    void* p = nullptr;
    if (cudaMalloc(&p, per_chunk * pbytes) != cudaSuccess) {
      cudaGetLastError();
      set_error("cudaMalloc failed for " + std::to_string(per_chunk) + " KV pages of " + std::to_string(pbytes) +
                " bytes");
      return SM_ERR_OOM;
    }
    m->page_chunks.push_back(p);
    for (size_t i = per_chunk; i-- > 0;) m->free_pages.push_back((float*)p + i * (size_t)m->kv_voff * 2);
  }
  float* pg = m->free_pages.back();
  m->free_pages.pop_back();
  m->page_refs[pg] = 1;
  // unwritten positions read as zeros, as in a freshly allocated SeqState
  CK(cudaMemsetAsync(pg, 0, pbytes, m->stream));
  *out = pg;
  return SM_OK;
}
static void page_release(sm_model* m, float* pg) {
  if (!pg) return;
  auto it = m->page_refs.find(pg);
  if (it == m->page_refs.end()) return;
  if (--it->second == 0) {
    m->page_refs.erase(it);
    m->free_pages.push_back(pg);  // reused in stream order: earlier reads are enqueued before any reuse
  }
}
// The device copy of the page array, after changes.
static int cache_sync(sm_model* m, sm_cache* c) {
  if (!c->dirty) return SM_OK;
  CK(cudaMemcpyAsync(c->pages_dev, c->pages.data(), c->pages.size() * sizeof(float*), cudaMemcpyHostToDevice,
                     m->stream));
  c->dirty = false;
  return SM_OK;
}
// Positions [len, upto) are about to be written: every page they touch is
// allocated, and a page shared with another cache is copied first.
static int cache_prepare(sm_model* m, sm_cache* c, uint64_t upto) {
  if (upto > c->cap) {
    set_error(std::to_string(upto) + " positions exceed the cache capacity " + std::to_string(c->cap));
    return SM_ERR_CAPACITY;
  }
  const uint64_t t1 = (upto + KV_PAGE - 1) / KV_PAGE;
  for (uint64_t t = c->len / KV_PAGE; t < t1; t++) {
    float*& pg = c->pages[t];
    if (!pg) {
      if (int rc = page_alloc(m, &pg)) return rc;
      c->dirty = true;
    } else if (m->page_refs[pg] > 1) {  // copy on write
      float* np = nullptr;
      if (int rc = page_alloc(m, &np)) return rc;
      CK(cudaMemcpyAsync(np, pg, (size_t)m->kv_voff * 2 * 4, cudaMemcpyDeviceToDevice, m->stream));
      page_release(m, pg);
      pg = np;
      c->dirty = true;
    }
  }
  return cache_sync(m, c);
}
// Drops the pages past position n.
static void cache_drop_after(sm_model* m, sm_cache* c, uint64_t n) {
  for (uint64_t t = (n + KV_PAGE - 1) / KV_PAGE; t < c->pages.size(); t++)
    if (c->pages[t]) {
      page_release(m, c->pages[t]);
      c->pages[t] = nullptr;
      c->dirty = true;
    }
}
static int cache_resize(sm_model* m, sm_cache* c, uint64_t cap) {
  const size_t np = (cap + KV_PAGE - 1) / KV_PAGE;
  float** d = nullptr;
  if (cudaMalloc((void**)&d, std::max<size_t>(np, 1) * sizeof(float*)) != cudaSuccess) {
    cudaGetLastError();
    set_error("cudaMalloc failed for a KV page table");
    return SM_ERR_OOM;
  }
  if (c->pages_dev) {
    cudaStreamSynchronize(m->stream);
    cudaFree(c->pages_dev);
  }
  c->pages_dev = d;
  c->pages.resize(np, nullptr);
  c->cap = cap;
  c->dirty = true;
  return cache_sync(m, c);
}
// Leading KV pages that every cache of a batch holds as the same physical
// page, all of whose positions are below every cache's length (the shared
// prefix of sequences cloned from one prefilled state: prefix.rs:59-109).
static uint32_t shared_prefix_pages(const sm_model* m, sm_cache* const* caches, uint64_t n) {
  if (n < 2 || m->c.head_dim % 32) return 0;
  uint64_t minlen = caches[0]->len;
  for (uint64_t i = 1; i < n; i++) minlen = std::min(minlen, caches[i]->len);
  uint64_t t = 0;
  for (; t < minlen / KV_PAGE; t++) {
    const float* p0 = caches[0]->pages[t];
    bool same = p0 != nullptr;
    for (uint64_t i = 1; same && i < n; i++) same = caches[i]->pages[t] == p0;
    if (!same) break;
  }
  return (uint32_t)t;
}
static SeqDesc seq_desc(const sm_model* m, const sm_cache* c) {
  return SeqDesc{c->pages_dev, (uint32_t)c->cap, m->kv_voff};
}

// Prefill / forward of n tokens of one cache, chunked by rows_max. The last
// token's logits end in m->logits row 0.
int forward_tokens(sm_model* m, sm_cache* c, const uint32_t* toks, uint64_t n) {
  if (n == 0) { set_error("forward_cached: empty token list"); return SM_ERR_ARG; }
  if (c->len + n > c->cap) {
    set_error("forward_cached: " + std::to_string(c->len + n) + " positions exceed the cache capacity " +
              std::to_string(c->cap));
    return SM_ERR_CAPACITY;
  }
  if (int rc = cache_prepare(m, c, c->len + n)) return rc;
  for (uint64_t i = 0; i < n; i++)
    if (toks[i] >= m->c.vocab_size) { set_error("token id out of range"); return SM_ERR_ARG; }
  cudaStream_t st = m->stream;
  for (uint64_t c0 = 0; c0 < n; c0 += m->rows_max) {
    const uint32_t rows = (uint32_t)std::min<uint64_t>(m->rows_max, n - c0);
    const bool last = c0 + rows == n;
    CK(cudaStreamSynchronize(st));  // pinned staging is reused
    for (uint32_t r = 0; r < rows; r++) {
      m->hin.tok[r] = toks[c0 + r];
      m->hin.rows[r] = RowDesc{0u, (uint32_t)(c->len + c0 + r)};
    }
    m->hin.seqs[0] = seq_desc(m, c);
    m->hin.sel[0] = rows - 1;
    CK(cudaMemcpyAsync(m->in_dev, m->in_host, m->in_bytes, cudaMemcpyHostToDevice, st));
    CK(run_rows(m, rows, last ? 1 : 0, st));
  }
  c->len += n;
  return SM_OK;
}

int sample_rows(sm_model* m, uint32_t rows, const uint8_t* mask_host, bool advance) {
  cudaStream_t st = m->stream;
  const uint8_t* mask = nullptr;
  if (mask_host) {
    CK(cudaMemcpyAsync(m->mask_dev, mask_host, (size_t)rows * m->c.vocab_size, cudaMemcpyHostToDevice, st));
    mask = m->mask_dev;
  }
  CK(launch_sample(m->logits, (uint32_t)m->c.vocab_size, rows, mask, m->din.sp, m->din.rng, m->dout.tok,
                   advance ? m->din.tok : nullptr, advance ? m->din.rows : nullptr, m->smp_scratch, st, ~0ull,
                   head_amax(m, rows), m->amax_n));
  CK(cudaMemcpyAsync(m->dout.rng, m->din.rng, rows * sizeof(uint64_t), cudaMemcpyDeviceToDevice, st));
  CK(cudaMemcpyAsync(m->out_host, m->out_dev, m->out_bytes, cudaMemcpyDeviceToHost, st));
  return SM_OK;
}

// One decode step of B sequences (one token each) as a CUDA graph:
// H2D of the step state, layer stack, head, sampler, D2H of tokens + RNG.
int decode_graph(sm_model* m, uint32_t B, cudaGraphExec_t* out) {
  auto it = m->graphs.find(B);
  if (it != m->graphs.end()) { *out = it->second; return SM_OK; }
  cudaStream_t st = m->stream;
  cudaGraph_t g = nullptr;
  CK(cudaStreamBeginCapture(st, cudaStreamCaptureModeThreadLocal));
  cudaError_t e = cudaMemcpyAsync(m->in_dev, m->in_host, m->in_bytes, cudaMemcpyHostToDevice, st);
  if (e == cudaSuccess) e = run_rows(m, B, B, st);
  if (e == cudaSuccess)
    e = launch_sample(m->logits, (uint32_t)m->c.vocab_size, B, nullptr, m->din.sp, m->din.rng, m->dout.tok, m->din.tok,
                      m->din.rows, m->smp_scratch, st, ~0ull, head_amax(m, B), m->amax_n);
  if (e == cudaSuccess) e = cudaMemcpyAsync(m->dout.rng, m->din.rng, B * sizeof(uint64_t), cudaMemcpyDeviceToDevice, st);
  if (e == cudaSuccess) e = cudaMemcpyAsync(m->out_host, m->out_dev, m->out_bytes, cudaMemcpyDeviceToHost, st);
  cudaError_t e2 = cudaStreamEndCapture(st, &g);
  if (e != cudaSuccess || e2 != cudaSuccess) {
    if (g) cudaGraphDestroy(g);
    cudaGetLastError();
    set_error(std::string("cuda: decode graph capture failed: ") + cudaGetErrorString(e != cudaSuccess ? e : e2));
    return SM_ERR_CUDA;
  }
  cudaGraphExec_t ex = nullptr;
  e = cudaGraphInstantiate(&ex, g, 0);
  cudaGraphDestroy(g);
  if (e != cudaSuccess) {
    set_error(std::string("cuda: graph instantiate: ") + cudaGetErrorString(e));
    return SM_ERR_CUDA;
  }
  m->graphs[B] = ex;
  *out = ex;
  return SM_OK;
}

// One decode step whose inputs (tokens, positions) were left on the device by
// the previous step's sampler; records the sampled tokens in m->hist.
int run_graph(sm_model* m, uint32_t B, cudaGraphExec_t* out) {
  auto it = m->run_graphs.find(B);
  if (it != m->run_graphs.end()) { *out = it->second; return SM_OK; }
  cudaStream_t st = m->stream;
  cudaGraph_t g = nullptr;
  CK(cudaStreamBeginCapture(st, cudaStreamCaptureModeThreadLocal));
  cudaError_t e = run_rows(m, B, B, st);
  if (e == cudaSuccess)
    e = launch_sample(m->logits, (uint32_t)m->c.vocab_size, B, nullptr, m->din.sp, m->din.rng, m->dout.tok, m->din.tok,
                      m->din.rows, m->smp_scratch, st, ~0ull, head_amax(m, B), m->amax_n);
  if (e == cudaSuccess) e = launch_record_tokens(m->dout.tok, B, m->hist, m->hist_ctr, HIST_TOKENS / B, st);
  cudaError_t e2 = cudaStreamEndCapture(st, &g);
  if (e != cudaSuccess || e2 != cudaSuccess) {
    if (g) cudaGraphDestroy(g);
    cudaGetLastError();
    set_error(std::string("cuda: decode-run graph capture failed: ") + cudaGetErrorString(e != cudaSuccess ? e : e2));
    return SM_ERR_CUDA;
  }
  size_t n_nodes = 0;
  uint64_t n_kernels = 0;
  if (cudaGraphGetNodes(g, nullptr, &n_nodes) == cudaSuccess && n_nodes) {
    std::vector<cudaGraphNode_t> nodes(n_nodes);
    if (cudaGraphGetNodes(g, nodes.data(), &n_nodes) == cudaSuccess)
      for (cudaGraphNode_t nd : nodes) {
        cudaGraphNodeType t;
        if (cudaGraphNodeGetType(nd, &t) == cudaSuccess && t == cudaGraphNodeTypeKernel) n_kernels++;
      }
  }
  cudaGetLastError();
  cudaGraphExec_t ex = nullptr;
  e = cudaGraphInstantiate(&ex, g, 0);
  cudaGraphDestroy(g);
  if (e != cudaSuccess) {
    set_error(std::string("cuda: graph instantiate: ") + cudaGetErrorString(e));
    return SM_ERR_CUDA;
  }
  m->run_graph_kernels[B] = n_kernels;
  m->run_graphs[B] = ex;
  *out = ex;
  return SM_OK;
}

int guard_model(const sm_model* m) {
  if (!m) { set_error("null model"); return SM_ERR_ARG; }
  return SM_OK;
}

// Compute entry points refuse a model whose bounded waits gave up earlier
// (its activations, KV or tensor-parallel exchange state are not valid).
int guard_live(const sm_model* m) {
  if (!m) { set_error("null model"); return SM_ERR_ARG; }
  if (m->failed) {
    set_error(m->tp ? "the model's tensor-parallel group failed earlier (a peer timed out); load it again"
                    : "the model failed earlier (a bounded wait gave up); load it again");
    return m->tp ? SM_ERR_PEER : SM_ERR_STATE;
  }
  return SM_OK;
}

// After the stream is synchronized: fails the call (and marks the model
// failed) if a bounded wait gave up during it. fetch: copy the error word
// first (paths whose step block did not bring it back).
int check_waits(sm_model* m, bool fetch) {
  if (fetch) CK(cudaMemcpy(m->hout.err, m->dout.err, 4, cudaMemcpyDeviceToHost));
  const uint32_t e = *m->hout.err;
  if (!e) return SM_OK;
  m->failed = true;
  if (e & TP_ERR_WAIT) {
    set_error("a tensor-parallel peer did not arrive within the wait bound (tp_wait_ms); the group is unusable");
    return SM_ERR_PEER;
  }
  set_error("a bounded wait in a GEMV gave up (a weight copy did not complete); results are invalid");
  return SM_ERR_CUDA;
}

void model_release(sm_model* m) {
  if (m && m->refs.fetch_sub(1) == 1) destroy_model(m);
}

}  // namespace

// ---------------------------------------------------------------- C ABI ----
extern "C" {

const char* sm_last_error(void) { return get_error().c_str(); }
int sm_abi_version(void) { return 2; }
int sm_tp_group_id(void* id_out) {
  if (!id_out) { set_error("null id"); return SM_ERR_ARG; }
  return tp_unique_id(id_out);
}
int sm_model_tp_abort(sm_model* m) {
  if (guard_model(m)) return SM_ERR_ARG;
  std::lock_guard<std::mutex> lk(m->mu);
  if (m->tp) m->failed = true;
  return SM_OK;
}
int sm_tp_plan(const sm_config* c, uint32_t rank, uint32_t size, sm_tp_shard* out) {
  if (!c || !out) { set_error("null argument"); return SM_ERR_ARG; }
  TpShard s;
  const std::string why =
      tp_plan(c->n_heads, c->n_kv_heads, c->head_dim, c->n_ff, c->vocab_size, 0, 0, rank, size ? size : 1, &s);
  if (!why.empty()) { set_error(why); return rank >= (size ? size : 1) ? SM_ERR_ARG : SM_ERR_UNSUPPORTED; }
  out->q_head0 = (uint64_t)rank * s.q_heads;
  out->q_heads = s.q_heads;
  out->kv_head0 = (uint64_t)rank * s.kv_heads;
  out->kv_heads = s.kv_heads;
  out->ff0 = (uint64_t)rank * s.ff;
  out->ff = s.ff;
  out->vocab0 = s.vocab0;
  out->vocab = s.vocab;
  return SM_OK;
}
uint64_t sm_rng_seed(uint64_t seed) { return seed + 0x9E3779B97F4A7C15ull; }

static int model_from_reader(std::unique_ptr<GgufReader> r, const sm_load_opts* opts, sm_model** out) {
  if (!r) return SM_ERR_FORMAT;
  if (!out) { set_error("null out"); return SM_ERR_ARG; }
  int ndev = 0;
  if (cudaGetDeviceCount(&ndev) != cudaSuccess || ndev == 0) {
    cudaGetLastError();
    set_error("no CUDA device available: the engine runs only on the GPU");
    return SM_ERR_CUDA;
  }
  auto* m = new sm_model();
  m->device = opts ? opts->device : 0;
  if (cudaSetDevice(m->device) != cudaSuccess || cudaStreamCreateWithFlags(&m->stream, cudaStreamNonBlocking) != cudaSuccess ||
      cudaStreamCreateWithFlags(&m->side.st, cudaStreamNonBlocking) != cudaSuccess ||
      cudaEventCreateWithFlags(&m->side.fork, cudaEventDisableTiming) != cudaSuccess ||
      cudaEventCreateWithFlags(&m->side.join, cudaEventDisableTiming) != cudaSuccess ||
      cudaEventCreateWithFlags(&m->qkv_join, cudaEventDisableTiming) != cudaSuccess ||
      gemv_tc_prepare() != cudaSuccess || gemv_tcb_prepare() != cudaSuccess ||
      gemv_umma_prepare() != cudaSuccess || attention_prepare() != cudaSuccess) {
    cudaGetLastError();
    const std::string msg = "cannot use CUDA device " + std::to_string(m->device);
    destroy_model(m);  // releases the streams and events made so far
    set_error(msg);
    return SM_ERR_CUDA;
  }
  int rc = load_model(*r, opts, m);
  if (rc) { std::string msg = get_error(); destroy_model(m); set_error(msg); return rc; }
  *out = m;
  return SM_OK;
}

int sm_model_load(const char* path, const sm_load_opts* opts, sm_model** out) {
  if (!path) { set_error("null path"); return SM_ERR_ARG; }
  auto r = GgufReader::open_file(path);
  if (!r) return get_error().rfind("io:", 0) == 0 ? SM_ERR_IO : SM_ERR_FORMAT;
  return model_from_reader(std::move(r), opts, out);
}

int sm_model_load_memory(const void* buf, uint64_t len, const sm_load_opts* opts, sm_model** out) {
  if (!buf) { set_error("null buffer"); return SM_ERR_ARG; }
  return model_from_reader(GgufReader::open_memory(buf, len), opts, out);
}

int sm_model_free(sm_model* m) {
  if (m && m->tp) {
    // Every rank frees its handle at the same point of the program: meet
    // there, then make no further exchanges (caches may outlive the handle).
    std::lock_guard<std::mutex> lk(m->mu);
    cudaSetDevice(m->device);
    cudaStreamSynchronize(m->stream);
    if (!m->failed) tp_group_barrier(m->tp);
    m->failed = true;
  }
  model_release(m);
  return SM_OK;
}

int sm_model_config(const sm_model* m, sm_config* out) {
  if (guard_model(m) || !out) return SM_ERR_ARG;
  *out = m->c;
  return SM_OK;
}

int sm_model_weight_bytes(const sm_model* m, uint64_t* out) {
  if (guard_model(m) || !out) return SM_ERR_ARG;
  *out = m->weight_bytes;
  return SM_OK;
}

int sm_model_step_io_bytes(const sm_model* m, uint64_t* h2d, uint64_t* d2h) {
  if (guard_model(m) || !h2d || !d2h) return SM_ERR_ARG;
  *h2d = m->in_bytes;
  *d2h = m->out_bytes;
  return SM_OK;
}

int sm_model_step_launches(const sm_model* m, uint64_t n_rows, uint64_t* out) {
  if (!m || !out) { set_error("null argument"); return SM_ERR_ARG; }
  std::lock_guard<std::mutex> lk(const_cast<sm_model*>(m)->mu);
  auto it = m->run_graph_kernels.find((uint32_t)n_rows);
  if (n_rows > 0xFFFFFFFFull || it == m->run_graph_kernels.end()) {
    set_error("sm_model_step_launches: no decode run of that many sequences has been made");
    return SM_ERR_STATE;
  }
  *out = it->second;
  return SM_OK;
}
int sm_model_stream(const sm_model* m, void** stream) {
  if (guard_model(m) || !stream) return SM_ERR_ARG;
  *stream = (void*)m->stream;
  return SM_OK;
}

// ------------------------------------------------------------- caches ----
int sm_cache_new(sm_model* m, uint64_t max_seq, sm_cache** out) {
  if (guard_model(m) || !out) return SM_ERR_ARG;
  if (max_seq == 0 || max_seq > m->max_ctx) {
    set_error("sm_cache_new: max_seq must be in 1.." + std::to_string(m->max_ctx) + " (the model's max_context)");
    return SM_ERR_CAPACITY;
  }
  std::lock_guard<std::mutex> lk(m->mu);
  cudaSetDevice(m->device);
  auto* c = new sm_cache();
  c->m = m;
  int rc = cache_resize(m, c, max_seq);
  if (rc) { delete c; return rc; }
  m->refs++;
  *out = c;
  return SM_OK;
}

int sm_cache_free(sm_cache* c) {
  if (!c) return SM_OK;
  sm_model* m = c->m;
  {
    std::lock_guard<std::mutex> lk(m->mu);
    cudaSetDevice(m->device);
    cudaStreamSynchronize(m->stream);
    for (float* pg : c->pages) page_release(m, pg);
    cudaFree(c->pages_dev);
    delete c;
  }
  model_release(m);
  return SM_OK;
}

int sm_cache_len(const sm_cache* c, uint64_t* out) {
  if (!c || !out) { set_error("null argument"); return SM_ERR_ARG; }
  *out = c->len;
  return SM_OK;
}
int sm_cache_capacity(const sm_cache* c, uint64_t* out) {
  if (!c || !out) { set_error("null argument"); return SM_ERR_ARG; }
  *out = c->cap;
  return SM_OK;
}
int sm_cache_advance(sm_cache* c, uint64_t n) {
  if (!c) { set_error("null cache"); return SM_ERR_ARG; }
  if (c->len + n > c->cap) { set_error("sm_cache_advance: beyond capacity"); return SM_ERR_CAPACITY; }
  sm_model* m = c->m;
  std::lock_guard<std::mutex> lk(m->mu);
  cudaSetDevice(m->device);
  if (int rc = cache_prepare(m, c, c->len + n)) return rc;  // the positions exist (zeros unless written)
  c->len += n;
  return SM_OK;
}
int sm_cache_reset(sm_cache* c) {
  if (!c) { set_error("null cache"); return SM_ERR_ARG; }
  sm_model* m = c->m;
  std::lock_guard<std::mutex> lk(m->mu);
  cudaSetDevice(m->device);
  cache_drop_after(m, c, 0);
  c->len = 0;
  return cache_sync(m, c);
}
int sm_cache_truncate(sm_cache* c, uint64_t len) {
  if (!c) { set_error("null cache"); return SM_ERR_ARG; }
  if (len > c->len) {
    set_error("truncate: " + std::to_string(len) + " > len=" + std::to_string(c->len) + " (a state cannot grow this way)");
    return SM_ERR_STATE;
  }
  sm_model* m = c->m;
  std::lock_guard<std::mutex> lk(m->mu);
  cudaSetDevice(m->device);
  cache_drop_after(m, c, len);
  c->len = len;
  return cache_sync(m, c);
}
int sm_cache_ensure_capacity(sm_cache* c, uint64_t min_cap) {
  if (!c) { set_error("null cache"); return SM_ERR_ARG; }
  if (min_cap <= c->cap) return SM_OK;
  sm_model* m = c->m;
  if (min_cap > m->max_ctx) { set_error("ensure_capacity: beyond the model's max_context"); return SM_ERR_CAPACITY; }
  std::lock_guard<std::mutex> lk(m->mu);
  cudaSetDevice(m->device);
  return cache_resize(m, c, min_cap);  // the pages stay: nothing is copied
}
int sm_cache_clone(const sm_cache* c, sm_cache** out) {
  if (!c || !out) { set_error("null argument"); return SM_ERR_ARG; }
  sm_model* m = c->m;
  std::lock_guard<std::mutex> lk(m->mu);
  cudaSetDevice(m->device);
  auto* n = new sm_cache();
  n->m = m;
  int rc = cache_resize(m, n, c->cap);
  if (rc) { delete n; return rc; }
  n->len = c->len;
  n->pages = c->pages;  // shared until one of them writes a page (cache_prepare)
  for (float* pg : n->pages)
    if (pg) m->page_refs[pg]++;
  n->dirty = true;
  if ((rc = cache_sync(m, n))) return rc;
  m->refs++;
  *out = n;
  return SM_OK;
}
int sm_model_kv_pages(const sm_model* m, uint64_t* held, uint64_t* allocated, uint64_t* kv_page_bytes) {
  if (!m || !held || !allocated || !kv_page_bytes) { set_error("null argument"); return SM_ERR_ARG; }
  std::lock_guard<std::mutex> lk(const_cast<sm_model*>(m)->mu);
  *held = m->page_refs.size();
  *allocated = m->page_refs.size() + m->free_pages.size();
  *kv_page_bytes = (uint64_t)m->kv_voff * 2 * 4;
  return SM_OK;
}
int sm_cache_read_kv(const sm_cache* c, uint64_t layer, uint64_t pos, float* k_out, float* v_out) {
  if (!c || !k_out || !v_out) { set_error("null argument"); return SM_ERR_ARG; }
  sm_model* m = c->m;
  if (layer >= m->c.n_layers || pos >= c->cap) { set_error("read_kv: index out of range"); return SM_ERR_ARG; }
  std::lock_guard<std::mutex> lk(m->mu);
  cudaSetDevice(m->device);
  CK(cudaStreamSynchronize(m->stream));
  const float* pg = c->pages[pos / KV_PAGE];
  if (!pg) {
    std::fill(k_out, k_out + m->kvd, 0.f);
    std::fill(v_out, v_out + m->kvd, 0.f);
    return SM_OK;
  }
  const size_t off = kv_page_off((uint32_t)layer, (uint32_t)pos, m->kvd);
  CK(cudaMemcpy(k_out, pg + off, m->kvd * 4, cudaMemcpyDeviceToHost));
  CK(cudaMemcpy(v_out, pg + m->kv_voff + off, m->kvd * 4, cudaMemcpyDeviceToHost));
  return SM_OK;
}

// Row `token` of the embedding table as the forward's first kernel produces it
// (qwen2.rs:468-472: the row dequantized exactly).
int sm_model_embedding(sm_model* m, uint32_t token, float* out) {
  if (guard_model(m) || !out) { set_error("sm_model_embedding: bad arguments"); return SM_ERR_ARG; }
  if (token >= m->c.vocab_size) { set_error("token id out of range"); return SM_ERR_ARG; }
  std::lock_guard<std::mutex> lk(m->mu);
  cudaSetDevice(m->device);
  CK(cudaStreamSynchronize(m->stream));  // the pinned staging block is free
  m->hin.tok[0] = token;
  CK(cudaMemcpyAsync(m->din.tok, m->hin.tok, sizeof(uint32_t), cudaMemcpyHostToDevice, m->stream));
  const uint32_t H = (uint32_t)m->c.n_embd;
  CK(launch_embed_norm(m->tok_embd.d, m->din.tok, 1, m->x, H, m->layers[0].attn_norm, m->xn, H, m->parts_a,
                       m->stream));
  CK(cudaMemcpyAsync(out, m->x, (size_t)H * 4, cudaMemcpyDeviceToHost, m->stream));
  CK(cudaStreamSynchronize(m->stream));
  return SM_OK;
}

// ------------------------------------------------------------ forward ----
int sm_forward_cached(sm_model* m, sm_cache* c, const uint32_t* toks, uint64_t n, float* logits_out) {
  if (guard_model(m) || !c || !toks || c->m != m) { set_error("sm_forward_cached: bad arguments"); return SM_ERR_ARG; }
  if (int g = guard_live(m)) return g;
  std::lock_guard<std::mutex> lk(m->mu);
  cudaSetDevice(m->device);
  int rc = forward_tokens(m, c, toks, n);
  if (rc) return rc;
  if (logits_out) {
    CK(cudaMemcpyAsync(logits_out, m->logits, m->c.vocab_size * 4, cudaMemcpyDeviceToHost, m->stream));
  }
  CK(cudaStreamSynchronize(m->stream));
  return check_waits(m, true);
}

int sm_forward_sample(sm_model* m, sm_cache* c, const uint32_t* toks, uint64_t n, const sm_sampler* s,
                      uint64_t* rng_state, const uint8_t* mask, uint32_t* out_token) {
  if (guard_model(m) || !c || !toks || !rng_state || !out_token || c->m != m) {
    set_error("sm_forward_sample: bad arguments");
    return SM_ERR_ARG;
  }
  int rc = check_sampler(s);
  if (rc) return rc;
  if ((rc = guard_live(m))) return rc;
  std::lock_guard<std::mutex> lk(m->mu);
  cudaSetDevice(m->device);
  if (n == 1 && !mask) {  // the decode step: graph replay
    if (c->len + 1 > c->cap) {
      set_error("decode: position " + std::to_string(c->len) + " is beyond the cache capacity " + std::to_string(c->cap));
      return SM_ERR_CAPACITY;
    }
    if (toks[0] >= m->c.vocab_size) { set_error("token id out of range"); return SM_ERR_ARG; }
    cudaGraphExec_t ex;
    if ((rc = decode_graph(m, 1, &ex))) return rc;
    if ((rc = cache_prepare(m, c, c->len + 1))) return rc;
    CK(cudaStreamSynchronize(m->stream));
    m->hin.tok[0] = toks[0];
    m->hin.rows[0] = RowDesc{0u, (uint32_t)c->len};
    m->hin.seqs[0] = seq_desc(m, c);
    m->hin.sp[0] = to_params(s);
    m->hin.rng[0] = *rng_state;
    m->hin.sel[0] = 0;
    CK(cudaGraphLaunch(ex, m->stream));
    CK(cudaStreamSynchronize(m->stream));
    if ((rc = check_waits(m, false))) return rc;
    c->len += 1;
    *out_token = m->hout.tok[0];
    *rng_state = m->hout.rng[0];
    return SM_OK;
  }
  if ((rc = forward_tokens(m, c, toks, n))) return rc;
  CK(cudaStreamSynchronize(m->stream));  // the staging block is free again
  m->hin.sp[0] = to_params(s);
  m->hin.rng[0] = *rng_state;
  // only sp/rng changed: copy the whole staging block again (small)
  CK(cudaMemcpyAsync(m->in_dev, m->in_host, m->in_bytes, cudaMemcpyHostToDevice, m->stream));
  if ((rc = sample_rows(m, 1, mask, false))) return rc;
  CK(cudaStreamSynchronize(m->stream));
  if ((rc = check_waits(m, false))) return rc;
  *out_token = m->hout.tok[0];
  *rng_state = m->hout.rng[0];
  return SM_OK;
}

static int decode_batch_impl(sm_model* m, sm_cache* const* caches, uint64_t n, const uint32_t* toks,
                             const sm_sampler* samplers, uint64_t* rng_states, uint32_t* out_tokens,
                             float* logits_out) {
  if (guard_model(m) || !caches || !toks || !rng_states || !out_tokens || n == 0) {
    set_error("sm_decode_batch: bad arguments");
    return SM_ERR_ARG;
  }
  if (n > m->rows_max) { set_error("sm_decode_batch: batch larger than the model's max_batch"); return SM_ERR_ARG; }
  if (int g = guard_live(m)) return g;
  for (uint64_t i = 0; i < n; i++) {
    int rc = check_sampler(samplers ? &samplers[i] : nullptr);
    if (rc) return rc;
    if (!caches[i] || caches[i]->m != m) { set_error("sm_decode_batch: cache of another model"); return SM_ERR_ARG; }
    if (caches[i]->len + 1 > caches[i]->cap) { set_error("sm_decode_batch: cache full"); return SM_ERR_CAPACITY; }
    if (toks[i] >= m->c.vocab_size) { set_error("token id out of range"); return SM_ERR_ARG; }
    for (uint64_t j = 0; j < i; j++)
      if (caches[j] == caches[i]) { set_error("sm_decode_batch: a cache appears twice"); return SM_ERR_ARG; }
  }
  std::lock_guard<std::mutex> lk(m->mu);
  cudaSetDevice(m->device);
  cudaGraphExec_t ex;
  int rc = decode_graph(m, (uint32_t)n, &ex);
  if (rc) return rc;
  for (uint64_t i = 0; i < n; i++)
    if ((rc = cache_prepare(m, caches[i], caches[i]->len + 1))) return rc;
  CK(cudaStreamSynchronize(m->stream));
  for (uint64_t i = 0; i < n; i++) {
    sm_cache* c = caches[i];
    m->hin.tok[i] = toks[i];
    m->hin.rows[i] = RowDesc{(uint32_t)i, (uint32_t)c->len};
    m->hin.seqs[i] = seq_desc(m, c);
    m->hin.sp[i] = to_params(samplers ? &samplers[i] : nullptr);
    m->hin.rng[i] = rng_states[i];
    m->hin.sel[i] = (uint32_t)i;
  }
  m->hin.shared[0] = shared_prefix_pages(m, caches, n);
  CK(cudaGraphLaunch(ex, m->stream));
  if (logits_out)  // the logits the step's sampler read (untouched until the next forward)
    CK(cudaMemcpyAsync(logits_out, m->logits, n * m->c.vocab_size * 4, cudaMemcpyDeviceToHost, m->stream));
  CK(cudaStreamSynchronize(m->stream));
  if ((rc = check_waits(m, false))) return rc;
  for (uint64_t i = 0; i < n; i++) {
    caches[i]->len += 1;
    out_tokens[i] = m->hout.tok[i];
    rng_states[i] = m->hout.rng[i];
  }
  return SM_OK;
}

int sm_decode_batch(sm_model* m, sm_cache* const* caches, uint64_t n, const uint32_t* toks, const sm_sampler* samplers,
                    uint64_t* rng_states, uint32_t* out_tokens) {
  return decode_batch_impl(m, caches, n, toks, samplers, rng_states, out_tokens, nullptr);
}

int sm_decode_batch_logits(sm_model* m, sm_cache* const* caches, uint64_t n, const uint32_t* toks,
                           const sm_sampler* samplers, uint64_t* rng_states, uint32_t* out_tokens, float* logits_out) {
  if (!logits_out) { set_error("sm_decode_batch_logits: null logits_out"); return SM_ERR_ARG; }
  return decode_batch_impl(m, caches, n, toks, samplers, rng_states, out_tokens, logits_out);
}

int sm_decode_run(sm_model* m, sm_cache* const* caches, uint64_t n, const uint32_t* toks, const sm_sampler* samplers,
                  uint64_t* rng_states, uint64_t n_steps, uint32_t* out_tokens, void* ev_begin, void* ev_end) {
  if (guard_model(m) || !caches || !toks || !rng_states || !out_tokens || n == 0) {
    set_error("sm_decode_run: bad arguments");
    return SM_ERR_ARG;
  }
  if (n > m->rows_max) { set_error("sm_decode_run: batch larger than the model's max_batch"); return SM_ERR_ARG; }
  if (int g = guard_live(m)) return g;
  if (n_steps == 0) return SM_OK;
  for (uint64_t i = 0; i < n; i++) {
    int rc = check_sampler(samplers ? &samplers[i] : nullptr);
    if (rc) return rc;
    if (!caches[i] || caches[i]->m != m) { set_error("sm_decode_run: cache of another model"); return SM_ERR_ARG; }
    if (caches[i]->len + n_steps > caches[i]->cap) { set_error("sm_decode_run: steps exceed the cache capacity"); return SM_ERR_CAPACITY; }
    if (toks[i] >= m->c.vocab_size) { set_error("token id out of range"); return SM_ERR_ARG; }
    for (uint64_t j = 0; j < i; j++)
      if (caches[j] == caches[i]) { set_error("sm_decode_run: a cache appears twice"); return SM_ERR_ARG; }
  }
  std::lock_guard<std::mutex> lk(m->mu);
  cudaSetDevice(m->device);
  cudaGraphExec_t ex;
  int rc = run_graph(m, (uint32_t)n, &ex);
  if (rc) return rc;
  for (uint64_t i = 0; i < n; i++)
    if ((rc = cache_prepare(m, caches[i], caches[i]->len + n_steps))) return rc;
  const uint64_t chunk = HIST_TOKENS / n;
  CK(cudaStreamSynchronize(m->stream));
  for (uint64_t i = 0; i < n; i++) {
    sm_cache* c = caches[i];
    m->hin.tok[i] = toks[i];
    m->hin.rows[i] = RowDesc{(uint32_t)i, (uint32_t)c->len};
    m->hin.seqs[i] = seq_desc(m, c);
    m->hin.sp[i] = to_params(samplers ? &samplers[i] : nullptr);
    m->hin.rng[i] = rng_states[i];
    m->hin.sel[i] = (uint32_t)i;
  }
  m->hin.shared[0] = shared_prefix_pages(m, caches, n);  // pages below every length stay shared during the run
  CK(cudaMemcpyAsync(m->in_dev, m->in_host, m->in_bytes, cudaMemcpyHostToDevice, m->stream));
  if (ev_begin) CK(cudaEventRecord((cudaEvent_t)ev_begin, m->stream));
  for (uint64_t s0 = 0; s0 < n_steps; s0 += chunk) {
    const uint64_t k = std::min(chunk, n_steps - s0);
    CK(cudaMemsetAsync(m->hist_ctr, 0, 4, m->stream));
    for (uint64_t s = 0; s < k; s++) CK(cudaGraphLaunch(ex, m->stream));
    CK(cudaMemcpyAsync(out_tokens + s0 * n, m->hist, k * n * 4, cudaMemcpyDeviceToHost, m->stream));
  }
  if (ev_end) CK(cudaEventRecord((cudaEvent_t)ev_end, m->stream));
  CK(cudaMemcpyAsync(m->hout.rng, m->din.rng, n * sizeof(uint64_t), cudaMemcpyDeviceToHost, m->stream));
  CK(cudaStreamSynchronize(m->stream));
  if ((rc = check_waits(m, true))) return rc;
  for (uint64_t i = 0; i < n; i++) {
    caches[i]->len += n_steps;
    rng_states[i] = m->hout.rng[i];
  }
  return SM_OK;
}

// ------------------------------------------------- kernel-level entries ----
// Sampler::sample[_masked] (sampling.rs:66-144) on host logits, on the current
// device: rows of `vocab` logits at logits + i * ld (ld = 0: every row samples
// the same logits), mask likewise (may be NULL).
int sm_sample(const float* logits, uint64_t n_rows, uint64_t ld, uint64_t vocab, const uint8_t* mask,
              const sm_sampler* samplers, uint64_t* rng_states, uint32_t* out_tokens) {
  if (!logits || !samplers || !rng_states || !out_tokens || !n_rows || !vocab || vocab > 0xFFFFFFFFull ||
      (ld && ld < vocab)) {
    set_error("sm_sample: bad arguments");
    return SM_ERR_ARG;
  }
  const uint64_t B = 64, uniq = ld ? std::min(n_rows, B) : 1, L = ld ? vocab : 0;
  const uint64_t sw = sample_scratch_words((uint32_t)vocab);
  struct Bufs {
    std::vector<void*> p;
    ~Bufs() { for (void* q : p) cudaFree(q); }
  } bufs;
  auto alloc = [&](size_t n, void** out) -> int {
    if (cudaMalloc(out, std::max<size_t>(n, 16)) != cudaSuccess) {
      cudaGetLastError();
      set_error("sm_sample: cudaMalloc failed");
      return SM_ERR_OOM;
    }
    bufs.p.push_back(*out);
    return SM_OK;
  };
  float* dl = nullptr;
  uint8_t* dm = nullptr;
  SampleParams* dp = nullptr;
  uint64_t* dr = nullptr;
  uint32_t *dt = nullptr, *ds = nullptr;
  int rc;
  if ((rc = alloc(uniq * vocab * 4, (void**)&dl)) || (mask && (rc = alloc(uniq * vocab, (void**)&dm))) ||
      (rc = alloc(B * sizeof(SampleParams), (void**)&dp)) || (rc = alloc(B * 8, (void**)&dr)) ||
      (rc = alloc(B * 4, (void**)&dt)) || (rc = alloc(B * sw * 4, (void**)&ds)))
    return rc;
  std::vector<SampleParams> hp(B);
  for (uint64_t r0 = 0; r0 < n_rows; r0 += B) {
    const uint64_t nb = std::min(B, n_rows - r0);
    if (ld || r0 == 0) {
      for (uint64_t i = 0; i < (ld ? nb : 1); i++) {
        CK(cudaMemcpy(dl + i * vocab, logits + (r0 + i) * ld, vocab * 4, cudaMemcpyHostToDevice));
        if (mask) CK(cudaMemcpy(dm + i * vocab, mask + (r0 + i) * ld, vocab, cudaMemcpyHostToDevice));
      }
    }
    for (uint64_t i = 0; i < nb; i++) hp[i] = to_params(&samplers[r0 + i]);
    CK(cudaMemcpy(dp, hp.data(), nb * sizeof(SampleParams), cudaMemcpyHostToDevice));
    CK(cudaMemcpy(dr, rng_states + r0, nb * 8, cudaMemcpyHostToDevice));
    CK(launch_sample(dl, (uint32_t)vocab, (uint32_t)nb, dm, dp, dr, dt, nullptr, nullptr, ds, 0, L));
    CK(cudaMemcpy(out_tokens + r0, dt, nb * 4, cudaMemcpyDeviceToHost));
    CK(cudaMemcpy(rng_states + r0, dr, nb * 8, cudaMemcpyDeviceToHost));
  }
  return SM_OK;
}

// softmax (sampling.rs:157-172) of rows x n device values (stream order).
int sm_softmax(const float* x_dev, uint64_t rows, uint64_t n, float* probs_dev, void* stream) {
  if (!x_dev || !probs_dev || rows > 0x7FFFFFFFull || n > 0xFFFFFFFFull) { set_error("sm_softmax: bad arguments"); return SM_ERR_ARG; }
  CK(launch_softmax(x_dev, (uint32_t)rows, (uint32_t)n, probs_dev, (cudaStream_t)stream));
  return SM_OK;
}

// The sampler's exp on n device values (stream order).
int sm_expf_ref(const float* x_dev, float* y_dev, uint64_t n, void* stream) {
  if (!x_dev || !y_dev) { set_error("null argument"); return SM_ERR_ARG; }
  CK(launch_expf_ref(x_dev, y_dev, n, (cudaStream_t)stream));
  return SM_OK;
}

struct sm_dweight {
  DW w;
  int device;
  // K-split scratch of its batch-1 tensor-core GEMV (counters zeroed)
  float* ks_part = nullptr;
  uint32_t* ks_cnt = nullptr;
  uint32_t ks_part_cap = 0, ks_cnt_cap = 0;
  // x image of its batched tcgen05 GEMV (up to 32 columns)
  uint8_t* xblob = nullptr;
  uint64_t xblob_cap = 0;
  // error word of the GEMVs' bounded waits (sm_gemv_status reads and clears it)
  uint32_t* err = nullptr;
};

int sm_dweight_upload(uint32_t type, const void* bytes, uint64_t n_out, uint64_t n_in, sm_dweight** out) {
  if (!bytes || !out) { set_error("null argument"); return SM_ERR_ARG; }
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) { cudaGetLastError(); set_error("no CUDA device"); return SM_ERR_CUDA; }
  auto* w = new sm_dweight();
  w->device = dev;
  int rc = upload_weight(type, (const uint8_t*)bytes, n_out, n_in, &w->w);
  if (rc) { delete w; return rc; }
  int sms = 0;
  GemvArgs probe{};
  probe.nseg = 1;
  probe.batch = 1;
  probe.seg[0] = seg(w->w, nullptr, 0, nullptr, EPI_STORE);
  uint64_t need_part = 0;
  uint32_t need_cnt = 0;
  if (cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) == cudaSuccess) {
    gemv_tc_scratch_need(probe, (uint32_t)sms, &need_part, &need_cnt);
    probe.batch = 32;  // the batched kernel's largest split
    probe.ldx = w->w.d.n_in;
    uint64_t pp = 0;
    uint32_t pc = 0;
    gemv_tcb_scratch_need(probe, (uint32_t)sms, &pp, &pc);
    need_part = std::max(need_part, pp);
    need_cnt = std::max(need_cnt, pc);
    gemv_umma_scratch_need(probe, (uint32_t)sms, &pp, &pc);
    need_part = std::max(need_part, pp);
    need_cnt = std::max(need_cnt, pc);
  }
  if (need_part && need_part <= 0xFFFFFFFFull) {
    if (cudaMalloc((void**)&w->ks_part, need_part * 4) != cudaSuccess ||
        cudaMalloc((void**)&w->ks_cnt, (size_t)need_cnt * 4) != cudaSuccess ||
        cudaMemset(w->ks_cnt, 0, (size_t)need_cnt * 4) != cudaSuccess) {
      cudaGetLastError();
      sm_dweight_free(w);
      set_error("cudaMalloc failed for the GEMV scratch");
      return SM_ERR_OOM;
    }
    w->ks_part_cap = (uint32_t)need_part;
    w->ks_cnt_cap = need_cnt;
  }
  if (cudaMalloc((void**)&w->err, 256) != cudaSuccess || cudaMemset(w->err, 0, 256) != cudaSuccess) {
    cudaGetLastError();
    w->err = nullptr;
    sm_dweight_free(w);
    set_error("cudaMalloc failed for the GEMV error word");
    return SM_ERR_OOM;
  }
  if (tiled_type(w->w.d.type)) {
    w->xblob_cap = gemv_umma_blob_bytes(w->w.d.n_in, 32);
    if (cudaMalloc((void**)&w->xblob, w->xblob_cap) != cudaSuccess) {
      cudaGetLastError();
      w->xblob = nullptr;
      sm_dweight_free(w);
      set_error("cudaMalloc failed for the GEMV scratch");
      return SM_ERR_OOM;
    }
  }
  *out = w;
  return SM_OK;
}
int sm_dweight_free(sm_dweight* w) {
  if (!w) return SM_OK;
  if (w->ks_part) cudaFree(w->ks_part);
  if (w->ks_cnt) cudaFree(w->ks_cnt);
  if (w->xblob) cudaFree(w->xblob);
  if (w->err) cudaFree(w->err);
  free_weight(w->w);
  delete w;
  return SM_OK;
}
int sm_dweight_bytes(const sm_dweight* w, uint64_t* out) {
  if (!w || !out) { set_error("null argument"); return SM_ERR_ARG; }
  *out = w->w.enc_bytes;
  return SM_OK;
}
int sm_dequant(const sm_dweight* w, float* out_dev, void* stream) {
  if (!w || !out_dev) { set_error("null argument"); return SM_ERR_ARG; }
  CK(launch_dequant(w->w.d, out_dev, (cudaStream_t)stream));
  return SM_OK;
}
int sm_gemv(const sm_dweight* w, const float* x_dev, float* y_dev, uint64_t batch, void* stream) {
  if (!w || !x_dev || !y_dev) { set_error("null argument"); return SM_ERR_ARG; }
  if (batch < 1 || batch > 32) { set_error("sm_gemv: batch must be 1..32"); return SM_ERR_ARG; }
  if (((uintptr_t)x_dev & 15) || (w->w.d.n_in & 3)) { set_error("sm_gemv: x must be 16-byte aligned"); return SM_ERR_ARG; }
  GemvArgs a{};
  a.x = x_dev;
  a.ldx = w->w.d.n_in;
  a.batch = (uint32_t)batch;
  a.nseg = 1;
  a.seg[0] = seg(w->w, y_dev, w->w.d.n_out, nullptr, EPI_STORE);
  a.ks_part = w->ks_part;
  a.ks_cnt = w->ks_cnt;
  a.ks_part_cap = w->ks_part_cap;
  a.ks_cnt_cap = w->ks_cnt_cap;
  a.xblob = w->xblob;
  a.xblob_cap = w->xblob_cap;
  a.err = w->err;
  CK(launch_gemv(a, (cudaStream_t)stream));
  return SM_OK;
}

int sm_gemv_status(const sm_dweight* w, void* stream) {
  if (!w) { set_error("null argument"); return SM_ERR_ARG; }
  cudaStream_t st = (cudaStream_t)stream;
  uint32_t h = 0;
  CK(cudaMemcpyAsync(&h, w->err, sizeof(h), cudaMemcpyDeviceToHost, st));
  CK(cudaStreamSynchronize(st));
  if (!h) return SM_OK;
  CK(cudaMemsetAsync(w->err, 0, sizeof(uint32_t), st));
  CK(cudaStreamSynchronize(st));
  set_error("a bounded wait in a GEMV on this weight gave up (a weight copy did not complete); its output is invalid");
  return SM_ERR_CUDA;
}

// Same product as sm_gemv, for callers that cannot allocate device memory: the
// batch-1 scratch is a fixed device array of the library (see gemv.cu).
int sm_gemv_noalloc(const sm_dweight* w, const float* x_dev, float* y_dev, uint64_t batch, void* stream) {
  if (!w || !x_dev || !y_dev) { set_error("null argument"); return SM_ERR_ARG; }
  if (batch < 1 || batch > 32) { set_error("sm_gemv_noalloc: batch must be 1..32"); return SM_ERR_ARG; }
  if (((uintptr_t)x_dev & 15) || (w->w.d.n_in & 3)) { set_error("sm_gemv_noalloc: x must be 16-byte aligned"); return SM_ERR_ARG; }
  int dev = -1;
  CK(cudaGetDevice(&dev));
  if (dev != w->device) {
    set_error("sm_gemv_noalloc: the weight lives on device " + std::to_string(w->device) + ", current device is " +
              std::to_string(dev));
    return SM_ERR_ARG;
  }
  GemvArgs a{};
  a.x = x_dev;
  a.ldx = w->w.d.n_in;
  a.batch = (uint32_t)batch;
  a.nseg = 1;
  a.seg[0] = seg(w->w, y_dev, w->w.d.n_out, nullptr, EPI_STORE);
  const cudaError_t e = launch_gemv_noalloc(a, (cudaStream_t)stream);
  if (e == cudaErrorNotSupported) {  // nothing was launched
    set_error("sm_gemv_noalloc: this shape's K-split needs more scratch than the fixed 256 KB array holds "
              "(Q4_K/Q6_K: roughly ceil(n_in / 8192) * n_out floats, rounded up to 16 rows, must be at most "
              "65536; 7168 for Q6_K); use sm_gemv");
    return SM_ERR_ARG;
  }
  CK(e);
  return SM_OK;
}

int sm_gemv_noalloc_status(void* stream) {
  uint32_t flag = 0;
  CK(gemv_noalloc_status((cudaStream_t)stream, &flag));
  if (!flag) return SM_OK;
  set_error("a bounded wait in an sm_gemv_noalloc call on this device gave up (a weight copy did not "
            "complete); that call's output is invalid");
  return SM_ERR_CUDA;
}

}  // extern "C"
