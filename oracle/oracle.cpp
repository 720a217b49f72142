// CPU ORACLE — test infrastructure only (see oracle.hpp for the scope).
// Restates the reference's Rust CPU path op for op; every function cites the
// reference file:line it follows. Built with -O2 -ffp-contract=off.
#include "oracle.hpp"

#include <fcntl.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include <immintrin.h>

#include <algorithm>
#include <cmath>
#include <cstring>
#include <condition_variable>
#include <functional>
#include <mutex>
#include <thread>

namespace orc {

// ---------------------------------------------------------------- types ----
bool is_quantized(uint32_t t) {  // types.rs:129-131 (Unknown counts as not quantized)
  switch (t) {
    case T_F32: case T_F16: case T_BF16: return false;
    case 2: case 3: case 6: case 7: case 8: case 9: case 10: case 11: case 12:
    case 13: case 14: case 15: case 16: case 17: case 18: case 19: case 20:
    case 21: case 22: case 23: case 24: return true;
    default: return false;
  }
}

void block_layout(uint32_t t, uint32_t* bs, uint32_t* tb) {  // types.rs:103-127
  uint32_t b = 32, s = 4;
  switch (t) {
    case 2: b = 32; s = 18; break;
    case 3: b = 32; s = 20; break;
    case 6: b = 32; s = 22; break;
    case 7: b = 32; s = 24; break;
    case 8: b = 32; s = 34; break;
    case 9: b = 32; s = 36; break;
    case 10: b = 256; s = 84; break;
    case 11: b = 256; s = 110; break;
    case 12: b = 256; s = 144; break;
    case 13: b = 256; s = 176; break;
    case 14: b = 256; s = 210; break;
    case 15: b = 256; s = 256; break;
    case 16: b = 256; s = 66; break;
    case 17: b = 256; s = 74; break;
    case 18: b = 256; s = 98; break;
    case 19: b = 256; s = 50; break;
    case 20: b = 256; s = 136; break;
    case 21: b = 256; s = 102; break;
    case 22: b = 256; s = 82; break;
    case 23: b = 256; s = 136; break;
    case 24: b = 256; s = 56; break;
    default: break;
  }
  *bs = b;
  *tb = s;
}

uint32_t type_size(uint32_t t) {  // types.rs:93-99 (BF16 counted as 4, as in the reference)
  return t == T_F16 ? 2 : 4;
}

// -------------------------------------------------------------- dequant ----
float fp16_to_f32(uint16_t h) {  // dequant.rs:12-33
  uint32_t sign = (h >> 15) & 1u;
  uint32_t exp = (h >> 10) & 0x1Fu;
  uint32_t frac = h & 0x3FFu;
  uint32_t e, f;
  if (exp == 0) {
    if (frac == 0) {
      e = 0;
      f = 0;
    } else {
      float val = (float)frac * 5.9604645e-8f;  // frac * 2^-24, exact
      return sign == 1 ? -val : val;
    }
  } else if (exp == 0x1F) {
    // NaN payload 0x200000 shifted by 13 overflows u32 to 0: NaN decodes to ±Inf.
    e = 0xFF;
    f = frac == 0 ? 0u : 0x200000u;
  } else {
    e = exp + 127 - 15;
    f = frac;
  }
  uint32_t bits = (sign << 31) | (e << 23) | (uint32_t)(f << 13);
  float out;
  std::memcpy(&out, &bits, 4);
  return out;
}

float bf16_to_f32(uint16_t h) {  // dequant.rs:36-38
  uint32_t bits = (uint32_t)h << 16;
  float out;
  std::memcpy(&out, &bits, 4);
  return out;
}

static inline uint16_t rd16(const uint8_t* p) { return (uint16_t)(p[0] | ((uint16_t)p[1] << 8)); }

void get_scale_min_k4(int j, const uint8_t* s, uint8_t* d, uint8_t* m) {  // dequant.rs:41-49
  if (j < 4) {
    *d = s[j] & 63;
    *m = s[j + 4] & 63;
  } else {
    *d = (uint8_t)((s[j + 4] & 0x0F) | ((s[j - 4] >> 6) << 4));
    *m = (uint8_t)((s[j + 4] >> 4) | ((s[j] >> 6) << 4));
  }
}

void dequant_q4_0(const uint8_t* b, float* out) {  // dequant.rs:54-63
  float d = fp16_to_f32(rd16(b));
  const uint8_t* qs = b + 2;
  for (int i = 0; i < 16; i++) {
    out[i] = d * (float)(qs[i] & 0x0F);
    out[i + 16] = d * (float)(qs[i] >> 4);
  }
}

void dequant_q8_0(const uint8_t* b, float* out) {  // dequant.rs:66-71
  float d = fp16_to_f32(rd16(b));
  for (int i = 0; i < 32; i++) out[i] = (float)(int8_t)b[2 + i] * d;
}

void dequant_q5_0(const uint8_t* b, float* out) {  // dequant.rs:79-94
  float d = fp16_to_f32(rd16(b));
  uint32_t qh = (uint32_t)b[2] | ((uint32_t)b[3] << 8) | ((uint32_t)b[4] << 16) | ((uint32_t)b[5] << 24);
  const uint8_t* qs = b + 6;
  for (int l = 0; l < 16; l++) {
    int32_t hi_lo = (int32_t)(((qh >> l) & 1u) << 4);
    int32_t hi_hi = (int32_t)(((qh >> (l + 16)) & 1u) << 4);
    int32_t q_lo = ((int32_t)(qs[l] & 0x0F) | hi_lo) - 16;
    int32_t q_hi = ((int32_t)(qs[l] >> 4) | hi_hi) - 16;
    out[l] = d * (float)q_lo;
    out[l + 16] = d * (float)q_hi;
  }
}

void dequant_q4_k(const uint8_t* b, float* out) {  // dequant.rs:98-124
  float d = fp16_to_f32(rd16(b));
  float mn = fp16_to_f32(rd16(b + 2));
  const uint8_t* scales = b + 4;
  const uint8_t* qs = b + 16;
  int is = 0, idx = 0, qoff = 0;
  for (int j = 0; j < 4; j++) {
    uint8_t ds1, ms1, ds2, ms2;
    get_scale_min_k4(is, scales, &ds1, &ms1);
    float d1 = d * (float)ds1;
    float m1 = mn * (float)ms1;
    get_scale_min_k4(is + 1, scales, &ds2, &ms2);
    float d2 = d * (float)ds2;
    float m2 = mn * (float)ms2;
    for (int l = 0; l < 32; l++) out[idx + l] = d1 * (float)(qs[qoff + l] & 0x0F) - m1;
    for (int l = 0; l < 32; l++) out[idx + 32 + l] = d2 * (float)(qs[qoff + l] >> 4) - m2;
    qoff += 32;
    idx += 64;
    is += 2;
  }
}

void dequant_q4_1(const uint8_t* b, float* out) {  // dequant.rs:128-136
  float d = fp16_to_f32(rd16(b));
  float dm = fp16_to_f32(rd16(b + 2));
  const uint8_t* qs = b + 4;
  for (int i = 0; i < 16; i++) {
    out[i] = d * (float)(qs[i] & 0x0F) + dm;
    out[i + 16] = d * (float)(qs[i] >> 4) + dm;
  }
}

void dequant_q6_k(const uint8_t* b, float* out) {  // dequant.rs:178-206
  const uint8_t* ql = b;
  const uint8_t* qh = b + 128;
  const uint8_t* sc = b + 192;
  float d = fp16_to_f32(rd16(b + 208));
  if (!std::isfinite(d)) {
    for (int i = 0; i < 256; i++) out[i] = 0.0f;
    return;
  }
  int yoff = 0;
  for (int n = 0; n < 2; n++) {
    int qloff = n * 64, qhoff = n * 32, scoff = n * 8;
    for (int is = 0; is < 2; is++) {  // is = l / 16: the scale is fixed over 16 values of l
      // (d * sc) * q, left to right as written in the reference
      const float s1 = d * (float)(int8_t)sc[scoff + is], s2 = d * (float)(int8_t)sc[scoff + is + 2];
      const float s3 = d * (float)(int8_t)sc[scoff + is + 4], s4 = d * (float)(int8_t)sc[scoff + is + 6];
      for (int l = 16 * is; l < 16 * is + 16; l++) {
        int32_t q1 = (int32_t)((ql[qloff + l] & 0x0F) | (((qh[qhoff + l] >> 0) & 3) << 4)) - 32;
        int32_t q2 = (int32_t)((ql[qloff + l + 32] & 0x0F) | (((qh[qhoff + l] >> 2) & 3) << 4)) - 32;
        int32_t q3 = (int32_t)((ql[qloff + l] >> 4) | (((qh[qhoff + l] >> 4) & 3) << 4)) - 32;
        int32_t q4 = (int32_t)((ql[qloff + l + 32] >> 4) | (((qh[qhoff + l] >> 6) & 3) << 4)) - 32;
        out[yoff + l] = s1 * (float)q1;
        out[yoff + l + 32] = s2 * (float)q2;
        out[yoff + l + 64] = s3 * (float)q3;
        out[yoff + l + 96] = s4 * (float)q4;
      }
    }
    yoff += 128;
  }
}

int dequantize(uint32_t type, uint64_t n, const uint8_t* raw, uint64_t raw_len, float* out,
               std::string* err) {  // dequant.rs:209-310
  for (uint64_t i = 0; i < n; i++) out[i] = 0.0f;
  auto blocks = [&](void (*fn)(const uint8_t*, float*), uint32_t bs, uint32_t tb) {
    uint64_t off = 0;
    // chunks_exact(tb): a trailing partial block is ignored
    for (uint64_t p = 0; p + tb <= raw_len; p += tb) {
      if (off + bs > n) break;
      fn(raw + p, out + off);
      off += bs;
    }
  };
  switch (type) {
    case T_F32:
      if (raw_len < n * 4) { if (err) *err = "truncated"; return -1; }
      std::memcpy(out, raw, n * 4);
      return 0;
    case T_F16:
      if (raw_len < n * 2) { if (err) *err = "truncated"; return -1; }
      for (uint64_t i = 0; i < n; i++) out[i] = fp16_to_f32(rd16(raw + 2 * i));
      return 0;
    case T_BF16:
      if (raw_len < n * 2) { if (err) *err = "truncated"; return -1; }
      for (uint64_t i = 0; i < n; i++) out[i] = bf16_to_f32(rd16(raw + 2 * i));
      return 0;
    case T_Q4_0: blocks(dequant_q4_0, 32, 18); return 0;
    case T_Q4_1: blocks(dequant_q4_1, 32, 20); return 0;
    case T_Q5_0: blocks(dequant_q5_0, 32, 22); return 0;
    case T_Q8_0: blocks(dequant_q8_0, 32, 34); return 0;
    case T_Q4K: blocks(dequant_q4_k, 256, 144); return 0;
    case T_Q6K: blocks(dequant_q6_k, 256, 210); return 0;
    default:
      // Q5_K exists in the reference (dequant.rs:141-172) with a non-standard
      // qh indexing; Q4_K_M files never hold Q5_K, so it is not restated.
      if (err) *err = "dequant not implemented for type " + std::to_string(type);
      return -1;
  }
}

// ----------------------------------------------------------------- GGUF ----
bool Value::as_u64(uint64_t* out) const {  // value.rs:61-73
  switch (type) {
    case 0: case 2: case 4: case 10: *out = u; return true;
    case 1: case 3: case 5: case 11: *out = (uint64_t)i; return true;
    default: return false;
  }
}
bool Value::as_f32(float* out) const {  // value.rs:82-88
  if (type == 6) { *out = (float)f; return true; }
  if (type == 12) { *out = (float)f; return true; }
  return false;
}

uint64_t TensorInfo::n_elements() const {  // lib.rs:81-83
  uint64_t p = 1;
  for (auto d : dims) p *= d;
  return p;
}
uint64_t TensorInfo::n_bytes() const {  // lib.rs:85-93
  if (is_quantized(type)) {
    uint32_t bs, tb;
    block_layout(type, &bs, &tb);
    return (n_elements() / bs) * tb;
  }
  return n_elements() * type_size(type);
}

Gguf::~Gguf() {
  if (map) munmap((void*)map, map_len);
}
const TensorInfo* Gguf::tensor(const std::string& name) const {
  for (auto& t : tensors)
    if (t.name == name) return &t;
  return nullptr;
}
const Value* Gguf::meta(const std::string& key) const {
  for (auto& kv : metadata)
    if (kv.first == key) return &kv.second;
  return nullptr;
}
const uint8_t* Gguf::raw(const TensorInfo& t, std::string* err) const {
  uint64_t abs = data_start + t.offset;
  if (abs > map_len || t.n_bytes() > map_len - abs) {
    if (err) *err = t.name + ": truncated tensor data";
    return nullptr;
  }
  return map + abs;
}

namespace {
struct Cursor {
  const uint8_t* p;
  size_t n, pos = 0;
  bool ok = true;
  bool need(size_t k) {
    if (!ok || n - pos < k) { ok = false; return false; }
    return true;
  }
  uint8_t u8() { if (!need(1)) return 0; return p[pos++]; }
  uint16_t u16() { if (!need(2)) return 0; uint16_t v; std::memcpy(&v, p + pos, 2); pos += 2; return v; }
  uint32_t u32() { if (!need(4)) return 0; uint32_t v; std::memcpy(&v, p + pos, 4); pos += 4; return v; }
  uint64_t u64() { if (!need(8)) return 0; uint64_t v; std::memcpy(&v, p + pos, 8); pos += 8; return v; }
  std::string str() {  // lib.rs:256-262
    uint64_t len = u64();
    if (!need(len)) return {};
    std::string s((const char*)p + pos, len);
    pos += len;
    return s;
  }
};

bool read_value(Cursor& c, uint32_t vt, Value& v, std::string* err, int depth) {  // value.rs:28-58
  v.type = vt;
  switch (vt) {
    case 0: v.u = c.u8(); break;
    case 1: v.i = (int8_t)c.u8(); break;
    case 2: v.u = c.u16(); break;
    case 3: v.i = (int16_t)c.u16(); break;
    case 4: v.u = c.u32(); break;
    case 5: v.i = (int32_t)c.u32(); break;
    case 6: { uint32_t b = c.u32(); float f; std::memcpy(&f, &b, 4); v.f = f; break; }
    case 7: v.b = c.u8() != 0; break;
    case 8: v.s = c.str(); break;
    case 9: {
      uint32_t et = c.u32();
      uint64_t n = c.u64();
      if (n > 100000000ull) { if (err) *err = "array count " + std::to_string(n); return false; }
      if (depth > 8) { if (err) *err = "nested arrays too deep"; return false; }
      v.elem_type = et;
      for (uint64_t k = 0; k < n && c.ok; k++) {
        Value e;
        if (!read_value(c, et, e, err, depth + 1)) return false;
        v.arr.push_back(std::move(e));
      }
      break;
    }
    case 10: v.u = c.u64(); break;
    case 11: v.i = (int64_t)c.u64(); break;
    case 12: { uint64_t b = c.u64(); std::memcpy(&v.f, &b, 8); break; }
    default: if (err) *err = "bad value type " + std::to_string(vt); return false;
  }
  if (!c.ok) { if (err) *err = "truncated header"; return false; }
  return true;
}
}  // namespace

std::unique_ptr<Gguf> gguf_open(const std::string& path, std::string* err) {  // lib.rs:114-179
  int fd = ::open(path.c_str(), O_RDONLY);
  if (fd < 0) { if (err) *err = "io: cannot open " + path; return nullptr; }
  struct stat st;
  if (fstat(fd, &st) != 0) { ::close(fd); if (err) *err = "io: stat"; return nullptr; }
  size_t len = (size_t)st.st_size;
  void* m = len ? mmap(nullptr, len, PROT_READ, MAP_PRIVATE, fd, 0) : nullptr;
  ::close(fd);
  if (len && m == MAP_FAILED) { if (err) *err = "io: mmap"; return nullptr; }
  auto g = std::make_unique<Gguf>();
  g->map = (const uint8_t*)m;
  g->map_len = len;
  Cursor c{g->map, len};
  uint32_t magic = c.u32();
  if (!c.ok) { if (err) *err = "io: unexpected eof"; return nullptr; }
  if (magic != 0x46554747u) { if (err) *err = "bad magic (expected GGUF)"; return nullptr; }
  g->version = c.u32();
  if (g->version != 3 && g->version != 2) {
    if (err) *err = "unsupported GGUF version " + std::to_string(g->version);
    return nullptr;
  }
  g->tensor_count = c.u64();
  g->kv_count = c.u64();
  if (!c.ok) { if (err) *err = "io: unexpected eof"; return nullptr; }
  for (uint64_t k = 0; k < g->kv_count; k++) {
    std::string key = c.str();
    uint32_t vt = c.u32();
    if (!c.ok) { if (err) *err = "io: unexpected eof"; return nullptr; }
    Value v;
    if (!read_value(c, vt, v, err, 0)) return nullptr;
    if (key == "general.alignment" && v.type == 4) g->alignment = v.u;  // lib.rs:138-142
    g->metadata.emplace_back(std::move(key), std::move(v));
  }
  for (uint64_t k = 0; k < g->tensor_count; k++) {
    TensorInfo t;
    t.name = c.str();
    uint32_t nd = c.u32();
    if (!c.ok) { if (err) *err = "io: unexpected eof"; return nullptr; }
    if (nd == 0 || nd > 8) {
      if (err) *err = "bad tensor: " + t.name + ": n_dims=" + std::to_string(nd) + " out of range";
      return nullptr;
    }
    for (uint32_t d = 0; d < nd; d++) t.dims.push_back(c.u64());
    t.type = c.u32();
    t.offset = c.u64();
    if (!c.ok) { if (err) *err = "io: unexpected eof"; return nullptr; }
    g->tensors.push_back(std::move(t));
  }
  uint64_t header_end = c.pos;
  if (g->alignment == 0) { if (err) *err = "bad alignment 0"; return nullptr; }
  g->data_start = g->tensor_count > 0
                      ? ((header_end + g->alignment - 1) / g->alignment) * g->alignment
                      : header_end;  // lib.rs:168-173
  return g;
}

// ---------------------------------------------------------------- model ----
// A persistent pool of worker threads: parallel_for splits [0, n) into
// contiguous chunks, one per thread, and returns when all are done. Which
// thread computes a chunk never changes a result (chunks are independent
// output elements).
namespace {
class Pool {
 public:
  ~Pool() {
    {
      std::lock_guard<std::mutex> lk(mu_);
      stop_ = true;
    }
    cv_.notify_all();
    for (auto& t : workers_) t.join();
  }
  void run(size_t parts, const std::function<void(size_t)>& fn) {
    std::lock_guard<std::mutex> serial(run_mu_);  // one parallel_for at a time
    {
      std::unique_lock<std::mutex> lk(mu_);
      while (workers_.size() + 1 < parts) {
        const size_t id = workers_.size() + 1;
        workers_.emplace_back([this, id] { loop(id); });
      }
      fn_ = &fn;
      parts_ = parts;
      pending_ = parts - 1;
      gen_++;
    }
    cv_.notify_all();
    fn(0);
    std::unique_lock<std::mutex> lk(mu_);
    done_.wait(lk, [this] { return pending_ == 0; });
    fn_ = nullptr;
  }

 private:
  void loop(size_t id) {
    uint64_t seen = 0;
    for (;;) {
      const std::function<void(size_t)>* fn = nullptr;
      {
        std::unique_lock<std::mutex> lk(mu_);
        cv_.wait(lk, [&] { return stop_ || gen_ != seen; });
        if (stop_) return;
        seen = gen_;
        if (id >= parts_) continue;
        fn = fn_;
      }
      (*fn)(id);
      std::lock_guard<std::mutex> lk(mu_);
      if (--pending_ == 0) done_.notify_one();
    }
  }
  std::mutex run_mu_, mu_;
  std::condition_variable cv_, done_;
  std::vector<std::thread> workers_;
  const std::function<void(size_t)>* fn_ = nullptr;
  size_t parts_ = 0, pending_ = 0;
  uint64_t gen_ = 0;
  bool stop_ = false;
};
Pool& pool() {
  static Pool p;
  return p;
}
}  // namespace

static void parallel_for(int threads, size_t n, const std::function<void(size_t, size_t)>& fn) {
  if (threads <= 1 || n < 2) { fn(0, n); return; }
  const size_t t = std::min<size_t>((size_t)threads, n), chunk = (n + t - 1) / t;
  const size_t parts = (n + chunk - 1) / chunk;
  pool().run(parts, [&](size_t i) { fn(i * chunk, std::min(n, (i + 1) * chunk)); });
}

void QWeight::row(size_t o, float* out) const {
  if (!dense.empty()) { std::memcpy(out, dense.data() + o * n_in, n_in * 4); return; }
  if (type == T_F32) { std::memcpy(out, raw + o * n_in * 4, n_in * 4); return; }
  uint32_t bs, tb;
  block_layout(type, &bs, &tb);
  size_t row_bytes = n_in / bs * tb;
  dequantize(type, n_in, raw + o * row_bytes, row_bytes, out, nullptr);
}

// Elements [d0, d0 + n) of row o: whole quant blocks (d0 and n multiples of
// the block size, which tile_width() guarantees).
void QWeight::row_range(size_t o, size_t d0, size_t n, float* out) const {
  if (!dense.empty()) { std::memcpy(out, dense.data() + o * n_in + d0, n * 4); return; }
  if (type == T_F32) { std::memcpy(out, raw + (o * n_in + d0) * 4, n * 4); return; }
  uint32_t bs, tb;
  block_layout(type, &bs, &tb);
  const size_t row_bytes = n_in / bs * tb;
  dequantize(type, n, raw + o * row_bytes + d0 / bs * tb, n / bs * tb, out, nullptr);
}
size_t QWeight::tile_width() const {
  if (!dense.empty() || type == T_F32) return 256;
  uint32_t bs, tb;
  block_layout(type, &bs, &tb);
  return bs >= 256 ? bs : 256 / bs * bs;
}

static bool load_weight(Gguf& g, const std::string& name, QWeight& w, std::string* err) {
  const TensorInfo* t = g.tensor(name);
  if (!t) { if (err) *err = name + ": tensor not found: " + name; return false; }
  const uint8_t* raw = g.raw(*t, err);
  if (!raw) return false;
  w.raw = raw;
  w.type = t->type;
  w.n_in = t->dims[0];
  w.n_out = t->n_elements() / w.n_in;
  uint32_t bs = 1, tb = 4;
  if (is_quantized(t->type)) block_layout(t->type, &bs, &tb);
  bool rows_ok = t->type == T_F32 || (is_quantized(t->type) && w.n_in % bs == 0 &&
                                      (t->type == T_Q4_0 || t->type == T_Q4_1 || t->type == T_Q5_0 ||
                                       t->type == T_Q8_0 || t->type == T_Q4K || t->type == T_Q6K));
  if (!rows_ok) {  // whole-tensor dequant, exactly like tensor_data_f32
    w.dense.assign(t->n_elements(), 0.f);
    if (dequantize(t->type, t->n_elements(), raw, t->n_bytes(), w.dense.data(), err) != 0) {
      *err = name + ": " + *err;
      return false;
    }
  }
  return true;
}

static bool load_f32(Gguf& g, const std::string& name, std::vector<float>& out, std::string* err) {
  const TensorInfo* t = g.tensor(name);
  if (!t) { if (err) *err = name + ": tensor not found: " + name; return false; }
  const uint8_t* raw = g.raw(*t, err);
  if (!raw) return false;
  out.assign(t->n_elements(), 0.f);
  if (dequantize(t->type, t->n_elements(), raw, t->n_bytes(), out.data(), err) != 0) {
    *err = name + ": " + *err;
    return false;
  }
  return true;
}

std::unique_ptr<Model> model_load(const std::string& path, int threads, std::string* err) {
  auto m = std::make_unique<Model>();
  m->threads = threads < 1 ? 1 : threads;
  m->g = gguf_open(path, err);
  if (!m->g) return nullptr;
  Gguf& g = *m->g;
  // Famiglia::detect (registry.rs:38-60)
  const Value* arch = g.meta("general.architecture");
  if (!arch || arch->type != 8) { *err = "missing metadata: general.architecture"; return nullptr; }
  if (arch->s != "qwen2" && arch->s != "llama") {
    *err = "architecture '" + arch->s + "' not supported (qwen2, llama)";
    return nullptr;
  }
  // Config::from_gguf (qwen2.rs:30-63)
  auto get_u = [&](const std::string& suf, size_t* out) -> bool {
    for (const char* pre : {"qwen2", "llama"}) {
      const Value* v = g.meta(std::string(pre) + "." + suf);
      if (v) {
        uint64_t u;
        if (!v->as_u64(&u)) { *err = std::string(pre) + "." + suf + ": unexpected type"; return false; }
        *out = (size_t)u;
        return true;
      }
    }
    *err = "missing metadata: " + suf;
    return false;
  };
  auto get_f = [&](const std::string& suf, float* out) -> bool {
    for (const char* pre : {"qwen2", "llama"}) {
      const Value* v = g.meta(std::string(pre) + "." + suf);
      if (v) {
        if (!v->as_f32(out)) { *err = std::string(pre) + "." + suf + ": unexpected type"; return false; }
        return true;
      }
    }
    *err = "missing metadata: " + suf;
    return false;
  };
  Config& c = m->c;
  if (!get_u("embedding_length", &c.n_embd) || !get_u("attention.head_count", &c.n_heads) ||
      !get_u("attention.head_count_kv", &c.n_kv_heads) || !get_u("block_count", &c.n_layers) ||
      !get_u("feed_forward_length", &c.n_ff) || !get_f("rope.freq_base", &c.rope_theta) ||
      !get_f("attention.layer_norm_rms_epsilon", &c.rms_eps))
    return nullptr;
  if (c.n_heads == 0 || c.n_kv_heads == 0) { *err = "zero heads"; return nullptr; }
  c.head_dim = c.n_embd / c.n_heads;
  const TensorInfo* te = g.tensor("token_embd.weight");
  if (!te) { *err = "tensor not found: token_embd.weight"; return nullptr; }
  if (te->dims.size() < 2) { *err = "token_embd.weight: expected 2 dims"; return nullptr; }
  c.vocab_size = te->dims[1];
  // Model::load (qwen2.rs:99-150)
  if (!load_weight(g, "token_embd.weight", m->tok_embd, err)) return nullptr;
  if (g.tensor("output.weight")) {
    if (!load_weight(g, "output.weight", m->output, err)) return nullptr;
  } else {
    m->output = m->tok_embd;  // tied embeddings (qwen2.rs:115-118)
  }
  if (!load_f32(g, "output_norm.weight", m->output_norm, err)) return nullptr;
  for (size_t i = 0; i < c.n_layers; i++) {
    LayerW L;
    std::string p = "blk." + std::to_string(i) + ".";
    auto opt = [&](const char* n, bool* has, std::vector<float>& b) -> bool {  // opt_bias (qwen2.rs:687-697)
      if (!g.tensor(p + n)) { *has = false; return true; }
      *has = true;
      return load_f32(g, p + n, b, err);
    };
    if (!opt("attn_q.bias", &L.has_bq, L.bq) || !opt("attn_k.bias", &L.has_bk, L.bk) ||
        !opt("attn_v.bias", &L.has_bv, L.bv))
      return nullptr;
    if (!load_f32(g, p + "attn_norm.weight", L.attn_norm, err) ||
        !load_weight(g, p + "attn_q.weight", L.wq, err) || !load_weight(g, p + "attn_k.weight", L.wk, err) ||
        !load_weight(g, p + "attn_v.weight", L.wv, err) ||
        !load_weight(g, p + "attn_output.weight", L.wo, err) ||
        !load_f32(g, p + "ffn_norm.weight", L.ffn_norm, err) ||
        !load_weight(g, p + "ffn_gate.weight", L.w_gate, err) ||
        !load_weight(g, p + "ffn_up.weight", L.w_up, err) ||
        !load_weight(g, p + "ffn_down.weight", L.w_down, err))
      return nullptr;
    m->layers.push_back(std::move(L));
  }
  return m;
}

SeqState SeqState::all_kv(size_t n_layers, size_t kv_dim, size_t max_seq) {  // state.rs:212-214, 72-74
  SeqState s;
  s.n_layers = n_layers;
  s.dim = kv_dim;
  s.cap = max_seq;
  s.k.assign(n_layers, std::vector<float>(max_seq * kv_dim, 0.f));
  s.v.assign(n_layers, std::vector<float>(max_seq * kv_dim, 0.f));
  return s;
}
void SeqState::ensure_capacity(size_t min_capacity) {  // state.rs:112-119, 323-329
  if (min_capacity <= cap) return;
  for (size_t l = 0; l < n_layers; l++) {
    k[l].resize(min_capacity * dim, 0.f);
    v[l].resize(min_capacity * dim, 0.f);
  }
  cap = min_capacity;
}
int SeqState::truncate(size_t new_len, std::string* err) {  // state.rs:341-360 (all-KV case)
  if (new_len > len) {
    if (err) *err = "truncate: " + std::to_string(new_len) + " > len=" + std::to_string(len);
    return -1;
  }
  len = new_len;
  return 0;
}

// y(seq×n_out) = x(seq×n_in) @ W^T, each sum sequential over d (qwen2.rs:663-674).
// Every output element is its own running sum, updated as sum = sum + w*x
// (a rounded product, then a rounded add) for d = 0, 1, ... in order, as the
// reference's loop does. The work is vectorized ACROSS independent sums: a
// lane of an 8-wide vector holds one row's sum (decode: 32 rows side by
// side, weights transposed so that one load brings w[o..o+7][d]) or one
// token's sum (prefill: one row, 32 tokens side by side, x transposed).
// Lanes never mix, so each result is bit-identical to the scalar loop.
typedef float v8f __attribute__((vector_size(32)));

static inline v8f v8_load(const float* p) {
  v8f v;
  std::memcpy(&v, p, sizeof(v));
  return v;
}
static inline v8f v8_splat(float f) { return v8f{f, f, f, f, f, f, f, f}; }

// wt[d][32] = rows[r][d] for r < 32, d < dl (dl a multiple of 8), by 8x8
// register transposes (pure data movement).
static void transpose_tile(const float* rows, size_t ld, size_t dl, float* wt) {
  for (size_t rb = 0; rb < 32; rb += 8)
    for (size_t d0 = 0; d0 < dl; d0 += 8) {
      __m256 r0 = _mm256_loadu_ps(rows + (rb + 0) * ld + d0), r1 = _mm256_loadu_ps(rows + (rb + 1) * ld + d0);
      __m256 r2 = _mm256_loadu_ps(rows + (rb + 2) * ld + d0), r3 = _mm256_loadu_ps(rows + (rb + 3) * ld + d0);
      __m256 r4 = _mm256_loadu_ps(rows + (rb + 4) * ld + d0), r5 = _mm256_loadu_ps(rows + (rb + 5) * ld + d0);
      __m256 r6 = _mm256_loadu_ps(rows + (rb + 6) * ld + d0), r7 = _mm256_loadu_ps(rows + (rb + 7) * ld + d0);
      __m256 t0 = _mm256_unpacklo_ps(r0, r1), t1 = _mm256_unpackhi_ps(r0, r1);
      __m256 t2 = _mm256_unpacklo_ps(r2, r3), t3 = _mm256_unpackhi_ps(r2, r3);
      __m256 t4 = _mm256_unpacklo_ps(r4, r5), t5 = _mm256_unpackhi_ps(r4, r5);
      __m256 t6 = _mm256_unpacklo_ps(r6, r7), t7 = _mm256_unpackhi_ps(r6, r7);
      __m256 u0 = _mm256_shuffle_ps(t0, t2, 0x44), u1 = _mm256_shuffle_ps(t0, t2, 0xEE);
      __m256 u2 = _mm256_shuffle_ps(t1, t3, 0x44), u3 = _mm256_shuffle_ps(t1, t3, 0xEE);
      __m256 u4 = _mm256_shuffle_ps(t4, t6, 0x44), u5 = _mm256_shuffle_ps(t4, t6, 0xEE);
      __m256 u6 = _mm256_shuffle_ps(t5, t7, 0x44), u7 = _mm256_shuffle_ps(t5, t7, 0xEE);
      float* o = wt + d0 * 32 + rb;
      _mm256_storeu_ps(o + 0 * 32, _mm256_permute2f128_ps(u0, u4, 0x20));
      _mm256_storeu_ps(o + 1 * 32, _mm256_permute2f128_ps(u1, u5, 0x20));
      _mm256_storeu_ps(o + 2 * 32, _mm256_permute2f128_ps(u2, u6, 0x20));
      _mm256_storeu_ps(o + 3 * 32, _mm256_permute2f128_ps(u3, u7, 0x20));
      _mm256_storeu_ps(o + 4 * 32, _mm256_permute2f128_ps(u0, u4, 0x31));
      _mm256_storeu_ps(o + 5 * 32, _mm256_permute2f128_ps(u1, u5, 0x31));
      _mm256_storeu_ps(o + 6 * 32, _mm256_permute2f128_ps(u2, u6, 0x31));
      _mm256_storeu_ps(o + 7 * 32, _mm256_permute2f128_ps(u3, u7, 0x31));
    }
}

static void matmul_rows(const QWeight& w, const float* x, size_t seq, float* y, int threads) {
  const size_t n_in = w.n_in, n_out = w.n_out;
  if (seq < 8) {
    // decode-sized: groups of 32 rows; K in tiles of (up to) 256 weights: the
    // tile of all 32 rows is dequantized, transposed to wt[d][32] and applied
    // to every token, each lane's running sum carried across tiles in d order.
    const size_t groups = (n_out + 31) / 32, TW = w.tile_width();
    parallel_for(threads, groups, [&](size_t gb, size_t ge) {
      std::vector<float> rows(32 * TW, 0.f), wt(32 * TW), acc(32 * seq);
      for (size_t gi = gb; gi < ge; gi++) {
        const size_t o0 = gi * 32, nr = std::min<size_t>(32, n_out - o0);
        std::fill(acc.begin(), acc.end(), 0.f);
        for (size_t d0 = 0; d0 < n_in; d0 += TW) {
          const size_t dl = std::min(TW, n_in - d0);
          for (size_t r = 0; r < nr; r++) w.row_range(o0 + r, d0, dl, rows.data() + r * TW);
          transpose_tile(rows.data(), TW, dl, wt.data());
          for (size_t s = 0; s < seq; s++) {
            const float* xs = x + s * n_in + d0;
            float* as = acc.data() + s * 32;
            v8f a0 = v8_load(as), a1 = v8_load(as + 8), a2 = v8_load(as + 16), a3 = v8_load(as + 24);
            const float* t = wt.data();
            for (size_t d = 0; d < dl; d++, t += 32) {
              const v8f xv = v8_splat(xs[d]);
              a0 = a0 + v8_load(t) * xv;
              a1 = a1 + v8_load(t + 8) * xv;
              a2 = a2 + v8_load(t + 16) * xv;
              a3 = a3 + v8_load(t + 24) * xv;
            }
            std::memcpy(as, &a0, 32);
            std::memcpy(as + 8, &a1, 32);
            std::memcpy(as + 16, &a2, 32);
            std::memcpy(as + 24, &a3, 32);
          }
        }
        for (size_t s = 0; s < seq; s++)
          for (size_t r = 0; r < nr; r++) y[s * n_out + o0 + r] = acc[s * 32 + r];
      }
    });
    return;
  }
  // prefill-sized: x transposed per group of 8 tokens (xt[g][d][8]); rows in
  // groups of 4 against pairs of token groups (8 independent vectors).
  const size_t ng = seq / 8, tail = seq - 8 * ng;
  std::vector<float> xt(ng * n_in * 8);
  for (size_t g = 0; g < ng; g++)
    for (size_t d = 0; d < n_in; d++)
      for (size_t l = 0; l < 8; l++) xt[(g * n_in + d) * 8 + l] = x[(8 * g + l) * n_in + d];
  const size_t rgroups = (n_out + 3) / 4;
  parallel_for(threads, rgroups, [&](size_t b, size_t e) {
    std::vector<float> rowbuf(4 * n_in, 0.f);
    for (size_t rg = b; rg < e; rg++) {
      const size_t o0 = rg * 4, nr = std::min<size_t>(4, n_out - o0);
      for (size_t r = 0; r < nr; r++) w.row(o0 + r, rowbuf.data() + r * n_in);
      const float* r0 = rowbuf.data();
      const float* r1 = r0 + n_in;
      const float* r2 = r1 + n_in;
      const float* r3 = r2 + n_in;
      auto store = [&](size_t g, size_t r, const v8f& a) {
        if (r < nr)
          for (size_t l = 0; l < 8; l++) y[(8 * g + l) * n_out + o0 + r] = a[l];
      };
      size_t g = 0;
      for (; g + 2 <= ng; g += 2) {
        v8f a00 = v8_splat(0.f), a01 = a00, a10 = a00, a11 = a00, a20 = a00, a21 = a00, a30 = a00, a31 = a00;
        const float* t0 = xt.data() + g * n_in * 8;
        const float* t1 = t0 + n_in * 8;
        for (size_t d = 0; d < n_in; d++) {
          const v8f x0 = v8_load(t0 + 8 * d), x1 = v8_load(t1 + 8 * d);
          const v8f w0 = v8_splat(r0[d]), w1 = v8_splat(r1[d]), w2 = v8_splat(r2[d]), w3 = v8_splat(r3[d]);
          a00 = a00 + w0 * x0; a01 = a01 + w0 * x1;
          a10 = a10 + w1 * x0; a11 = a11 + w1 * x1;
          a20 = a20 + w2 * x0; a21 = a21 + w2 * x1;
          a30 = a30 + w3 * x0; a31 = a31 + w3 * x1;
        }
        store(g, 0, a00); store(g + 1, 0, a01); store(g, 1, a10); store(g + 1, 1, a11);
        store(g, 2, a20); store(g + 1, 2, a21); store(g, 3, a30); store(g + 1, 3, a31);
      }
      for (; g < ng; g++) {
        v8f a0 = v8_splat(0.f), a1 = a0, a2 = a0, a3 = a0;
        const float* t0 = xt.data() + g * n_in * 8;
        for (size_t d = 0; d < n_in; d++) {
          const v8f x0 = v8_load(t0 + 8 * d);
          a0 = a0 + v8_splat(r0[d]) * x0;
          a1 = a1 + v8_splat(r1[d]) * x0;
          a2 = a2 + v8_splat(r2[d]) * x0;
          a3 = a3 + v8_splat(r3[d]) * x0;
        }
        store(g, 0, a0); store(g, 1, a1); store(g, 2, a2); store(g, 3, a3);
      }
      for (size_t s = 8 * ng; s < 8 * ng + tail; s++) {
        const float* xs = x + s * n_in;
        for (size_t r = 0; r < nr; r++) {
          const float* rr = rowbuf.data() + r * n_in;
          float sum = 0.f;
          for (size_t d = 0; d < n_in; d++) sum += rr[d] * xs[d];
          y[s * n_out + o0 + r] = sum;
        }
      }
    }
  });
}

static void rmsnorm_into(const float* x, float* out, size_t seq, size_t n, const float* w,
                         float eps) {  // qwen2.rs:647-660
  for (size_t s = 0; s < seq; s++) {
    const float* row = x + s * n;
    float ss = 0.f;
    for (size_t i = 0; i < n; i++) ss += row[i] * row[i];
    ss /= (float)n;
    float inv = 1.0f / std::sqrt(ss + eps);
    for (size_t i = 0; i < n; i++) out[s * n + i] = row[i] * inv * w[i];
  }
}

static void add_bias_rows(float* y, const std::vector<float>& b, bool has, size_t seq,
                          size_t n) {  // qwen2.rs:676-683
  if (!has) return;
  for (size_t s = 0; s < seq; s++)
    for (size_t i = 0; i < n; i++) y[s * n + i] += b[i];
}

static void rope_norm_offset(float* x, size_t seq, size_t n_heads, size_t hd, float theta,
                             size_t pos0) {  // qwen2.rs:708-724 (NEOX half-split)
  size_t half = hd / 2;
  for (size_t s = 0; s < seq; s++)
    for (size_t h = 0; h < n_heads; h++) {
      size_t base = (s * n_heads + h) * hd;
      for (size_t i = 0; i < half; i++) {
        float freq = powf(theta, -(2.0f * (float)i) / (float)hd);
        float angle = (float)(s + pos0) * freq;
        float sn = sinf(angle), cs = cosf(angle);
        float x0 = x[base + i], x1 = x[base + i + half];
        x[base + i] = x0 * cs - x1 * sn;
        x[base + i + half] = x0 * sn + x1 * cs;
      }
    }
}

static void softmax_row(float* x, size_t n) {  // qwen2.rs:726-741
  float mx = -INFINITY;
  for (size_t i = 0; i < n; i++)
    if (x[i] > mx) mx = x[i];
  float sum = 0.f;
  for (size_t i = 0; i < n; i++) {
    x[i] = expf(x[i] - mx);
    sum += x[i];
  }
  for (size_t i = 0; i < n; i++) x[i] /= sum;
}

void softmax_row_ref(float* x, size_t n) { softmax_row(x, n); }  // sampling.rs:157-172 (same steps)

static inline float silu(float x) { return x / (1.0f + expf(-x)); }  // qwen2.rs:743-745

void logits_from_hidden(const Model& m, const float* last_hidden, float* logits) {  // qwen2.rs:425-446
  const size_t ne = m.c.n_embd;
  std::vector<float> last(ne);
  float ss = 0.f;  // rmsnorm_row (qwen2.rs:748-756)
  for (size_t i = 0; i < ne; i++) ss += last_hidden[i] * last_hidden[i];
  float inv = 1.0f / std::sqrt(ss / (float)ne + m.c.rms_eps);
  for (size_t i = 0; i < ne; i++) last[i] = last_hidden[i] * inv * m.output_norm[i];
  matmul_rows(m.output, last.data(), 1, logits, m.threads);
}

int forward_cached(const Model& m, const uint32_t* tokens, size_t seq, SeqState& cache, float* logits,
                   std::string* err) {  // qwen2.rs:460-561
  const Config& c = m.c;
  const size_t pos0 = cache.len, ne = c.n_embd, hd = c.head_dim, kv_dim = c.n_kv_heads * hd;
  if (seq == 0) { *err = "forward_cached: empty token list"; return -1; }
  if (pos0 + seq > cache.cap) {
    *err = "forward_cached: " + std::to_string(pos0 + seq) + " positions exceed capacity " +
           std::to_string(cache.cap);
    return -1;
  }
  for (size_t s = 0; s < seq; s++)
    if (tokens[s] >= c.vocab_size) { *err = "token id out of range"; return -1; }
  std::vector<float> x(seq * ne);
  for (size_t s = 0; s < seq; s++) m.tok_embd.row(tokens[s], x.data() + s * ne);  // :468-472
  std::vector<float> normed(seq * ne), q(seq * ne), k_new(seq * kv_dim), v_new(seq * kv_dim),
      attn_out(seq * ne), tmp1(seq * std::max(c.n_ff, ne)), tmp2(seq * std::max(c.n_ff, ne));
  const size_t heads_per_kv = c.n_heads / c.n_kv_heads;
  const float scale = 1.0f / std::sqrt((float)hd);
  for (size_t li = 0; li < c.n_layers; li++) {
    const LayerW& L = m.layers[li];
    rmsnorm_into(x.data(), normed.data(), seq, ne, L.attn_norm.data(), c.rms_eps);
    matmul_rows(L.wq, normed.data(), seq, q.data(), m.threads);
    matmul_rows(L.wk, normed.data(), seq, k_new.data(), m.threads);
    matmul_rows(L.wv, normed.data(), seq, v_new.data(), m.threads);
    add_bias_rows(q.data(), L.bq, L.has_bq, seq, ne);
    add_bias_rows(k_new.data(), L.bk, L.has_bk, seq, kv_dim);
    add_bias_rows(v_new.data(), L.bv, L.has_bv, seq, kv_dim);
    rope_norm_offset(q.data(), seq, c.n_heads, hd, c.rope_theta, pos0);
    rope_norm_offset(k_new.data(), seq, c.n_kv_heads, hd, c.rope_theta, pos0);
    std::memcpy(cache.k[li].data() + pos0 * kv_dim, k_new.data(), seq * kv_dim * 4);
    std::memcpy(cache.v[li].data() + pos0 * kv_dim, v_new.data(), seq * kv_dim * 4);
    const float* k_all = cache.k[li].data();
    const float* v_all = cache.v[li].data();
    // attention (qwen2.rs:502-533); heads are independent
    parallel_for(m.threads, c.n_heads, [&](size_t hb, size_t he) {
      std::vector<float> sc(pos0 + seq);
      for (size_t s = 0; s < seq; s++)
        for (size_t h = hb; h < he; h++) {
          size_t kvh = h / heads_per_kv, abs_s = pos0 + s;
          for (size_t t = 0; t <= abs_s; t++) {
            size_t q_off = s * ne + h * hd, k_off = t * kv_dim + kvh * hd;
            float dot = 0.f;
            for (size_t d = 0; d < hd; d++) dot += q[q_off + d] * k_all[k_off + d];
            sc[t] = dot * scale;
          }
          softmax_row(sc.data(), abs_s + 1);
          size_t o_off = s * ne + h * hd;
          for (size_t d = 0; d < hd; d++) attn_out[o_off + d] = 0.f;
          for (size_t t = 0; t <= abs_s; t++) {
            float w = sc[t];
            size_t v_off = t * kv_dim + kvh * hd;
            for (size_t d = 0; d < hd; d++) attn_out[o_off + d] += w * v_all[v_off + d];
          }
        }
    });
    matmul_rows(L.wo, attn_out.data(), seq, tmp1.data(), m.threads);
    for (size_t i = 0; i < seq * ne; i++) x[i] += tmp1[i];
    rmsnorm_into(x.data(), normed.data(), seq, ne, L.ffn_norm.data(), c.rms_eps);
    float* gate = tmp1.data();
    float* up = tmp2.data();
    matmul_rows(L.w_gate, normed.data(), seq, gate, m.threads);
    matmul_rows(L.w_up, normed.data(), seq, up, m.threads);
    for (size_t i = 0; i < seq * c.n_ff; i++) gate[i] = silu(gate[i]) * up[i];
    float* down = tmp2.data();
    matmul_rows(L.w_down, gate, seq, down, m.threads);
    for (size_t i = 0; i < seq * ne; i++) x[i] += down[i];
  }
  cache.advance(seq);
  logits_from_hidden(m, x.data() + (seq - 1) * ne, logits);
  return 0;
}

// ------------------------------------------------------------- sampling ----
uint64_t Rng::next_u64() {  // sampling.rs:28-34
  s += 0x9E3779B97F4A7C15ull;
  uint64_t z = s;
  z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
  z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
  return z ^ (z >> 31);
}
float Rng::next_f32() {  // sampling.rs:37-40
  return (float)((double)(next_u64() >> 11) / (double)(1ull << 53));
}

size_t argmax(const float* x, size_t n) {  // sampling.rs:147-155
  size_t best = 0;
  for (size_t i = 1; i < n; i++)
    if (x[i] > x[best]) best = i;
  return best;
}

size_t Sampler::sample(const float* logits, size_t n, Rng& rng) const {  // sampling.rs:94-144
  if (temperature <= 0.0f) return argmax(logits, n);
  std::vector<float> probs(n);
  for (size_t i = 0; i < n; i++) probs[i] = logits[i] / temperature;
  softmax_row(probs.data(), n);  // sampling.rs:157-172 is the same function
  std::vector<size_t> idx(n);
  for (size_t i = 0; i < n; i++) idx[i] = i;
  // descending probability, ties by ascending index
  std::stable_sort(idx.begin(), idx.end(), [&](size_t a, size_t b) {
    float pa = probs[a], pb = probs[b];
    if (pb < pa) return true;   // b.partial_cmp(a) == Less  => a first
    if (pb > pa) return false;
    return a < b;               // Equal (or unordered) => index order
  });
  if (top_k >= 0) {
    size_t k = std::max<size_t>(std::min<size_t>((size_t)top_k, idx.size()), 1);
    idx.resize(k);
  }
  if (top_p >= 0.0f) {
    float cum = 0.f;
    size_t cut = idx.size();
    for (size_t i = 0; i < idx.size(); i++) {
      cum += probs[idx[i]];
      if (cum >= top_p) { cut = i + 1; break; }
    }
    idx.resize(std::max<size_t>(cut, 1));
  }
  float total = 0.f;
  for (size_t j : idx) total += probs[j];
  float r = rng.next_f32() * total;
  for (size_t j : idx) {
    r -= probs[j];
    if (r <= 0.0f) return j;
  }
  return idx.back();
}

size_t Sampler::sample_masked(const float* logits, const uint8_t* mask, size_t n,
                              Rng& rng) const {  // sampling.rs:66-88
  std::vector<float> masked(n);
  for (size_t i = 0; i < n; i++) masked[i] = mask[i] ? logits[i] : -INFINITY;
  return sample(masked.data(), n, rng);
}

}  // namespace orc
