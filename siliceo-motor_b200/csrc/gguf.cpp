// GGUF reader / writer (see gguf.hpp for the format).
#include "gguf.hpp"

#include <fcntl.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include <cstring>

#include "common.hpp"

namespace sm {

// ---------------------------------------------------------------- common ----
static thread_local std::string g_err;
void set_error(const std::string& msg) { g_err = msg; }
const std::string& get_error() { return g_err; }

uint16_t f32_to_fp16(float f) {
  uint32_t x;
  std::memcpy(&x, &f, 4);
  uint32_t sign = (x >> 16) & 0x8000u;
  uint32_t absx = x & 0x7FFFFFFFu;
  if (absx >= 0x7F800000u) return (uint16_t)(sign | (absx > 0x7F800000u ? 0x7E00u : 0x7C00u));
  if (absx >= 0x477FF000u) return (uint16_t)(sign | 0x7C00u);  // rounds to >= 65520: inf
  if (absx < 0x38800000u) {                                     // below 2^-14: subnormal half
    if (absx < 0x33000000u) return (uint16_t)sign;              // below 2^-25: zero
    uint32_t e = absx >> 23;
    uint32_t mant = (absx & 0x7FFFFFu) | 0x800000u;
    uint32_t shift = 126 - e;  // = 14 - (e - 127) + 23 - 10 - 1 + 1
    // value = mant * 2^(e-150); half subnormal unit = 2^-24 => q = mant >> (126-e)
    uint32_t q = mant >> shift;
    uint32_t rem = mant & ((1u << shift) - 1);
    uint32_t half = 1u << (shift - 1);
    if (rem > half || (rem == half && (q & 1))) q++;
    return (uint16_t)(sign | q);
  }
  uint32_t e = (absx >> 23) - 127 + 15;
  uint32_t mant = absx & 0x7FFFFFu;
  uint32_t q = (e << 10) | (mant >> 13);
  uint32_t rem = mant & 0x1FFFu;
  if (rem > 0x1000u || (rem == 0x1000u && (q & 1))) q++;
  return (uint16_t)(sign | q);
}

float fp16_to_f32_ref(uint16_t h) {
  uint32_t sign = (h >> 15) & 1u, exp = (h >> 10) & 0x1Fu, frac = h & 0x3FFu, e, fr;
  if (exp == 0) {
    if (frac == 0) { e = 0; fr = 0; }
    else { float v = (float)frac * 5.9604645e-8f; return sign ? -v : v; }
  } else if (exp == 0x1F) { e = 0xFF; fr = frac ? 0x200000u : 0u; }
  else { e = exp + 112; fr = frac; }
  uint32_t bits = (sign << 31) | (e << 23) | (uint32_t)(fr << 13);
  float out;
  std::memcpy(&out, &bits, 4);
  return out;
}

// ----------------------------------------------------------------- value ----
bool GgufValue::as_u64(uint64_t* out) const {
  switch (type) {
    case 0: case 2: case 4: case 10: *out = u; return true;
    case 1: case 3: case 5: case 11: *out = (uint64_t)i; return true;
    default: return false;
  }
}
bool GgufValue::as_f32(float* out) const {
  if (type == 6 || type == 12) { *out = (float)f; return true; }
  return false;
}

uint64_t GgufTensor::n_elements() const {
  uint64_t p = 1;
  for (auto d : dims) p *= d;
  return p;
}
uint64_t GgufTensor::n_bytes() const {
  uint32_t bs = 1, tb = 4;
  if (!qtype_layout(type, &bs, &tb)) return n_elements() * 4;
  return n_elements() / bs * tb;
}

// ---------------------------------------------------------------- reader ----
namespace {
struct Cur {
  const uint8_t* p;
  size_t n, pos = 0;
  bool ok = true;
  bool need(uint64_t k) {
    if (!ok || n - pos < k) { ok = false; return false; }
    return true;
  }
  template <class T> T get() {
    T v{};
    if (!need(sizeof(T))) return v;
    std::memcpy(&v, p + pos, sizeof(T));
    pos += sizeof(T);
    return v;
  }
  std::string str() {
    uint64_t l = get<uint64_t>();
    if (!need(l)) return {};
    std::string s((const char*)p + pos, l);
    pos += l;
    return s;
  }
};
bool read_val(Cur& c, uint32_t vt, GgufValue& v, int depth) {
  v.type = vt;
  switch (vt) {
    case 0: v.u = c.get<uint8_t>(); break;
    case 1: v.i = c.get<int8_t>(); break;
    case 2: v.u = c.get<uint16_t>(); break;
    case 3: v.i = c.get<int16_t>(); break;
    case 4: v.u = c.get<uint32_t>(); break;
    case 5: v.i = c.get<int32_t>(); break;
    case 6: v.f = c.get<float>(); break;
    case 7: v.u = c.get<uint8_t>() != 0; break;
    case 8: v.s = c.str(); break;
    case 9: {
      v.elem_type = c.get<uint32_t>();
      uint64_t n = c.get<uint64_t>();
      if (n > 100000000ull || depth > 8) { set_error("gguf: bad array"); return false; }
      for (uint64_t k = 0; k < n && c.ok; k++) {
        GgufValue e;
        if (!read_val(c, v.elem_type, e, depth + 1)) return false;
        v.arr.push_back(std::move(e));
      }
      break;
    }
    case 10: v.u = c.get<uint64_t>(); break;
    case 11: v.i = c.get<int64_t>(); break;
    case 12: v.f = c.get<double>(); break;
    default: set_error("gguf: bad value type " + std::to_string(vt)); return false;
  }
  if (!c.ok) { set_error("gguf: truncated header"); return false; }
  return true;
}
}  // namespace

std::unique_ptr<GgufReader> GgufReader::open_file(const std::string& path) {
  int fd = ::open(path.c_str(), O_RDONLY);
  if (fd < 0) { set_error("io: cannot open " + path); return nullptr; }
  struct stat st;
  if (fstat(fd, &st) != 0 || st.st_size == 0) { ::close(fd); set_error("io: empty or unreadable " + path); return nullptr; }
  void* m = mmap(nullptr, (size_t)st.st_size, PROT_READ, MAP_PRIVATE, fd, 0);
  ::close(fd);
  if (m == MAP_FAILED) { set_error("io: mmap failed for " + path); return nullptr; }
  std::unique_ptr<GgufReader> r(new GgufReader());
  r->base_ = (const uint8_t*)m;
  r->len_ = (size_t)st.st_size;
  r->mapped_ = true;
  if (!r->parse()) return nullptr;
  return r;
}

std::unique_ptr<GgufReader> GgufReader::open_memory(const void* buf, size_t len) {
  std::unique_ptr<GgufReader> r(new GgufReader());
  r->base_ = (const uint8_t*)buf;
  r->len_ = len;
  if (!r->parse()) return nullptr;
  return r;
}

GgufReader::~GgufReader() {
  if (mapped_ && base_) munmap((void*)base_, len_);
}

bool GgufReader::parse() {
  Cur c{base_, len_};
  uint32_t magic = c.get<uint32_t>();
  if (!c.ok) { set_error("gguf: unexpected eof"); return false; }
  if (magic != 0x46554747u) { set_error("gguf: bad magic (expected GGUF)"); return false; }
  version = c.get<uint32_t>();
  if (version != 2 && version != 3) { set_error("gguf: unsupported version " + std::to_string(version)); return false; }
  uint64_t n_t = c.get<uint64_t>(), n_kv = c.get<uint64_t>();
  if (!c.ok) { set_error("gguf: unexpected eof"); return false; }
  for (uint64_t k = 0; k < n_kv; k++) {
    std::string key = c.str();
    uint32_t vt = c.get<uint32_t>();
    if (!c.ok) { set_error("gguf: unexpected eof"); return false; }
    GgufValue v;
    if (!read_val(c, vt, v, 0)) return false;
    if (key == "general.alignment" && v.type == 4) alignment = v.u;
    metadata.emplace_back(std::move(key), std::move(v));
  }
  for (uint64_t k = 0; k < n_t; k++) {
    GgufTensor t;
    t.name = c.str();
    uint32_t nd = c.get<uint32_t>();
    if (!c.ok) { set_error("gguf: unexpected eof"); return false; }
    if (nd == 0 || nd > 8) { set_error("gguf: bad tensor " + t.name + ": n_dims out of range"); return false; }
    for (uint32_t d = 0; d < nd; d++) t.dims.push_back(c.get<uint64_t>());
    t.type = c.get<uint32_t>();
    t.offset = c.get<uint64_t>();
    if (!c.ok) { set_error("gguf: unexpected eof"); return false; }
    tensors.push_back(std::move(t));
  }
  if (alignment == 0) { set_error("gguf: alignment 0"); return false; }
  data_start = n_t ? (c.pos + alignment - 1) / alignment * alignment : c.pos;
  return true;
}

const GgufTensor* GgufReader::tensor(const std::string& name) const {
  for (auto& t : tensors)
    if (t.name == name) return &t;
  return nullptr;
}
const GgufValue* GgufReader::meta(const std::string& key) const {
  for (auto& kv : metadata)
    if (kv.first == key) return &kv.second;
  return nullptr;
}
const uint8_t* GgufReader::data(const GgufTensor& t) const {
  uint64_t abs = data_start + t.offset;
  if (abs > len_ || t.n_bytes() > len_ - abs) return nullptr;
  return base_ + abs;
}

// ---------------------------------------------------------------- writer ----
namespace {
template <class T> void put(std::vector<uint8_t>& b, T v) {
  size_t o = b.size();
  b.resize(o + sizeof(T));
  std::memcpy(b.data() + o, &v, sizeof(T));
}
void put_str(std::vector<uint8_t>& b, const std::string& s) {
  put<uint64_t>(b, s.size());
  b.insert(b.end(), s.begin(), s.end());
}
}  // namespace

void GgufWriter::kv_u32(const std::string& k, uint32_t v) { put_str(kv_, k); put<uint32_t>(kv_, 4); put<uint32_t>(kv_, v); n_kv_++; }
void GgufWriter::kv_f32(const std::string& k, float v) { put_str(kv_, k); put<uint32_t>(kv_, 6); put<float>(kv_, v); n_kv_++; }
void GgufWriter::kv_str(const std::string& k, const std::string& v) { put_str(kv_, k); put<uint32_t>(kv_, 8); put_str(kv_, v); n_kv_++; }

void GgufWriter::add_tensor(const std::string& name, const std::vector<uint64_t>& dims, uint32_t type) {
  GgufTensor t;
  t.name = name;
  t.dims = dims;
  t.type = type;
  t.offset = data_bytes_;
  offsets_.push_back(t.offset);
  data_bytes_ += (t.n_bytes() + alignment - 1) / alignment * alignment;
  infos_.push_back(std::move(t));
}

std::vector<uint8_t> GgufWriter::header() const {
  std::vector<uint8_t> b;
  put<uint32_t>(b, 0x46554747u);
  put<uint32_t>(b, 3);
  put<uint64_t>(b, infos_.size());
  put<uint64_t>(b, n_kv_);
  b.insert(b.end(), kv_.begin(), kv_.end());
  for (auto& t : infos_) {
    put_str(b, t.name);
    put<uint32_t>(b, (uint32_t)t.dims.size());
    for (auto d : t.dims) put<uint64_t>(b, d);
    put<uint32_t>(b, t.type);
    put<uint64_t>(b, t.offset);
  }
  while (b.size() % alignment) b.push_back(0);
  return b;
}

}  // namespace sm
