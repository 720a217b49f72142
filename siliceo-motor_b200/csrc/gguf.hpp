// GGUF v2/v3 container: a streaming-free reader over a read-only mapping and
// a writer for the synthetic model files. Format as parsed by the reference
// (crates/s-gguf/src/lib.rs:114-179, value.rs:28-58): little-endian header
// {magic "GGUF", version, tensor_count u64, kv_count u64}, kv pairs, tensor
// infos {name, n_dims u32, dims u64[n], type u32, offset u64}, then the data
// section aligned to general.alignment (default 32).
#pragma once
#include <cstdint>
#include <map>
#include <memory>
#include <string>
#include <vector>

namespace sm {

struct GgufValue {
  uint32_t type = 0;  // 0=u8 1=i8 2=u16 3=i16 4=u32 5=i32 6=f32 7=bool 8=str 9=array 10=u64 11=i64 12=f64
  uint64_t u = 0;
  int64_t i = 0;
  double f = 0;
  std::string s;
  uint32_t elem_type = 0;
  std::vector<GgufValue> arr;
  bool as_u64(uint64_t* out) const;
  bool as_f32(float* out) const;
};

struct GgufTensor {
  std::string name;
  std::vector<uint64_t> dims;
  uint32_t type = 0;
  uint64_t offset = 0;
  uint64_t n_elements() const;
  uint64_t n_bytes() const;
};

class GgufReader {
 public:
  // Opens a file (mmap) or wraps a caller-owned buffer. Returns nullptr and
  // sets the engine error on failure.
  static std::unique_ptr<GgufReader> open_file(const std::string& path);
  static std::unique_ptr<GgufReader> open_memory(const void* buf, size_t len);
  ~GgufReader();
  uint32_t version = 0;
  uint64_t alignment = 32, data_start = 0;
  std::vector<std::pair<std::string, GgufValue>> metadata;
  std::vector<GgufTensor> tensors;
  const GgufTensor* tensor(const std::string& name) const;
  const GgufValue* meta(const std::string& key) const;
  const uint8_t* data(const GgufTensor& t) const;  // nullptr if out of bounds
 private:
  bool parse();
  const uint8_t* base_ = nullptr;
  size_t len_ = 0;
  bool mapped_ = false;
};

class GgufWriter {
 public:
  void kv_u32(const std::string& k, uint32_t v);
  void kv_f32(const std::string& k, float v);
  void kv_str(const std::string& k, const std::string& v);
  // Registers a tensor; its bytes are supplied later, in the same order.
  void add_tensor(const std::string& name, const std::vector<uint64_t>& dims, uint32_t type);
  // Serialises header + infos; returns the header bytes, padded to alignment.
  std::vector<uint8_t> header() const;
  uint64_t tensor_offset(size_t i) const { return offsets_[i]; }
  uint64_t data_bytes() const { return data_bytes_; }
  size_t n_tensors() const { return infos_.size(); }
  uint64_t alignment = 32;

 private:
  std::vector<uint8_t> kv_;
  uint64_t n_kv_ = 0;
  std::vector<GgufTensor> infos_;
  std::vector<uint64_t> offsets_;
  uint64_t data_bytes_ = 0;
};

}  // namespace sm
