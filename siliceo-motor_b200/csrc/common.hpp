// Shared host-side definitions of the B200 decode engine.
#pragma once
#include <cstddef>
#include <cstdint>
#include <cstring>
#include <string>
#include <vector>

namespace sm {

// ggml type codes as stored in GGUF tensor infos (reference:
// crates/s-gguf/src/types.rs:33-61).
enum QType : uint32_t {
  QT_F32 = 0, QT_F16 = 1, QT_Q4_0 = 2, QT_Q4_1 = 3, QT_Q5_0 = 6, QT_Q8_0 = 8,
  QT_Q4K = 12, QT_Q5K = 13, QT_Q6K = 14, QT_BF16 = 30,
};

// (elements per block, bytes per block) for the types the engine handles
// (types.rs:103-127).
inline bool qtype_layout(uint32_t t, uint32_t* bs, uint32_t* tb) {
  switch (t) {
    case QT_F32: *bs = 1; *tb = 4; return true;
    case QT_F16: *bs = 1; *tb = 2; return true;
    case QT_BF16: *bs = 1; *tb = 2; return true;
    case QT_Q4_0: *bs = 32; *tb = 18; return true;
    case QT_Q4_1: *bs = 32; *tb = 20; return true;
    case QT_Q5_0: *bs = 32; *tb = 22; return true;
    case QT_Q8_0: *bs = 32; *tb = 34; return true;
    case QT_Q4K: *bs = 256; *tb = 144; return true;
    case QT_Q5K: *bs = 256; *tb = 176; return true;
    case QT_Q6K: *bs = 256; *tb = 210; return true;
    default: return false;
  }
}

inline uint64_t qtype_row_bytes(uint32_t t, uint64_t n_in) {
  uint32_t bs = 1, tb = 4;
  qtype_layout(t, &bs, &tb);
  return n_in / bs * tb;
}

// IEEE binary16 <-> f32 (round to nearest even on the way down).
uint16_t f32_to_fp16(float f);
// Reference decoding of fp16 (dequant.rs:12-33), NaN -> ±Inf quirk included.
float fp16_to_f32_ref(uint16_t h);

// Thread-local error string returned through the C ABI.
void set_error(const std::string& msg);
const std::string& get_error();

}  // namespace sm
