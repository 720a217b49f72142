// The N(0, std) stream of the synthetic models (synth.cpp): element e of a
// tensor is half of a Box-Muller draw from splitmix64(key + (e >> 1) * phi)
// (the cosine half for even e, the sine half for odd e). Built with vector
// math (-ffast-math, AVX2 vector logf/sinf/cosf): the values are fixed by
// this build, not bit-equal to a scalar libm; the models are only defined by
// the files this library writes.
#include <algorithm>
#include <cmath>
#include <cstdint>

namespace sm {
namespace {
inline uint64_t mix64(uint64_t z) {
  z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
  z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
  return z ^ (z >> 31);
}
// Draws [p0, p0 + np): x[2i] = cosine half, x[2i + 1] = sine half of draw p0 + i.
void draw_pairs(uint64_t key, uint64_t p0, uint32_t np, float stdv, float* c, float* s) {
  float u1[256], u2[256];
  for (uint32_t i = 0; i < np; i++) {
    const uint64_t h = mix64(key + (p0 + i) * 0x9E3779B97F4A7C15ull);
    u1[i] = ((float)(h >> 40) + 0.5f) * (1.0f / 16777216.0f);
    u2[i] = ((float)((h >> 16) & 0xFFFFFFu) + 0.5f) * (1.0f / 16777216.0f);
  }
#pragma omp simd
  for (uint32_t i = 0; i < np; i++) {
    const float r = sqrtf(-2.0f * logf(u1[i]));
    const float th = 6.283185307179586f * u2[i];
    c[i] = stdv * (r * cosf(th));
    s[i] = stdv * (r * sinf(th));
  }
}
}  // namespace

void normal_fill(uint64_t key, uint64_t e0, uint64_t n, float stdv, float* x) {
  float c[256], s[256];
  const uint64_t end = e0 + n, pend = (end + 1) >> 1;
  for (uint64_t p = e0 >> 1; p < pend; p += 256) {
    const uint32_t np = (uint32_t)std::min<uint64_t>(256, pend - p);
    draw_pairs(key, p, np, stdv, c, s);
    for (uint32_t i = 0; i < np; i++) {
      const uint64_t e = 2 * (p + i);
      if (e >= e0 && e < end) x[e - e0] = c[i];
      if (e + 1 >= e0 && e + 1 < end) x[e + 1 - e0] = s[i];
    }
  }
}

}  // namespace sm
