// expf as the reference's sampler computes it: Rust's f32::exp, which on
// x86-64 Linux is glibc's expf. glibc's result is the correctly rounded one
// except for about 1e-4 of the inputs, where it is off by one ulp; the
// sampler's probabilities (sampling.rs:94-144) must equal the reference's bit
// for bit, so this function reproduces glibc's results on x <= 0 (the domain
// of exp(p - max p)).
//
// Method (own derivation, standard textbook range reduction): with
// k = round(x * 32 / ln2) = 32 q + j (0 <= j < 32), r = x - k ln2 / 32
// (|r| <= ln2 / 64, Cody-Waite split of ln2 / 32 so that k * C1 is exact),
// exp(x) = 2^q * 2^(j/32) * exp(r), with exp(r) by its Taylor polynomial to
// degree 6 (truncation below 2^-57) and 2^(j/32) correctly rounded doubles.
// Every double operation is written out with round-to-nearest intrinsics on
// the device and plain operators on the host (built without contraction), so
// the host twin computes the same double y (relative error below 2^-50) and
// the same float round(y). The inputs where glibc's expf differs from
// round(y) are listed in a table made at build time by calling glibc
// (gen_expf_table.cpp, exhaustive over [-104, 0]); a table lookup happens only
// when y lies within EXPF_NEAR float ulps of a rounding midpoint (where
// every listed input lies) or the result is below the normal range.
#pragma once
#include <stdint.h>

#ifdef __CUDACC__
#define EXPF_HD __host__ __device__ __forceinline__
#else
#define EXPF_HD inline
#endif

namespace sm {

// 2^(j/32), j = 0..31, correctly rounded to double.
#define SM_EXP2_32_TABLE                                                                                          \
  {0x1.0000000000000p+0, 0x1.059b0d3158574p+0, 0x1.0b5586cf9890fp+0, 0x1.11301d0125b51p+0,                        \
   0x1.172b83c7d517bp+0, 0x1.1d4873168b9aap+0, 0x1.2387a6e756238p+0, 0x1.29e9df51fdee1p+0,                        \
   0x1.306fe0a31b715p+0, 0x1.371a7373aa9cbp+0, 0x1.3dea64c123422p+0, 0x1.44e086061892dp+0,                        \
   0x1.4bfdad5362a27p+0, 0x1.5342b569d4f82p+0, 0x1.5ab07dd485429p+0, 0x1.6247eb03a5585p+0,                        \
   0x1.6a09e667f3bcdp+0, 0x1.71f75e8ec5f74p+0, 0x1.7a11473eb0187p+0, 0x1.82589994cce13p+0,                        \
   0x1.8ace5422aa0dbp+0, 0x1.93737b0cdc5e5p+0, 0x1.9c49182a3f090p+0, 0x1.a5503b23e255dp+0,                        \
   0x1.ae89f995ad3adp+0, 0x1.b7f76f2fb5e47p+0, 0x1.c199bdd85529cp+0, 0x1.cb720dcef9069p+0,                        \
   0x1.d5818dcfba487p+0, 0x1.dfc97337b9b5fp+0, 0x1.ea4afa2a490dap+0, 0x1.f50765b6e4540p+0}

// A lookup is made when the 29 bits a float rounding drops from y's double
// mantissa are within EXPF_NEAR_BITS of the midpoint 2^28, i.e. y within
// 2^-9 float ulp of a rounding midpoint (about 0.4% of the inputs). Every
// input where glibc's expf misrounds lies there: measured over the whole
// domain by the generator, which fails otherwise.
constexpr int64_t EXPF_NEAR_BITS = int64_t(1) << 20;
// Below this input glibc's result is subnormal or zero: always looked up.
constexpr float EXPF_SUBNORMAL_BELOW = -87.0f;

#ifdef __CUDA_ARCH__
#define EXPF_ADD(a, b) __dadd_rn(a, b)
#define EXPF_MUL(a, b) __dmul_rn(a, b)
#define EXPF_D2F(a) __double2float_rn(a)
#define EXPF_RINT(a) __double2ll_rn(a)
#else
#define EXPF_ADD(a, b) ((a) + (b))
#define EXPF_MUL(a, b) ((a) * (b))
#define EXPF_D2F(a) ((float)(a))
#define EXPF_RINT(a) ((long long)__builtin_rint(a))
#endif

struct ExpfEval {
  double y;  // exp(x) to within 2^-50 relative
  float f;   // round(y)
  bool check;  // glibc may differ from f: consult the exception table
};

// exp(x) in double, and its float rounding, for finite x in [-104, 0].
EXPF_HD ExpfEval expf_eval(float x, const double* t32) {
  const double xd = (double)x;
  const long long k = EXPF_RINT(EXPF_MUL(xd, 0x1.71547652b82fep+5));
  const double kd = (double)k;
  const double r = EXPF_ADD(EXPF_ADD(xd, -EXPF_MUL(kd, 0x1.62e42ff000000p-6)), -EXPF_MUL(kd, -0x1.718432a1b0e26p-40));
  double p = 0x1.6c16c16c16c17p-10;  // 1/720
  p = EXPF_ADD(EXPF_MUL(p, r), 0x1.1111111111111p-7);  // 1/120
  p = EXPF_ADD(EXPF_MUL(p, r), 0x1.5555555555555p-5);  // 1/24
  p = EXPF_ADD(EXPF_MUL(p, r), 0x1.5555555555555p-3);  // 1/6
  p = EXPF_ADD(EXPF_MUL(p, r), 0.5);
  p = EXPF_ADD(EXPF_MUL(p, r), 1.0);
  p = EXPF_ADD(EXPF_MUL(p, r), 1.0);
  const long long q = k >> 5;  // floor(k / 32)
  const int j = (int)(k & 31);
  double y = EXPF_MUL(t32[j], p);
  // times 2^q (q >= -151): exact, done in two steps to stay in range
  const long long q1 = q / 2, q2 = q - q1;
  union {
    double d;
    uint64_t u;
  } s1, s2;
  s1.u = (uint64_t)(q1 + 1023) << 52;
  s2.u = (uint64_t)(q2 + 1023) << 52;
  y = EXPF_MUL(EXPF_MUL(y, s1.d), s2.d);
  ExpfEval e;
  e.y = y;
  e.f = EXPF_D2F(y);
  union {
    double d;
    uint64_t u;
  } yb;
  yb.d = y;
  const int64_t dropped = (int64_t)(yb.u & ((uint64_t(1) << 29) - 1));
  const int64_t dist = dropped - (int64_t(1) << 28);
  e.check = x < EXPF_SUBNORMAL_BELOW || (dist < EXPF_NEAR_BITS && dist > -EXPF_NEAR_BITS);
  return e;
}

#undef EXPF_ADD
#undef EXPF_MUL
#undef EXPF_D2F
#undef EXPF_RINT

}  // namespace sm
