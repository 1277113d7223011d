// Host fast paths of the scalar rules in csrc/common/ngl_scalar.h for the
// buffer loops of the host library.  Each returns the same bits as the rule
// it replaces, for every input: q823_from_f32 and eb_code are compared with
// the scalar rules over all 2^32 float bit patterns by
// tests/test_host_fast_paths.py.
//
// * Rounding half away from zero of a float s with |s| < 2^31: s +- 0.5 is
//   exact in double (a float has 24 significant bits), so truncating the sum
//   toward zero is the rounded value.  No libm call, and the loops vectorize.
// * Division by 2^23 or 2^64 of a value whose result is normal or zero is
//   exact, so it is the same as multiplying by 2^-23 or 2^-64.
// * maxNum(m, |x|) with m never NaN is "|x| > m ? |x| : m" (a NaN |x| never
//   compares greater).  For a signaling NaN glibc's fmaxf returns NaN while
//   this, like Rust's f32::max, skips it; the host inputs of absmax are
//   conversions of Q8.23 integers, which are never NaN.
// The device keeps the rules of ngl_scalar.h.
#pragma once
#include <cmath>
#include <cstddef>
#include <cstdint>

#include "../common/ngl_scalar.h"

// Loops that use a fused multiply-add get an FMA-instruction clone next to
// the baseline one (GCC function multiversioning, chosen once at load time).
// Both compute the correctly rounded fma of the reference rule (the baseline
// through libm's fmaf), so the results are identical; -ffp-contract=off
// keeps every other multiply and add separate in both clones.
// Loops written to vectorize get AVX-512 and AVX2 clones the same way (the
// AVX-512 one has 64-bit multiplies and a rounded u64 -> f32 conversion);
// they hold only exact operations, so every clone gives the same bits.
// ThreadSanitizer builds take the baseline only: the clones' load-time
// resolvers would run instrumented before the sanitizer's runtime is up.
#if defined(__GNUC__) && !defined(__clang__) && defined(__x86_64__) && !defined(__SANITIZE_THREAD__)
#define NGL_HOST_FMA_CLONES __attribute__((target_clones("fma", "default")))
#define NGL_HOST_VEC_CLONES __attribute__((target_clones("arch=x86-64-v4", "arch=x86-64-v3", "default")))
#else
#define NGL_HOST_FMA_CLONES
#define NGL_HOST_VEC_CLONES
#endif

namespace ngl {
namespace host {
namespace fast {

// ngl::q823_from_f32: saturating at +-2^31, NaN -> 0, else round half away.
inline int32_t q823_from_f32(float v) {
  const float s = v * kQScale;
  if (s >= 2147483648.0f) return INT32_MAX;
  if (s <= -2147483648.0f) return INT32_MIN;
  if (s != s) return 0;
  const double d = s;
  return (int32_t)(d + (d < 0.0 ? -0.5 : 0.5));  // the conversion truncates toward zero
}

// ngl::q823_to_f32: q / 2^23 (exact: the result is zero or at least 2^-23).
inline float q823_to_f32(int32_t q) { return (float)q * 0x1p-23f; }

// ngl::eb_code: round(v / scale), clamped to i16.  |x| < 32767 rounds inside
// the i16 range with no clamping; everything else (large, inf, NaN) takes the
// scalar rule.
inline int16_t eb_code(float v, float scale) {
  const float x = v / scale;
  if (!(std::fabs(x) < 32767.0f)) return ngl::eb_code(v, scale);
  const double d = x;
  return (int16_t)(int32_t)(d + (d < 0.0 ? -0.5 : 0.5));
}

// ngl::eb_code without a branch (for vectorized loops): round half away in
// double (exact for every float: below 2^31 the +-0.5 sum is exact, above it
// the value is already an integer and clamps), then the clamp as maxNum /
// minNum.  "d >= -32768 ? d : -32768" sends NaN to -32768, as the reference's
// f32::max(-32768.0) does; infinities clamp to the nearer end.
inline int16_t eb_code_bf(float v, float scale) {
  const double d = (double)(v / scale);
  double r = std::trunc(d + (d < 0.0 ? -0.5 : 0.5));
  r = r >= -32768.0 ? r : -32768.0;
  r = r <= 32767.0 ? r : 32767.0;
  return (int16_t)(int32_t)r;
}

// u64 -> f32 rounded to nearest even without a branch on the top bit (the
// hash's top bit is random, so a branch mispredicts half the time): below
// 2^63 the signed conversion is exact-rounded; at or above, halve with the
// low bit kept as a sticky bit, convert, and double.
inline float u64_to_f32(uint64_t x) {
  const float lo = (float)(int64_t)x;
  const float hi = 2.0f * (float)(int64_t)((x >> 1) | (x & 1u));
  return (int64_t)x >= 0 ? lo : hi;
}

// ngl::compat_stochastic_round with the division by 2^64 as a multiply.
inline int32_t stochastic_round(float value, uint64_t seed, uint64_t counter) {
  const float fl = std::floor(value);
  const float frac = value - fl;
  const float r = u64_to_f32(fmix64(seed ^ counter)) * 0x1p-64f;
  const int32_t fi = sat_f32_to_i32(fl);
  return (r < frac) ? (int32_t)((uint32_t)fi + 1u) : fi;
}

// Rust f32::max fold of |x| from 0 (maxNum: NaN elements are skipped).
inline float absmax(const float* f, size_t n) {
  float m = 0.0f;
  for (size_t i = 0; i < n; ++i) {
    const float a = std::fabs(f[i]);
    m = a > m ? a : m;
  }
  return m;
}

}  // namespace fast
}  // namespace host
}  // namespace ngl
