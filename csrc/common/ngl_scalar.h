// Scalar semantics shared by the C++ host oracle and the sm_100a kernels.
//
// Every function here restates one piece of the reference's Rust arithmetic
// with the exact same IEEE-754 binary32 operation order, so that a value
// computed on the host and one computed on the device are bit-identical:
//
//   * Q8.23 conversion: nangila-math/src/fixed_point.rs:34-60
//   * saturating add/sub and mul_scalar: nangila-math/src/ops.rs:6-49
//   * no_std FixedQ rounding (s +/- 0.5 then truncate): nangila-edge/src/lib.rs:18-41
//   * Rust float->int `as` casts saturate and send NaN to 0.
//
// Host code must be compiled with -ffp-contract=off; device code uses the
// explicitly rounded intrinsics so nvcc cannot contract a*b+c into an FMA.
#pragma once
#include <stdint.h>

#if defined(__CUDACC__)
#define NGL_HD __host__ __device__ __forceinline__
#else
#define NGL_HD inline
#endif

#if defined(__CUDA_ARCH__)
#define NGL_FMUL(a, b) __fmul_rn((a), (b))
#define NGL_FADD(a, b) __fadd_rn((a), (b))
#define NGL_FSUB(a, b) __fsub_rn((a), (b))
#define NGL_FDIV(a, b) __fdiv_rn((a), (b))
#define NGL_FMA(a, b, c) __fmaf_rn((a), (b), (c))
#else
#include <cmath>
#define NGL_FMUL(a, b) ((float)(a) * (float)(b))
#define NGL_FADD(a, b) ((float)(a) + (float)(b))
#define NGL_FSUB(a, b) ((float)(a) - (float)(b))
#define NGL_FDIV(a, b) ((float)(a) / (float)(b))
#define NGL_FMA(a, b, c) std::fma((float)(a), (float)(b), (float)(c))
#endif

namespace ngl {

constexpr int kFracBits = 23;
constexpr float kQScale = 8388608.0f;  // 2^23

NGL_HD bool is_nan(float x) { return x != x; }

NGL_HD float f_round(float x) {
#if defined(__CUDA_ARCH__)
  return roundf(x);
#else
  return std::round(x);
#endif
}
NGL_HD float f_floor(float x) {
#if defined(__CUDA_ARCH__)
  return floorf(x);
#else
  return std::floor(x);
#endif
}
NGL_HD float f_abs(float x) {
#if defined(__CUDA_ARCH__)
  return fabsf(x);
#else
  return std::fabs(x);
#endif
}
// IEEE maxNum: a NaN operand is ignored (Rust f32::max / f32::min).
NGL_HD float f_max(float a, float b) {
#if defined(__CUDA_ARCH__)
  return fmaxf(a, b);
#else
  return std::fmax(a, b);
#endif
}
NGL_HD float f_min(float a, float b) {
#if defined(__CUDA_ARCH__)
  return fminf(a, b);
#else
  return std::fmin(a, b);
#endif
}

// Rust `x as i32` for f32: truncate toward zero, saturate, NaN -> 0.
NGL_HD int32_t sat_f32_to_i32(float x) {
  if (is_nan(x)) return 0;
  if (x >= 2147483648.0f) return INT32_MAX;
  if (x <= -2147483648.0f) return INT32_MIN;
  return (int32_t)x;
}
// Rust `x as i64` for f32.
NGL_HD int64_t sat_f32_to_i64(float x) {
  if (is_nan(x)) return 0;
  if (x >= 9223372036854775808.0f) return INT64_MAX;
  if (x <= -9223372036854775808.0f) return INT64_MIN;
  return (int64_t)x;
}
// Rust `x as i16` / `x as i8` for f32.
NGL_HD int16_t sat_f32_to_i16(float x) {
  if (is_nan(x)) return 0;
  if (x >= 32767.0f) return 32767;
  if (x <= -32768.0f) return -32768;
  return (int16_t)x;
}
NGL_HD int8_t sat_f32_to_i8(float x) {
  if (is_nan(x)) return 0;
  if (x >= 127.0f) return 127;
  if (x <= -128.0f) return -128;
  return (int8_t)x;
}

// FixedPointBuffer::from_f32 element (fixed_point.rs:34-53).
NGL_HD int32_t q823_from_f32(float v) {
  float s = NGL_FMUL(v, kQScale);
#if defined(__CUDA_ARCH__)
  // roundf (half away from zero), then a saturating conversion: >= 2^31 ->
  // INT32_MAX, <= -2^31 -> INT32_MIN, NaN -> 0, the same cases as below.
  int32_t r;
  asm("cvt.rzi.sat.s32.f32 %0, %1;" : "=r"(r) : "f"(roundf(s)));
  return r;
#else
  if (s >= 2147483648.0f) return INT32_MAX;   // i32::MAX as f32 == 2^31
  if (s <= -2147483648.0f) return INT32_MIN;
  if (is_nan(s)) return 0;
  return (int32_t)f_round(s);                 // half away from zero
#endif
}
// FixedPointBuffer::to_f32 element (fixed_point.rs:56-60): q / 2^23.  On the
// device as q * 2^-23: a power-of-two scale of (float)q (0 or |.| >= 1) is
// exact, so the product equals the quotient bit for bit.
NGL_HD float q823_to_f32(int32_t q) {
#if defined(__CUDA_ARCH__)
  return __fmul_rn((float)q, 1.1920928955078125e-07f);
#else
  return NGL_FDIV((float)q, kQScale);
#endif
}

NGL_HD int32_t sat_add_i32(int32_t a, int32_t b) {
#if defined(__CUDA_ARCH__)
  int32_t r;
  asm("add.sat.s32 %0, %1, %2;" : "=r"(r) : "r"(a), "r"(b));
  return r;
#else
  int64_t s = (int64_t)a + (int64_t)b;
  if (s > INT32_MAX) return INT32_MAX;
  if (s < INT32_MIN) return INT32_MIN;
  return (int32_t)s;
#endif
}
NGL_HD int32_t sat_sub_i32(int32_t a, int32_t b) {
#if defined(__CUDA_ARCH__)
  int32_t r;
  asm("sub.sat.s32 %0, %1, %2;" : "=r"(r) : "r"(a), "r"(b));
  return r;
#else
  int64_t s = (int64_t)a - (int64_t)b;
  if (s > INT32_MAX) return INT32_MAX;
  if (s < INT32_MIN) return INT32_MIN;
  return (int32_t)s;
#endif
}
// mul_scalar's fixed-point scalar: (s * 2^23) as i64 (ops.rs:38).
NGL_HD int64_t q823_scalar_fixed(float s) { return sat_f32_to_i64(NGL_FMUL(s, kQScale)); }
// mul_scalar element: ((v as i64) * sf) >> 23, clamped to i32 (ops.rs:40-46).
// The i64 product wraps like a Rust release build.
NGL_HD int32_t q823_mul_fixed(int32_t v, int64_t sf) {
  uint64_t p = (uint64_t)(int64_t)v * (uint64_t)sf;
  int64_t sh = ((int64_t)p) >> kFracBits;
  if (sh > INT32_MAX) return INT32_MAX;
  if (sh < INT32_MIN) return INT32_MIN;
  return (int32_t)sh;
}

// nangila-edge FixedQ::from_f32 element: s +/- 0.5 in f32, then truncate.
NGL_HD int32_t fixedq_from_f32(float x) {
  float s = NGL_FMUL(x, kQScale);
  if (s >= 2147483648.0f) return INT32_MAX;
  if (s <= -2147483648.0f) return INT32_MIN;
  float r = (s >= 0.0f) ? NGL_FADD(s, 0.5f) : NGL_FSUB(s, 0.5f);
  return sat_f32_to_i32(r);
}
NGL_HD float fixedq_to_f32(int32_t y) { return NGL_FMUL((float)y, 1.0f / kQScale); }

// Error-bounded INT16 code: round(v / scale) clamped with max/min then `as i16`
// (error_bounded.rs:41-46, block_sparse.rs:38-39, rle.rs:30-31).
NGL_HD int16_t eb_code(float v, float scale) {
  float q = f_round(NGL_FDIV(v, scale));
  float c = f_min(f_max(q, -32768.0f), 32767.0f);
  return sat_f32_to_i16(c);
}

// MurmurHash3 fmix64 (the code's `hash_u64`, unified_quantizer.rs:400-412).
NGL_HD uint64_t fmix64(uint64_t h) {
  h ^= h >> 33;
  h *= 0xff51afd7ed558ccdULL;
  h ^= h >> 33;
  h *= 0xc4ceb9fe1a85ec53ULL;
  h ^= h >> 33;
  return h;
}
// Rust `u64 as f32` (round to nearest even).  Host and device both convert
// with correct rounding.
NGL_HD float u64_to_f32(uint64_t x) { return (float)x; }

// stochastic_round(value) with the counter PRNG (unified_quantizer.rs:378-398).
NGL_HD int32_t compat_stochastic_round(float value, uint64_t seed, uint64_t counter) {
  float fl = f_floor(value);
  float frac = NGL_FSUB(value, fl);
  uint64_t h = fmix64(seed ^ counter);
  float r = NGL_FDIV(u64_to_f32(h), 18446744073709551616.0f);  // u64::MAX as f32 == 2^64
  int32_t fi = sat_f32_to_i32(fl);
  return (r < frac) ? (int32_t)((uint32_t)fi + 1u) : fi;
}

}  // namespace ngl
