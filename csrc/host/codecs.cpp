// Bit-exact host restatement of the reference's Rust codecs.
// Reference locations are given per function.
#include <algorithm>
#include <cmath>
#include <cstring>

#include "../common/ngl_scalar.h"
#include "nangila_host.hpp"
#include "fast_scalar.h"

namespace ngl {
namespace host {

namespace {
inline void put_u32(Bytes& b, uint32_t v) {
  b.push_back((uint8_t)v);
  b.push_back((uint8_t)(v >> 8));
  b.push_back((uint8_t)(v >> 16));
  b.push_back((uint8_t)(v >> 24));
}
inline void put_i16(Bytes& b, int16_t v) {
  uint16_t u = (uint16_t)v;
  b.push_back((uint8_t)u);
  b.push_back((uint8_t)(u >> 8));
}
inline uint32_t get_u32(const uint8_t* p) {
  return (uint32_t)p[0] | ((uint32_t)p[1] << 8) | ((uint32_t)p[2] << 16) | ((uint32_t)p[3] << 24);
}
inline int16_t get_i16(const uint8_t* p) { return (int16_t)(uint16_t)((uint16_t)p[0] | ((uint16_t)p[1] << 8)); }

Floats to_f32(const int32_t* r, size_t n) { return q823_to_f32(r, n); }
Fixed from_f32(const Floats& f) { return q823_from_f32(f.data(), f.size()); }
inline size_t div_ceil(size_t a, size_t b) { return (a + b - 1) / b; }
}  // namespace

// ---------------------------------------------------------------- nangila-math
Fixed q823_from_f32(const float* x, size_t n) {
  Fixed out(n);
  for (size_t i = 0; i < n; ++i) out[i] = fast::q823_from_f32(x[i]);
  return out;
}
Floats q823_to_f32(const int32_t* q, size_t n) {
  Floats out(n);
  for (size_t i = 0; i < n; ++i) out[i] = fast::q823_to_f32(q[i]);
  return out;
}
Fixed q823_add(const int32_t* a, size_t na, const int32_t* b, size_t nb) {
  if (na != nb) throw ShapeMismatch(na, nb);
  Fixed out(na);
  for (size_t i = 0; i < na; ++i) out[i] = sat_add_i32(a[i], b[i]);
  return out;
}
Fixed q823_sub(const int32_t* a, size_t na, const int32_t* b, size_t nb) {
  if (na != nb) throw ShapeMismatch(na, nb);
  Fixed out(na);
  for (size_t i = 0; i < na; ++i) out[i] = sat_sub_i32(a[i], b[i]);
  return out;
}
Fixed q823_mul_scalar(const int32_t* a, size_t n, float s) {
  const int64_t sf = q823_scalar_fixed(s);
  Fixed out(n);
  for (size_t i = 0; i < n; ++i) out[i] = q823_mul_fixed(a[i], sf);
  return out;
}
// MomentumPredictor::update after the first observation (momentum.rs:41-48):
// state.mul_scalar(beta).add(obs.mul_scalar(1 - beta)), element by element
// in one pass with the same rules as the three buffer ops.
Fixed q823_momentum_update(const int32_t* state, const int32_t* obs, size_t n, float beta, float one_minus_beta) {
  const int64_t sb = q823_scalar_fixed(beta), so = q823_scalar_fixed(one_minus_beta);
  Fixed out(n);
  for (size_t i = 0; i < n; ++i) out[i] = sat_add_i32(q823_mul_fixed(state[i], sb), q823_mul_fixed(obs[i], so));
  return out;
}
Fixed fixedq_from_f32(const float* x, size_t n) {
  Fixed out(n);
  for (size_t i = 0; i < n; ++i) out[i] = ngl::fixedq_from_f32(x[i]);
  return out;
}
Floats fixedq_to_f32(const int32_t* q, size_t n) {
  Floats out(n);
  for (size_t i = 0; i < n; ++i) out[i] = ngl::fixedq_to_f32(q[i]);
  return out;
}

// ------------------------------------------- UnifiedQuantizer: stochastic mode
// unified_quantizer.rs:171-223
namespace detail {
// Stochastic codes of f / scale clamped to [qlo, qhi]: fast::stochastic_round
// written out so the loop vectorizes (clones in fast_scalar.h).
NGL_HOST_VEC_CLONES
void stochastic_codes(const float* f, size_t n, float scale, uint64_t seed, uint64_t c0, int32_t qlo, int32_t qhi,
                      int8_t* q) {
  for (size_t i = 0; i < n; ++i) {
    const float v = f[i] / scale;
    const float fl = std::floor(v);
    const float frac = v - fl;
    const float r = (float)fmix64(seed ^ (c0 + i)) * 0x1p-64f;  // h / 2^64: exact scaling
    const int32_t fi = sat_f32_to_i32(fl);
    const int32_t qq = (r < frac) ? (int32_t)((uint32_t)fi + 1u) : fi;
    q[i] = (int8_t)std::min(std::max(qq, qlo), qhi);
  }
}
}  // namespace detail

QuantOut stochastic_quantize(const int32_t* r, size_t n, int bits, uint64_t seed, uint64_t* counter) {
  QuantOut out{{}, 1.0f};
  Floats f = to_f32(r, n);
  if (f.empty()) return out;
  const float max_val = fast::absmax(f.data(), f.size());
  float scale = 1.0f;
  if (max_val > 1e-9f) {
    int levels = (bits >= 1 && bits < 31) ? ((1 << bits) - 1) : 255;
    scale = max_val / ((float)levels / 2.0f);
  }
  out.scale = scale;
  const uint64_t c0 = *counter;  // element i uses counter c0 + i
  if (bits == 4) {
    std::vector<int8_t> q(n);
    detail::stochastic_codes(f.data(), n, scale, seed, c0, -8, 7, q.data());
    out.bytes.assign((n + 1) / 2, 0);
    uint8_t* o = out.bytes.data();
    // first element of a pair -> high nibble
    for (size_t j = 0; j < n / 2; ++j)
      o[j] = (uint8_t)((((uint8_t)q[2 * j] & 0x0F) << 4) | ((uint8_t)q[2 * j + 1] & 0x0F));
    if (n & 1) o[n / 2] = (uint8_t)(((uint8_t)q[n - 1] & 0x0F) << 4);
    *counter = c0 + n;
  } else if (bits == 8) {
    out.bytes.resize(n);
    detail::stochastic_codes(f.data(), n, scale, seed, c0, -128, 127, reinterpret_cast<int8_t*>(out.bytes.data()));
    *counter = c0 + n;
  } else {
    // Fallback: deterministic INT8 rounding with Rust f32::clamp (NaN stays
    // NaN and then casts to 0).
    out.bytes.reserve(n);
    for (size_t i = 0; i < n; ++i) {
      float q = f_round(f[i] / scale);
      if (!is_nan(q)) q = std::min(std::max(q, -128.0f), 127.0f);
      out.bytes.push_back((uint8_t)sat_f32_to_i8(q));
    }
  }
  return out;
}

// unified_quantizer.rs:225-250
Fixed stochastic_dequantize(const uint8_t* b, size_t nb, float scale, int bits) {
  if (bits == 4) {
    Fixed out(nb * 2);  // two values per byte: an odd length gains a trailing 0 (Q10)
    for (size_t i = 0; i < nb; ++i) {
      const int8_t high = (int8_t)(uint8_t)(b[i] & 0xF0);   // high nibble, sign in bit 7
      const int8_t low = (int8_t)(uint8_t)(b[i] << 4);
      out[2 * i] = fast::q823_from_f32((float)(high >> 4) * scale);
      out[2 * i + 1] = fast::q823_from_f32((float)(low >> 4) * scale);
    }
    return out;
  }
  Fixed out(nb);
  for (size_t i = 0; i < nb; ++i) out[i] = fast::q823_from_f32((float)(int8_t)b[i] * scale);
  return out;
}

// unified_quantizer.rs:253-279 (same layout as nangila-hpc ErrorBounded)
QuantOut unified_eb_quantize(const int32_t* r, size_t n, float eps) { return eb_quantize(r, n, eps); }
Fixed unified_eb_dequantize(const uint8_t* b, size_t nb, float scale) { return eb_dequantize(b, nb, scale); }

// ------------------------------------------------------ UnifiedQuantizer: top-k
// unified_quantizer.rs:285-303
float topk_threshold(const float* x, size_t n, float k_percent) {
  if (n == 0) return 1e-9f;
  Floats a(n);
  for (size_t i = 0; i < n; ++i) a[i] = f_abs(x[i]);
  float kf = f_floor((float)n * k_percent);
  size_t keep = 0;
  if (!is_nan(kf) && kf > 0.0f) keep = (kf >= 1.8446744e19f) ? SIZE_MAX : (size_t)kf;
  if (keep == 0) return 1e-9f;
  size_t idx = n - std::min(keep, n);
  std::nth_element(a.begin(), a.begin() + idx, a.end());
  return f_max(a[idx], 1e-9f);
}

// unified_quantizer.rs:285-335
QuantOut topk_quantize(const int32_t* r, size_t n, float k_percent) {
  QuantOut out{{}, 1.0f};
  Floats f = to_f32(r, n);
  if (n == 0) return out;
  const float threshold = topk_threshold(f.data(), n, k_percent);
  float max_val = 0.0f;
  for (float x : f) max_val = f_max(max_val, f_abs(x));
  const float scale = max_val > 1e-9f ? max_val / 127.0f : 1.0f;
  out.scale = scale;
  out.bytes.reserve(4 + n / 4);
  put_u32(out.bytes, (uint32_t)n);
  for (size_t s = 0; s < n; s += 32) {
    size_t len = std::min<size_t>(32, n - s);
    uint32_t mask = 0;
    uint8_t vals[32];
    int nv = 0;
    for (size_t i = 0; i < len; ++i) {
      float v = f[s + i];
      if (f_abs(v) >= threshold) {
        mask |= 1u << i;
        float q = f_round(v / scale);
        if (!is_nan(q)) q = std::min(std::max(q, -128.0f), 127.0f);
        vals[nv++] = (uint8_t)sat_f32_to_i8(q);
      }
    }
    put_u32(out.bytes, mask);
    out.bytes.insert(out.bytes.end(), vals, vals + nv);
  }
  return out;
}

// unified_quantizer.rs:337-375
Fixed topk_dequantize(const uint8_t* b, size_t nb, float scale) {
  if (nb < 4) return Fixed();
  const size_t n = get_u32(b);
  Floats rec;
  rec.reserve(std::min<size_t>(n, nb * 32 + 32));
  size_t ptr = 4;
  const size_t num_blocks = div_ceil(n, 32);
  for (size_t blk = 0; blk < num_blocks; ++blk) {
    if (ptr + 4 > nb) break;
    uint32_t mask = get_u32(b + ptr);
    ptr += 4;
    size_t block_len = (blk == num_blocks - 1) ? n - blk * 32 : 32;
    for (size_t i = 0; i < block_len; ++i) {
      if ((mask >> i) & 1u) {
        if (ptr < nb) {
          rec.push_back((float)(int8_t)b[ptr] * scale);
          ptr += 1;
        } else {
          rec.push_back(0.0f);
        }
      } else {
        rec.push_back(0.0f);
      }
    }
  }
  rec.resize(n, 0.0f);
  return from_f32(rec);
}

// ------------------------------------------------------------------ nangila-hpc
// error_bounded.rs:29-68
Bytes eb_pack_codes(const int16_t* q, size_t n) {
  Bytes out(n * 2);
  for (size_t i = 0; i < n; ++i) {
    const uint16_t c = (uint16_t)q[i];
    out[2 * i] = (uint8_t)(c & 0xFF);
    out[2 * i + 1] = (uint8_t)(c >> 8);
  }
  return out;
}
QuantOut eb_quantize(const int32_t* r, size_t n, float eps) {
  const float scale = 2.0f * eps;
  QuantOut out{{}, scale};
  out.bytes.resize(n * 2);
  uint8_t* o = out.bytes.data();
  for (size_t i = 0; i < n; ++i) {
    const uint16_t c = (uint16_t)fast::eb_code(fast::q823_to_f32(r[i]), scale);
    o[2 * i] = (uint8_t)(c & 0xFF);
    o[2 * i + 1] = (uint8_t)(c >> 8);
  }
  return out;
}
Fixed eb_dequantize(const uint8_t* b, size_t nb, float scale) {
  Fixed out(nb / 2);
  for (size_t i = 0; i + 2 <= nb; i += 2) out[i / 2] = fast::q823_from_f32((float)get_i16(b + i) * scale);
  return out;
}

// rle.rs:21-99
QuantOut rle_quantize(const int32_t* r, size_t n, float eps) {
  QuantOut out{{}, 1.0f};
  if (n == 0) return out;
  const float scale = 2.0f * eps;
  out.scale = scale;
  std::vector<int16_t> q(n);
  for (size_t i = 0; i < n; ++i) q[i] = fast::eb_code(fast::q823_to_f32(r[i]), scale);
  out.bytes = rle_encode_i16(q.data(), n);
  return out;
}
Bytes rle_encode_i16(const int16_t* q, size_t n) {
  Bytes out;
  size_t i = 0;
  while (i < n) {
    size_t start = i;
    if (q[i] == 0) {
      while (i < n && q[i] == 0 && (i - start) < 128) ++i;
      out.push_back((uint8_t)(128 + (i - start) - 1));
    } else {
      while (i < n && q[i] != 0 && (i - start) < 128) ++i;
      size_t count = i - start;
      out.push_back((uint8_t)(count - 1));
      for (size_t j = 0; j < count; ++j) put_i16(out, q[start + j]);
    }
  }
  return out;
}
std::vector<int16_t> rle_decode_i16(const uint8_t* b, size_t nb) {
  std::vector<int16_t> out;
  size_t ptr = 0;
  while (ptr < nb) {
    uint8_t op = b[ptr++];
    if (op >= 128) {
      out.insert(out.end(), (size_t)(op - 128 + 1), (int16_t)0);
    } else {
      size_t count = (size_t)op + 1;
      for (size_t k = 0; k < count; ++k) {
        if (ptr + 2 > nb) break;
        out.push_back(get_i16(b + ptr));
        ptr += 2;
      }
    }
  }
  return out;
}
Fixed rle_dequantize(const uint8_t* b, size_t nb, float scale) {
  std::vector<int16_t> q = rle_decode_i16(b, nb);
  Fixed out(q.size());
  for (size_t i = 0; i < q.size(); ++i) out[i] = fast::q823_from_f32((float)q[i] * scale);
  return out;
}

// block_sparse.rs:21-92
Bytes bs_pack_codes(const int16_t* q, size_t n) {
  Bytes out;
  out.reserve(4 + n * 2);
  put_u32(out, (uint32_t)n);
  for (size_t s = 0; s < n; s += 32) {
    const size_t len = std::min<size_t>(32, n - s);
    uint32_t mask = 0;
    for (size_t i = 0; i < len; ++i)
      if (q[s + i] != 0) mask |= 1u << i;
    put_u32(out, mask);
    for (size_t i = 0; i < len; ++i)
      if (q[s + i] != 0) put_i16(out, q[s + i]);
  }
  return out;
}
QuantOut bs_quantize(const int32_t* r, size_t n, float eps) {
  const float scale = 2.0f * eps;
  std::vector<int16_t> q(n);
  for (size_t i = 0; i < n; ++i) q[i] = fast::eb_code(fast::q823_to_f32(r[i]), scale);
  return QuantOut{bs_pack_codes(q.data(), n), scale};
}
Fixed bs_dequantize(const uint8_t* b, size_t nb, float scale) {
  if (nb < 4) return Fixed();
  const size_t n = get_u32(b);
  size_t ptr = 4;
  const size_t num_blocks = div_ceil(n, 32);
  Floats rec;
  rec.reserve(std::min<size_t>(n, nb * 16 + 32));
  for (size_t blk = 0; blk < num_blocks; ++blk) {
    if (ptr + 4 > nb) break;
    uint32_t mask = get_u32(b + ptr);
    ptr += 4;
    size_t block_len = (blk == num_blocks - 1) ? n - blk * 32 : 32;
    for (size_t i = 0; i < block_len; ++i) {
      if ((mask >> i) & 1u) {
        if (ptr + 2 <= nb) {
          rec.push_back((float)get_i16(b + ptr) * scale);
          ptr += 2;
        } else {
          rec.push_back(0.0f);
        }
      } else {
        rec.push_back(0.0f);
      }
    }
  }
  if (rec.size() > n) rec.resize(n);
  return from_f32(rec);
}

// block_sparse_rle.rs:26-131
Bytes bsrle_pack_codes(const int16_t* q, size_t n) {
  const size_t num_blocks = div_ceil(n, 32);
  std::vector<uint32_t> masks(num_blocks);
  for (size_t blk = 0; blk < num_blocks; ++blk) {
    uint32_t m = 0;
    size_t s = blk * 32, len = std::min<size_t>(32, n - s);
    for (size_t i = 0; i < len; ++i)
      if (q[s + i] != 0) m |= 1u << i;
    masks[blk] = m;
  }
  Bytes out;
  out.reserve(4 + num_blocks * 6);
  put_u32(out, (uint32_t)n);
  size_t blk = 0;
  while (blk < num_blocks) {
    size_t count = 1;
    if (masks[blk] == 0) {
      while (blk + count < num_blocks && masks[blk + count] == 0 && count < 128) ++count;
      out.push_back((uint8_t)(0x80 | (count - 1)));
      blk += count;
      continue;
    }
    while (blk + count < num_blocks && masks[blk + count] != 0 && count < 128) ++count;
    out.push_back((uint8_t)(count - 1));
    for (size_t j = 0; j < count; ++j) {
      size_t bb = blk + j;
      put_u32(out, masks[bb]);
      size_t s = bb * 32, len = std::min<size_t>(32, n - s);
      for (size_t i = 0; i < len; ++i)
        if (q[s + i] != 0) put_i16(out, q[s + i]);
    }
    blk += count;
  }
  return out;
}
QuantOut bsrle_quantize(const int32_t* r, size_t n, float eps) {
  const float scale = 2.0f * eps;
  std::vector<int16_t> q(n);
  for (size_t i = 0; i < n; ++i) q[i] = fast::eb_code(fast::q823_to_f32(r[i]), scale);
  return QuantOut{bsrle_pack_codes(q.data(), n), scale};
}
Fixed bsrle_dequantize(const uint8_t* b, size_t nb, float scale) {
  if (nb < 4) return Fixed();
  const size_t n = get_u32(b);
  const size_t num_blocks = div_ceil(n, 32);
  Floats rec;
  rec.reserve(std::min<size_t>(n, nb * 4096 + 32));
  size_t ptr = 4, blk = 0;
  while (blk < num_blocks && ptr < nb) {
    uint8_t op = b[ptr++];
    if (op & 0x80) {
      size_t count = (size_t)(op & 0x7F) + 1;
      for (size_t k = 0; k < count; ++k) {
        size_t block_len = (blk + k == num_blocks - 1) ? n - (blk + k) * 32 : 32;
        rec.insert(rec.end(), block_len, 0.0f);
      }
      blk += count;
    } else {
      size_t count = (size_t)op + 1;
      for (size_t k = 0; k < count; ++k) {
        if (ptr + 4 > nb) break;
        uint32_t mask = get_u32(b + ptr);
        ptr += 4;
        size_t block_len = (blk == num_blocks - 1) ? n - blk * 32 : 32;
        for (size_t i = 0; i < block_len; ++i) {
          if ((mask >> i) & 1u) {
            if (ptr + 2 <= nb) {
              rec.push_back((float)get_i16(b + ptr) * scale);
              ptr += 2;
            } else {
              rec.push_back(0.0f);
            }
          } else {
            rec.push_back(0.0f);
          }
        }
        blk += 1;
      }
    }
  }
  if (rec.size() > n) rec.resize(n);
  return from_f32(rec);
}

}  // namespace host
}  // namespace ngl
