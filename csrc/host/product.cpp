// Host oracle of the product wire format used by the fused all-reduce kernel
// (csrc/cuda/fused_kernels.cu).  Same per-element arithmetic
// (csrc/common/ngl_product.h).  Blocks are independent and the noise is
// counter-based, so the block loops run on host threads (parallel.h) with
// results that do not depend on the thread count.
#include <algorithm>
#include <cmath>
#include <cstring>
#include <numeric>

#include "../common/ngl_product.h"
#include "nangila_host.hpp"
#include "fast_scalar.h"
#include "parallel.h"

namespace ngl {
namespace host {

namespace {
inline size_t nchunks_of(size_t n) { return ((n + kBlock - 1) / kBlock + kChunkBlocks - 1) / kChunkBlocks; }
// Block b of a dense chunked payload: scale and code pointers.
inline float* dense_scale(uint8_t* wire, size_t b, size_t cr) {
  return reinterpret_cast<float*>(wire + (b / kChunkBlocks) * cr) + (b % kChunkBlocks);
}
inline uint8_t* dense_codes(uint8_t* wire, size_t b, size_t cr, size_t bpb) {
  return wire + (b / kChunkBlocks) * cr + 4 * kChunkBlocks + (b % kChunkBlocks) * bpb;
}
inline float dense_scale_c(const uint8_t* wire, size_t b, size_t cr) {
  float s;
  std::memcpy(&s, wire + (b / kChunkBlocks) * cr + 4 * (b % kChunkBlocks), 4);
  return s;
}
}  // namespace

size_t product_wire_bytes(size_t n, int mode, int k) { return nchunks_of(n) * (size_t)chunk_record_bytes(mode, k); }

TopoChunks product_topology(size_t nchunks, double drop, uint64_t seed, uint64_t stream) {
  TopoChunks t;
  if (nchunks == 0) return t;
  drop = std::min(1.0, std::max(0.0, drop));
  int64_t keep = (int64_t)std::floor((double)nchunks * (1.0 - drop));
  keep = std::max<int64_t>(1, std::min<int64_t>(keep, (int64_t)nchunks));
  t.ndrop = (int64_t)nchunks - keep;
  const uint64_t h = fmix64(seed ^ (stream * 0x9E3779B97F4A7C15ull));
  const uint64_t nc = (uint64_t)nchunks;
  uint64_t a = nc > 1 ? 1 + h % (nc - 1) : 1;
  while (std::gcd(a, nc) != 1) a = a + 1 < nc ? a + 1 : 1;
  t.a = a;
  t.b = fmix64(h ^ 0xD1B54A32D192ED03ull) % nc;
  return t;
}

void product_encode(const float* g, const float* pred, const float* e_in, size_t n, const ProductParams& p,
                    uint8_t* wire, float* e_out) {
  const int32_t qmax = p.bits == 4 ? 7 : 127;
  const float qmaxf = (float)qmax;
  const size_t nblk = (n + kBlock - 1) / kBlock;
  const size_t bpb = p.bits == 4 ? kInt4BlockBytes : kInt8BlockBytes;
  const size_t cr = chunk_record_bytes(p.bits == 4 ? 0 : 1, 0);
  std::memset(wire, 0, nchunks_of(n) * cr);
  const uint64_t nch = nchunks_of(n);
  parallel_for(nblk, 64, [&](size_t lo, size_t hi) {
    for (size_t b = lo; b < hi; ++b) {
      float c[kBlock];
      int32_t q[kBlock];
      const size_t base = b * kBlock;
      const size_t len = std::min<size_t>(kBlock, n - base);
      if (topo_passenger(b / kChunkBlocks, p.topo_a, p.topo_b, p.topo_ndrop, nch)) {
        // passenger: zero record, the whole residual goes to the error feedback
        if (p.error_feedback && e_out)
          for (size_t i = 0; i < len; ++i)
            e_out[base + i] = product_residual(g[base + i], pred ? pred[base + i] : 0.0f, e_in ? e_in[base + i] : 0.0f);
        continue;
      }
      float absmax = 0.0f;
      for (size_t i = 0; i < kBlock; ++i) {
        if (i < len) {
          float pr = pred ? pred[base + i] : 0.0f;
          float e = (p.error_feedback && e_in) ? e_in[base + i] : 0.0f;
          c[i] = product_residual(g[base + i], pr, e);
          // maxNum fold; c is an arithmetic result, so never a signaling NaN
          const float a = f_abs(c[i]);
          absmax = a > absmax ? a : absmax;
        } else {
          c[i] = 0.0f;
        }
      }
      const float s = product_scale(absmax, qmaxf);
      const float inv = product_inv(s);
      *dense_scale(wire, b, cr) = s;
      for (size_t i = 0; i < kBlock; i += 4) {
        U32x4 r = {0, 0, 0, 0};
        if (p.stochastic) r = product_noise4(p.seed, p.rank, p.bucket, p.step, (uint32_t)((base + i) / 4));
        const uint32_t rb[4] = {r.x, r.y, r.z, r.w};
        for (int j = 0; j < 4; ++j) {
          const size_t k = i + j;
          if (k >= len) {
            q[k] = 0;
            continue;
          }
          q[k] = p.stochastic ? product_code_sr(c[k], inv, u01_from_bits(rb[j]), qmax) : product_code_rn(c[k], inv, qmax);
          if (p.error_feedback && e_out) e_out[base + k] = NGL_FSUB(c[k], product_deq(q[k], s));
        }
      }
      uint8_t* out = dense_codes(wire, b, cr, bpb);
      if (p.bits == 4) {
        for (size_t j = 0; j < kInt4BlockBytes; ++j) out[j] = (uint8_t)((nib(q[2 * j]) << 4) | nib(q[2 * j + 1]));
      } else {
        for (size_t j = 0; j < kInt8BlockBytes; ++j) out[j] = (uint8_t)(int8_t)q[j];
      }
    }
  });
}

namespace detail {
// Range bodies of the loops that use a fused multiply-add: named functions,
// so each carries its FMA clone (a lambda would not inherit it).
NGL_HOST_FMA_CLONES
void reduce_range(const uint8_t* const* wires, int world, int bits, const float* pred, float inv_world,
                  float* avg_out, size_t lo, size_t hi) {
  const size_t bpb = bits == 4 ? kInt4BlockBytes : kInt8BlockBytes;
  const size_t cr = chunk_record_bytes(bits == 4 ? 0 : 1, 0);
  for (size_t i = lo; i < hi; ++i) {
    const size_t b = i / kBlock, k = i % kBlock;
    float acc = 0.0f;
    for (int r = 0; r < world; ++r) {
      const uint8_t* blk = dense_codes(const_cast<uint8_t*>(wires[r]), b, cr, bpb);
      int32_t q;
      if (bits == 4) {
        uint32_t byte = blk[k / 2];
        q = sext4((k & 1) ? (byte & 0xF) : (byte >> 4));
      } else {
        q = (int8_t)blk[k];
      }
      acc = product_accum(acc, q, dense_scale_c(wires[r], b, cr));
    }
    avg_out[i] = product_average(pred ? pred[i] : 0.0f, acc, inv_world);
  }
}

NGL_HOST_FMA_CLONES
void ema_range(float* state, const float* avg, float beta, bool first, size_t lo, size_t hi) {
  const float omb = 1.0f - beta;
  for (size_t i = lo; i < hi; ++i) state[i] = ngl::product_ema(state[i], avg[i], beta, omb, first);
}
}  // namespace detail

void product_reduce(const uint8_t* const* wires, int world, size_t n, int bits, const float* pred, float inv_world,
                    float* avg_out) {
  parallel_for(n, 1u << 15, [&](size_t lo, size_t hi) {
    detail::reduce_range(wires, world, bits, pred, inv_world, avg_out, lo, hi);
  });
}

void product_ema(float* state, const float* avg, size_t n, float beta, bool first) {
  parallel_for(n, 1u << 15, [&](size_t lo, size_t hi) { detail::ema_range(state, avg, beta, first, lo, hi); });
}

namespace {
inline uint32_t fbits(float x) {
  uint32_t u;
  std::memcpy(&u, &x, 4);
  return u;
}
}  // namespace

void product_topk_encode(const float* g, const float* pred, const float* e_in, size_t n, int k, bool ef,
                         uint8_t* records, float* e_out, const TopoChunks& topo) {
  const size_t nblk = (n + kBlock - 1) / kBlock;
  const int rb = topk_record_bytes(k);
  std::memset(records, 0, nchunks_of(n) * kChunkBlocks * rb);
  const uint64_t nch = nchunks_of(n);
  parallel_for(nblk, 64, [&](size_t lo, size_t hi) {
    for (size_t b = lo; b < hi; ++b) {
      float c[kBlock];
      uint32_t mag[kBlock];
      const size_t base = b * kBlock;
      const int len = (int)std::min<size_t>(kBlock, n - base);
      if (topo_passenger(b / kChunkBlocks, topo.a, topo.b, topo.ndrop, nch)) {
        if (ef && e_out)
          for (int i = 0; i < len; ++i)
            e_out[base + i] = product_residual(g[base + i], pred ? pred[base + i] : 0.0f, e_in ? e_in[base + i] : 0.0f);
        continue;
      }
      float absmax = 0.0f;
      for (int i = 0; i < len; ++i) {
        c[i] = product_residual(g[base + i], pred ? pred[base + i] : 0.0f, (ef && e_in) ? e_in[base + i] : 0.0f);
        mag[i] = fbits(f_abs(c[i]));
        const float a = f_abs(c[i]);  // maxNum fold; c is never a signaling NaN
        absmax = a > absmax ? a : absmax;
      }
      const int keff = std::min(k, len);
      // Threshold: largest T with count(mag >= T) >= keff (bitwise search).
      uint32_t T = 0;
      for (int bit = 31; bit >= 0; --bit) {
        uint32_t cand = T | (1u << bit);
        int cnt = 0;
        for (int i = 0; i < len; ++i) cnt += mag[i] >= cand;
        if (cnt >= keff) T = cand;
      }
      int gt = 0;
      for (int i = 0; i < len; ++i) gt += mag[i] > T;
      int eq_budget = keff - gt;
      const float s = product_scale(absmax, 127.0f);
      const float inv = product_inv(s);
      uint8_t* rec = records + b * rb;
      std::memcpy(rec, &s, 4);
      int out = 0;
      for (int i = 0; i < len; ++i) {
        bool sel = mag[i] > T;
        if (!sel && mag[i] == T && eq_budget > 0) {
          sel = true;
          --eq_budget;
        }
        if (sel) {
          int32_t q = product_code_rn(c[i], inv, 127);
          rec[4 + out] = (uint8_t)i;
          rec[4 + k + out] = (uint8_t)(int8_t)q;
          ++out;
          if (ef && e_out) e_out[base + i] = NGL_FSUB(c[i], product_deq(q, s));
        } else if (ef && e_out) {
          e_out[base + i] = c[i];
        }
      }
    }
  });
}

namespace detail {
NGL_HOST_FMA_CLONES
void topk_reduce_range(const uint8_t* const* records, int world, size_t n, int k, const float* pred,
                       float inv_world, float* avg_out, size_t lo, size_t hi) {
  const int rb = topk_record_bytes(k);
  for (size_t b = lo; b < hi; ++b) {
    float acc[kBlock];
    const size_t base = b * kBlock;
    const int len = (int)std::min<size_t>(kBlock, n - base);
    for (int i = 0; i < kBlock; ++i) acc[i] = 0.0f;
    for (int r = 0; r < world; ++r) {
      const uint8_t* rec = records[r] + b * rb;
      float s;
      std::memcpy(&s, rec, 4);
      const int keff = std::min(k, len);  // records of a short last block are padded
      for (int j = 0; j < keff; ++j) {
        int idx = rec[4 + j];
        int32_t q = (int8_t)rec[4 + k + j];
        acc[idx] = product_accum(acc[idx], q, s);
      }
    }
    for (int i = 0; i < len; ++i) avg_out[base + i] = product_average(pred ? pred[base + i] : 0.0f, acc[i], inv_world);
  }
}
}  // namespace detail

void product_topk_reduce(const uint8_t* const* records, int world, size_t n, int k, const float* pred,
                         float inv_world, float* avg_out) {
  const size_t nblk = (n + kBlock - 1) / kBlock;
  parallel_for(nblk, 64, [&](size_t lo, size_t hi) {
      detail::topk_reduce_range(records, world, n, k, pred, inv_world, avg_out, lo, hi);
  });
}

namespace detail {
NGL_HOST_FMA_CLONES
void twoshot_range(const uint8_t* const* wires, int world, size_t n, int bits, const float* pred, float inv_world,
                   float* avg_out, size_t lo, size_t hi) {
  const size_t bpb = bits == 4 ? kInt4BlockBytes : kInt8BlockBytes;
  const size_t cr = chunk_record_bytes(bits == 4 ? 0 : 1, 0);
  for (size_t b = lo; b < hi; ++b) {
    float m[kBlock];
    const size_t base = b * kBlock;
    const size_t len = std::min<size_t>(kBlock, n - base);
    float absmax = 0.0f;
    for (size_t k = 0; k < kBlock; ++k) {
      float acc = 0.0f;
      if (k < len) {
        for (int r = 0; r < world; ++r) {
          const uint8_t* blk = dense_codes(const_cast<uint8_t*>(wires[r]), b, cr, bpb);
          int32_t q;
          if (bits == 4) {
            uint32_t byte = blk[k / 2];
            q = sext4((k & 1) ? (byte & 0xF) : (byte >> 4));
          } else {
            q = (int8_t)blk[k];
          }
          acc = product_accum(acc, q, dense_scale_c(wires[r], b, cr));
        }
      }
      m[k] = NGL_FMUL(acc, inv_world);
      const float a = f_abs(m[k]);  // maxNum fold; m is never a signaling NaN
      absmax = a > absmax ? a : absmax;
    }
    const float s2 = product_scale(absmax, 127.0f);
    const float inv2 = product_inv(s2);
    for (size_t k = 0; k < len; ++k) {
      const float d = product_accum(0.0f, product_code_rn(m[k], inv2, 127), s2);
      avg_out[base + k] = product_average(pred ? pred[base + k] : 0.0f, d, 1.0f);
    }
  }
}
}  // namespace detail

// Two-shot: the chunk owner reduces, re-encodes the mean residual as INT8
// with per-block scales (round to nearest), every rank decodes that.
void product_reduce_twoshot(const uint8_t* const* wires, int world, size_t n, int bits, const float* pred,
                            float inv_world, float* avg_out) {
  const size_t nblk = (n + kBlock - 1) / kBlock;
  parallel_for(nblk, 64, [&](size_t lo, size_t hi) {
      detail::twoshot_range(wires, world, n, bits, pred, inv_world, avg_out, lo, hi);
  });
}

}  // namespace host
}  // namespace ngl
