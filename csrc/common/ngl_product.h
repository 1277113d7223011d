// Product wire format of the fused compressed all-reduce: per-element math
// shared by the host oracle (csrc/host) and the sm_100a kernels (csrc/cuda).
//
// The reference hook (python/nangila_ddp/comm_hook.py:146-290) quantizes a
// whole bucket with one absmax scale and floor(x + U - 0.5) noise.  The
// product format keeps the reference's nibble order (element 2i in the high
// nibble, comm_hook.py:83-93) but uses one fp32 scale per 256-element block,
// unbiased floor(x + U) rounding with U from Philox4x32-10, error feedback,
// and a deterministic rank-ordered FMA reduction so that every rank computes
// bit-identical averages and predictor states.
#pragma once
#include "ngl_scalar.h"

namespace ngl {

constexpr int kBlock = 256;          // elements per scale block
constexpr int kInt4BlockBytes = 128; // packed nibbles per block
constexpr int kInt8BlockBytes = 256;

// ---------------------------------------------------------------------------
// Philox4x32-10 counter-based generator (Salmon, Moraes, Dror, Shaw,
// "Parallel Random Numbers: As Easy as 1, 2, 3", SC'11).  Written from the
// paper's round function: two 32x32->64 multiplies per round, a Weyl key
// schedule, ten rounds.
// ---------------------------------------------------------------------------
struct U32x4 { uint32_t x, y, z, w; };

NGL_HD void mulhilo32(uint32_t a, uint32_t b, uint32_t& hi, uint32_t& lo) {
#if defined(__CUDA_ARCH__)
  lo = a * b;
  hi = __umulhi(a, b);
#else
  uint64_t p = (uint64_t)a * (uint64_t)b;
  lo = (uint32_t)p;
  hi = (uint32_t)(p >> 32);
#endif
}

NGL_HD U32x4 philox4x32_10(U32x4 c, uint32_t k0, uint32_t k1) {
  const uint32_t M0 = 0xD2511F53u, M1 = 0xCD9E8D57u;
  const uint32_t W0 = 0x9E3779B9u, W1 = 0xBB67AE85u;
#if defined(__CUDA_ARCH__)
#pragma unroll
#endif
  for (int r = 0; r < 10; ++r) {
    uint32_t hi0, lo0, hi1, lo1;
    mulhilo32(M0, c.x, hi0, lo0);
    mulhilo32(M1, c.z, hi1, lo1);
    U32x4 n;
    n.x = hi1 ^ c.y ^ k0;
    n.y = lo1;
    n.z = hi0 ^ c.w ^ k1;
    n.w = lo0;
    c = n;
    k0 += W0;
    k1 += W1;
  }
  return c;
}

// Uniform in [0, 1) with 24 random bits: exact in binary32.
NGL_HD float u01_from_bits(uint32_t b) { return (float)(b >> 8) * (1.0f / 16777216.0f); }

// Noise for the 4 consecutive elements 4*group .. 4*group+3 of one bucket.
// Key = (seed, rank); counter = (group, bucket, step).
NGL_HD U32x4 product_noise4(uint64_t seed, uint32_t rank, uint32_t bucket, uint64_t step,
                            uint32_t group) {
  U32x4 c;
  c.x = group;
  c.y = bucket;
  c.z = (uint32_t)step;
  c.w = (uint32_t)(step >> 32);
  uint32_t k0 = (uint32_t)seed;
  uint32_t k1 = (uint32_t)(seed >> 32) ^ (rank * 0x9E3779B9u);
  return philox4x32_10(c, k0, k1);
}

// ---------------------------------------------------------------------------
// Block quantizer.  s = absmax / qmax; inv = 1 / s (0 when s == 0).
// ---------------------------------------------------------------------------
NGL_HD float product_scale(float absmax, float qmax) { return NGL_FDIV(absmax, qmax); }
NGL_HD float product_inv(float s) { return (s > 0.0f && s < 3.0e38f) ? NGL_FDIV(1.0f, s) : 0.0f; }

NGL_HD int32_t clamp_i32(int32_t q, int32_t lo, int32_t hi) { return q < lo ? lo : (q > hi ? hi : q); }

// Unbiased stochastic rounding: floor(c * inv + u).
NGL_HD int32_t product_code_sr(float c, float inv, float u, int32_t qmax) {
  float t = NGL_FADD(NGL_FMUL(c, inv), u);
  return clamp_i32(sat_f32_to_i32(f_floor(t)), -qmax - 1, qmax);
}
// Deterministic round to nearest (half away from zero).
NGL_HD int32_t product_code_rn(float c, float inv, int32_t qmax) {
  return clamp_i32(sat_f32_to_i32(f_round(NGL_FMUL(c, inv))), -qmax - 1, qmax);
}
NGL_HD float product_deq(int32_t q, float s) { return NGL_FMUL((float)q, s); }

// Two's-complement nibble helpers (element 2i -> high nibble).
NGL_HD uint32_t nib(int32_t q) { return (uint32_t)q & 0xFu; }
NGL_HD int32_t sext4(uint32_t v) { return ((int32_t)(v << 28)) >> 28; }

// Residual with error feedback: c = (g - pred) + e.
NGL_HD float product_residual(float g, float pred, float e) { return NGL_FADD(NGL_FSUB(g, pred), e); }

// Average of the W ranks: acc accumulated in rank order with FMA.
NGL_HD float product_accum(float acc, int32_t q, float s) { return NGL_FMA((float)q, s, acc); }
NGL_HD float product_average(float pred, float acc, float inv_world) {
  return NGL_FADD(pred, NGL_FMUL(acc, inv_world));
}
// EMA predictor update (fp32; the first observation is copied).
NGL_HD float product_ema(float state, float avg, float beta, float one_minus_beta, bool first) {
  return first ? avg : NGL_FMA(beta, state, NGL_FMUL(one_minus_beta, avg));
}

// Top-k record size in bytes for k kept elements of a 256-block:
// fp32 scale, k uint8 indices, k int8 values, padded to 4 bytes.
NGL_HD int topk_record_bytes(int k) { return (4 + 2 * k + 3) & ~3; }
// Wire payloads are sequences of chunk records, one per 8 consecutive
// 256-blocks (the last chunk is padded with empty blocks):
//   INT4 / INT8: [8 x f32 scale][8 x 128 | 256 code bytes]
//   top-k:       8 x top-k block record
constexpr int kChunkBlocks = 8;
NGL_HD int chunk_record_bytes(int mode, int k) {
  return mode == 0 ? 4 * kChunkBlocks + kChunkBlocks * kInt4BlockBytes
       : mode == 1 ? 4 * kChunkBlocks + kChunkBlocks * kInt8BlockBytes
                   : kChunkBlocks * topk_record_bytes(k);
}

// Static topology drop at chunk granularity (all ranks agree): chunk c of
// nchunks is a passenger iff (c * a + b) mod nchunks < ndrop, with a coprime
// to nchunks so the map is a permutation and exactly ndrop chunks drop.
NGL_HD bool topo_passenger(uint64_t c, uint64_t a, uint64_t b, int64_t ndrop, uint64_t nchunks) {
  return ndrop > 0 && (int64_t)((c * a + b) % nchunks) < ndrop;
}

// Kept elements per 256-block for a keep fraction.
inline int topk_per_block(double frac) {
  int k = (int)(frac * kBlock + 0.5);
  if (k < 1) k = 1;
  if (k > kBlock) k = kBlock;
  return k;
}

}  // namespace ngl
