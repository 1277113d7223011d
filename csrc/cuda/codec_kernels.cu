// sm_100a codec kernels: Q8.23 math, the fused HPC closed-loop step, the
// reference's byte formats (error-bounded INT16, BlockSparse,
// BlockSparse+RLE, element RLE, stochastic INT4/INT8, top-k) on the device.
//
// Reference hot loops restated here (all scalar Rust loops in the reference):
//   nangila-math/src/fixed_point.rs:34-60, ops.rs:6-49        -> q823_* kernels
//   nangila-hpc/src/error_bounded.rs:29-68, linear.rs:26-57     -> hpc_step, eb_*
//   nangila-hpc/src/block_sparse.rs:21-92                      -> bs_encode + walker
//   nangila-hpc/src/block_sparse_rle.rs:26-131                 -> bsrle_encode + walker
//   nangila-hpc/src/rle.rs:21-99                               -> rle_encode + walker
//   nangila-core/src/unified_quantizer.rs:171-375              -> stochastic_*, topk_*
//
// Variable-length encoders compute every item's output offset with a
// single-pass decoupled look-back scan across tiles (tile status words in
// scratch, dynamic tile ids from an atomic counter); every spin on a
// predecessor tile is bounded and reports through the status word.
#include "codecs.h"
#include "ngl_cuda.cuh"

namespace ngl {
namespace codec {

using dev::kFull;
using dev::max64;
using dev::min64;

constexpr int kThreads = 256;
constexpr uint64_t kSpinLimitNs = 2000000000ull;  // 2 s per look-back wait

__device__ __forceinline__ int64_t gtid() { return (int64_t)blockIdx.x * blockDim.x + threadIdx.x; }
__device__ __forceinline__ int64_t gstride() { return (int64_t)gridDim.x * blockDim.x; }

inline int grid_for(int64_t n, int per_thread = 4) {
  int64_t g = (n + (int64_t)kThreads * per_thread - 1) / ((int64_t)kThreads * per_thread);
  if (g < 1) g = 1;
  if (g > 148 * 16) g = 148 * 16;
  return (int)g;
}

// ================================================================ Q8.23 (K2)
__global__ void k_from_f32(const float* __restrict__ x, int32_t* __restrict__ q, int64_t n) {
  for (int64_t i = gtid(); i < n; i += gstride()) q[i] = q823_from_f32(x[i]);
}
__global__ void k_to_f32(const int32_t* __restrict__ q, float* __restrict__ x, int64_t n) {
  for (int64_t i = gtid(); i < n; i += gstride()) x[i] = q823_to_f32(q[i]);
}
__global__ void k_addsub(const int32_t* __restrict__ a, const int32_t* __restrict__ b, int32_t* __restrict__ o,
                         int64_t n, int sub) {
  for (int64_t i = gtid(); i < n; i += gstride()) o[i] = sub ? sat_sub_i32(a[i], b[i]) : sat_add_i32(a[i], b[i]);
}
__global__ void k_mul_scalar(const int32_t* __restrict__ a, int32_t* __restrict__ o, int64_t n, int64_t sf) {
  for (int64_t i = gtid(); i < n; i += gstride()) o[i] = q823_mul_fixed(a[i], sf);
}

cudaError_t from_f32_dev(const float* x, int32_t* q, int64_t n, cudaStream_t s) {
  if (n > 0) k_from_f32<<<grid_for(n), kThreads, 0, s>>>(x, q, n);
  return cudaGetLastError();
}
cudaError_t to_f32_dev(const int32_t* q, float* x, int64_t n, cudaStream_t s) {
  if (n > 0) k_to_f32<<<grid_for(n), kThreads, 0, s>>>(q, x, n);
  return cudaGetLastError();
}
cudaError_t q823_addsub(const int32_t* a, const int32_t* b, int32_t* out, int64_t n, bool sub, cudaStream_t s) {
  if (n > 0) k_addsub<<<grid_for(n), kThreads, 0, s>>>(a, b, out, n, sub ? 1 : 0);
  return cudaGetLastError();
}
cudaError_t q823_mul_scalar(const int32_t* a, int32_t* out, int64_t n, float scalar, cudaStream_t s) {
  // (scalar * 2^23) as i64 computed on the host with the same f32 multiply.
  const int64_t sf = q823_scalar_fixed(scalar);
  if (n > 0) k_mul_scalar<<<grid_for(n), kThreads, 0, s>>>(a, out, n, sf);
  return cudaGetLastError();
}

// ======================================================= error-bounded (K3)
__global__ void k_eb_encode(const int32_t* __restrict__ r, int16_t* __restrict__ c, int64_t n, float scale) {
  for (int64_t i = gtid(); i < n; i += gstride()) c[i] = eb_code(q823_to_f32(r[i]), scale);
}
__global__ void k_eb_decode(const int16_t* __restrict__ c, int32_t* __restrict__ o, int64_t n, float scale) {
  for (int64_t i = gtid(); i < n; i += gstride()) o[i] = q823_from_f32(NGL_FMUL((float)c[i], scale));
}

// One closed-loop step for a snapshot: predict, residual, code, reconstruct,
// track the max error.  Four elements per thread with 16-byte accesses.
// `vec` is set by the launcher only when x, st, stm1, recon are 16-byte and
// codes 8-byte aligned; otherwise every access is scalar.
__global__ void k_hpc_step(const float* __restrict__ x, const int32_t* __restrict__ st,
                           const int32_t* __restrict__ stm1, int hist, float scale, int16_t* __restrict__ codes,
                           int32_t* __restrict__ recon, uint32_t* __restrict__ maxerr, int64_t n, int vec) {
  float emax = 0.0f;
  const int64_t n4 = n / 4;
  for (int64_t v = gtid(); v < n4 + (n % 4 ? 1 : 0); v += gstride()) {
    const int64_t i0 = v * 4;
    const bool full = vec && i0 + 4 <= n;
    float xs[4];
    int32_t s0[4] = {0, 0, 0, 0}, s1[4] = {0, 0, 0, 0};
    if (full) {
      const float4 xv = *reinterpret_cast<const float4*>(x + i0);
      xs[0] = xv.x; xs[1] = xv.y; xs[2] = xv.z; xs[3] = xv.w;
      if (hist >= 1) {
        const int4 a = *reinterpret_cast<const int4*>(st + i0);
        s0[0] = a.x; s0[1] = a.y; s0[2] = a.z; s0[3] = a.w;
      }
      if (hist >= 2) {
        const int4 b = *reinterpret_cast<const int4*>(stm1 + i0);
        s1[0] = b.x; s1[1] = b.y; s1[2] = b.z; s1[3] = b.w;
      }
    } else {
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        xs[j] = (i0 + j < n) ? x[i0 + j] : 0.0f;
        if (hist >= 1 && i0 + j < n) s0[j] = st[i0 + j];
        if (hist >= 2 && i0 + j < n) s1[j] = stm1[i0 + j];
      }
    }
    int16_t c[4];
    int32_t rc[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int32_t xq = q823_from_f32(xs[j]);
      int32_t pred = 0;
      if (hist >= 2) pred = sat_add_i32(s0[j], sat_sub_i32(s0[j], s1[j]));
      else if (hist == 1) pred = s0[j];
      const int32_t r = hist >= 1 ? sat_sub_i32(xq, pred) : xq;
      c[j] = eb_code(q823_to_f32(r), scale);
      const int32_t d = q823_from_f32(NGL_FMUL((float)c[j], scale));
      rc[j] = hist >= 1 ? sat_add_i32(pred, d) : d;
      if (i0 + j < n) emax = fmaxf(emax, fabsf(NGL_FSUB(q823_to_f32(xq), q823_to_f32(rc[j]))));
    }
    if (full) {
      *reinterpret_cast<int4*>(recon + i0) = make_int4(rc[0], rc[1], rc[2], rc[3]);
      *reinterpret_cast<uint2*>(codes + i0) =
          make_uint2(((uint32_t)(uint16_t)c[0]) | ((uint32_t)(uint16_t)c[1] << 16),
                     ((uint32_t)(uint16_t)c[2]) | ((uint32_t)(uint16_t)c[3] << 16));
    } else {
      for (int j = 0; j < 4; ++j)
        if (i0 + j < n) {
          recon[i0 + j] = rc[j];
          codes[i0 + j] = c[j];
        }
    }
  }
  const uint32_t m = __reduce_max_sync(kFull, __float_as_uint(emax));
  if ((threadIdx.x & 31) == 0 && maxerr != nullptr) atomicMax(maxerr, m);
}

// Linear-predictor add-back over T snapshots: parallel over elements,
// sequential over steps (the reference's chain: empty, s_t, 2 s_t - s_{t-1}).
// Add-back chain over T residual snapshots; writes the Q8.23 values in place
// (f32out == nullptr) or their fp32 conversions to f32out (one pass fewer).
__global__ void k_linear_addback(int32_t* __restrict__ res, float* __restrict__ f32out, int64_t P, int64_t T) {
  for (int64_t i = gtid(); i < P; i += gstride()) {
    int32_t a = 0, b = 0;  // s_t, s_{t-1}
    int32_t nxt = T > 0 ? res[i] : 0;
    for (int64_t t = 0; t < T; ++t) {
      const int32_t d = nxt;  // loaded one step ahead
      if (t + 1 < T) nxt = res[(t + 1) * P + i];
      int32_t rc;
      if (t == 0) rc = d;
      else if (t == 1) rc = sat_add_i32(a, d);
      else rc = sat_add_i32(sat_add_i32(a, sat_sub_i32(a, b)), d);
      if (f32out) __stcs(f32out + t * P + i, q823_to_f32(rc));
      else res[t * P + i] = rc;
      b = a;
      a = rc;
    }
  }
}

// Whole-trajectory closed loop: thread owns 4 consecutive coordinates and
// walks all T steps with the LinearPredictor history (s_t, s_{t-1}) in
// registers; per element-step it reads the fp32 snapshot value and writes
// the INT16 code.  Same arithmetic as k_hpc_step, step by step.
__global__ void __launch_bounds__(kThreads) k_hpc_encode_all(const float* __restrict__ x, int16_t* __restrict__ codes,
                                                             uint32_t* __restrict__ maxerr, int64_t P, int64_t T,
                                                             float scale, int vec) {
  float emax = 0.0f;
  const int64_t nv = (P + 3) / 4;
  for (int64_t v = gtid(); v < nv; v += gstride()) {
    const int64_t i0 = v * 4;
    const bool full = vec && i0 + 4 <= P;
    int32_t a[4] = {0, 0, 0, 0}, b[4] = {0, 0, 0, 0};  // s_t, s_{t-1}
    float4 nxt = full ? __ldcs(reinterpret_cast<const float4*>(x + i0)) : make_float4(0.f, 0.f, 0.f, 0.f);
    for (int64_t t = 0; t < T; ++t) {
      const float* xt = x + t * P;
      float xs[4];
      if (full) {
        const float4 xv = nxt;  // prefetched one step ahead: two loads in flight
        if (t + 1 < T) nxt = __ldcs(reinterpret_cast<const float4*>(xt + P + i0));
        xs[0] = xv.x; xs[1] = xv.y; xs[2] = xv.z; xs[3] = xv.w;
      } else {
#pragma unroll
        for (int j = 0; j < 4; ++j) xs[j] = (i0 + j < P) ? xt[i0 + j] : 0.0f;
      }
      int16_t c[4];
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const int32_t xq = q823_from_f32(xs[j]);
        int32_t pred = 0;
        if (t >= 2) pred = sat_add_i32(a[j], sat_sub_i32(a[j], b[j]));
        else if (t == 1) pred = a[j];
        const int32_t r = t >= 1 ? sat_sub_i32(xq, pred) : xq;
        c[j] = eb_code(q823_to_f32(r), scale);
        const int32_t d = q823_from_f32(NGL_FMUL((float)c[j], scale));
        const int32_t rc = t >= 1 ? sat_add_i32(pred, d) : d;
        if (i0 + j < P) emax = fmaxf(emax, fabsf(NGL_FSUB(q823_to_f32(xq), q823_to_f32(rc))));
        b[j] = a[j];
        a[j] = rc;
      }
      int16_t* ct = codes + t * P;
      if (full) {
        __stcs(reinterpret_cast<uint2*>(ct + i0),
               make_uint2(((uint32_t)(uint16_t)c[0]) | ((uint32_t)(uint16_t)c[1] << 16),
                          ((uint32_t)(uint16_t)c[2]) | ((uint32_t)(uint16_t)c[3] << 16)));
      } else {
        for (int j = 0; j < 4; ++j)
          if (i0 + j < P) ct[i0 + j] = c[j];
      }
    }
  }
  const uint32_t m = __reduce_max_sync(kFull, __float_as_uint(emax));
  if ((threadIdx.x & 31) == 0 && maxerr != nullptr) atomicMax(maxerr, m);
}

// Whole-trajectory EB decode + LinearPredictor add-back: codes [T, P] ->
// Q8.23 reconstructions [T, P] (the chain kept in registers).
__global__ void __launch_bounds__(kThreads) k_eb_decode_all(const int16_t* __restrict__ codes,
                                                            int32_t* __restrict__ out, float* __restrict__ f32out,
                                                            int64_t P, int64_t T, const float* __restrict__ scales) {
  for (int64_t i = gtid(); i < P; i += gstride()) {
    int32_t a = 0, b = 0;
    for (int64_t t = 0; t < T; ++t) {
      const int32_t d = q823_from_f32(NGL_FMUL((float)__ldcs(codes + t * P + i), scales[t]));
      int32_t rc;
      if (t == 0) rc = d;
      else if (t == 1) rc = sat_add_i32(a, d);
      else rc = sat_add_i32(sat_add_i32(a, sat_sub_i32(a, b)), d);
      if (f32out) __stcs(f32out + t * P + i, q823_to_f32(rc));
      else out[t * P + i] = rc;
      b = a;
      a = rc;
    }
  }
}

cudaError_t hpc_encode_all(const float* x, int16_t* codes, uint32_t* maxerr_bits, int64_t P, int64_t T, float scale,
                           cudaStream_t s) {
  const int vec = ((reinterpret_cast<uintptr_t>(x) & 15u) == 0) && ((reinterpret_cast<uintptr_t>(codes) & 7u) == 0) &&
                  (P % 4 == 0);
  if (P > 0 && T > 0)
    k_hpc_encode_all<<<grid_for((P + 3) / 4, 1), kThreads, 0, s>>>(x, codes, maxerr_bits, P, T, scale, vec);
  return cudaGetLastError();
}
cudaError_t eb_decode_all(const int16_t* codes, int32_t* out, int64_t P, int64_t T, const float* scales,
                          cudaStream_t s, float* f32out) {
  if (P > 0 && T > 0) k_eb_decode_all<<<grid_for(P, 1), kThreads, 0, s>>>(codes, out, f32out, P, T, scales);
  return cudaGetLastError();
}

cudaError_t eb_encode(const int32_t* r, int16_t* codes, int64_t n, float scale, cudaStream_t s) {
  if (n > 0) k_eb_encode<<<grid_for(n), kThreads, 0, s>>>(r, codes, n, scale);
  return cudaGetLastError();
}
cudaError_t eb_decode(const int16_t* codes, int32_t* out, int64_t n, float scale, cudaStream_t s) {
  if (n > 0) k_eb_decode<<<grid_for(n), kThreads, 0, s>>>(codes, out, n, scale);
  return cudaGetLastError();
}
cudaError_t hpc_step(const float* x, const int32_t* s_t, const int32_t* s_tm1, int hist, float scale, int16_t* codes,
                     int32_t* recon, uint32_t* maxerr_bits, int64_t n, cudaStream_t s) {
  auto a16 = [](const void* p) { return p == nullptr || (reinterpret_cast<uintptr_t>(p) & 15u) == 0; };
  const int vec = a16(x) && a16(s_t) && a16(s_tm1) && a16(recon) && (reinterpret_cast<uintptr_t>(codes) & 7u) == 0;
  if (n > 0)
    k_hpc_step<<<grid_for(n, 4), kThreads, 0, s>>>(x, s_t, s_tm1, hist, scale, codes, recon, maxerr_bits, n, vec);
  return cudaGetLastError();
}
cudaError_t linear_addback(int32_t* res, int64_t particles, int64_t steps, cudaStream_t s, float* f32out) {
  if (particles > 0 && steps > 0)
    k_linear_addback<<<grid_for(particles, 1), kThreads, 0, s>>>(res, f32out, particles, steps);
  return cudaGetLastError();
}

// ================================================ decoupled look-back scan
// Status word: bits 63..62 state (1 = aggregate, 2 = inclusive prefix),
// bits 61..0 value.  Warp 0 of the tile publishes and looks back over 32
// predecessors at a time.
constexpr uint64_t kStAgg = 1ull << 62, kStInc = 2ull << 62, kValMask = (1ull << 62) - 1;

__device__ __forceinline__ void st_release_gpu(uint64_t* p, uint64_t v) {
  asm volatile("st.release.gpu.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}
__device__ __forceinline__ uint64_t ld_acquire_gpu(const uint64_t* p) {
  uint64_t v;
  asm volatile("ld.acquire.gpu.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}

struct OpSum {
  __device__ static uint64_t id() { return 0; }
  __device__ static uint64_t op(uint64_t a, uint64_t b) { return a + b; }
};
struct OpMax {
  __device__ static uint64_t id() { return 0; }
  __device__ static uint64_t op(uint64_t a, uint64_t b) { return a > b ? a : b; }
};

template <class Op>
__device__ __forceinline__ uint64_t warp_reduce_op(uint64_t v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = Op::op(v, __shfl_xor_sync(kFull, v, o));
  return v;
}

// Called by every thread of the CTA; returns the exclusive prefix of this
// tile (all threads).  On a timeout it records the status and returns the
// identity (the caller's output is then invalid; status says so).
template <class Op>
__device__ uint64_t lookback(uint64_t* status_arr, int64_t tile, uint64_t agg, int* status, uint64_t* s_slot) {
  const int lane = threadIdx.x & 31;
  if (threadIdx.x < 32) {
    uint64_t excl = Op::id();
    if (tile == 0) {
      if (lane == 0) st_release_gpu(&status_arr[0], kStInc | (agg & kValMask));
    } else {
      if (lane == 0) st_release_gpu(&status_arr[tile], kStAgg | (agg & kValMask));
      int64_t base = tile - 1;
      bool timed_out = false;
      while (true) {
        const int64_t idx = base - lane;
        uint64_t s = idx >= 0 ? ld_acquire_gpu(&status_arr[idx]) : (kStInc | Op::id());
        const uint64_t t0 = dev::globaltimer();
        while (__any_sync(kFull, (s >> 62) == 0)) {  // uniform loop condition
          if ((s >> 62) == 0) s = ld_acquire_gpu(&status_arr[idx]);
          const bool late = dev::globaltimer() - t0 > kSpinLimitNs;
          if (__any_sync(kFull, late)) {  // uniform exit
            timed_out = true;
            break;
          }
        }
        if (timed_out) break;
        const uint32_t inc = __ballot_sync(kFull, (s >> 62) == 2);
        const int stop = inc ? (__ffs(inc) - 1) : 31;
        uint64_t v = lane <= stop ? (s & kValMask) : Op::id();
        excl = Op::op(excl, warp_reduce_op<Op>(v));
        if (inc) break;
        base -= 32;
      }
      if (timed_out) {
        if (lane == 0) dev::set_status(status, dev::kTimeoutLookback, (int)tile, -1);
        excl = Op::id();
      }
      if (lane == 0) st_release_gpu(&status_arr[tile], kStInc | (Op::op(excl, agg) & kValMask));
    }
    if (lane == 0) *s_slot = excl;
  }
  __syncthreads();
  const uint64_t r = *s_slot;
  __syncthreads();
  return r;
}

// Block-wide exclusive scan of one u64 per thread (256 threads).
template <class Op>
__device__ uint64_t block_excl_scan(uint64_t v, uint64_t* s_warp, uint64_t* total) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  uint64_t x = v;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const uint64_t y = __shfl_up_sync(kFull, x, o);
    if (lane >= o) x = Op::op(x, y);
  }
  if (lane == 31) s_warp[warp] = x;
  __syncthreads();
  if (warp == 0) {
    uint64_t w = lane < (kThreads / 32) ? s_warp[lane] : Op::id();
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const uint64_t y = __shfl_up_sync(kFull, w, o);
      if (lane >= o) w = Op::op(w, y);
    }
    if (lane < (kThreads / 32)) s_warp[lane] = w;  // inclusive prefix of warps
  }
  __syncthreads();
  const uint64_t wbase = warp ? s_warp[warp - 1] : Op::id();
  const uint64_t excl_in_warp = __shfl_up_sync(kFull, x, 1);
  const uint64_t r = Op::op(wbase, lane ? excl_in_warp : Op::id());
  if (total) *total = s_warp[kThreads / 32 - 1];
  __syncthreads();
  return r;
}

int64_t pack_scratch_words(int64_t n, int64_t ns) {
  const int64_t nblk = (n + 31) / 32;
  const int64_t tiles = (nblk + kPackTileBlocks - 1) / kPackTileBlocks;
  return tiles * ns + 2;  // status per tile of every stream, tile counter
}

// ==================================================== mask packers (K4, K8)
struct SrcBS {  // BlockSparse from i16 codes: kept iff q != 0, value q
  const int16_t* q;
  static constexpr int kVBytes = 2;
  __device__ __forceinline__ bool get(int64_t i, int32_t& v) const {
    v = q[i];
    return v != 0;
  }
  __device__ __forceinline__ SrcBS at(int64_t off) const { return SrcBS{q + off}; }
};
struct SrcTopK {  // top-k compat from Q8.23: kept iff |x| >= thr
  const int32_t* r;
  const float* thr;
  const float* scale;
  static constexpr int kVBytes = 1;
  __device__ __forceinline__ bool get(int64_t i, int32_t& v) const {
    const float x = q823_to_f32(r[i]);
    const bool keep = fabsf(x) >= *thr;
    float q = f_round(NGL_FDIV(x, *scale));
    if (!is_nan(q)) q = fminf(fmaxf(q, -128.0f), 127.0f);
    v = sat_f32_to_i8(q);
    return keep;
  }
  __device__ __forceinline__ SrcTopK at(int64_t off) const { return SrcTopK{r + off, thr, scale}; }
};

__device__ __forceinline__ void put_u32_bytes(uint8_t* p, uint32_t v) {
  p[0] = (uint8_t)v;
  p[1] = (uint8_t)(v >> 8);
  p[2] = (uint8_t)(v >> 16);
  p[3] = (uint8_t)(v >> 24);
}

// Batched over `ns` streams of n elements each (stream s: input src.at(s *
// in_stride), output out + s * out_stride, length totals[s]); each stream
// has its own tile-status range, tile ids are global.
template <class Src>
__global__ void __launch_bounds__(kThreads) k_mask_pack(Src src0, int64_t n, int ns, int64_t in_stride,
                                                        uint8_t* __restrict__ out0, int64_t out_stride,
                                                        uint64_t* scratch, uint64_t* totals, int* status) {
  __shared__ uint64_t s_warp[kThreads / 32];
  __shared__ uint64_t s_slot;
  __shared__ int64_t s_tile;
  __shared__ uint32_t s_mask[kPackTileBlocks];
  const int64_t nblk = (n + 31) / 32;
  const int64_t tps = (nblk + kPackTileBlocks - 1) / kPackTileBlocks;
  const int64_t ntiles_all = tps * ns;
  unsigned long long* ctr = reinterpret_cast<unsigned long long*>(scratch + ntiles_all);
  if (threadIdx.x == 0) s_tile = (int64_t)atomicAdd(ctr, 1ull);
  __syncthreads();
  const int64_t gtile = s_tile;
  if (gtile >= ntiles_all) return;
  const int64_t sidx = gtile / tps, tile = gtile % tps;
  const Src src = src0.at(sidx * in_stride);
  uint8_t* out = out0 + sidx * out_stride;
  uint64_t* st = scratch + sidx * tps;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int64_t blk0 = tile * kPackTileBlocks + (int64_t)warp * kPackBlocksPerWarp;
  // pass 1: masks (kept in shared memory) and this warp's byte count
  uint64_t wsum = 0;
  for (int j = 0; j < kPackBlocksPerWarp; ++j) {
    const int64_t blk = blk0 + j;
    const int64_t i = blk * 32 + lane;
    int32_t v = 0;
    const bool keep = (blk < nblk && i < n) ? src.get(i, v) : false;
    const uint32_t m = __ballot_sync(kFull, keep);
    if (lane == 0) s_mask[warp * kPackBlocksPerWarp + j] = m;
    if (blk < nblk) wsum += 4 + Src::kVBytes * __popc(m);
  }
  uint64_t tile_agg;
  const uint64_t wexcl = block_excl_scan<OpSum>(lane == 0 ? wsum : 0, s_warp, &tile_agg);
  const uint64_t warp_base = __shfl_sync(kFull, wexcl, 0);
  const uint64_t excl = lookback<OpSum>(st, tile, tile_agg, status, &s_slot);
  if (tile == 0 && threadIdx.x == 0) put_u32_bytes(out, (uint32_t)n);
  // pass 2: write masks and kept values (inputs re-read from L2)
  uint64_t off = 4 + excl + warp_base;
  const uint32_t lt = (1u << lane) - 1u;
  for (int j = 0; j < kPackBlocksPerWarp; ++j) {
    const int64_t blk = blk0 + j;
    if (blk >= nblk) break;
    const uint32_t m = s_mask[warp * kPackBlocksPerWarp + j];
    if (lane == 0) put_u32_bytes(out + off, m);
    if ((m >> lane) & 1u) {
      int32_t v = 0;
      src.get(blk * 32 + lane, v);
      const uint64_t pos = off + 4 + Src::kVBytes * __popc(m & lt);
      if (Src::kVBytes == 2) {
        out[pos] = (uint8_t)v;
        out[pos + 1] = (uint8_t)((uint32_t)v >> 8);
      } else {
        out[pos] = (uint8_t)v;
      }
    }
    off += 4 + Src::kVBytes * __popc(m);
  }
  if (tile == tps - 1 && threadIdx.x == 0) totals[sidx] = 4 + excl + tile_agg;
}

__global__ void k_fill_u64(uint64_t* p, int64_t n, uint64_t v) {
  for (int64_t i = gtid(); i < n; i += gstride()) p[i] = v;
}

template <class Src>
cudaError_t launch_pack(const Src& src, int64_t n, int ns, int64_t in_stride, uint8_t* out, int64_t out_stride,
                        uint64_t* scratch, uint64_t* totals, int* status, cudaStream_t s) {
  const int64_t nblk = (n + 31) / 32;
  const int64_t tps = (nblk + kPackTileBlocks - 1) / kPackTileBlocks;
  if (ns <= 0) return cudaSuccess;
  cudaError_t e = cudaMemsetAsync(scratch, 0, (tps * ns + 2) * sizeof(uint64_t), s);
  if (e != cudaSuccess) return e;
  if (tps == 0) {
    // Empty inputs still write the u32 header (n = 0).
    for (int i = 0; i < ns; ++i) {
      e = cudaMemsetAsync(out + (int64_t)i * out_stride, 0, 4, s);
      if (e != cudaSuccess) return e;
    }
    k_fill_u64<<<1, 32, 0, s>>>(totals, ns, 4);
    return cudaGetLastError();
  }
  k_mask_pack<Src><<<(unsigned)(tps * ns), kThreads, 0, s>>>(src, n, ns, in_stride, out, out_stride, scratch, totals,
                                                             status);
  return cudaGetLastError();
}

cudaError_t bs_encode(const int16_t* q, int64_t n, uint8_t* out, uint64_t* scratch, uint64_t* total_bytes,
                      int* status, cudaStream_t s) {
  return launch_pack(SrcBS{q}, n, 1, 0, out, 0, scratch, total_bytes, status, s);
}
cudaError_t bs_encode_batch(const int16_t* q, int64_t n, int ns, uint8_t* out, int64_t out_stride, uint64_t* scratch,
                            uint64_t* totals, int* status, cudaStream_t s) {
  return launch_pack(SrcBS{q}, n, ns, n, out, out_stride, scratch, totals, status, s);
}
cudaError_t topk_encode(const int32_t* r, int64_t n, const float* threshold, const float* scale, uint8_t* out,
                        uint64_t* scratch, uint64_t* total_bytes, int* status, cudaStream_t s) {
  return launch_pack(SrcTopK{r, threshold, scale}, n, 1, 0, out, 0, scratch, total_bytes, status, s);
}

// ================================================= run-length encoders (K5, K6)
// Items are 32-blocks (BlockSparse+RLE, item kept iff its mask != 0) or
// single codes (RLE, kept iff code != 0).  A run starts at an item whose
// kind differs from its predecessor, and every 128 items into a run; each
// run head carries a one-byte opcode.  Pass 1 scans twice with look-back
// (segment start by max-scan, byte offsets by sum-scan) and writes the item
// payloads; pass 2 writes the opcodes (run length found by scanning ahead).
//
// Every launch encodes `ns` streams of n codes (stream s at q + s * n, its
// bytes at out + s * out_stride, its length in totals[s]).  Scratch layout
// (u64 words): [ns x (max status, sum status) per tile][tile counter, pad]
// [ns x item head offsets][ns x item kinds (bytes)][ns x block masks (u32)].
struct RunScratch {
  int64_t nitems, tps;
  int ns;
  uint64_t* base;
  __device__ __host__ uint64_t* st_max(int64_t s) const { return base + s * 2 * tps; }
  __device__ __host__ uint64_t* st_sum(int64_t s) const { return base + s * 2 * tps + tps; }
  __device__ __host__ unsigned long long* ctr() const {
    return reinterpret_cast<unsigned long long*>(base + (int64_t)ns * 2 * tps);
  }
  __device__ __host__ int64_t* offs() const { return reinterpret_cast<int64_t*>(base + (int64_t)ns * 2 * tps + 2); }
  __device__ __host__ uint8_t* types() const { return reinterpret_cast<uint8_t*>(offs() + (int64_t)ns * nitems); }
  __device__ __host__ uint32_t* masks() const {
    const int64_t tb = ((int64_t)ns * nitems + 7) / 8;  // u64 words of kinds
    return reinterpret_cast<uint32_t*>(offs() + (int64_t)ns * nitems + tb);
  }
};

int64_t run_scratch_words(int64_t items, int64_t ns) {
  const int64_t tiles = (items + kRunTileItems - 1) / kRunTileItems;
  return 2 * tiles * ns + 2 + items * ns + (items * ns + 7) / 8 + (items * ns + 1) / 2;
}

// One warp per 32-block of every stream: mask bit i = code i is non-zero.
__global__ void k_block_masks(const int16_t* __restrict__ q, int64_t n, int64_t nblk, int64_t total_blk,
                              uint32_t* __restrict__ masks) {
  const int lane = threadIdx.x & 31;
  for (int64_t b = gtid() >> 5; b < total_blk; b += gstride() >> 5) {
    const int64_t sidx = b / nblk, lb = b - sidx * nblk;
    const int64_t e = lb * 32 + lane;
    const uint32_t m = __ballot_sync(kFull, e < n && q[sidx * n + e] != 0);
    if (lane == 0) masks[b] = m;
  }
}

template <bool BLOCKS>
__global__ void __launch_bounds__(kThreads) k_run_pass1(const int16_t* __restrict__ q0, int64_t n, RunScratch sc,
                                                        uint8_t* __restrict__ out0, int64_t out_stride,
                                                        uint64_t* totals, int* status) {
  constexpr int IPT = kRunTileItems / kThreads;  // 16 items per thread
  __shared__ uint64_t s_warp[kThreads / 32];
  __shared__ uint64_t s_slot;
  __shared__ int64_t s_tile;
  __shared__ uint32_t s_rel[BLOCKS ? kRunTileItems : 1];  // payload offset in the tile (~0u: none)
  __shared__ uint32_t s_m[BLOCKS ? kRunTileItems : 1];
  const int64_t nitems = sc.nitems, tps = sc.tps;
  if (threadIdx.x == 0) s_tile = (int64_t)atomicAdd(sc.ctr(), 1ull);
  __syncthreads();
  const int64_t gtile = s_tile;
  if (gtile >= tps * sc.ns) return;
  const int64_t sidx = gtile / tps, tile = gtile - sidx * tps;
  const int16_t* q = q0 + sidx * n;
  uint8_t* out = out0 + sidx * out_stride;
  int64_t* offs = sc.offs() + sidx * nitems;
  uint8_t* types = sc.types() + sidx * nitems;
  const uint32_t* masks = sc.masks() + sidx * nitems;
  const int64_t i0 = tile * kRunTileItems + (int64_t)threadIdx.x * IPT;
  uint32_t m[IPT];
  bool nz[IPT];
  bool prev_nz = false;
  if (i0 > 0 && i0 - 1 < nitems) prev_nz = BLOCKS ? (masks[i0 - 1] != 0) : (q[i0 - 1] != 0);
  // pass A: segment starts (max-scan of change positions)
  uint64_t seg = 0;
  bool any_change = false;
#pragma unroll
  for (int j = 0; j < IPT; ++j) {
    const int64_t i = i0 + j;
    m[j] = 0;
    nz[j] = false;
    if (i < nitems) {
      if (BLOCKS) {
        m[j] = masks[i];
        nz[j] = m[j] != 0;
      } else {
        nz[j] = q[i] != 0;
      }
      const bool p = j == 0 ? prev_nz : nz[j - 1];
      if (i == 0 || nz[j] != p) {
        seg = (uint64_t)i;
        any_change = true;
      }
    }
  }
  uint64_t tile_max;
  const uint64_t thr_excl_max = block_excl_scan<OpMax>(any_change ? seg : 0, s_warp, &tile_max);
  const uint64_t tile_excl_max = lookback<OpMax>(sc.st_max(sidx), tile, tile_max, status, &s_slot);
  // pass B: run heads and byte sizes
  uint64_t run_start = OpMax::op(tile_excl_max, thr_excl_max);
  uint64_t sizes[IPT];
  bool head[IPT];
  uint64_t tsum = 0;
#pragma unroll
  for (int j = 0; j < IPT; ++j) {
    const int64_t i = i0 + j;
    sizes[j] = 0;
    head[j] = false;
    if (i < nitems) {
      const bool p = j == 0 ? prev_nz : nz[j - 1];
      if (i == 0 || nz[j] != p) run_start = (uint64_t)i;
      head[j] = (((uint64_t)i - run_start) % 128) == 0;
      uint64_t sz = head[j] ? 1 : 0;
      if (nz[j]) sz += BLOCKS ? (4 + 2 * (uint64_t)__popc(m[j])) : 2;
      sizes[j] = sz;
      tsum += sz;
    }
  }
  uint64_t tile_sum;
  const uint64_t thr_excl_sum = block_excl_scan<OpSum>(tsum, s_warp, &tile_sum);
  const uint64_t tile_excl_sum = lookback<OpSum>(sc.st_sum(sidx), tile, tile_sum, status, &s_slot);
  const uint64_t hdr = BLOCKS ? 4 : 0;
  if (BLOCKS && tile == 0 && threadIdx.x == 0) put_u32_bytes(out, (uint32_t)n);
  const uint64_t tbase = hdr + tile_excl_sum;
  uint64_t rel = thr_excl_sum;
#pragma unroll
  for (int j = 0; j < IPT; ++j) {
    const int64_t i = i0 + j;
    if (i < nitems) {
      types[i] = (uint8_t)(nz[j] ? 1 : 0);
      offs[i] = head[j] ? (int64_t)(tbase + rel) : -1;
      const uint64_t p = rel + (head[j] ? 1 : 0);
      if (BLOCKS) {
        s_rel[threadIdx.x * IPT + j] = nz[j] ? (uint32_t)p : ~0u;
        s_m[threadIdx.x * IPT + j] = m[j];
      } else if (nz[j]) {
        const uint16_t v = (uint16_t)q[i];
        out[tbase + p] = (uint8_t)v;
        out[tbase + p + 1] = (uint8_t)(v >> 8);
      }
    } else if (BLOCKS) {
      s_rel[threadIdx.x * IPT + j] = ~0u;
    }
    rel += sizes[j];
  }
  if (BLOCKS) {
    // Payload of every kept block, one warp per block: lane e loads code e
    // (coalesced) and stores it at its rank among the kept codes.
    __syncthreads();
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const uint32_t lt = (1u << lane) - 1u;
    constexpr int kU = 4;  // blocks per round: their loads are issued before any store
    constexpr int kW = kThreads / 32;
    for (int j0 = warp; j0 < kRunTileItems; j0 += kU * kW) {
      uint32_t r[kU], mm[kU];
      uint16_t v[kU];
#pragma unroll
      for (int u = 0; u < kU; ++u) {
        const int j = j0 + u * kW;
        r[u] = j < kRunTileItems ? s_rel[j] : ~0u;
        mm[u] = r[u] != ~0u ? s_m[j] : 0u;
        v[u] = ((mm[u] >> lane) & 1u) ? (uint16_t)q[(tile * kRunTileItems + j) * 32 + lane] : (uint16_t)0;
      }
#pragma unroll
      for (int u = 0; u < kU; ++u) {
        if (r[u] == ~0u) continue;
        uint8_t* dst = out + tbase + r[u];
        if (lane == 0) put_u32_bytes(dst, mm[u]);
        if ((mm[u] >> lane) & 1u) {
          const uint32_t pos = 4 + 2 * __popc(mm[u] & lt);
          dst[pos] = (uint8_t)v[u];
          dst[pos + 1] = (uint8_t)(v[u] >> 8);
        }
      }
    }
  }
  if (tile == tps - 1 && threadIdx.x == 0) totals[sidx] = hdr + tile_excl_sum + tile_sum;
}

// Pass 2: opcode of every run head = kind bit | (run length - 1).
__global__ void k_run_pass2(RunScratch sc, uint8_t* __restrict__ out0, int64_t out_stride) {
  const int64_t nitems = sc.nitems, all = nitems * sc.ns;
  const int64_t* offs = sc.offs();
  const uint8_t* types = sc.types();
  for (int64_t i = gtid(); i < all; i += gstride()) {
    const int64_t o = offs[i];
    if (o < 0) continue;
    const int64_t sidx = i / nitems, li = i - sidx * nitems;
    const uint8_t t = types[i];
    int count = 1;
    while (count < 128 && li + count < nitems && types[i + count] == t) ++count;
    out0[sidx * out_stride + o] = t ? (uint8_t)(count - 1) : (uint8_t)(0x80 | (count - 1));
  }
}

// Empty streams: header only (BlockSparse+RLE writes u32 n = 0).
__global__ void k_run_empty(uint8_t* out0, int64_t out_stride, int ns, bool blocks, uint64_t* totals) {
  for (int64_t i = gtid(); i < ns; i += gstride()) {
    if (blocks) put_u32_bytes(out0 + i * out_stride, 0u);
    totals[i] = blocks ? 4 : 0;
  }
}

template <bool BLOCKS>
cudaError_t launch_run(const int16_t* q, int64_t n, int ns, uint8_t* out, int64_t out_stride, uint64_t* scratch,
                       uint64_t* totals, int* status, cudaStream_t s) {
  if (ns <= 0) return cudaSuccess;
  const int64_t nitems = BLOCKS ? (n + 31) / 32 : n;
  const int64_t tps = (nitems + kRunTileItems - 1) / kRunTileItems;
  if (tps == 0) {
    k_run_empty<<<1, 128, 0, s>>>(out, out_stride, ns, BLOCKS, totals);
    return cudaGetLastError();
  }
  RunScratch sc{nitems, tps, ns, scratch};
  cudaError_t e = cudaMemsetAsync(scratch, 0, (2 * tps * ns + 2) * sizeof(uint64_t), s);
  if (e != cudaSuccess) return e;
  if (BLOCKS) {
    const int64_t total_blk = nitems * ns;
    int64_t g = (total_blk * 32 + kThreads - 1) / kThreads;
    if (g > 148 * 32) g = 148 * 32;
    k_block_masks<<<(unsigned)g, kThreads, 0, s>>>(q, n, nitems, total_blk, sc.masks());
  }
  k_run_pass1<BLOCKS><<<(unsigned)(tps * ns), kThreads, 0, s>>>(q, n, sc, out, out_stride, totals, status);
  e = cudaGetLastError();
  if (e != cudaSuccess) return e;
  k_run_pass2<<<grid_for(nitems * ns, 1), kThreads, 0, s>>>(sc, out, out_stride);
  return cudaGetLastError();
}

cudaError_t bsrle_encode(const int16_t* q, int64_t n, uint8_t* out, uint64_t* scratch, uint64_t* total_bytes,
                         int* status, cudaStream_t s) {
  return launch_run<true>(q, n, 1, out, 0, scratch, total_bytes, status, s);
}
cudaError_t rle_encode(const int16_t* q, int64_t n, uint8_t* out, uint64_t* scratch, uint64_t* total_bytes,
                       int* status, cudaStream_t s) {
  return launch_run<false>(q, n, 1, out, 0, scratch, total_bytes, status, s);
}
cudaError_t bsrle_encode_batch(const int16_t* q, int64_t n, int ns, uint8_t* out, int64_t out_stride,
                               uint64_t* scratch, uint64_t* totals, int* status, cudaStream_t s) {
  return launch_run<true>(q, n, ns, out, out_stride, scratch, totals, status, s);
}
cudaError_t rle_encode_batch(const int16_t* q, int64_t n, int ns, uint8_t* out, int64_t out_stride,
                             uint64_t* scratch, uint64_t* totals, int* status, cudaStream_t s) {
  return launch_run<false>(q, n, ns, out, out_stride, scratch, totals, status, s);
}

// ============================================================ stream decode
// Walk: one thread per stream reproduces the reference decoder's control
// flow and records, per decoded 32-block or RLE opcode, a descriptor
// (out offset | length << 48, input offset + 1 or 0 for zeros).
__device__ __forceinline__ uint32_t rd_u32(const uint8_t* p) {
  return (uint32_t)p[0] | ((uint32_t)p[1] << 8) | ((uint32_t)p[2] << 16) | ((uint32_t)p[3] << 24);
}

// Position after reading `cnt` values of `vb` bytes from `vals` where only
// whole values inside the stream are consumed (the reference decoder pushes
// 0 for the rest without advancing).
__device__ __forceinline__ int64_t advance_values(int64_t vals, int64_t len, int cnt, int vb) {
  const int64_t room = len > vals ? (len - vals) / vb : 0;
  return vals + (int64_t)vb * min64((int64_t)cnt, room);
}

constexpr int kWalkWin = 32768;  // bytes of a stream staged in shared memory at a time

// BlockSparse (fallback without scratch), top-k compat and element RLE.
// One CTA per stream: all threads stage a window of the stream into shared
// memory with 16-byte loads, then thread 0 runs the reference decoder's
// control flow from shared memory (a resumable state machine, so tokens may
// straddle windows) and records one descriptor per decoded 32-block or RLE
// opcode (one 16-byte store each).  Tokens are processed only while they lie
// entirely in the window (or the window reaches the end of the stream).
template <int KIND>
__global__ void __launch_bounds__(kThreads) k_walk(const uint8_t* __restrict__ data, const int64_t* __restrict__ soff,
                                                   int nstreams, int64_t out_cap, int64_t* __restrict__ out_len,
                                                   int64_t* __restrict__ table, int64_t table_cap, int* status) {
  constexpr int VB = KIND == 1 ? 1 : 2;
  constexpr int kMaxTok = KIND == 3 ? 257 : 4 + 32 * VB;
  static_assert(KIND != 2, "BlockSparse+RLE streams use k_walk_bsrle");
  constexpr int kWin = kWalkWin;
  __shared__ __align__(16) uint32_t win32[kWin / 4 + 4];
  __shared__ int64_t s_ptr;
  __shared__ int s_done;
  const int sidx = blockIdx.x;
  if (sidx >= nstreams) return;
  const uint8_t* b = data + soff[sidx];
  const int64_t len = soff[sidx + 1] - soff[sidx];
  int64_t* row = table + (int64_t)sidx * (2 * table_cap + 2);
  longlong2* tab = reinterpret_cast<longlong2*>(row + 2);
  const uint8_t* win = reinterpret_cast<const uint8_t*>(win32);
  // walker state (thread 0)
  int64_t ptr = 0, out = 0, nent = 0, blk = 0, n = 0, nblk = 0;
  bool overflow = false, done = false;
  if (threadIdx.x == 0) {
    if (KIND != 3) {
      if (len < 4) {
        done = true;
      } else {
        n = (int64_t)rd_u32(b);
        nblk = (n + 31) / 32;
        ptr = 4;
      }
    }
    s_ptr = ptr;
    s_done = done ? 1 : 0;
  }
  __syncthreads();
  while (!s_done) {
    const int64_t p0 = s_ptr;
    const int64_t base = p0 - (int64_t)(reinterpret_cast<uintptr_t>(b + p0) & 15u);
    const int64_t hi = min64(len, base + kWin);
    const int cnt = (int)(hi - base);
    const uint4* src = reinterpret_cast<const uint4*>(b + base);
    for (int i = threadIdx.x; i < cnt / 16; i += blockDim.x) reinterpret_cast<uint4*>(win32)[i] = src[i];
    for (int i = (cnt / 16) * 16 + threadIdx.x; i < cnt; i += blockDim.x)
      reinterpret_cast<uint8_t*>(win32)[i] = b[base + i];
    __syncthreads();
    if (threadIdx.x == 0) {
      const bool last = hi == len;
      const int lim = last ? cnt : cnt - kMaxTok;  // tokens must start at or before lim
      int q = (int)(ptr - base);                    // window-relative position
      const int qlen = (int)min64(len - base, (int64_t)1 << 30);
      auto u32 = [&](int x) -> uint32_t {
        const uint32_t w0 = win32[x >> 2], w1 = win32[(x >> 2) + 1];
        return __funnelshift_r(w0, w1, (x & 3) * 8);
      };
      auto emit = [&](int64_t o, int64_t l, int64_t in_plus1) {
        if (nent >= table_cap) {
          overflow = true;
          return;
        }
        tab[nent] = make_longlong2(o | (l << 48), in_plus1);
        ++nent;
      };
      while (!done && !overflow && (q <= lim || last)) {
        if (KIND == 0 || KIND == 1) {
          if (blk >= nblk || q + 4 > qlen) {
            done = true;
            break;
          }
          const uint32_t m = u32(q);
          const int64_t bl = blk == nblk - 1 ? n - blk * 32 : 32;
          emit(out, bl, base + q + 1);
          out += bl;
          const int c = __popc(bl >= 32 ? m : (m & ((1u << bl) - 1u)));
          const int vals = q + 4;
          const int room = qlen > vals ? (qlen - vals) / VB : 0;
          q = vals + VB * (c < room ? c : room);
          ++blk;
        } else {  // element RLE
          if (q >= qlen) {
            done = true;
            break;
          }
          const uint32_t op = win[q++];
          if (op >= 128) {
            out += (int64_t)op - 128 + 1;  // zeros: the output is zero-filled already
          } else {
            const int c = (int)op + 1;
            const int room = (qlen - q) / 2;
            const int avail = c < room ? c : room;
            if (avail > 0) emit(out, avail, base + q + 1);
            q += 2 * avail;
            out += avail;
          }
        }
      }
      ptr = base + q;
      if (overflow) done = true;
      if (!done && ptr >= len) done = true;
      s_ptr = ptr;
      s_done = done ? 1 : 0;
    }
    __syncthreads();
  }
  if (threadIdx.x == 0) {
    int64_t ol;
    if (KIND == 3) ol = out;
    else if (len < 4) ol = 0;
    else if (KIND == 1) ol = n;  // top-k pads to n
    else ol = min64(out, n);
    out_len[sidx] = ol;
    row[0] = nent;
    if (overflow || ol > out_cap) dev::set_status(status, dev::kBounds, sidx, (int)nent);
  }
}

// BlockSparse+RLE walk with warp specialisation.  Fixed windows: window k
// is home to the tokens starting in [k W, (k+1) W) and is staged with kROV
// more bytes, so every such token (at most 69 bytes) lies inside it.  While
// thread 0 walks window k, warps 1..7 stage window k+1 into the other buffer
// and fill its advance table (per byte position: 4 + 2 x the kept values of
// a block starting there, clamped to the whole values left), so a literal
// block costs the walker one byte load and an add.  Zero runs emit nothing
// (the output is zero-filled).  Same descriptors, lengths and status as the
// generic walker.
constexpr int kRW = 8192;
constexpr int kROV = 96;
constexpr int kRBuf = kRW + kROV + 32;

__device__ __forceinline__ void bsrle_prep(const uint8_t* b, int64_t len, int k, uint32_t* win, uint8_t* adv,
                                           int tid, int nthreads, bool all_threads) {
  const int64_t start = (int64_t)k * kRW;
  const int mis = (int)(reinterpret_cast<uintptr_t>(b + start) & 15u);
  const int64_t base = start - mis;
  const int64_t hi = min64(len, start + kRW + kROV);
  const int cnt = (int)(hi - base);
  const uint4* src = reinterpret_cast<const uint4*>(b + base);
  for (int i = tid; i < cnt / 16; i += nthreads) reinterpret_cast<uint4*>(win)[i] = src[i];
  for (int i = (cnt / 16) * 16 + tid; i < cnt; i += nthreads) reinterpret_cast<uint8_t*>(win)[i] = b[base + i];
  if (all_threads) __syncthreads();
  else asm volatile("bar.sync 1, %0;" ::"r"(nthreads) : "memory");
  const int qlen = (int)min64(len - base, (int64_t)1 << 30);
  for (int x = tid; x < cnt; x += nthreads) {
    uint32_t a = 0;
    if (x + 4 <= qlen) {
      const uint32_t w0 = win[x >> 2], w1 = win[(x >> 2) + 1];
      const int ad = 2 * __popc(__funnelshift_r(w0, w1, (x & 3) * 8)), rem = (qlen - (x + 4)) & ~1;
      a = 4 + (ad < rem ? ad : rem);
    }
    adv[x] = (uint8_t)a;
  }
}

__global__ void __launch_bounds__(kThreads) k_walk_bsrle(const uint8_t* __restrict__ data,
                                                         const int64_t* __restrict__ soff, int nstreams,
                                                         int64_t out_cap, int64_t* __restrict__ out_len,
                                                         int64_t* __restrict__ table, int64_t table_cap, int* status) {
  __shared__ __align__(16) uint32_t win[2][kRBuf / 4 + 4];
  __shared__ uint8_t adv[2][kRBuf];
  __shared__ int s_done;
  const int sidx = blockIdx.x;
  if (sidx >= nstreams) return;
  const uint8_t* b = data + soff[sidx];
  const int64_t len = soff[sidx + 1] - soff[sidx];
  int64_t* row = table + (int64_t)sidx * (2 * table_cap + 2);
  longlong2* tab = reinterpret_cast<longlong2*>(row + 2);
  const int64_t nwin = (len + kRW - 1) / kRW;
  // walker state (thread 0)
  int64_t ptr = 4, nent = 0, blk = 0, n = 0, nblk = 0;
  int lit = 0;
  bool done = false;
  if (threadIdx.x == 0) {
    if (len < 4) {
      done = true;
    } else {
      n = (int64_t)rd_u32(b);
      nblk = (n + 31) / 32;
      if (nblk > table_cap) {  // one descriptor per literal block at most
        dev::set_status(status, dev::kBounds, sidx, -1);
        done = true;
      }
    }
    s_done = done ? 1 : 0;
  }
  if (nwin > 0) bsrle_prep(b, len, 0, win[0], adv[0], threadIdx.x, blockDim.x, true);
  __syncthreads();
  for (int64_t k = 0; k < nwin && !s_done; ++k) {
    const int cur = (int)(k & 1);
    if (threadIdx.x >= 32) {
      if (k + 1 < nwin) bsrle_prep(b, len, (int)(k + 1), win[cur ^ 1], adv[cur ^ 1], threadIdx.x - 32,
                                   blockDim.x - 32, false);
    } else if (threadIdx.x == 0) {
      const int64_t start = k * kRW;
      const int64_t base = start - (int64_t)(reinterpret_cast<uintptr_t>(b + start) & 15u);
      const int64_t hi = min64(len, start + kRW + kROV);
      const bool last = hi == len;
      const int qlen = (int)min64(len - base, (int64_t)1 << 30);
      const int home_end = (int)(start + kRW - base);  // tokens starting before it belong here
      const uint8_t* wb = reinterpret_cast<const uint8_t*>(win[cur]);
      const uint8_t* av = adv[cur];
      int q = (int)(ptr - base);
      while (!done && (last || q < home_end)) {
        if (lit == 0) {
          if (!(blk < nblk && q < qlen)) {
            done = true;
            break;
          }
          const uint32_t op = wb[q++];
          if (op & 0x80u) blk += (int64_t)(op & 0x7fu) + 1;
          else lit = (int)op + 1;
          continue;
        }
        // full blocks before the last one, while a block fits (window, stream)
        {
          const int qstop = last ? qlen - 4 : home_end - 1;
          const int kmax = (int)min64((int64_t)lit, nblk - 1 - blk);
          longlong2* tp = tab + nent;
          const int64_t d0 = (blk * 32) | (32ll << 48), in0 = base + 1;
          int j = 0;
          while (j < kmax && q <= qstop) {
            tp[j] = make_longlong2(d0 + 32ll * j, in0 + q);
            q += av[q];
            ++j;
          }
          nent += j;
          blk += j;
          lit -= j;
        }
        if (lit == 0 || (!last && q >= home_end)) continue;
        if (blk >= nblk) {  // later blocks add nothing
          done = true;
          break;
        }
        if (q + 4 > qlen) {  // the literal run ends early; an opcode may follow
          lit = 0;
          continue;
        }
        // the stream's last block (its mask is read by the expansion)
        const int64_t l = n - blk * 32;
        tab[nent++] = make_longlong2((blk * 32) | (l << 48), base + q + 1);
        q += av[q];  // only decides when the walk ends: nothing follows the last block
        ++blk;
        --lit;
      }
      ptr = base + q;
      if (!done && last) done = true;
      s_done = done ? 1 : 0;
    }
    __syncthreads();
  }
  if (threadIdx.x == 0) {
    const int64_t ol = len < 4 ? 0 : min64(blk * 32, n);
    out_len[sidx] = ol;
    row[0] = nent;
    if (ol > out_cap) dev::set_status(status, dev::kBounds, sidx, (int)nent);
  }
}

// Expansion of element-RLE descriptors: one warp per descriptor; lanes write
// elements.
__global__ void k_expand(int kind, const uint8_t* __restrict__ data, const int64_t* __restrict__ soff,
                         const float* __restrict__ scales, int nstreams, int32_t* __restrict__ out, int64_t out_cap,
                         const int64_t* __restrict__ out_len, const int64_t* __restrict__ table, int64_t table_cap) {
  const int lane = threadIdx.x & 31;
  const int64_t wid = gtid() >> 5, nw = gstride() >> 5;
  const int64_t total = (int64_t)nstreams * table_cap;
  for (int64_t e = wid; e < total; e += nw) {
    const int64_t sidx = e / table_cap, ent = e % table_cap;
    const int64_t* row = table + sidx * (2 * table_cap + 2);
    if (ent >= row[0]) continue;  // past this stream's last descriptor
    const int64_t* tab = row + 2;
    const int64_t w0 = tab[2 * ent];
    const int64_t o = w0 & ((1ll << 48) - 1), l = (int64_t)((uint64_t)w0 >> 48), in1 = tab[2 * ent + 1];
    const uint8_t* b = data + soff[sidx];
    const int64_t len = soff[sidx + 1] - soff[sidx];
    const float sc = scales[sidx];
    const int64_t lim = min64(out_len[sidx], out_cap);
    int32_t* dst = out + sidx * out_cap;
    if (kind == 3) {
      for (int64_t j = lane; j < l; j += 32) {
        if (o + j >= lim) break;
        int32_t v = 0;
        if (in1) {
          const int64_t p = in1 - 1 + 2 * j;
          const int16_t c = (int16_t)((uint16_t)b[p] | ((uint16_t)b[p + 1] << 8));
          v = q823_from_f32(NGL_FMUL((float)c, sc));
        }
        dst[o + j] = v;
      }
    } else {
      if (lane < l && o + lane < lim) {
        int32_t v = 0;
        if (in1) {
          const int64_t mo = in1 - 1;
          const uint32_t m = rd_u32(b + mo);
          if ((m >> lane) & 1u) {
            const int vb = kind == 1 ? 1 : 2;
            const int64_t p = mo + 4 + (int64_t)vb * __popc(m & ((1u << lane) - 1u));
            if (kind == 1) {
              if (p < len) v = q823_from_f32(NGL_FMUL((float)(int8_t)b[p], sc));
            } else if (p + 2 <= len) {
              const int16_t c = (int16_t)((uint16_t)b[p] | ((uint16_t)b[p + 1] << 8));
              v = q823_from_f32(NGL_FMUL((float)c, sc));
            }
          }
        }
        dst[o + lane] = v;
      }
    }
  }
}

// Block descriptors (BlockSparse, top-k compat, BlockSparse+RLE): one warp
// per 32 consecutive descriptors of a stream.  Every lane first loads one
// descriptor and its mask (32 independent loads in flight), then the warp
// writes the 32 blocks in turn, coalesced, with each block's descriptor
// broadcast by shuffle; the value loads of successive blocks pipeline.
__global__ void __launch_bounds__(kThreads) k_expand_blocks(int kind, const uint8_t* __restrict__ data,
                                                            const int64_t* __restrict__ soff,
                                                            const float* __restrict__ scales, int nstreams,
                                                            int32_t* __restrict__ out, int64_t out_cap,
                                                            const int64_t* __restrict__ out_len,
                                                            const int64_t* __restrict__ table, int64_t table_cap) {
  const int lane = threadIdx.x & 31;
  const int vb = kind == 1 ? 1 : 2;
  const int64_t groups = (table_cap + 31) / 32;
  const int64_t wid = gtid() >> 5, nw = gstride() >> 5;
  const uint32_t lt = (1u << lane) - 1u;
  for (int64_t gi = wid; gi < (int64_t)nstreams * groups; gi += nw) {
    const int64_t sidx = gi / groups, g0 = (gi - sidx * groups) * 32;
    const int64_t* row = table + sidx * (2 * table_cap + 2);
    const int64_t count = row[0];
    if (g0 >= count) continue;  // uniform across the warp
    const int nd = (int)min64(32, count - g0);
    const uint8_t* b = data + soff[sidx];
    const int64_t len = soff[sidx + 1] - soff[sidx];
    const float sc = scales[sidx];
    const int64_t lim = min64(out_len[sidx], out_cap);
    int32_t* dst = out + sidx * out_cap;
    long long w0 = 0, in1 = 0;
    uint32_t m = 0;
    if (lane < nd) {
      const longlong2 dd = reinterpret_cast<const longlong2*>(row + 2)[g0 + lane];
      w0 = dd.x;
      in1 = dd.y;
      if (in1) m = rd_u32(b + in1 - 1);
    }
    for (int d = 0; d < nd; ++d) {
      const long long wd = __shfl_sync(kFull, w0, d);
      const long long id = __shfl_sync(kFull, in1, d);
      const uint32_t md = __shfl_sync(kFull, m, d);
      const int64_t o = wd & ((1ll << 48) - 1), l = (int64_t)((unsigned long long)wd >> 48);
      if (lane < l && o + lane < lim) {
        int32_t v = 0;
        if (id && ((md >> lane) & 1u)) {
          const int64_t p = id - 1 + 4 + (int64_t)vb * __popc(md & lt);
          if (kind == 1) {
            if (p < len) v = q823_from_f32(NGL_FMUL((float)(int8_t)b[p], sc));
          } else if (p + 2 <= len) {
            const int16_t c = (int16_t)((uint16_t)b[p] | ((uint16_t)b[p + 1] << 8));
            v = q823_from_f32(NGL_FMUL((float)c, sc));
          }
        }
        dst[o + lane] = v;
      }
    }
  }
}

// Top-k pads the decoded stream with zeros up to n (the walk reports n).
// ------------------------------------- parallel BlockSparse-family decode
// A BlockSparse (or top-k compat) stream is a chain of blocks [u32 mask]
// [VB bytes per set bit]: each block's position depends on every earlier
// mask, so a single thread walking it is latency bound.  Blocks are at most
// kMaxBlk = 4 + 32 VB bytes, so the chain enters a window [start, start + W)
// of the stream at one of kCand candidate offsets (even offsets for VB = 2,
// where every position is even; every offset for VB = 1).
//   A  one thread per (window, candidate) walks from the candidate to the
//      window's end: exit offset into the next window and block count.
//   B  one CTA per stream stages the candidate tables in shared memory and
//      chains them from the stream start: true entry and first block index of
//      every window.
//   C  one thread per window re-walks from its true entry with the exact
//      reference rules (last-block mask, truncated values, block limit) and
//      writes the block descriptors; the expansion kernel then writes values.
// Window size: 16 KB when the streams hold enough windows to fill the GPU
// (the per-stream chain of phase B stays short), 4 KB for small inputs
// (more, shorter speculative walks).  Measured on B200: a 64 Mi-element
// stream decodes in 1.4 ms at 16 KB vs 1.8 ms at 4 KB, a 16 Mi-element one
// in 0.60 ms at 4 KB vs 0.79 ms at 16 KB.
constexpr int64_t kBsWinLarge = 16384, kBsWinSmall = 4096;
inline int64_t bs_window(int64_t total_bytes) { return total_bytes / kBsWinLarge >= 2048 ? kBsWinLarge : kBsWinSmall; }
constexpr uint32_t kExitEnd = 255u;  // the stream ends inside the window

template <int VB>
struct BsGeom {
  static constexpr int kMaxBlk = 4 + 32 * VB;
  static constexpr int kStep = VB == 2 ? 2 : 1;
  static constexpr int kCand = kMaxBlk / kStep;  // 34 or 36
};

__device__ __forceinline__ uint32_t rd_u32_bytes(const uint8_t* p) {
  return (uint32_t)__ldg(p) | ((uint32_t)__ldg(p + 1) << 8) | ((uint32_t)__ldg(p + 2) << 16) |
         ((uint32_t)__ldg(p + 3) << 24);
}

// Window ranges: win_off[s] = first window of stream s (prefix over streams
// of ceil((len_s - 4) / W)), win_off[ns] = total.
__global__ void k_bs_win_offsets(const int64_t* __restrict__ soff, int ns, int64_t win, int64_t max_windows,
                                 int64_t* __restrict__ win_off, int* status) {
  if (blockIdx.x != 0 || threadIdx.x != 0) return;
  int64_t acc = 0;
  for (int i = 0; i < ns; ++i) {
    win_off[i] = acc;
    const int64_t len = soff[i + 1] - soff[i];
    acc += len > 4 ? (len - 4 + win - 1) / win : 0;
  }
  win_off[ns] = acc;
  // streams that overlap or lie outside `data` can need more windows than
  // the scratch holds: report instead of decoding part of them
  if (acc > max_windows) dev::set_status(status, dev::kBounds, -1, (int)min64(acc, 0x7fffffff));
}

__device__ __forceinline__ int stream_of_window(const int64_t* win_off, int ns, int64_t w) {
  int lo = 0, hi = ns - 1;  // last s with win_off[s] <= w
  while (lo < hi) {
    const int mid = (lo + hi + 1) >> 1;
    if (win_off[mid] <= w) lo = mid;
    else hi = mid - 1;
  }
  return lo;
}

template <int VB>
__global__ void __launch_bounds__(kThreads) k_bs_spec(const uint8_t* __restrict__ data, const int64_t* __restrict__ soff,
                                                      int ns, int64_t win, const int64_t* __restrict__ win_off,
                                                      int64_t max_windows, uint32_t* __restrict__ spec) {
  using G = BsGeom<VB>;
  const int64_t total = min64(win_off[ns], max_windows) * G::kCand;
  for (int64_t t = gtid(); t < total; t += gstride()) {
    const int64_t gw = t / G::kCand;
    const int cand = (int)(t - gw * G::kCand);
    const int s = stream_of_window(win_off, ns, gw);
    const int64_t w = gw - win_off[s];
    const uint8_t* b = data + soff[s];
    const int64_t len = soff[s + 1] - soff[s];
    const int64_t start = 4 + w * win, end = start + win;
    int64_t q = start + (int64_t)cand * G::kStep;
    uint32_t cnt = 0, exit = kExitEnd;
    while (true) {
      if (q >= end) {
        exit = (uint32_t)(q - end);
        break;
      }
      if (q + 4 > len) break;  // the stream ends here
      const int c = __popc(rd_u32_bytes(b + q));
      q = advance_values(q + 4, len, c, VB);
      ++cnt;
    }
    spec[t] = exit | (cnt << 8);
  }
}

// One CTA per stream: chain the windows.  entry[w] = true first block
// position in window w (-1: inactive), base[w] = its block index.
template <int VB>
__global__ void __launch_bounds__(kThreads) k_bs_chain(const uint8_t* __restrict__ data, const int64_t* __restrict__ soff,
                                                       int ns, int64_t win, const int64_t* __restrict__ win_off,
                                                       int64_t max_windows, const uint32_t* __restrict__ spec,
                                                       int64_t* __restrict__ entry, int64_t* __restrict__ base) {
  using G = BsGeom<VB>;
  constexpr int kChunk = 96;  // windows staged per round
  __shared__ uint32_t tab[kChunk * G::kCand];
  __shared__ int64_t s_e, s_base;
  __shared__ int s_stop;
  const int s = blockIdx.x;
  if (s >= ns) return;
  const int64_t w0 = win_off[s];
  const int64_t nw = min64(win_off[s + 1], max_windows) - min64(w0, max_windows);
  const int64_t len = soff[s + 1] - soff[s];
  if (threadIdx.x == 0) {
    const uint8_t* b = data + soff[s];
    int64_t nblk = 0;
    if (len >= 4) nblk = ((int64_t)rd_u32_bytes(b) + 31) / 32;
    s_e = 4;
    s_base = 0;
    s_stop = (len < 4 || nblk == 0) ? 1 : 0;
  }
  __syncthreads();
  for (int64_t c0 = 0; c0 < nw; c0 += kChunk) {
    const int nc = (int)min64(kChunk, nw - c0);
    if (!s_stop)
      for (int i = threadIdx.x; i < nc * G::kCand; i += blockDim.x) tab[i] = spec[(w0 + c0) * G::kCand + i];
    __syncthreads();
    if (threadIdx.x == 0) {
      int64_t e = s_e, bs = s_base;
      bool stop = s_stop != 0;
      for (int i = 0; i < nc; ++i) {
        const int64_t w = c0 + i;
        if (stop) {
          entry[w0 + w] = -1;
          continue;
        }
        const int64_t start = 4 + w * win;
        entry[w0 + w] = e;
        base[w0 + w] = bs;
        const uint32_t f = tab[i * G::kCand + (int)((e - start) / G::kStep)];
        const uint32_t ex = f & 0xffu;
        if (ex == kExitEnd) {
          stop = true;  // the chain ends inside this window
          continue;
        }
        bs += f >> 8;
        e = start + win + ex;
      }
      s_e = e;
      s_base = bs;
      s_stop = stop ? 1 : 0;
    }
    __syncthreads();
  }
}

// One thread per window: exact walk from the true entry, descriptors by
// block index; row[0] of the stream = decoded block count (atomicMax of the
// block index each window reached, capped at the header's block count).
template <int VB>
__global__ void __launch_bounds__(kThreads) k_bs_emit(const uint8_t* __restrict__ data, const int64_t* __restrict__ soff,
                                                      int ns, int64_t win, const int64_t* __restrict__ win_off,
                                                      int64_t max_windows, const int64_t* __restrict__ entry,
                                                      const int64_t* __restrict__ base, int64_t* __restrict__ table,
                                                      int64_t table_cap, int* status) {
  const int64_t total = min64(win_off[ns], max_windows);
  for (int64_t gw = gtid(); gw < total; gw += gstride()) {
    int64_t q = entry[gw];
    if (q < 0) continue;
    const int s = stream_of_window(win_off, ns, gw);
    const int64_t w = gw - win_off[s];
    const uint8_t* b = data + soff[s];
    const int64_t len = soff[s + 1] - soff[s];
    const int64_t n = (int64_t)rd_u32_bytes(b);
    const int64_t nblk = (n + 31) / 32;
    const int64_t end = 4 + (w + 1) * win;
    int64_t* row = table + (int64_t)s * (2 * table_cap + 2);
    longlong2* tab = reinterpret_cast<longlong2*>(row + 2);
    int64_t blk = base[gw];
    while (q < end && blk < nblk && q + 4 <= len) {
      if (blk >= table_cap) {
        dev::set_status(status, dev::kBounds, s, (int)blk);
        break;
      }
      const uint32_t m = rd_u32_bytes(b + q);
      const int64_t bl = blk == nblk - 1 ? n - blk * 32 : 32;
      tab[blk] = make_longlong2((blk * 32) | (bl << 48), q + 1);
      const int c = __popc(bl >= 32 ? m : (m & ((1u << bl) - 1u)));
      q = advance_values(q + 4, len, c, VB);
      ++blk;
    }
    // A window entered after the last block carries a speculative base >=
    // nblk: the chain decoded all nblk blocks.
    atomicMax(reinterpret_cast<unsigned long long*>(row), (unsigned long long)min64(blk, nblk));
  }
}

// Decoded length per stream: BlockSparse min(blocks * 32, n), top-k n.
__global__ void k_bs_len(const uint8_t* __restrict__ data, const int64_t* __restrict__ soff, int ns, int kind,
                         const int64_t* __restrict__ table, int64_t table_cap, int64_t out_cap,
                         int64_t* __restrict__ out_len, int* status) {
  for (int64_t s = gtid(); s < ns; s += gstride()) {
    const int64_t len = soff[s + 1] - soff[s];
    int64_t ol = 0;
    if (len >= 4) {
      const int64_t n = (int64_t)rd_u32_bytes(data + soff[s]);
      const int64_t blocks = table[s * (2 * table_cap + 2)];
      ol = kind == 1 ? n : min64(blocks * 32, n);
    }
    out_len[s] = ol;
    if (ol > out_cap) dev::set_status(status, dev::kBounds, (int)s, -1);
  }
}

int64_t bs_decode_scratch_words(int64_t total_bytes, int64_t nstreams) {
  const int64_t wins = total_bytes / bs_window(total_bytes) + 2 * nstreams + 1;
  // win_off (ns + 1), entry + base (2 per window), candidate tables (u32)
  return (nstreams + 1) + 2 * wins + (wins * 36 + 1) / 2;
}

template <int VB>
cudaError_t launch_bs_parallel(int kind, const uint8_t* data, const int64_t* soff, int ns, int64_t out_cap,
                               int64_t* out_len, int64_t* table, int64_t table_cap, int* status, uint64_t* scratch,
                               int64_t total_bytes, cudaStream_t s) {
  using G = BsGeom<VB>;
  const int64_t win = bs_window(total_bytes);
  const int64_t max_w = total_bytes / win + 2 * (int64_t)ns + 1;
  int64_t* win_off = reinterpret_cast<int64_t*>(scratch);
  int64_t* entry = win_off + ns + 1;
  int64_t* base = entry + max_w;
  uint32_t* spec = reinterpret_cast<uint32_t*>(base + max_w);
  // row[0] of every stream starts at 0 (atomicMax of block counts)
  cudaError_t e = cudaMemset2DAsync(table, (size_t)(2 * table_cap + 2) * sizeof(int64_t), 0, sizeof(int64_t),
                                    (size_t)ns, s);
  if (e != cudaSuccess) return e;
  k_bs_win_offsets<<<1, 32, 0, s>>>(soff, ns, win, max_w, win_off, status);
  const int64_t cand = max_w * G::kCand;
  int64_t g = (cand + kThreads - 1) / kThreads;
  if (g > 148 * 16) g = 148 * 16;
  k_bs_spec<VB><<<(unsigned)(g > 0 ? g : 1), kThreads, 0, s>>>(data, soff, ns, win, win_off, max_w, spec);
  k_bs_chain<VB><<<ns, kThreads, 0, s>>>(data, soff, ns, win, win_off, max_w, spec, entry, base);
  int64_t g2 = (max_w + kThreads - 1) / kThreads;
  if (g2 > 148 * 8) g2 = 148 * 8;
  k_bs_emit<VB><<<(unsigned)(g2 > 0 ? g2 : 1), kThreads, 0, s>>>(data, soff, ns, win, win_off, max_w, entry, base,
                                                                 table, table_cap, status);
  k_bs_len<<<(unsigned)((ns + kThreads - 1) / kThreads), kThreads, 0, s>>>(data, soff, ns, kind, table, table_cap,
                                                                          out_cap, out_len, status);
  return cudaGetLastError();
}

__global__ void k_zero_fill(int32_t* out, int64_t out_cap, const int64_t* out_len, int nstreams) {
  for (int64_t i = gtid(); i < (int64_t)nstreams * out_cap; i += gstride()) out[i] = 0;
}

cudaError_t stream_decode(int kind, const uint8_t* data, const int64_t* stream_off, const float* scales, int nstreams,
                          int32_t* out, int64_t out_cap, int64_t* out_len, int64_t* table, int64_t table_cap,
                          int* status, uint64_t* scratch, int64_t total_bytes, cudaStream_t s) {
  if (nstreams <= 0) return cudaSuccess;
  if (kind == 1) {
    k_zero_fill<<<grid_for((int64_t)nstreams * out_cap), kThreads, 0, s>>>(out, out_cap, out_len, nstreams);
  }
  cudaError_t e = cudaSuccess;
  if (kind == 0 && scratch) e = launch_bs_parallel<2>(kind, data, stream_off, nstreams, out_cap, out_len, table, table_cap, status, scratch, total_bytes, s);
  else if (kind == 1 && scratch) e = launch_bs_parallel<1>(kind, data, stream_off, nstreams, out_cap, out_len, table, table_cap, status, scratch, total_bytes, s);
  else if (kind == 0) k_walk<0><<<nstreams, kThreads, 0, s>>>(data, stream_off, nstreams, out_cap, out_len, table, table_cap, status);
  else if (kind == 1) k_walk<1><<<nstreams, kThreads, 0, s>>>(data, stream_off, nstreams, out_cap, out_len, table, table_cap, status);
  else if (kind == 2) k_walk_bsrle<<<nstreams, kThreads, 0, s>>>(data, stream_off, nstreams, out_cap, out_len, table, table_cap, status);
  else k_walk<3><<<nstreams, kThreads, 0, s>>>(data, stream_off, nstreams, out_cap, out_len, table, table_cap, status);
  if (e != cudaSuccess) return e;
  e = cudaGetLastError();
  if (e != cudaSuccess) return e;
  if (kind != 3) {  // block descriptors: 32 per warp
    const int64_t warps = (int64_t)nstreams * ((table_cap + 31) / 32);
    int64_t g = (warps * 32 + kThreads - 1) / kThreads;
    if (g > 148 * 32) g = 148 * 32;
    if (g < 1) g = 1;
    k_expand_blocks<<<(unsigned)g, kThreads, 0, s>>>(kind, data, stream_off, scales, nstreams, out, out_cap, out_len,
                                                     table, table_cap);
    return cudaGetLastError();
  }
  const int64_t warps = (int64_t)nstreams * table_cap;
  int64_t g = (warps * 32 + kThreads - 1) / kThreads;
  if (g > 148 * 32) g = 148 * 32;
  if (g < 1) g = 1;
  k_expand<<<(unsigned)g, kThreads, 0, s>>>(kind, data, stream_off, scales, nstreams, out, out_cap, out_len, table,
                                           table_cap);
  return cudaGetLastError();
}

// ===================================================== stochastic compat (K7)
__global__ void k_absmax(const int32_t* __restrict__ r, int64_t n, uint32_t* max_bits) {
  float m = 0.0f;
  for (int64_t i = gtid(); i < n; i += gstride()) m = fmaxf(m, fabsf(q823_to_f32(r[i])));
  const uint32_t w = __reduce_max_sync(kFull, __float_as_uint(m));
  if ((threadIdx.x & 31) == 0) atomicMax(max_bits, w);
}

__device__ __forceinline__ float compat_scale(float max_val, int bits) {
  if (!(max_val > 1e-9f)) return 1.0f;
  const int levels = (bits >= 1 && bits < 31) ? ((1 << bits) - 1) : 255;
  return NGL_FDIV(max_val, NGL_FDIV((float)levels, 2.0f));
}

__global__ void k_stochastic_encode(const int32_t* __restrict__ r, int64_t n, int bits, uint64_t seed,
                                    uint64_t counter, const uint32_t* max_bits, float* scale_out,
                                    uint8_t* __restrict__ out) {
  const float scale = compat_scale(__uint_as_float(*max_bits), bits);
  if (gtid() == 0) *scale_out = scale;
  if (bits == 4) {
    const int64_t nb = (n + 1) / 2;
    for (int64_t j = gtid(); j < nb; j += gstride()) {
      uint8_t byte = 0;
      for (int k = 0; k < 2; ++k) {
        const int64_t i = 2 * j + k;
        if (i >= n) break;
        int32_t q = compat_stochastic_round(NGL_FDIV(q823_to_f32(r[i]), scale), seed, counter + (uint64_t)i);
        q = q < -8 ? -8 : (q > 7 ? 7 : q);
        const uint8_t nb4 = (uint8_t)((int8_t)q & 0x0F);
        byte |= k == 0 ? (uint8_t)(nb4 << 4) : nb4;
      }
      out[j] = byte;
    }
  } else if (bits == 8) {
    for (int64_t i = gtid(); i < n; i += gstride()) {
      int32_t q = compat_stochastic_round(NGL_FDIV(q823_to_f32(r[i]), scale), seed, counter + (uint64_t)i);
      q = q < -128 ? -128 : (q > 127 ? 127 : q);
      out[i] = (uint8_t)(int8_t)q;
    }
  } else {
    for (int64_t i = gtid(); i < n; i += gstride()) {
      float q = f_round(NGL_FDIV(q823_to_f32(r[i]), scale));
      if (!is_nan(q)) q = fminf(fmaxf(q, -128.0f), 127.0f);
      out[i] = (uint8_t)sat_f32_to_i8(q);
    }
  }
}

__global__ void k_stochastic_decode(const uint8_t* __restrict__ b, int64_t nbytes, int bits, float scale,
                                    int32_t* __restrict__ out) {
  for (int64_t i = gtid(); i < nbytes; i += gstride()) {
    if (bits == 4) {
      const int32_t hi = ((int32_t)((uint32_t)b[i] << 24)) >> 28;
      const int32_t lo = ((int32_t)((uint32_t)b[i] << 28)) >> 28;
      out[2 * i] = q823_from_f32(NGL_FMUL((float)hi, scale));
      out[2 * i + 1] = q823_from_f32(NGL_FMUL((float)lo, scale));
    } else {
      out[i] = q823_from_f32(NGL_FMUL((float)(int8_t)b[i], scale));
    }
  }
}

cudaError_t absmax_f32_of_fixed(const int32_t* r, int64_t n, uint32_t* max_bits, cudaStream_t s) {
  cudaError_t e = cudaMemsetAsync(max_bits, 0, sizeof(uint32_t), s);
  if (e != cudaSuccess) return e;
  if (n > 0) k_absmax<<<grid_for(n), kThreads, 0, s>>>(r, n, max_bits);
  return cudaGetLastError();
}
cudaError_t stochastic_encode(const int32_t* r, int64_t n, int bits, uint64_t seed, uint64_t counter,
                              const uint32_t* max_bits, float* scale_out, uint8_t* out, cudaStream_t s) {
  k_stochastic_encode<<<grid_for(n > 0 ? n : 1), kThreads, 0, s>>>(r, n, bits, seed, counter, max_bits, scale_out,
                                                                   out);
  return cudaGetLastError();
}
cudaError_t stochastic_decode(const uint8_t* b, int64_t nbytes, int bits, float scale, int32_t* out,
                              cudaStream_t s) {
  if (nbytes > 0) k_stochastic_decode<<<grid_for(nbytes), kThreads, 0, s>>>(b, nbytes, bits, scale, out);
  return cudaGetLastError();
}

// ============================================ top-k radix-select threshold (K8)
// Pass p histograms digit p (MSB first) of the |x| bit patterns that match
// the prefix selected by passes 0..p-1; every CTA re-derives that prefix
// from the previous histograms (256 bins each), so no host round trip.
__device__ void select_prefix(const uint32_t* hist, int passes, int64_t target, uint32_t* prefix_out,
                              int64_t* target_out) {
  uint32_t prefix = 0;
  for (int p = 0; p < passes; ++p) {
    const uint32_t* h = hist + p * 256;
    int64_t acc = 0;
    int d = 255;
    for (; d > 0; --d) {
      if (acc + (int64_t)h[d] >= target) break;
      acc += h[d];
    }
    target -= acc;
    prefix = (prefix << 8) | (uint32_t)d;
  }
  *prefix_out = prefix;
  *target_out = target;
}

__global__ void k_radix_hist(const int32_t* __restrict__ r, int64_t n, int pass, int64_t keep,
                             uint32_t* __restrict__ hist) {
  __shared__ uint32_t sh[256];
  __shared__ uint32_t s_prefix;
  for (int i = threadIdx.x; i < 256; i += blockDim.x) sh[i] = 0;
  if (threadIdx.x == 0) {
    int64_t t;
    select_prefix(hist, pass, keep, &s_prefix, &t);
  }
  __syncthreads();
  const uint32_t prefix = s_prefix;
  const int shift = 24 - 8 * pass;
  for (int64_t i = gtid(); i < n; i += gstride()) {
    const uint32_t u = __float_as_uint(fabsf(q823_to_f32(r[i])));
    if (pass == 0 || (u >> (shift + 8)) == prefix) atomicAdd(&sh[(u >> shift) & 0xffu], 1u);
  }
  __syncthreads();
  for (int i = threadIdx.x; i < 256; i += blockDim.x)
    if (sh[i]) atomicAdd(&hist[pass * 256 + i], sh[i]);
}

__global__ void k_radix_final(const uint32_t* hist, int64_t keep, const uint32_t* max_bits, float* thr,
                              float* scale) {
  if (threadIdx.x != 0 || blockIdx.x != 0) return;
  if (keep == 0) {
    *thr = 1e-9f;
  } else {
    uint32_t prefix;
    int64_t t;
    select_prefix(hist, 4, keep, &prefix, &t);
    *thr = fmaxf(__uint_as_float(prefix), 1e-9f);
  }
  const float mx = __uint_as_float(*max_bits);
  *scale = mx > 1e-9f ? NGL_FDIV(mx, 127.0f) : 1.0f;
}

cudaError_t topk_threshold(const int32_t* r, int64_t n, int64_t keep, uint32_t* hist, const uint32_t* max_bits,
                           float* threshold, float* scale, cudaStream_t s) {
  cudaError_t e = cudaMemsetAsync(hist, 0, 4 * 256 * sizeof(uint32_t), s);
  if (e != cudaSuccess) return e;
  if (keep > n) keep = n;
  if (keep > 0)
    for (int p = 0; p < 4; ++p) k_radix_hist<<<grid_for(n), kThreads, 0, s>>>(r, n, p, keep, hist);
  k_radix_final<<<1, 32, 0, s>>>(hist, keep, max_bits, threshold, scale);
  return cudaGetLastError();
}

}  // namespace codec
}  // namespace ngl
