// Device-side helpers shared by the sm_100a kernels: memory-ordering PTX for
// cross-GPU flags, bounded waits, vector I/O for fp32/bf16 buckets.
#pragma once
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "common/ngl_product.h"

namespace ngl {
namespace dev {

constexpr unsigned kFull = 0xffffffffu;

__device__ __forceinline__ int64_t min64(int64_t a, int64_t b) { return a < b ? a : b; }
__device__ __forceinline__ int64_t max64(int64_t a, int64_t b) { return a > b ? a : b; }

// Error codes written to the status word (never a trap).
enum Status : int {
  kOk = 0,
  kTimeoutPayload = 1,   // a peer's payload flag never arrived
  kTimeoutResult = 2,    // a two-shot result flag never arrived
  kBadHeader = 3,        // payload header did not match (n / epoch)
  kBounds = 4,           // bounds check failed (NGL_BOUNDS_CHECK builds)
  kTimeoutCopy = 5,      // a bulk copy into shared memory never completed
  kTimeoutLookback = 6,  // a scan's look-back wait on a predecessor tile expired
};

__device__ __forceinline__ uint64_t globaltimer() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}
__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ void st_release_sys(uint32_t* p, uint32_t v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ int ld_volatile_i32(const int* p) {
  int v;
  asm volatile("ld.volatile.global.s32 %0, [%1];" : "=r"(v) : "l"(p));
  return v;
}

// Record the first error (code + two context words) without trapping.
__device__ __forceinline__ void set_status(int* status, int code, int a, int b) {
  if (status == nullptr) return;
  if (atomicCAS(status, 0, code) == 0) {
    status[1] = a;
    status[2] = b;
  }
}

// Spin until *flag == want, a deadline passes, or another CTA reports an
// error.  Returns false on give-up (caller records the status).
__device__ __forceinline__ bool wait_flag(const uint32_t* flag, uint32_t want, uint64_t timeout_ns,
                                          const int* status) {
  if (ld_acquire_sys(flag) == want) return true;
  const uint64_t t0 = globaltimer();
  uint32_t spins = 0;
  while (true) {
    if (ld_acquire_sys(flag) == want) return true;
    if ((++spins & 63u) == 0) {
      if (globaltimer() - t0 > timeout_ns) return false;
      if (status != nullptr && ld_volatile_i32(status) != 0) return false;
    }
    __nanosleep(64);
  }
}

// Warp reductions.
__device__ __forceinline__ float warp_absmax(float v) {
  float m = fabsf(v);
  if (m != m) m = 0.0f;  // NaN ignored, like fmax
  uint32_t u = __reduce_max_sync(kFull, __float_as_uint(m));
  return __uint_as_float(u);
}
__device__ __forceinline__ int warp_excl_scan(int v, int lane) {
  int x = v;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    int y = __shfl_up_sync(kFull, x, o);
    if (lane >= o) x += y;
  }
  return x - v;
}

// ---- 8 consecutive elements per lane: vector loads of fp32 / bf16 ----
template <typename T>
struct Vec8;

template <>
struct Vec8<float> {
  static __device__ __forceinline__ void load(const float* p, float (&v)[8]) {
    float4 a = *reinterpret_cast<const float4*>(p);
    float4 b = *reinterpret_cast<const float4*>(p + 4);
    v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w;
    v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
  }
  static __device__ __forceinline__ void store(float* p, const float (&v)[8]) {
    *reinterpret_cast<float4*>(p) = make_float4(v[0], v[1], v[2], v[3]);
    *reinterpret_cast<float4*>(p + 4) = make_float4(v[4], v[5], v[6], v[7]);
  }
  static __device__ __forceinline__ float get(const float* p) { return *p; }
  static __device__ __forceinline__ void put(float* p, float v) { *p = v; }
};

template <>
struct Vec8<__nv_bfloat16> {
  static __device__ __forceinline__ void load(const __nv_bfloat16* p, float (&v)[8]) {
    uint4 u = *reinterpret_cast<const uint4*>(p);
    const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      v[2 * i] = __uint_as_float(w[i] << 16);
      v[2 * i + 1] = __uint_as_float(w[i] & 0xffff0000u);
    }
  }
  static __device__ __forceinline__ void store(__nv_bfloat16* p, const float (&v)[8]) {
    uint32_t w[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      __nv_bfloat162 h = __floats2bfloat162_rn(v[2 * i], v[2 * i + 1]);
      w[i] = *reinterpret_cast<uint32_t*>(&h);
    }
    *reinterpret_cast<uint4*>(p) = make_uint4(w[0], w[1], w[2], w[3]);
  }
  static __device__ __forceinline__ float get(const __nv_bfloat16* p) { return __bfloat162float(*p); }
  static __device__ __forceinline__ void put(__nv_bfloat16* p, float v) { *p = __float2bfloat16_rn(v); }
};

// Load 8 elements starting at element `e0` of which `valid` (0..8) are in
// range; out-of-range lanes read 0.  `vec_ok` selects the vector path.
// ---- bounds-checked debug builds (-DNGL_BOUNDS_CHECK)
// NGL_BOUNDS_UNIFORM(cond, status, a, b): when cond fails, record kBounds
// with (a, b) in the status word and leave the kernel.  Only for conditions
// that are uniform across the CTA at that point (no thread may be left
// waiting at a barrier).  Compiled out in release builds.
#ifdef NGL_BOUNDS_CHECK
#define NGL_BOUNDS_UNIFORM(cond, status, a, b)                           \
  do {                                                                   \
    if (!(cond)) {                                                       \
      if (threadIdx.x == 0) ::ngl::dev::set_status((status), ::ngl::dev::kBounds, (a), (b)); \
      return;                                                            \
    }                                                                    \
  } while (0)
#else
#define NGL_BOUNDS_UNIFORM(cond, status, a, b) \
  do {                                         \
  } while (0)
#endif

// ---- bulk copies global -> shared with an mbarrier (no tensor map, no multicast)
__device__ __forceinline__ uint32_t smem_u32(const void* p) { return (uint32_t)__cvta_generic_to_shared(p); }
__device__ __forceinline__ void mbar_init(uint64_t* m, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(m)), "r"(count) : "memory");
}
__device__ __forceinline__ void fence_mbar_init() { asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory"); }
__device__ __forceinline__ void fence_proxy_async_smem() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }
__device__ __forceinline__ void mbar_expect_tx(uint64_t* m, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(m)), "r"(bytes) : "memory");
}
// src, dst 16-byte aligned, bytes a multiple of 16; src is this GPU's memory.
__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, uint32_t bytes, uint64_t* m) {
  asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                   smem_u32(dst)),
               "l"(src), "r"(bytes), "r"(smem_u32(m))
               : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint64_t* m, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}\n"
      : "=r"(ok)
      : "r"(smem_u32(m)), "r"(parity)
      : "memory");
  return ok != 0;
}
// Bounded wait for phase `parity` of an mbarrier: false after limit_ns.
__device__ __forceinline__ bool mbar_wait(uint64_t* m, uint32_t parity, uint64_t limit_ns) {
  if (mbar_try_wait(m, parity)) return true;
  const uint64_t t0 = globaltimer();
  while (!mbar_try_wait(m, parity))
    if (globaltimer() - t0 > limit_ns) return false;
  return true;
}

// ---- L2 eviction-priority loads (createpolicy + ld.global.L2::cache_hint)
// A policy marks a fraction of the accessed lines evict_first (streamed
// once) or evict_last (read again soon by this kernel: kept over normal
// lines).  fp32 only; the caller checks alignment (16 bytes).
__device__ __forceinline__ uint64_t l2_policy_evict_last(float fraction) {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_last.b64 %0, %1;" : "=l"(p) : "f"(fraction));
  return p;
}
__device__ __forceinline__ uint64_t l2_policy_evict_first() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(p));
  return p;
}
__device__ __forceinline__ float4 ld_f4_policy(const float* p, uint64_t pol) {
  float4 v;
  asm volatile("ld.global.L2::cache_hint.v4.f32 {%0, %1, %2, %3}, [%4], %5;"
               : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w)
               : "l"(p), "l"(pol));
  return v;
}
// 8 fp32 elements at base + e0 through an L2 policy (scalar tail as load8).
__device__ __forceinline__ void load8_policy(const float* base, int64_t e0, int valid, uint64_t pol,
                                             float (&v)[8]) {
  if (valid == 8) {
    const float4 a = ld_f4_policy(base + e0, pol), b = ld_f4_policy(base + e0 + 4, pol);
    v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w;
    v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
  } else {
#pragma unroll
    for (int j = 0; j < 8; ++j) v[j] = (j < valid) ? base[e0 + j] : 0.0f;
  }
}

template <typename T>
__device__ __forceinline__ void load8(const T* base, int64_t e0, int valid, bool vec_ok, float (&v)[8]) {
  if (valid == 8 && vec_ok) {
    Vec8<T>::load(base + e0, v);
  } else {
#pragma unroll
    for (int j = 0; j < 8; ++j) v[j] = (j < valid) ? Vec8<T>::get(base + e0 + j) : 0.0f;
  }
}
template <typename T>
__device__ __forceinline__ void store8(T* base, int64_t e0, int valid, bool vec_ok, const float (&v)[8]) {
  if (valid == 8 && vec_ok) {
    Vec8<T>::store(base + e0, v);
  } else {
#pragma unroll
    for (int j = 0; j < 8; ++j)
      if (j < valid) Vec8<T>::put(base + e0 + j, v[j]);
  }
}

}  // namespace dev
}  // namespace ngl
