// Synthetic workload generators on the device (sm_100a): AR(1) gradient
// streams and Brownian particle trajectories with a periodic box, the input
// shapes of the mode-switching and LAMMPS-compression workloads at sizes
// where host generation would dominate a run.
//
// Random numbers: Philox4x32-10 (Salmon et al., "Parallel random numbers:
// as easy as 1, 2, 3", SC'11) keyed by the seed, one counter per (element,
// step, stream); Gaussian variates by the Box-Muller transform (Box and
// Muller, 1958) on the first two words, uniforms from the top 24 bits.
// log/sqrt/sincospi are CUDA's own functions.
//
// The reference generates its workloads on the host with closed-form
// signals (examples/mode_switching/src/main.rs:87-93,
// examples/lammps_compress/src/main.rs:311-322); these generators have no
// counterpart there.
#include <cuda_runtime.h>
#include <stdint.h>

#include "common/ngl_product.h"
#include "synth.h"

namespace ngl {
namespace synth {
namespace {

constexpr int kThreads = 256;

__device__ __forceinline__ U32x4 draw(uint64_t seed, uint64_t i, uint32_t step, uint32_t stream) {
  const U32x4 c = {(uint32_t)i, (uint32_t)(i >> 32), step, stream};
  return philox4x32_10(c, (uint32_t)seed, (uint32_t)(seed >> 32));
}
// Uniform in (0, 1]: top 24 bits, offset by one ulp of 2^-24.
__device__ __forceinline__ float u01_open0(uint32_t b) { return ((float)(b >> 8) + 1.0f) * (1.0f / 16777216.0f); }
__device__ __forceinline__ float gauss(const U32x4& r) {
  const float u1 = u01_open0(r.x), u2 = u01_open0(r.y);
  const float rad = sqrtf(-2.0f * logf(u1));
  float s, c;
  sincospif(2.0f * u2, &s, &c);
  return rad * c;
}

__global__ void __launch_bounds__(kThreads) k_ar1(float* __restrict__ out, int64_t n, int steps, uint64_t seed,
                                                  float rho, float sigma, float sigma0, float sparse_frac,
                                                  float sparse_scale) {
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
    const U32x4 r0 = draw(seed, (uint64_t)i, 0u, 0x41523100u);
    const float scale = u01_open0(r0.z) <= sparse_frac ? sparse_scale : 1.0f;
    float g = __fmul_rn(sigma0, gauss(r0));
    for (int t = 0; t < steps; ++t) {
      if (t) g = __fadd_rn(__fmul_rn(rho, g), __fmul_rn(sigma, gauss(draw(seed, (uint64_t)i, (uint32_t)t, 0x41523101u))));
      __stcs(out + (int64_t)t * n + i, __fmul_rn(g, scale));
    }
  }
}

// x in [lo, lo + box): x - box * floor((x - lo) / box).
__device__ __forceinline__ float wrap(float x, float lo, float box) {
  const float y = __fsub_rn(x, lo);
  return __fadd_rn(lo, __fsub_rn(y, __fmul_rn(box, floorf(__fdiv_rn(y, box)))));
}

__global__ void __launch_bounds__(kThreads) k_brownian(float* __restrict__ out, int64_t n, int steps, uint64_t seed,
                                                       float sigma, float box, float lo, int periodic) {
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
    float x = __fadd_rn(lo, __fmul_rn(box, u01_open0(draw(seed, (uint64_t)i, 0u, 0x4C4D5000u).x) - (1.0f / 16777216.0f)));
    for (int t = 0; t < steps; ++t) {
      if (t) {
        x = __fadd_rn(x, __fmul_rn(sigma, gauss(draw(seed, (uint64_t)i, (uint32_t)t, 0x4C4D5001u))));
        if (periodic) x = wrap(x, lo, box);
      }
      __stcs(out + (int64_t)t * n + i, x);
    }
  }
}

int grid_for(int64_t n) {
  int sms = 148;
  int dev = 0;
  if (cudaGetDevice(&dev) == cudaSuccess) cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const int64_t want = (n + kThreads - 1) / kThreads;
  const int64_t cap = (int64_t)sms * 8;
  return (int)(want < 1 ? 1 : (want < cap ? want : cap));
}

}  // namespace

cudaError_t ar1(float* out, int64_t n, int steps, uint64_t seed, float rho, float sigma, float sigma0,
                float sparse_frac, float sparse_scale, cudaStream_t s) {
  if (n <= 0 || steps <= 0) return cudaSuccess;
  k_ar1<<<grid_for(n), kThreads, 0, s>>>(out, n, steps, seed, rho, sigma, sigma0, sparse_frac, sparse_scale);
  return cudaGetLastError();
}

cudaError_t brownian(float* out, int64_t n, int steps, uint64_t seed, float sigma, float box, float lo, bool periodic,
                     cudaStream_t s) {
  if (n <= 0 || steps <= 0) return cudaSuccess;
  k_brownian<<<grid_for(n), kThreads, 0, s>>>(out, n, steps, seed, sigma, box, lo, periodic ? 1 : 0);
  return cudaGetLastError();
}

}  // namespace synth
}  // namespace ngl
