// Device generators of synthetic workloads (csrc/cuda/synth_kernels.cu).
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>

namespace ngl {
namespace synth {

// out [steps, n]: g_0 = sigma0 * z, g_t = rho * g_{t-1} + sigma * z_t, each
// element scaled by sparse_scale with probability sparse_frac (fixed per
// element).  z ~ N(0, 1).
cudaError_t ar1(float* out, int64_t n, int steps, uint64_t seed, float rho, float sigma, float sigma0,
                float sparse_frac, float sparse_scale, cudaStream_t s);
// out [steps, n]: x_0 uniform in [lo, lo + box), x_t = x_{t-1} + sigma * z_t,
// wrapped into [lo, lo + box) when periodic.
cudaError_t brownian(float* out, int64_t n, int steps, uint64_t seed, float sigma, float box, float lo, bool periodic,
                     cudaStream_t s);

}  // namespace synth
}  // namespace ngl
