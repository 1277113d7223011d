// Torch bindings of the device workload generators.
#include <torch/extension.h>

#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>

#include "synth.h"

namespace {

torch::Tensor make_out(int64_t steps, int64_t n, int64_t device) {
  TORCH_CHECK(steps >= 0 && n >= 0, "sizes must be non-negative");
  return torch::empty({steps, n}, torch::TensorOptions().dtype(torch::kFloat32).device(torch::kCUDA, device));
}

torch::Tensor synth_ar1(int64_t n, int64_t steps, int64_t seed, double rho, double sigma, double sigma0,
                        double sparse_frac, double sparse_scale, int64_t device) {
  c10::cuda::CUDAGuard g((c10::DeviceIndex)device);
  auto out = make_out(steps, n, device);
  const cudaError_t e = ngl::synth::ar1(out.data_ptr<float>(), n, (int)steps, (uint64_t)seed, (float)rho, (float)sigma,
                                        (float)sigma0, (float)sparse_frac, (float)sparse_scale,
                                        at::cuda::getCurrentCUDAStream());
  TORCH_CHECK(e == cudaSuccess, "synth_ar1: ", cudaGetErrorString(e));
  return out;
}

torch::Tensor synth_brownian(int64_t n, int64_t steps, int64_t seed, double sigma, double box, double lo,
                             bool periodic, int64_t device) {
  c10::cuda::CUDAGuard g((c10::DeviceIndex)device);
  auto out = make_out(steps, n, device);
  const cudaError_t e = ngl::synth::brownian(out.data_ptr<float>(), n, (int)steps, (uint64_t)seed, (float)sigma,
                                             (float)box, (float)lo, periodic, at::cuda::getCurrentCUDAStream());
  TORCH_CHECK(e == cudaSuccess, "synth_brownian: ", cudaGetErrorString(e));
  return out;
}

}  // namespace

void register_synth(pybind11::module& m) {
  m.def("synth_ar1", &synth_ar1, pybind11::arg("n"), pybind11::arg("steps"), pybind11::arg("seed") = 0,
        pybind11::arg("rho") = 0.9, pybind11::arg("sigma") = 1e-3, pybind11::arg("sigma0") = 1e-2,
        pybind11::arg("sparse_frac") = 0.7, pybind11::arg("sparse_scale") = 0.01, pybind11::arg("device") = 0);
  m.def("synth_brownian", &synth_brownian, pybind11::arg("n"), pybind11::arg("steps"), pybind11::arg("seed") = 0,
        pybind11::arg("sigma") = 0.01, pybind11::arg("box") = 100.0, pybind11::arg("lo") = 0.0,
        pybind11::arg("periodic") = true, pybind11::arg("device") = 0);
}
