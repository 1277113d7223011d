// Module definition of mini_nangila_b200._cuda (sm_100a kernels).
#include <torch/extension.h>

void register_fused(pybind11::module& m);
void register_symm(pybind11::module& m);
void register_codecs(pybind11::module& m);
void register_synth(pybind11::module& m);

PYBIND11_MODULE(TORCH_EXTENSION_NAME, m) {
  m.doc() = "sm_100a kernels: fused compressed all-reduce, codecs, symmetric memory";
  m.attr("ARCH") = "sm_100a";
  register_fused(m);
  register_symm(m);
  register_codecs(m);
  register_synth(m);
}
