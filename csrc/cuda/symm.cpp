// Symmetric peer memory for the fused all-reduce: one cudaMalloc'd region per
// rank, exported with CUDA IPC and mapped into every other rank's address
// space so kernels can store to (and load from) peers over NVLink / NVSwitch.
// The handles travel through the process group (see parallel/symm.py); this
// file only allocates, exports, opens and closes.
#include <cuda_runtime.h>
#include <pybind11/pybind11.h>
#include <pybind11/stl.h>

#include <cstring>
#include <stdexcept>
#include <string>
#include <vector>

namespace {

void check(cudaError_t e, const char* what) {
  if (e != cudaSuccess) throw std::runtime_error(std::string(what) + ": " + cudaGetErrorString(e));
}

class SymmRegion {
 public:
  SymmRegion(int64_t bytes, int64_t device) : bytes_(bytes), device_((int)device) {
    if (bytes <= 0) throw std::runtime_error("SymmRegion: bytes must be positive");
    check(cudaSetDevice(device_), "cudaSetDevice");
    check(cudaMalloc(&local_, (size_t)bytes), "cudaMalloc(symmetric region)");
    check(cudaMemset(local_, 0, (size_t)bytes), "cudaMemset(symmetric region)");
    check(cudaDeviceSynchronize(), "cudaDeviceSynchronize");
  }
  ~SymmRegion() {
    try {
      close();
    } catch (...) {
    }
  }

  pybind11::bytes ipc_handle() const {
    cudaIpcMemHandle_t h;
    check(cudaIpcGetMemHandle(&h, local_), "cudaIpcGetMemHandle");
    return pybind11::bytes(reinterpret_cast<const char*>(&h), sizeof(h));
  }

  // Map every other rank's region; handles[r] is rank r's ipc_handle().
  void open(const std::vector<std::string>& handles, int64_t rank) {
    check(cudaSetDevice(device_), "cudaSetDevice");
    peers_.assign(handles.size(), nullptr);
    for (size_t r = 0; r < handles.size(); ++r) {
      if ((int64_t)r == rank) {
        peers_[r] = local_;
        continue;
      }
      if (handles[r].size() != sizeof(cudaIpcMemHandle_t)) throw std::runtime_error("bad IPC handle size");
      cudaIpcMemHandle_t h;
      std::memcpy(&h, handles[r].data(), sizeof(h));
      void* p = nullptr;
      check(cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess), "cudaIpcOpenMemHandle");
      peers_[r] = p;
    }
    rank_ = rank;
  }

  std::vector<int64_t> ptrs() const {
    std::vector<int64_t> out;
    for (void* p : peers_) out.push_back(reinterpret_cast<int64_t>(p));
    if (out.empty()) out.push_back(reinterpret_cast<int64_t>(local_));
    return out;
  }
  int64_t local_ptr() const { return reinterpret_cast<int64_t>(local_); }
  int64_t bytes() const { return bytes_; }

  // Unmap the peers' regions (call on every rank, then barrier, then close).
  void close_peers() {
    if (peers_.empty()) return;
    cudaSetDevice(device_);
    for (size_t r = 0; r < peers_.size(); ++r)
      if ((int64_t)r != rank_ && peers_[r] != nullptr) cudaIpcCloseMemHandle(peers_[r]);
    peers_.clear();
  }
  void close() {
    close_peers();
    if (local_ == nullptr) return;
    cudaSetDevice(device_);
    cudaFree(local_);
    local_ = nullptr;
  }

 private:
  int64_t bytes_;
  int device_;
  int64_t rank_ = -1;
  void* local_ = nullptr;
  std::vector<void*> peers_;
};

}  // namespace

void register_symm(pybind11::module& m) {
  pybind11::class_<SymmRegion>(m, "SymmRegion")
      .def(pybind11::init<int64_t, int64_t>())
      .def("ipc_handle", &SymmRegion::ipc_handle)
      .def("open", &SymmRegion::open)
      .def("ptrs", &SymmRegion::ptrs)
      .def("local_ptr", &SymmRegion::local_ptr)
      .def("bytes", &SymmRegion::bytes)
      .def("close_peers", &SymmRegion::close_peers)
      .def("close", &SymmRegion::close);
}
