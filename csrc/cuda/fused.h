// Parameters and launchers of the fused compressed all-reduce kernels
// (csrc/cuda/fused_kernels.cu).  Plain CUDA: no torch headers, so the kernel
// translation unit compiles quickly; csrc/cuda/fused_bind.cpp adapts tensors.
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>

namespace ngl {
namespace dev {

constexpr int kWarps = 8;
constexpr int kThreads = kWarps * 32;
constexpr int kChunkBlocks = kWarps;  // one 256-block per warp per chunk
constexpr int kMaxWorld = 8;
constexpr int kTopkMaxRec = 520;      // topk_record_bytes(256) rounded up

enum Mode : int { kInt4 = 0, kInt8 = 1, kTopK = 2 };

struct QParams {
  uint64_t seed;
  uint64_t step;
  uint32_t bucket;
  uint32_t rank;
  int stochastic;
  int use_ef;
  int use_pred;
};
struct FParams {
  float inv_world;
  float beta;
  float omb;
  int first;
  int use_pred;
};

struct FusedParams {
  void* grad;
  float* pred;
  float* ef;
  int64_t n;
  int nblk;
  int nchunks;
  int k;          // top-k per block
  int rec_bytes;  // top-k record bytes
  int world;
  int rank;
  uint8_t* sym[kMaxWorld];
  int64_t flags_off;   // u64 flags [2][world][max_chunks]
  int64_t rflags_off;  // u64 result flags [2][max_chunks]
  int64_t inbox_off;   // [2][world] slots of slot_bytes
  int64_t slot_bytes;
  int64_t result_off;  // [2] result regions of result_bytes
  int64_t result_bytes;
  int max_chunks;
  uint32_t epoch;
  uint32_t tag;
  int parity;
  QParams q;
  FParams f;
  int* status;
  uint64_t timeout_ns;
};

struct ReduceSrcs {
  const uint8_t* p[kMaxWorld];
};

enum DType : int { kF32 = 0, kBF16 = 1 };
enum Variant : int { kVariantSingle = 0, kVariantOneShot = 1, kVariantTwoShot = 2 };

cudaError_t launch_fused(const FusedParams& P, int mode, int dtype, int variant, int grid, cudaStream_t stream);
cudaError_t launch_encode(const void* g, const float* pred, const float* ef_in, float* ef_out, int64_t n, int k,
                          const QParams& qp, uint8_t* out, int mode, int dtype, int grid, cudaStream_t stream);
cudaError_t launch_reduce(const ReduceSrcs& srcs, int world, void* out, float* pred, int64_t n, int k,
                          const FParams& fp, int mode, int dtype, int grid, cudaStream_t stream);

}  // namespace dev
}  // namespace ngl
