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
constexpr int kMaxWorld = 8;
constexpr int kMaxCols = 2048;        // max CTAs of one launch (flag columns)
constexpr int kTopkMaxRec = 520;      // topk_record_bytes(256)
constexpr int kMaxChunkRec = 8 * kTopkMaxRec;

enum Mode : int { kInt4 = 0, kInt8 = 1, kTopK = 2 };
enum FlagKind : int { kFlagPayload = 0, kFlagResult = 1 };

// Static topology drop at chunk granularity: chunk c (of nchunks) is a
// passenger iff (c * a + b) mod nchunks < ndrop.  Passengers are neither
// encoded nor sent; they reconstruct to the prediction and keep their whole
// residual in the error feedback.  ndrop = 0 disables it.
struct Topo {
  uint32_t a;
  uint32_t b;
  int ndrop;
};

struct QParams {
  uint64_t seed;
  uint64_t step;
  uint32_t bucket;
  uint32_t rank;
  int stochastic;
  int use_ef;
  int use_pred;
  Topo topo;
  // Exchange kernels: fraction of the predictor's lines read in phase 1 with
  // the L2 evict_last policy, so phase 2's re-read hits L2 (0: no policy).
  float pred_keep;
};
// One fp32 parameter of a bucket for the optimizer fused into the decode
// phase: its gradient occupies bucket elements [off, off + numel).
struct OptSeg {
  int64_t off;
  int64_t numel;
  float* p;
  float* m;  // first moment
  float* v;  // second moment
};
// AdamW with decoupled weight decay (Loshchilov & Hutter), applied to every
// averaged gradient element as it is written: segs == nullptr turns it off.
// Host-computed per step: decay = 1 - lr * weight_decay, step_size =
// lr / (1 - beta1^t), inv_bc2_sqrt = 1 / sqrt(1 - beta2^t).
struct OptParams {
  const OptSeg* segs;  // device array sorted by off
  int nsegs;
  int64_t base;        // bucket element of this launch's element 0 (segmented buckets)
  float beta1, beta2, eps, decay, step_size, inv_bc2_sqrt;
};
struct FParams {
  float inv_world;
  float beta;
  float omb;
  int first;
  int use_pred;
  Topo topo;
  int pred_stream;  // phase 2 reads the predictor with the evict_first policy
  OptParams opt;
};

// Symmetric region of every rank (same layout on all ranks):
//   flags_off : u64 flags [2 parity][2 kinds][world src][kMaxCols]
//   inbox_off : [2 parity][world src] slots of slot_bytes (chunk records)
//   result_off: [2 parity] two-shot result regions of result_bytes
struct FusedParams {
  void* grad;
  float* pred;
  float* ef;
  int64_t n;
  int nblk;
  int nchunks;
  int k;           // top-k per block
  int rec_bytes;   // top-k block record bytes
  int chunk_bytes; // wire bytes per chunk record for this mode
  int world;
  int rank;
  uint8_t* sym[kMaxWorld];
  int64_t flags_off;
  int64_t inbox_off;
  int64_t slot_bytes;
  int64_t result_off;
  int64_t result_bytes;
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

// Grid used for a launch: a pure function of (nchunks, mode, dtype, variant,
// cap) on a given GPU model, so every rank launches the same grid.
// opt: the instance that applies the fused optimizer (its occupancy differs).
int fused_grid(int nchunks, int mode, int dtype, int variant, int cap, int device, int opt = 0);
cudaError_t launch_fused(const FusedParams& P, int mode, int dtype, int variant, int grid, cudaStream_t stream);
cudaError_t launch_encode(const void* g, const float* pred, const float* ef_in, float* ef_out, int64_t n, int k,
                          const QParams& qp, uint8_t* out, int mode, int dtype, int grid, cudaStream_t stream);
// Check of the shared-memory prefetch pipeline: dst = src through it.
cudaError_t launch_pipe_copy(const float* src, float* dst, int64_t n, int grid, int vec, int* status,
                             cudaStream_t stream);
cudaError_t launch_reduce(const ReduceSrcs& srcs, int world, void* out, float* pred, int64_t n, int k,
                          const FParams& fp, int mode, int dtype, int grid, cudaStream_t stream);

}  // namespace dev
}  // namespace ngl
