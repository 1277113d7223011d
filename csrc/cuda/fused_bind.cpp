// Torch-facing side of the fused compressed all-reduce: tensor checks,
// geometry, epoch bookkeeping and launches on the current CUDA stream.
#include <torch/extension.h>

#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>

#include <algorithm>
#include <cstring>

#include "common/ngl_product.h"
#include "fused.h"

namespace {
using namespace ngl::dev;

int num_sms(int device) {
  static int cached[64] = {0};
  if (device >= 0 && device < 64 && cached[device]) return cached[device];
  int v = 0;
  cudaDeviceGetAttribute(&v, cudaDevAttrMultiProcessorCount, device);
  if (device >= 0 && device < 64) cached[device] = v;
  return v;
}

int64_t nchunks_of(int64_t n) { return ((n + 255) / 256 + ngl::kChunkBlocks - 1) / ngl::kChunkBlocks; }
// Wire bytes of one rank's payload for a bucket of n elements.
int64_t payload_bytes(int64_t n, int64_t mode, int64_t k) {
  return nchunks_of(n) * ngl::chunk_record_bytes((int)mode, (int)k);
}

void check_dev(const torch::Tensor& t, const char* what) {
  TORCH_CHECK(t.is_cuda(), what, " must be a CUDA tensor");
  TORCH_CHECK(t.is_contiguous(), what, " must be contiguous");
  TORCH_CHECK(reinterpret_cast<uintptr_t>(t.data_ptr()) % 16 == 0, what, " must be 16-byte aligned");
}
int dtype_code(torch::ScalarType t) {
  if (t == torch::kFloat32) return kF32;
  if (t == torch::kBFloat16) return kBF16;
  TORCH_CHECK(false, "bucket dtype must be float32 or bfloat16");
  return -1;
}
Topo topo_of(const std::vector<int64_t>& t, int64_t nchunks) {
  Topo r{1u, 0u, 0};
  if (t.empty()) return r;
  TORCH_CHECK(t.size() == 3, "topology must be (a, b, ndrop)");
  TORCH_CHECK(t[0] > 0 && t[1] >= 0 && t[2] >= 0 && t[2] < std::max<int64_t>(nchunks, 1) &&
                  (nchunks == 0 || (t[0] < std::max<int64_t>(nchunks, 2) && t[1] < nchunks)),
              "topology (a, b, ndrop) out of range for ", nchunks, " chunks");
  r.a = (uint32_t)t[0];
  r.b = (uint32_t)t[1];
  r.ndrop = (int)t[2];
  return r;
}

void check_launch(cudaError_t e, const char* what) {
  TORCH_CHECK(e == cudaSuccess, what, " launch failed: ", cudaGetErrorString(e));
}

// Persistent state of one process's fused communicator: the symmetric-region
// pointers of every rank, the geometry, the epoch counter, the status word.
class FusedComm {
 public:
  FusedComm(int64_t world, int64_t rank, std::vector<int64_t> sym_ptrs, int64_t flags_off, int64_t inbox_off,
            int64_t slot_bytes, int64_t result_off, int64_t result_bytes, torch::Tensor status)
      : world_(world), rank_(rank), status_(status) {
    TORCH_CHECK(world >= 1 && world <= kMaxWorld, "world size must be in [1, 8]");
    TORCH_CHECK(world == 1 || (int64_t)sym_ptrs.size() == world, "need one symmetric pointer per rank");
    TORCH_CHECK(status.is_cuda() && status.scalar_type() == torch::kInt32 && status.numel() >= 4,
                "status must be int32[>=4] on the device");
    std::memset(&base_, 0, sizeof(base_));
    for (int i = 0; i < (int)sym_ptrs.size() && i < kMaxWorld; ++i)
      base_.sym[i] = reinterpret_cast<uint8_t*>(sym_ptrs[i]);
    base_.world = (int)world;
    base_.rank = (int)rank;
    base_.flags_off = flags_off;
    base_.inbox_off = inbox_off;
    base_.slot_bytes = slot_bytes;
    base_.result_off = result_off;
    base_.result_bytes = result_bytes;
    base_.status = status.data_ptr<int>();
  }

  // Launch the fused kernel on the current stream; returns the epoch used.
  // variant: 0 = auto-single (world 1), 1 = one-shot, 2 = two-shot.
  // opt_segs: optional uint8 CUDA tensor holding opt_nsegs OptSeg records
  // (the fused AdamW of the decode phase); opt_hyper = (beta1, beta2, eps,
  // decay, step_size, inv_bc2_sqrt); opt_base = bucket element of grad[0].
  int64_t run(torch::Tensor grad, c10::optional<torch::Tensor> pred, c10::optional<torch::Tensor> ef, int64_t mode,
              int64_t k, int64_t variant, bool stochastic, int64_t seed, int64_t bucket, int64_t step, double beta,
              bool first, int64_t max_ctas, int64_t timeout_ns, int64_t tag, std::vector<int64_t> topo,
              c10::optional<torch::Tensor> opt_segs, int64_t opt_nsegs, int64_t opt_base,
              std::vector<double> opt_hyper) {
    check_dev(grad, "bucket");
    const int64_t n = grad.numel();
    FusedParams P = base_;
    P.grad = grad.data_ptr();
    P.pred = nullptr;
    P.ef = nullptr;
    if (pred.has_value()) {
      check_dev(*pred, "predictor state");
      TORCH_CHECK(pred->scalar_type() == torch::kFloat32 && pred->numel() == n, "predictor state must be fp32[n]");
      P.pred = pred->data_ptr<float>();
    }
    if (ef.has_value()) {
      check_dev(*ef, "error feedback");
      TORCH_CHECK(ef->scalar_type() == torch::kFloat32 && ef->numel() == n, "error feedback must be fp32[n]");
      P.ef = ef->data_ptr<float>();
    }
    TORCH_CHECK(mode >= 0 && mode <= 2, "mode must be 0 (int4), 1 (int8) or 2 (top-k)");
    P.n = n;
    P.nblk = (int)((n + ngl::kBlock - 1) / ngl::kBlock);
    P.nchunks = (P.nblk + ngl::kChunkBlocks - 1) / ngl::kChunkBlocks;
    P.k = (int)k;
    P.rec_bytes = ngl::topk_record_bytes((int)k);
    P.chunk_bytes = ngl::chunk_record_bytes((int)mode, (int)k);
    if (world_ == 1) variant = kVariantSingle;
    TORCH_CHECK(variant != kVariantSingle || world_ == 1, "the single-rank kernel needs world size 1");
    if (mode == kTopK) {
      TORCH_CHECK(k >= 1 && k <= 256, "top-k per block must be in [1, 256]");
      TORCH_CHECK(variant != kVariantTwoShot, "two-shot is implemented for dense modes only");
    }
    if (world_ > 1) {
      const int64_t need = payload_bytes(n, mode, k);
      TORCH_CHECK(need <= base_.slot_bytes, "payload (", need, " B) exceeds the inbox slot (", base_.slot_bytes, " B)");
      if (variant == kVariantTwoShot)
        TORCH_CHECK(payload_bytes(n, kInt8, 0) <= base_.result_bytes, "two-shot result exceeds its region");
    }
    epoch_ += 1;
    P.epoch = (uint32_t)epoch_;
    P.parity = (int)(epoch_ & 1);
    P.tag = (uint32_t)tag;
    P.q.seed = (uint64_t)seed;
    P.q.step = (uint64_t)step;
    P.q.bucket = (uint32_t)bucket;
    P.q.rank = (uint32_t)rank_;
    P.q.stochastic = stochastic ? 1 : 0;
    P.q.use_ef = P.ef != nullptr;
    P.q.use_pred = P.pred != nullptr;
    P.f.inv_world = 1.0f / (float)world_;
    P.f.beta = (float)beta;
    P.f.omb = 1.0f - (float)beta;
    P.f.first = first ? 1 : 0;
    P.f.use_pred = P.pred != nullptr;
    P.q.topo = topo_of(topo, P.nchunks);
    P.f.topo = P.q.topo;
    // Exchange kernels read the predictor in both phases: keep (at most
    // l2_keep_bytes of) it in L2 between them.
    P.q.pred_keep = 0.0f;
    if (variant != kVariantSingle && P.pred != nullptr && l2_keep_bytes_ > 0 && n > 0)
      P.q.pred_keep = (float)std::min(1.0, (double)l2_keep_bytes_ / (4.0 * (double)n));
    P.f.pred_stream = P.q.pred_keep > 0.0f ? 1 : 0;
    std::memset(&P.f.opt, 0, sizeof(P.f.opt));
    if (opt_segs.has_value()) {
      TORCH_CHECK(opt_segs->is_cuda() && opt_segs->scalar_type() == torch::kUInt8 && opt_segs->is_contiguous(),
                  "optimizer segments must be a contiguous uint8 CUDA tensor");
      TORCH_CHECK(opt_nsegs >= 1 && opt_segs->numel() == opt_nsegs * (int64_t)sizeof(OptSeg),
                  "optimizer segment table size mismatch");
      TORCH_CHECK(opt_hyper.size() == 6, "optimizer scalars must be (beta1, beta2, eps, decay, step_size, "
                                         "inv_bc2_sqrt)");
      TORCH_CHECK(grad.scalar_type() == torch::kFloat32, "the fused optimizer needs an fp32 bucket");
      P.f.opt.segs = reinterpret_cast<const OptSeg*>(opt_segs->data_ptr());
      P.f.opt.nsegs = (int)opt_nsegs;
      P.f.opt.base = opt_base;
      P.f.opt.beta1 = (float)opt_hyper[0];
      P.f.opt.beta2 = (float)opt_hyper[1];
      P.f.opt.eps = (float)opt_hyper[2];
      P.f.opt.decay = (float)opt_hyper[3];
      P.f.opt.step_size = (float)opt_hyper[4];
      P.f.opt.inv_bc2_sqrt = (float)opt_hyper[5];
    }
    P.timeout_ns = (uint64_t)timeout_ns;
    if (P.nblk == 0) return epoch_;
    const c10::cuda::CUDAGuard guard(grad.device());
    cudaStream_t stream = at::cuda::getCurrentCUDAStream();
    const int dev = grad.get_device();
    const int grid = fused_grid(P.nchunks, (int)mode, dtype_code(grad.scalar_type()), (int)variant, (int)max_ctas, dev,
                                P.f.opt.segs != nullptr ? 1 : 0);
    check_launch(launch_fused(P, (int)mode, dtype_code(grad.scalar_type()), (int)variant, grid, stream), "fused");
    return epoch_;
  }

  int64_t epoch() const { return epoch_; }
  void set_epoch(int64_t e) { epoch_ = e; }
  int64_t l2_keep_bytes() const { return l2_keep_bytes_; }
  void set_l2_keep_bytes(int64_t b) { l2_keep_bytes_ = b < 0 ? 0 : b; }

 private:
  // Predictor bytes held in L2 between the phases of an exchange kernel
  // (48 MB of the 126 MB L2 by default; 0 turns the policy off).
  int64_t l2_keep_bytes_ = int64_t(48) << 20;
  int64_t world_, rank_;
  torch::Tensor status_;
  FusedParams base_;
  int64_t epoch_ = 0;
};

// Encode one rank's payload on the device (same layout as an inbox slot).
std::vector<torch::Tensor> product_encode_cuda(torch::Tensor g, c10::optional<torch::Tensor> pred,
                                               c10::optional<torch::Tensor> ef, int64_t mode, int64_t k,
                                               bool stochastic, int64_t seed, int64_t rank, int64_t bucket,
                                               int64_t step, std::vector<int64_t> topo) {
  check_dev(g, "g");
  const int64_t n = g.numel();
  const int nblk = (int)((n + 255) / 256);
  const int64_t bytes = payload_bytes(n, mode, k);
  auto out = torch::zeros({bytes}, g.options().dtype(torch::kUInt8));
  torch::Tensor ef_out =
      ef.has_value() ? torch::empty_like(*ef) : torch::empty({0}, g.options().dtype(torch::kFloat32));
  QParams qp;
  qp.seed = (uint64_t)seed;
  qp.step = (uint64_t)step;
  qp.bucket = (uint32_t)bucket;
  qp.rank = (uint32_t)rank;
  qp.stochastic = stochastic;
  qp.use_ef = ef.has_value();
  qp.use_pred = pred.has_value();
  qp.topo = topo_of(topo, nchunks_of(n));
  qp.pred_keep = 0.0f;
  if (pred.has_value()) check_dev(*pred, "pred");
  if (ef.has_value()) check_dev(*ef, "ef");
  if (nblk == 0) return {out, ef_out};
  const c10::cuda::CUDAGuard guard(g.device());
  cudaStream_t stream = at::cuda::getCurrentCUDAStream();
  const int grid = std::min((nblk + kWarps - 1) / kWarps, 4 * num_sms(g.get_device()));
  check_launch(launch_encode(g.data_ptr(), pred.has_value() ? pred->data_ptr<float>() : nullptr,
                             ef.has_value() ? ef->data_ptr<float>() : nullptr,
                             ef.has_value() ? ef_out.data_ptr<float>() : nullptr, n, (int)k, qp,
                             out.data_ptr<uint8_t>(), (int)mode, dtype_code(g.scalar_type()), grid, stream),
               "encode");
  return {out, ef_out};
}

// Rank-ordered reduction of W payloads on one device; updates `pred` (EMA)
// in place when given and returns the averaged bucket.
torch::Tensor product_reduce_cuda(std::vector<torch::Tensor> payloads, int64_t n, int64_t mode, int64_t k,
                                  c10::optional<torch::Tensor> pred, double beta, bool first, double inv_world,
                                  torch::ScalarType out_dtype, std::vector<int64_t> topo) {
  TORCH_CHECK(!payloads.empty() && (int)payloads.size() <= kMaxWorld, "1..8 payloads");
  ReduceSrcs s;
  std::memset(&s, 0, sizeof(s));
  for (size_t i = 0; i < payloads.size(); ++i) {
    check_dev(payloads[i], "payload");
    s.p[i] = payloads[i].data_ptr<uint8_t>();
  }
  auto out = torch::empty({n}, payloads[0].options().dtype(out_dtype));
  const int nblk = (int)((n + 255) / 256);
  if (nblk == 0) return out;
  FParams fp;
  fp.inv_world = (float)inv_world;
  fp.beta = (float)beta;
  fp.omb = 1.0f - (float)beta;
  fp.first = first;
  fp.use_pred = pred.has_value();
  fp.topo = topo_of(topo, nchunks_of(n));
  fp.pred_stream = 0;
  std::memset(&fp.opt, 0, sizeof(fp.opt));
  if (pred.has_value()) check_dev(*pred, "pred");
  const c10::cuda::CUDAGuard guard(payloads[0].device());
  cudaStream_t stream = at::cuda::getCurrentCUDAStream();
  const int grid = std::min((nblk + kWarps - 1) / kWarps, 4 * num_sms(payloads[0].get_device()));
  check_launch(launch_reduce(s, (int)payloads.size(), out.data_ptr(),
                             pred.has_value() ? pred->data_ptr<float>() : nullptr, n, (int)k, fp, (int)mode,
                             dtype_code(out_dtype), grid, stream),
               "reduce");
  return out;
}

}  // namespace

void register_fused(pybind11::module& m) {
  pybind11::class_<FusedComm>(m, "FusedComm")
      .def(pybind11::init<int64_t, int64_t, std::vector<int64_t>, int64_t, int64_t, int64_t, int64_t, int64_t,
                          torch::Tensor>())
      .def("run", &FusedComm::run, pybind11::arg("grad"), pybind11::arg("pred"), pybind11::arg("ef"),
           pybind11::arg("mode"), pybind11::arg("k"), pybind11::arg("variant"), pybind11::arg("stochastic"),
           pybind11::arg("seed"), pybind11::arg("bucket"), pybind11::arg("step"), pybind11::arg("beta"),
           pybind11::arg("first"), pybind11::arg("max_ctas"), pybind11::arg("timeout_ns"), pybind11::arg("tag"),
           pybind11::arg("topo") = std::vector<int64_t>{},
           pybind11::arg("opt_segs") = c10::optional<torch::Tensor>(), pybind11::arg("opt_nsegs") = 0,
           pybind11::arg("opt_base") = 0, pybind11::arg("opt_hyper") = std::vector<double>{})
      .def_property("epoch", &FusedComm::epoch, &FusedComm::set_epoch)
      .def_property("l2_keep_bytes", &FusedComm::l2_keep_bytes, &FusedComm::set_l2_keep_bytes);
  m.def("product_encode", &product_encode_cuda, pybind11::arg("g"), pybind11::arg("pred"), pybind11::arg("ef"),
        pybind11::arg("mode"), pybind11::arg("k"), pybind11::arg("stochastic"), pybind11::arg("seed"),
        pybind11::arg("rank"), pybind11::arg("bucket"), pybind11::arg("step"),
        pybind11::arg("topo") = std::vector<int64_t>{});
  m.def("product_reduce", &product_reduce_cuda, pybind11::arg("payloads"), pybind11::arg("n"), pybind11::arg("mode"),
        pybind11::arg("k"), pybind11::arg("pred"), pybind11::arg("beta"), pybind11::arg("first"),
        pybind11::arg("inv_world"), pybind11::arg("out_dtype"), pybind11::arg("topo") = std::vector<int64_t>{});
  m.def("payload_bytes", &payload_bytes);
  m.def("opt_seg_bytes", []() { return (int64_t)sizeof(OptSeg); });
  m.def("pipe_copy", [](torch::Tensor src, int64_t grid, torch::Tensor status, bool vec) {
    check_dev(src, "src");
    TORCH_CHECK(src.scalar_type() == torch::kFloat32, "src must be float32");
    auto dst = torch::empty_like(src);
    const c10::cuda::CUDAGuard guard(src.device());
    check_launch(launch_pipe_copy(src.data_ptr<float>(), dst.data_ptr<float>(), src.numel(), (int)grid, vec ? 1 : 0,
                                  status.data_ptr<int>(), at::cuda::getCurrentCUDAStream()),
                 "pipe_copy");
    return dst;
  });
  m.def("fused_grid", [](int64_t n, int64_t mode, bool bf16, int64_t variant, int64_t cap, int64_t device, bool opt) {
    const int nchunks = (int)nchunks_of(n);
    return fused_grid(nchunks, (int)mode, bf16 ? kBF16 : kF32, (int)variant, (int)cap, (int)device, opt ? 1 : 0);
  }, pybind11::arg("n"), pybind11::arg("mode"), pybind11::arg("bf16"), pybind11::arg("variant"), pybind11::arg("cap"),
     pybind11::arg("device"), pybind11::arg("opt") = false);
}
