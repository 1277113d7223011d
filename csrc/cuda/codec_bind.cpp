// Torch-facing side of the codec kernels (csrc/cuda/codec_kernels.cu).
// Encoders return (uint8 CUDA tensor of the exact byte stream, scale);
// decoders take a uint8 CUDA tensor and return int32 Q8.23 values.
#include <torch/extension.h>

#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>

#include <cmath>

#include "codecs.h"
#include "common/ngl_scalar.h"

namespace {
using namespace ngl::codec;

void ck(cudaError_t e, const char* what) { TORCH_CHECK(e == cudaSuccess, what, ": ", cudaGetErrorString(e)); }
cudaStream_t cur() { return at::cuda::getCurrentCUDAStream(); }
void need(const torch::Tensor& t, torch::ScalarType dt, const char* what) {
  TORCH_CHECK(t.is_cuda() && t.is_contiguous() && t.scalar_type() == dt, what, " must be a contiguous CUDA ", dt,
              " tensor");
}
torch::Tensor status_tensor(const torch::Tensor& like) {
  return torch::zeros({4}, like.options().dtype(torch::kInt32));
}
void check_status(const torch::Tensor& st, const char* what) {
  auto h = st.cpu();
  const int* p = h.data_ptr<int>();
  TORCH_CHECK(p[0] == 0, what, " failed: device status ", p[0], " (", p[1], ", ", p[2], ")");
}

// ---- Q8.23
torch::Tensor from_f32(torch::Tensor x) {
  need(x, torch::kFloat32, "x");
  c10::cuda::CUDAGuard g(x.device());
  auto q = torch::empty_like(x, x.options().dtype(torch::kInt32));
  ck(from_f32_dev(x.data_ptr<float>(), q.data_ptr<int32_t>(), x.numel(), cur()), "q823_from_f32");
  return q;
}
torch::Tensor to_f32(torch::Tensor q) {
  need(q, torch::kInt32, "q");
  c10::cuda::CUDAGuard g(q.device());
  auto x = torch::empty_like(q, q.options().dtype(torch::kFloat32));
  ck(to_f32_dev(q.data_ptr<int32_t>(), x.data_ptr<float>(), q.numel(), cur()), "q823_to_f32");
  return x;
}
torch::Tensor addsub(torch::Tensor a, torch::Tensor b, bool sub) {
  need(a, torch::kInt32, "a");
  need(b, torch::kInt32, "b");
  TORCH_CHECK(a.numel() == b.numel(), "Shape mismatch: ", a.numel(), " vs ", b.numel());
  c10::cuda::CUDAGuard g(a.device());
  auto o = torch::empty_like(a);
  ck(q823_addsub(a.data_ptr<int32_t>(), b.data_ptr<int32_t>(), o.data_ptr<int32_t>(), a.numel(), sub, cur()),
     "q823_addsub");
  return o;
}
torch::Tensor mul_scalar(torch::Tensor a, double s) {
  need(a, torch::kInt32, "a");
  c10::cuda::CUDAGuard g(a.device());
  auto o = torch::empty_like(a);
  ck(q823_mul_scalar(a.data_ptr<int32_t>(), o.data_ptr<int32_t>(), a.numel(), (float)s, cur()), "q823_mul_scalar");
  return o;
}

// ---- error-bounded codes
torch::Tensor eb_codes(torch::Tensor r, double scale) {
  need(r, torch::kInt32, "residual");
  c10::cuda::CUDAGuard g(r.device());
  auto c = torch::empty({r.numel()}, r.options().dtype(torch::kInt16));
  ck(eb_encode(r.data_ptr<int32_t>(), c.data_ptr<int16_t>(), r.numel(), (float)scale, cur()), "eb_encode");
  return c;
}
torch::Tensor eb_decode_bytes(torch::Tensor b, double scale) {
  need(b, torch::kUInt8, "bytes");
  c10::cuda::CUDAGuard g(b.device());
  const int64_t n = b.numel() / 2;
  auto even = b.narrow(0, 0, 2 * n).contiguous();
  if (reinterpret_cast<uintptr_t>(even.data_ptr()) % 2 != 0) even = even.clone();  // i16 loads need 2-byte alignment
  auto out = torch::empty({n}, b.options().dtype(torch::kInt32));
  ck(eb_decode(reinterpret_cast<const int16_t*>(even.data_ptr<uint8_t>()), out.data_ptr<int32_t>(), n, (float)scale,
               cur()),
     "eb_decode");
  return out;
}

// ---- variable-length encoders from i16 codes: kind 0 BS, 2 BSRLE, 3 RLE
torch::Tensor pack_codes(torch::Tensor codes, int64_t kind) {
  need(codes, torch::kInt16, "codes");
  c10::cuda::CUDAGuard g(codes.device());
  const int64_t n = codes.numel();
  const int64_t nblk = (n + 31) / 32;
  int64_t cap, words;
  if (kind == 0) {
    cap = 4 + nblk * 68;
    words = pack_scratch_words(n);
  } else if (kind == 2) {
    cap = 4 + nblk * 69;
    words = run_scratch_words(nblk);
  } else {
    cap = 3 * n + 1;
    words = run_scratch_words(n);
  }
  auto opt = codes.options();
  auto out = torch::empty({std::max<int64_t>(cap, 4)}, opt.dtype(torch::kUInt8));
  auto scratch = torch::empty({std::max<int64_t>(words, 1)}, opt.dtype(torch::kInt64));
  auto total = torch::zeros({1}, opt.dtype(torch::kInt64));
  auto st = status_tensor(codes);
  auto* sp = reinterpret_cast<uint64_t*>(scratch.data_ptr<int64_t>());
  auto* tp = reinterpret_cast<uint64_t*>(total.data_ptr<int64_t>());
  const int16_t* q = codes.data_ptr<int16_t>();
  if (kind == 0) ck(bs_encode(q, n, out.data_ptr<uint8_t>(), sp, tp, st.data_ptr<int>(), cur()), "bs_encode");
  else if (kind == 2) ck(bsrle_encode(q, n, out.data_ptr<uint8_t>(), sp, tp, st.data_ptr<int>(), cur()), "bsrle_encode");
  else ck(rle_encode(q, n, out.data_ptr<uint8_t>(), sp, tp, st.data_ptr<int>(), cur()), "rle_encode");
  const int64_t len = total.item<int64_t>();
  check_status(st, "encoder");
  TORCH_CHECK(len <= out.numel(), "encoder overflow");
  return out.narrow(0, 0, len);
}

// ---- stream decoders (one or many streams)
std::vector<torch::Tensor> decode_streams(torch::Tensor data, torch::Tensor stream_off, torch::Tensor scales,
                                          int64_t kind, int64_t out_cap, int64_t table_cap) {
  need(data, torch::kUInt8, "data");
  need(stream_off, torch::kInt64, "stream_off");
  need(scales, torch::kFloat32, "scales");
  c10::cuda::CUDAGuard g(data.device());
  const int64_t ns = stream_off.numel() - 1;
  TORCH_CHECK(ns >= 0 && scales.numel() >= ns, "one scale per stream");
  auto opt = data.options();
  auto out = torch::zeros({std::max<int64_t>(ns * out_cap, 1)}, opt.dtype(torch::kInt32));
  auto out_len = torch::zeros({std::max<int64_t>(ns, 1)}, opt.dtype(torch::kInt64));
  auto table = torch::empty({std::max<int64_t>(ns * (2 * table_cap + 2), 1)}, opt.dtype(torch::kInt64));
  auto st = status_tensor(data);
  torch::Tensor scratch;
  uint64_t* sp = nullptr;
  if (kind == 0 || kind == 1) {
    scratch = torch::empty({bs_decode_scratch_words(data.numel(), ns)}, opt.dtype(torch::kInt64));
    sp = reinterpret_cast<uint64_t*>(scratch.data_ptr<int64_t>());
  }
  ck(stream_decode((int)kind, data.data_ptr<uint8_t>(), stream_off.data_ptr<int64_t>(), scales.data_ptr<float>(),
                   (int)ns, out.data_ptr<int32_t>(), out_cap, out_len.data_ptr<int64_t>(), table.data_ptr<int64_t>(),
                   table_cap, st.data_ptr<int>(), sp, data.numel(), cur()),
     "stream_decode");
  check_status(st, "stream_decode");
  return {out, out_len};
}

// ---- reference stochastic codec
std::tuple<torch::Tensor, double> stochastic_q(torch::Tensor r, int64_t bits, int64_t seed, int64_t counter) {
  need(r, torch::kInt32, "residual");
  c10::cuda::CUDAGuard g(r.device());
  const int64_t n = r.numel();
  auto opt = r.options();
  if (n == 0) return {torch::empty({0}, opt.dtype(torch::kUInt8)), 1.0};
  auto mx = torch::zeros({1}, opt.dtype(torch::kInt32));
  auto sc = torch::zeros({1}, opt.dtype(torch::kFloat32));
  const int64_t nb = bits == 4 ? (n + 1) / 2 : n;
  auto out = torch::empty({nb}, opt.dtype(torch::kUInt8));
  auto* mp = reinterpret_cast<uint32_t*>(mx.data_ptr<int32_t>());
  ck(absmax_f32_of_fixed(r.data_ptr<int32_t>(), n, mp, cur()), "absmax");
  ck(stochastic_encode(r.data_ptr<int32_t>(), n, (int)bits, (uint64_t)seed, (uint64_t)counter, mp,
                       sc.data_ptr<float>(), out.data_ptr<uint8_t>(), cur()),
     "stochastic_encode");
  return {out, (double)sc.item<float>()};
}
torch::Tensor stochastic_dq(torch::Tensor b, double scale, int64_t bits) {
  need(b, torch::kUInt8, "bytes");
  c10::cuda::CUDAGuard g(b.device());
  const int64_t n = bits == 4 ? 2 * b.numel() : b.numel();
  auto out = torch::empty({n}, b.options().dtype(torch::kInt32));
  ck(stochastic_decode(b.data_ptr<uint8_t>(), b.numel(), (int)bits, (float)scale, out.data_ptr<int32_t>(), cur()),
     "stochastic_decode");
  return out;
}

// ---- reference top-k codec
std::tuple<torch::Tensor, double> topk_q(torch::Tensor r, double k_percent) {
  need(r, torch::kInt32, "residual");
  c10::cuda::CUDAGuard g(r.device());
  const int64_t n = r.numel();
  auto opt = r.options();
  if (n == 0) return {torch::empty({0}, opt.dtype(torch::kUInt8)), 1.0};
  // keep = floor((n as f32) * k) as usize (Rust f32 arithmetic)
  const float kf = std::floor((float)n * (float)k_percent);
  int64_t keep = 0;
  if (!(kf != kf) && kf > 0.0f) keep = kf >= 9.2e18f ? INT64_MAX : (int64_t)kf;
  auto mx = torch::zeros({1}, opt.dtype(torch::kInt32));
  auto thr_sc = torch::zeros({2}, opt.dtype(torch::kFloat32));
  auto hist = torch::empty({4 * 256 + 4}, opt.dtype(torch::kInt32));
  auto* mp = reinterpret_cast<uint32_t*>(mx.data_ptr<int32_t>());
  ck(absmax_f32_of_fixed(r.data_ptr<int32_t>(), n, mp, cur()), "absmax");
  ck(topk_threshold(r.data_ptr<int32_t>(), n, keep, reinterpret_cast<uint32_t*>(hist.data_ptr<int32_t>()), mp,
                    thr_sc.data_ptr<float>(), thr_sc.data_ptr<float>() + 1, cur()),
     "topk_threshold");
  const int64_t nblk = (n + 31) / 32;
  auto out = torch::empty({4 + nblk * 36}, opt.dtype(torch::kUInt8));
  auto scratch = torch::empty({pack_scratch_words(n)}, opt.dtype(torch::kInt64));
  auto total = torch::zeros({1}, opt.dtype(torch::kInt64));
  auto st = status_tensor(r);
  ck(topk_encode(r.data_ptr<int32_t>(), n, thr_sc.data_ptr<float>(), thr_sc.data_ptr<float>() + 1,
                 out.data_ptr<uint8_t>(), reinterpret_cast<uint64_t*>(scratch.data_ptr<int64_t>()),
                 reinterpret_cast<uint64_t*>(total.data_ptr<int64_t>()), st.data_ptr<int>(), cur()),
     "topk_encode");
  const int64_t len = total.item<int64_t>();
  check_status(st, "topk_encode");
  const double scale = (double)thr_sc[1].item<float>();
  return {out.narrow(0, 0, len), scale};
}
torch::Tensor topk_threshold_t(torch::Tensor r, double k_percent) {
  need(r, torch::kInt32, "residual");
  c10::cuda::CUDAGuard g(r.device());
  const int64_t n = r.numel();
  const float kf = std::floor((float)n * (float)k_percent);
  int64_t keep = (!(kf != kf) && kf > 0.0f) ? (int64_t)kf : 0;
  auto opt = r.options();
  auto mx = torch::zeros({1}, opt.dtype(torch::kInt32));
  auto thr_sc = torch::zeros({2}, opt.dtype(torch::kFloat32));
  auto hist = torch::empty({4 * 256 + 4}, opt.dtype(torch::kInt32));
  auto* mp = reinterpret_cast<uint32_t*>(mx.data_ptr<int32_t>());
  ck(absmax_f32_of_fixed(r.data_ptr<int32_t>(), n, mp, cur()), "absmax");
  ck(topk_threshold(r.data_ptr<int32_t>(), n, keep, reinterpret_cast<uint32_t*>(hist.data_ptr<int32_t>()), mp,
                    thr_sc.data_ptr<float>(), thr_sc.data_ptr<float>() + 1, cur()),
     "topk_threshold");
  return thr_sc;
}

// ---- HPC closed-loop step and add-back chain
void hpc_step_t(torch::Tensor x, torch::Tensor s_t, torch::Tensor s_tm1, int64_t hist, double scale,
                torch::Tensor codes, torch::Tensor recon, torch::Tensor maxerr_bits) {
  need(x, torch::kFloat32, "x");
  need(codes, torch::kInt16, "codes");
  need(recon, torch::kInt32, "recon");
  need(maxerr_bits, torch::kInt32, "maxerr");
  c10::cuda::CUDAGuard g(x.device());
  const int64_t n = x.numel();
  TORCH_CHECK(codes.numel() >= n && recon.numel() >= n, "output too small");
  if (hist >= 1) TORCH_CHECK(s_t.numel() == n && s_t.scalar_type() == torch::kInt32, "s_t must be int32[n]");
  if (hist >= 2) TORCH_CHECK(s_tm1.numel() == n && s_tm1.scalar_type() == torch::kInt32, "s_tm1 must be int32[n]");
  ck(hpc_step(x.data_ptr<float>(), hist >= 1 ? s_t.data_ptr<int32_t>() : nullptr,
              hist >= 2 ? s_tm1.data_ptr<int32_t>() : nullptr, (int)hist, (float)scale, codes.data_ptr<int16_t>(),
              recon.data_ptr<int32_t>(), reinterpret_cast<uint32_t*>(maxerr_bits.data_ptr<int32_t>()), n, cur()),
     "hpc_step");
}
void linear_addback_t(torch::Tensor res, int64_t particles, int64_t steps) {
  need(res, torch::kInt32, "res");
  TORCH_CHECK(res.numel() >= particles * steps, "res too small");
  c10::cuda::CUDAGuard g(res.device());
  ck(linear_addback(res.data_ptr<int32_t>(), particles, steps, cur()), "linear_addback");
}

// ---- .nz pipelines: all steps on the device, one host sync at the end
// Encode T snapshots (x: [T, P] fp32) with the LinearPredictor closed loop.
// codec: 1 EB, 2 EB+RLE, 3 EB+BlockSparse, 4 EB+BlockSparse+RLE.
// Returns (payloads [T, cap] u8, lengths [T] i64, maxerr f32 scalar tensor).
std::vector<torch::Tensor> nz_encode_steps(torch::Tensor x, int64_t codec, double eps) {
  need(x, torch::kFloat32, "snapshots");
  TORCH_CHECK(x.dim() == 2, "snapshots must be [steps, particles]");
  TORCH_CHECK(codec >= 1 && codec <= 4, "codec must be 1..4");
  c10::cuda::CUDAGuard g(x.device());
  const int64_t T = x.size(0), P = x.size(1);
  const float scale = 2.0f * (float)eps;
  const int64_t nblk = (P + 31) / 32;
  const int64_t cap = codec == 1 ? 2 * P : codec == 2 ? 3 * P + 1 : codec == 3 ? 4 + nblk * 68 : 4 + nblk * 69;
  const int64_t capA = (std::max<int64_t>(cap, 4) + 15) / 16 * 16;
  auto opt = x.options();
  auto maxerr = torch::zeros({1}, opt.dtype(torch::kInt32));
  auto st = status_tensor(x);
  cudaStream_t s = cur();
  // Closed loop of every element over all steps in one kernel.  EB payloads
  // are the codes themselves (row t of [T, P] i16 = 2P bytes); the packers
  // encode every step's codes.
  auto all_codes = torch::empty({T, P}, opt.dtype(torch::kInt16));
  ck(hpc_encode_all(x.data_ptr<float>(), all_codes.data_ptr<int16_t>(),
                    reinterpret_cast<uint32_t*>(maxerr.data_ptr<int32_t>()), P, T, scale, s),
     "hpc_encode_all");
  auto mx = maxerr.view(torch::kFloat32);
  if (codec == 1) {
    auto lens = torch::full({T}, 2 * P, opt.dtype(torch::kInt64));
    return {all_codes.view(torch::kUInt8).view({T, 2 * P}), lens, mx, st};
  }
  auto payload = torch::empty({T, capA}, opt.dtype(torch::kUInt8));
  auto lens = torch::zeros({T}, opt.dtype(torch::kInt64));
  auto* lp = reinterpret_cast<uint64_t*>(lens.data_ptr<int64_t>());
  if (codec == 3) {
    // All steps in one launch (tile ranges and look-back status per step).
    auto scratch = torch::empty({pack_scratch_words(P, T)}, opt.dtype(torch::kInt64));
    ck(bs_encode_batch(all_codes.data_ptr<int16_t>(), P, (int)T, payload.data_ptr<uint8_t>(), capA,
                       reinterpret_cast<uint64_t*>(scratch.data_ptr<int64_t>()), lp, st.data_ptr<int>(), s),
       "bs_encode_batch");
    return {payload, lens, mx, st};
  }
  const int64_t items = codec == 4 ? nblk : P;
  auto scratch = torch::empty({run_scratch_words(items, T)}, opt.dtype(torch::kInt64));
  auto* sp = reinterpret_cast<uint64_t*>(scratch.data_ptr<int64_t>());
  if (codec == 2) {
    ck(rle_encode_batch(all_codes.data_ptr<int16_t>(), P, (int)T, payload.data_ptr<uint8_t>(), capA, sp, lp,
                        st.data_ptr<int>(), s),
       "rle_encode_batch");
  } else {
    ck(bsrle_encode_batch(all_codes.data_ptr<int16_t>(), P, (int)T, payload.data_ptr<uint8_t>(), capA, sp, lp,
                          st.data_ptr<int>(), s),
       "bsrle_encode_batch");
  }
  return {payload, lens, mx, st};
}

// Decode T step payloads (concatenated, offsets [T+1]) back to values with
// the LinearPredictor add-back.  Returns fp32 [T, P].
torch::Tensor nz_decode_steps(torch::Tensor data, torch::Tensor offsets, torch::Tensor scales, int64_t codec,
                              int64_t P) {
  need(data, torch::kUInt8, "data");
  need(offsets, torch::kInt64, "offsets");
  need(scales, torch::kFloat32, "scales");
  c10::cuda::CUDAGuard g(data.device());
  const int64_t T = offsets.numel() - 1;
  auto opt = data.options();
  torch::Tensor res;
  if (codec == 1) {
    // EB payloads: 2P bytes each (shorter, truncated ones decode to fewer
    // values followed by zeros); gather them into [T, P] codes, then decode
    // and add back in one kernel.
    auto offs_h = offsets.cpu();
    const int64_t* oh = offs_h.data_ptr<int64_t>();
    bool dense = true;
    for (int64_t t = 0; t < T && dense; ++t) dense = (oh[t + 1] - oh[t] == 2 * P) && (oh[t] % 2 == 0);
    torch::Tensor codes;
    if (dense && oh[0] == 0) {
      codes = data.narrow(0, 0, 2 * P * T).view(torch::kInt16).view({T, P});
    } else {
      codes = torch::zeros({T, P}, opt.dtype(torch::kInt16));
      for (int64_t t = 0; t < T; ++t) {
        const int64_t nb = std::min<int64_t>((oh[t + 1] - oh[t]) / 2, P) * 2;
        if (nb > 0)
          ck(cudaMemcpyAsync(codes[t].data_ptr<int16_t>(), data.data_ptr<uint8_t>() + oh[t], nb,
                             cudaMemcpyDeviceToDevice, cur()),
             "gather codes");
      }
    }
    // decode + add-back + fp32 conversion in one pass over [T, P]
    auto outf = torch::empty({T, P}, opt.dtype(torch::kFloat32));
    ck(eb_decode_all(codes.data_ptr<int16_t>(), nullptr, P, T, scales.data_ptr<float>(), cur(),
                     outf.data_ptr<float>()),
       "eb_decode_all");
    return outf;
  } else {
    const int kind = codec == 2 ? 3 : codec == 3 ? 0 : 2;
    const int64_t nblk = (P + 31) / 32;
    int64_t tcap = kind == 3 ? (data.numel() / std::max<int64_t>(T, 1) + 2) : nblk;
    if (kind == 3) {
      auto offs_h = offsets.cpu();
      int64_t mx = 1;
      for (int64_t t = 0; t < T; ++t)
        mx = std::max(mx, offs_h.data_ptr<int64_t>()[t + 1] - offs_h.data_ptr<int64_t>()[t]);
      tcap = mx;
    }
    auto r = decode_streams(data, offsets, scales, kind, P, tcap);
    res = r[0].view({T, P});
  }
  // add-back + fp32 conversion in one pass
  auto outf = torch::empty({T, P}, opt.dtype(torch::kFloat32));
  ck(linear_addback(res.data_ptr<int32_t>(), P, T, cur(), outf.data_ptr<float>()), "linear_addback");
  return outf;
}

}  // namespace

void register_codecs(pybind11::module& m) {
  m.def("nz_encode_steps", &nz_encode_steps);
  m.def("nz_decode_steps", &nz_decode_steps);
  m.def("q823_from_f32", &from_f32);
  m.def("q823_to_f32", &to_f32);
  m.def("q823_addsub", &addsub);
  m.def("q823_mul_scalar", &mul_scalar);
  m.def("eb_codes", &eb_codes);
  m.def("eb_decode", &eb_decode_bytes);
  m.def("pack_codes", &pack_codes);
  m.def("decode_streams", &decode_streams);
  m.def("stochastic_quantize", &stochastic_q);
  m.def("stochastic_dequantize", &stochastic_dq);
  m.def("topk_quantize", &topk_q);
  m.def("topk_threshold", &topk_threshold_t);
  m.def("hpc_step", &hpc_step_t);
  m.def("linear_addback", &linear_addback_t);
}
