// Launch API of the sm_100a codec kernels (csrc/cuda/codec_kernels.cu):
// Q8.23 elementwise math, the fused HPC closed-loop step, the error-bounded,
// BlockSparse, BlockSparse+RLE and RLE encoders/decoders, the reference's
// stochastic INT4/INT8 codec and its top-k codec with a radix-select
// threshold.  Every byte stream is identical to the host library's.
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>

namespace ngl {
namespace codec {

constexpr int kPackThreads = 256;
constexpr int kPackBlocksPerWarp = 64;                            // 32-element blocks per warp per tile
constexpr int kPackTileBlocks = (kPackThreads / 32) * kPackBlocksPerWarp;  // 512 blocks = 16384 elements
constexpr int kRunTileItems = 4096;                               // items per tile of the run-length encoders

// Scratch words needed by the look-back encoders for n elements.
int64_t pack_scratch_words(int64_t n, int64_t nstreams = 1);
int64_t run_scratch_words(int64_t items, int64_t nstreams = 1);

// ---- Q8.23 (K2) ----
cudaError_t from_f32_dev(const float* x, int32_t* q, int64_t n, cudaStream_t s);
cudaError_t to_f32_dev(const int32_t* q, float* x, int64_t n, cudaStream_t s);
cudaError_t q823_addsub(const int32_t* a, const int32_t* b, int32_t* out, int64_t n, bool sub, cudaStream_t s);
cudaError_t q823_mul_scalar(const int32_t* a, int32_t* out, int64_t n, float scalar, cudaStream_t s);

// ---- Error-bounded INT16 (K3) ----
// codes[i] = round(to_f32(r[i]) / scale) clamped to i16.
cudaError_t eb_encode(const int32_t* r, int16_t* codes, int64_t n, float scale, cudaStream_t s);
// out[i] = from_f32(codes[i] * scale)
cudaError_t eb_decode(const int16_t* codes, int32_t* out, int64_t n, float scale, cudaStream_t s);
// Fused closed-loop step of the LinearPredictor + EB codec for one snapshot:
// x -> Q8.23; pred = hist>=2 ? s_t + (s_t - s_tm1) : hist==1 ? s_t : none;
// r = x - pred; codes = EB(r); recon = pred + from_f32(codes * scale);
// maxerr (float bits, atomicMax) = max |to_f32(x) - to_f32(recon)|.
cudaError_t hpc_step(const float* x, const int32_t* s_t, const int32_t* s_tm1, int hist, float scale, int16_t* codes,
                     int32_t* recon, uint32_t* maxerr_bits, int64_t n, cudaStream_t s);
// Whole trajectory at once (all T snapshots of P values): the closed loop
// of every element runs its T steps with the predictor history in
// registers; codes [T, P].  Identical codes to T calls of hpc_step.
cudaError_t hpc_encode_all(const float* x, int16_t* codes, uint32_t* maxerr_bits, int64_t P, int64_t T, float scale,
                           cudaStream_t s);
// EB decode of codes [T, P] with the add-back chain -> Q8.23 values [T, P]
// in `out`, or (f32out != nullptr) their fp32 conversions in f32out.
cudaError_t eb_decode_all(const int16_t* codes, int32_t* out, int64_t P, int64_t T, const float* scales,
                          cudaStream_t s, float* f32out = nullptr);
// Linear predictor add-back over T decoded residual snapshots:
// recon_t = pred_t + res_t with the predictor's history chain, in place, or
// (f32out != nullptr) as fp32 values in f32out.
cudaError_t linear_addback(int32_t* res, int64_t particles, int64_t steps, cudaStream_t s, float* f32out = nullptr);

// ---- Mask packers (BlockSparse, top-k compat) with decoupled look-back ----
// BlockSparse from i16 codes: [u32 n] then per 32-block [u32 mask][i16 per
// set bit].  Top-k compat from Q8.23 residuals: [u32 n] then per 32-block
// [u32 mask][i8 per kept], kept iff |x| >= *threshold, value
// round(x / *scale) clamped to i8.
// scratch: pack_scratch_words(n) u64 words; total_bytes: one u64.
cudaError_t bs_encode(const int16_t* q, int64_t n, uint8_t* out, uint64_t* scratch, uint64_t* total_bytes,
                      int* status, cudaStream_t s);
cudaError_t topk_encode(const int32_t* r, int64_t n, const float* threshold, const float* scale, uint8_t* out,
                        uint64_t* scratch, uint64_t* total_bytes, int* status, cudaStream_t s);
// BlockSparse over `ns` streams of n codes (stream i at q + i * n) in one
// launch; stream i's bytes at out + i * out_stride, length totals[i].
// scratch: pack_scratch_words(n, ns) words.
cudaError_t bs_encode_batch(const int16_t* q, int64_t n, int ns, uint8_t* out, int64_t out_stride, uint64_t* scratch,
                            uint64_t* totals, int* status, cudaStream_t s);

// ---- Run-length encoders from i16 codes ----
// BlockSparse+RLE ([u32 n], opcode runs over 32-blocks) and element RLE
// (opcode runs over codes, no header).  scratch: run_scratch_words(items).
cudaError_t bsrle_encode(const int16_t* q, int64_t n, uint8_t* out, uint64_t* scratch, uint64_t* total_bytes,
                         int* status, cudaStream_t s);
cudaError_t rle_encode(const int16_t* q, int64_t n, uint8_t* out, uint64_t* scratch, uint64_t* total_bytes,
                       int* status, cudaStream_t s);
// Both over `ns` streams of n codes in one launch sequence (stream i at
// q + i * n, bytes at out + i * out_stride, length totals[i]); scratch:
// run_scratch_words(items per stream, ns).
cudaError_t bsrle_encode_batch(const int16_t* q, int64_t n, int ns, uint8_t* out, int64_t out_stride,
                               uint64_t* scratch, uint64_t* totals, int* status, cudaStream_t s);
cudaError_t rle_encode_batch(const int16_t* q, int64_t n, int ns, uint8_t* out, int64_t out_stride,
                             uint64_t* scratch, uint64_t* totals, int* status, cudaStream_t s);

// ---- Stream decoders: header walk + parallel expansion ----
// kind: 0 = BlockSparse (i16), 1 = top-k compat (i8), 2 = BlockSparse+RLE, 3 = RLE.
// Stream i is data[stream_off[i] .. stream_off[i+1]) with scale scales[i];
// it decodes into out[i * out_cap ...] (Q8.23) and out_len[i] receives the
// decoded length the reference's decoder produces (status kBounds when that
// exceeds out_cap, or a stream needs more than table_cap descriptors).
// table: nstreams * (2 * table_cap + 2) int64 words (count + descriptors).
// scratch (kinds 0 and 1): bs_decode_scratch_words(total_bytes, nstreams)
// u64 words, total_bytes = data bytes covered by all streams; with scratch
// those kinds decode window-parallel, without it by the one-thread walk.
int64_t bs_decode_scratch_words(int64_t total_bytes, int64_t nstreams);
cudaError_t stream_decode(int kind, const uint8_t* data, const int64_t* stream_off, const float* scales, int nstreams,
                          int32_t* out, int64_t out_cap, int64_t* out_len, int64_t* table, int64_t table_cap,
                          int* status, uint64_t* scratch, int64_t total_bytes, cudaStream_t s);

// ---- Reference stochastic INT4/INT8 codec (K7) ----
cudaError_t absmax_f32_of_fixed(const int32_t* r, int64_t n, uint32_t* max_bits, cudaStream_t s);
cudaError_t stochastic_encode(const int32_t* r, int64_t n, int bits, uint64_t seed, uint64_t counter,
                              const uint32_t* max_bits, float* scale_out, uint8_t* out, cudaStream_t s);
cudaError_t stochastic_decode(const uint8_t* b, int64_t nbytes, int bits, float scale, int32_t* out,
                              cudaStream_t s);

// ---- Top-k compat threshold by radix select (K8) ----
// Finds the value at ascending rank (n - keep) of |to_f32(r)| with four 8-bit
// radix passes; writes max(value, 1e-9) to *threshold (1e-9 when keep == 0)
// and max|x|/127 (or 1) to *scale.  hist: 4 x 256 u32 + 4 words scratch.
cudaError_t topk_threshold(const int32_t* r, int64_t n, int64_t keep, uint32_t* hist, const uint32_t* max_bits,
                           float* threshold, float* scale, cudaStream_t s);

}  // namespace codec
}  // namespace ngl
