// Native host library: bit-exact C++17 restatement of the reference's Rust
// crates (nangila-math, nangila-core, nangila-ai, nangila-hpc, nangila-twin,
// the NZCP container of examples/lammps_compress) plus the host oracle of the
// product wire format used by the fused GPU all-reduce.
//
// It is the CPU test oracle for every kernel, the CPU baseline the benches
// time (the codecs and the .nz pipeline run on one thread, as the reference's
// binaries; the product-format oracle, which also carries the CPU DDP hook,
// splits its block loops over NGL_HOST_THREADS / OMP_NUM_THREADS threads with
// results that do not depend on the count), and the reader/writer of the
// on-disk formats.
#pragma once
#include <cstddef>
#include <cstdint>
#include <stdexcept>
#include <string>
#include <vector>

namespace ngl {
namespace host {

using Bytes = std::vector<uint8_t>;
using Fixed = std::vector<int32_t>;
using Floats = std::vector<float>;

struct ShapeMismatch : std::runtime_error {
  size_t a, b;
  ShapeMismatch(size_t a_, size_t b_)
      : std::runtime_error("Shape mismatch: " + std::to_string(a_) + " vs " + std::to_string(b_)), a(a_), b(b_) {}
};

// ---- nangila-math (fixed_point.rs, ops.rs) and nangila-edge (lib.rs) ----
Fixed q823_from_f32(const float* x, size_t n);
Floats q823_to_f32(const int32_t* q, size_t n);
Fixed q823_add(const int32_t* a, size_t na, const int32_t* b, size_t nb);
Fixed q823_sub(const int32_t* a, size_t na, const int32_t* b, size_t nb);
Fixed q823_mul_scalar(const int32_t* a, size_t n, float s);
// state.mul_scalar(beta).add(obs.mul_scalar(one_minus_beta)) in one pass.
Fixed q823_momentum_update(const int32_t* state, const int32_t* obs, size_t n, float beta, float one_minus_beta);
Fixed fixedq_from_f32(const float* x, size_t n);
Floats fixedq_to_f32(const int32_t* q, size_t n);

// ---- nangila-core UnifiedQuantizer (unified_quantizer.rs) ----
struct QuantOut {
  Bytes bytes;
  float scale;
};
// Stochastic INT4/INT8; `counter` is the persistent PRNG counter, advanced by
// one per element quantized with the hash PRNG.
QuantOut stochastic_quantize(const int32_t* r, size_t n, int bits, uint64_t seed, uint64_t* counter);
Fixed stochastic_dequantize(const uint8_t* b, size_t nb, float scale, int bits);
QuantOut unified_eb_quantize(const int32_t* r, size_t n, float eps);
Fixed unified_eb_dequantize(const uint8_t* b, size_t nb, float scale);
QuantOut topk_quantize(const int32_t* r, size_t n, float k_percent);
Fixed topk_dequantize(const uint8_t* b, size_t nb, float scale);
// Threshold that quantize_topk keeps (|x| >= threshold), for tests.
float topk_threshold(const float* x, size_t n, float k_percent);

// ---- nangila-hpc ----
QuantOut eb_quantize(const int32_t* r, size_t n, float eps);     // error_bounded.rs
Fixed eb_dequantize(const uint8_t* b, size_t nb, float scale);
QuantOut rle_quantize(const int32_t* r, size_t n, float eps);    // rle.rs
Fixed rle_dequantize(const uint8_t* b, size_t nb, float scale);
QuantOut bs_quantize(const int32_t* r, size_t n, float eps);     // block_sparse.rs
Fixed bs_dequantize(const uint8_t* b, size_t nb, float scale);
QuantOut bsrle_quantize(const int32_t* r, size_t n, float eps);  // block_sparse_rle.rs
Fixed bsrle_dequantize(const uint8_t* b, size_t nb, float scale);
// Byte streams of already computed error-bounded i16 codes (what the EB,
// BlockSparse and BlockSparse+RLE quantizers emit for those codes).
Bytes eb_pack_codes(const int16_t* q, size_t n);
Bytes bs_pack_codes(const int16_t* q, size_t n);
Bytes bsrle_pack_codes(const int16_t* q, size_t n);
// Raw i16 element RLE used by the rotor twin's top-k path (client.rs:41-66).
Bytes rle_encode_i16(const int16_t* q, size_t n);
std::vector<int16_t> rle_decode_i16(const uint8_t* b, size_t nb);

// ---- Predictors (momentum.rs, linear.rs) ----
class MomentumPredictor {
 public:
  explicit MomentumPredictor(float beta) : beta_(beta) {}
  Fixed predict() const { return has_ ? state_ : Fixed(); }
  void update(const int32_t* obs, size_t n);
  void reset() { has_ = false; state_.clear(); }
  bool has_state() const { return has_; }
  float beta() const { return beta_; }
  const Fixed& state() const { return state_; }
  void set_state(const Fixed& s, bool has) { state_ = s; has_ = has; }

 private:
  float beta_;
  bool has_ = false;
  Fixed state_;
};

class LinearPredictor {
 public:
  Fixed predict() const;
  void update(const int32_t* obs, size_t n);
  void reset() { n_hist_ = 0; s_t_.clear(); s_tm1_.clear(); }
  int history() const { return n_hist_; }
  const Fixed& s_t() const { return s_t_; }
  const Fixed& s_tm1() const { return s_tm1_; }
  void set_history(const Fixed& st, const Fixed& stm1, int n) { s_t_ = st; s_tm1_ = stm1; n_hist_ = n; }

 private:
  int n_hist_ = 0;  // 0, 1 or 2 snapshots held
  Fixed s_t_, s_tm1_;
};

// ---- TopologyMask (topology.rs) ----
struct TopologyMask {
  std::vector<uint64_t> driver_indices;
  std::vector<uint64_t> passenger_indices;
  float threshold = 0.0f;
  uint64_t total_layers = 0;

  static TopologyMask from_variance_threshold(const float* v, size_t n, float drop_percent);
  static TopologyMask all_drivers(uint64_t n);
  bool is_driver(uint64_t i) const;
  bool is_passenger(uint64_t i) const;
  float compression_factor() const;
  float passenger_percentage() const;
  Bytes to_bytes() const;                      // bincode 1.3 default layout
  static TopologyMask from_bytes(const uint8_t* b, size_t n);  // throws on malformed input
};

// ---- NZCP container (examples/lammps_compress/src/main.rs:90-127) ----
enum NzCodec : uint8_t { kNzEB = 1, kNzRLE = 2, kNzBS = 3, kNzBSRLE = 4 };
struct NzStats {
  size_t total_raw = 0;
  size_t total_comp = 0;
  float max_abs_err = 0.0f;
};
// Closed-loop LinearPredictor compression of `steps` snapshots of
// `particles` floats each into an in-memory .nz image.
Bytes nz_compress(const float* data, size_t particles, size_t steps, int codec, float eps, NzStats* stats);
struct NzHeader {
  uint8_t version = 1;
  uint8_t codec = 1;
  uint32_t particles = 0;
  uint32_t steps = 0;
};
NzHeader nz_read_header(const uint8_t* b, size_t n);
// Decode every step.  add_back=false returns the residual stream exactly as
// the reference's read_and_decompress does (main.rs:249-309); add_back=true
// runs the LinearPredictor closed loop and returns the reconstructed values.
Floats nz_decompress(const uint8_t* b, size_t n, bool add_back);

// Synthetic LAMMPS-like generator of the reference (main.rs:311-322).
Floats lammps_generate_synthetic(size_t particles, size_t steps);

// LAMMPS ASCII dump I/O (main.rs:324-419): one flattened [x0, y0, z0, x1, ...]
// snapshot per ITEM: TIMESTEP block; std::runtime_error with the reference's
// messages on malformed input.  The writer emits the reference's synthetic
// dump (cos/sin/cos(0.5) of phase 0.1 t + 0.001 i, six decimals).
std::vector<Floats> lammps_read_dump(const std::string& path);
std::vector<Floats> lammps_read_dump_text(const char* text, size_t size);
void lammps_write_dump(const std::string& path, size_t atoms, size_t steps);

// ---- Product wire format (fused GPU all-reduce oracle) ----
struct ProductParams {
  int bits = 4;            // 4 or 8
  bool stochastic = true;
  bool error_feedback = true;
  uint64_t seed = 0;
  uint32_t rank = 0;
  uint32_t bucket = 0;
  uint64_t step = 0;
  // static topology drop (topo_passenger); ndrop = 0 keeps every chunk
  uint64_t topo_a = 0, topo_b = 0;
  int64_t topo_ndrop = 0;
};
// Topology drop parameters of a bucket of nchunks chunk records: exactly
// nchunks - max(1, floor(nchunks * (1 - drop))) chunks become passengers,
// spread by a keyed permutation of (seed, stream).
struct TopoChunks {
  uint64_t a = 1, b = 0;
  int64_t ndrop = 0;
};
TopoChunks product_topology(size_t nchunks, double drop, uint64_t seed, uint64_t stream);
// Encode one rank's residual c = g - pred + e into the chunked wire payload
// (product_wire_bytes bytes); writes the new error feedback when e_out is set.
size_t product_wire_bytes(size_t n, int mode, int k);
void product_encode(const float* g, const float* pred, const float* e_in, size_t n, const ProductParams& p,
                    uint8_t* wire, float* e_out);
// Rank-ordered reduction of W payloads: avg = pred + (sum_r q_r s_r) / W.
void product_reduce(const uint8_t* const* wires, int world, size_t n, int bits, const float* pred, float inv_world,
                    float* avg_out);
// Two-shot: the mean residual re-encoded as INT8 per block, then decoded.
void product_reduce_twoshot(const uint8_t* const* wires, int world, size_t n, int bits, const float* pred,
                            float inv_world, float* avg_out);
// EMA predictor update; `first` copies avg into the state.
void product_ema(float* state, const float* avg, size_t n, float beta, bool first);
// Per-256-block top-k: fixed-size records (scale, ascending indices, int8
// values), 8 per chunk; decode-sum in rank order.
void product_topk_encode(const float* g, const float* pred, const float* e_in, size_t n, int k, bool ef,
                         uint8_t* records, float* e_out, const TopoChunks& topo = TopoChunks());
void product_topk_reduce(const uint8_t* const* records, int world, size_t n, int k, const float* pred,
                         float inv_world, float* avg_out);

}  // namespace host
}  // namespace ngl
