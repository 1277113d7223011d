// Predictors, TopologyMask and the NZCP container of the host library.
#include <algorithm>
#include <cmath>
#include <cstring>

#include "../common/ngl_scalar.h"
#include "nangila_host.hpp"
#include "fast_scalar.h"

namespace ngl {
namespace host {

namespace {
inline void put_u32(Bytes& b, uint32_t v) {
  for (int i = 0; i < 4; ++i) b.push_back((uint8_t)(v >> (8 * i)));
}
inline void put_u64(Bytes& b, uint64_t v) {
  for (int i = 0; i < 8; ++i) b.push_back((uint8_t)(v >> (8 * i)));
}
inline void put_f32(Bytes& b, float f) {
  uint32_t u;
  std::memcpy(&u, &f, 4);
  put_u32(b, u);
}
inline uint32_t get_u32(const uint8_t* p) {
  return (uint32_t)p[0] | ((uint32_t)p[1] << 8) | ((uint32_t)p[2] << 16) | ((uint32_t)p[3] << 24);
}
inline uint64_t get_u64(const uint8_t* p) { return (uint64_t)get_u32(p) | ((uint64_t)get_u32(p + 4) << 32); }
inline float get_f32(const uint8_t* p) {
  uint32_t u = get_u32(p);
  float f;
  std::memcpy(&f, &u, 4);
  return f;
}
}  // namespace

// ------------------------------------------------ MomentumPredictor (momentum.rs)
void MomentumPredictor::update(const int32_t* obs, size_t n) {
  if (!has_) {
    state_.assign(obs, obs + n);
    has_ = true;
    return;
  }
  Fixed decayed = q823_mul_scalar(state_.data(), state_.size(), beta_);
  Fixed scaled = q823_mul_scalar(obs, n, 1.0f - beta_);
  state_ = q823_add(decayed.data(), decayed.size(), scaled.data(), scaled.size());
}

// -------------------------------------------------- LinearPredictor (linear.rs)
Fixed LinearPredictor::predict() const {
  if (n_hist_ >= 2) {
    Fixed diff = q823_sub(s_t_.data(), s_t_.size(), s_tm1_.data(), s_tm1_.size());
    return q823_add(s_t_.data(), s_t_.size(), diff.data(), diff.size());
  }
  if (n_hist_ == 1) return s_t_;
  return Fixed();
}
void LinearPredictor::update(const int32_t* obs, size_t n) {
  if (n_hist_ >= 1) s_tm1_.swap(s_t_);
  s_t_.assign(obs, obs + n);
  n_hist_ = std::min(n_hist_ + 1, 2);
}

// ----------------------------------------------------- TopologyMask (topology.rs)
TopologyMask TopologyMask::from_variance_threshold(const float* v, size_t n, float drop_percent) {
  TopologyMask m;
  if (n == 0) return m;
  // f32::clamp(0.0, 1.0); NaN stays NaN
  float drop = drop_percent;
  if (!is_nan(drop)) drop = std::min(std::max(drop, 0.0f), 1.0f);
  std::vector<std::pair<uint64_t, float>> iv(n);
  for (size_t i = 0; i < n; ++i) iv[i] = {i, v[i]};
  // Stable sort, variance descending; NaN compares Equal.
  std::stable_sort(iv.begin(), iv.end(), [](const auto& a, const auto& b) { return a.second > b.second; });
  float nd = std::ceil((float)n * (1.0f - drop));
  size_t num_drivers = 0;
  if (!is_nan(nd) && nd > 0.0f) num_drivers = (size_t)nd;
  num_drivers = std::min(std::max<size_t>(num_drivers, 1), n);
  for (size_t i = 0; i < num_drivers; ++i) m.driver_indices.push_back(iv[i].first);
  for (size_t i = num_drivers; i < n; ++i) m.passenger_indices.push_back(iv[i].first);
  std::sort(m.driver_indices.begin(), m.driver_indices.end());
  std::sort(m.passenger_indices.begin(), m.passenger_indices.end());
  m.threshold = num_drivers < n ? iv[num_drivers - 1].second : 0.0f;
  m.total_layers = n;
  return m;
}
TopologyMask TopologyMask::all_drivers(uint64_t n) {
  TopologyMask m;
  for (uint64_t i = 0; i < n; ++i) m.driver_indices.push_back(i);
  m.total_layers = n;
  return m;
}
bool TopologyMask::is_driver(uint64_t i) const {
  return std::binary_search(driver_indices.begin(), driver_indices.end(), i);
}
bool TopologyMask::is_passenger(uint64_t i) const {
  return std::binary_search(passenger_indices.begin(), passenger_indices.end(), i);
}
float TopologyMask::compression_factor() const {
  if (driver_indices.empty()) return 1.0f;
  return (float)total_layers / (float)driver_indices.size();
}
float TopologyMask::passenger_percentage() const {
  if (total_layers == 0) return 0.0f;
  return ((float)passenger_indices.size() / (float)total_layers) * 100.0f;
}
// bincode 1.3 default options: fixed-width little-endian integers, u64 lengths
// and usize as u64, fields in declaration order (topology.rs:12-24).
Bytes TopologyMask::to_bytes() const {
  Bytes b;
  b.reserve(28 + 8 * (driver_indices.size() + passenger_indices.size()));
  put_u64(b, driver_indices.size());
  for (uint64_t x : driver_indices) put_u64(b, x);
  put_u64(b, passenger_indices.size());
  for (uint64_t x : passenger_indices) put_u64(b, x);
  put_f32(b, threshold);
  put_u64(b, total_layers);
  return b;
}
TopologyMask TopologyMask::from_bytes(const uint8_t* p, size_t n) {
  TopologyMask m;
  size_t off = 0;
  auto need = [&](size_t k) {
    if (off + k > n) throw std::runtime_error("Deserialization error: io error: unexpected end of file");
  };
  auto read_vec = [&](std::vector<uint64_t>& out) {
    need(8);
    uint64_t len = get_u64(p + off);
    off += 8;
    if (len > (n - off) / 8) throw std::runtime_error("Deserialization error: io error: unexpected end of file");
    out.resize(len);
    for (uint64_t i = 0; i < len; ++i) {
      out[i] = get_u64(p + off);
      off += 8;
    }
  };
  read_vec(m.driver_indices);
  read_vec(m.passenger_indices);
  need(4);
  m.threshold = get_f32(p + off);
  off += 4;
  need(8);
  m.total_layers = get_u64(p + off);
  return m;
}

// -------------------------------------------------- NZCP container (.nz files)
namespace {
Fixed nz_dequantize(int codec, const uint8_t* b, size_t n, float scale) {
  switch (codec) {
    case kNzEB: return eb_dequantize(b, n, scale);
    case kNzRLE: return rle_dequantize(b, n, scale);
    case kNzBS: return bs_dequantize(b, n, scale);
    case kNzBSRLE: return bsrle_dequantize(b, n, scale);
  }
  throw std::runtime_error("unknown codec " + std::to_string(codec));
}
}  // namespace

namespace detail {
// One closed-loop step of the LinearPredictor + error-bounded codes for n
// values x (hist = snapshots in the predictor's history): the codes, the
// reconstruction (the new history), and the largest |x - recon| as float
// bits.  Every codec's decoder returns code * scale for each element, so the
// reconstruction comes from the codes without decoding the step's bytes.
// Written out so it vectorizes; only exact operations, and the error maximum
// is an integer max of the bit patterns of non-negative floats, which does
// not depend on the order.
NGL_HOST_VEC_CLONES
uint32_t hpc_step(const float* x, const int32_t* s_t, const int32_t* s_tm1, int hist, float scale, size_t n,
                  int16_t* codes, int32_t* recon) {
  uint32_t maxbits = 0;
  for (size_t i = 0; i < n; ++i) {
    const int32_t q = fast::q823_from_f32(x[i]);
    const int32_t p = hist >= 2 ? sat_add_i32(s_t[i], sat_sub_i32(s_t[i], s_tm1[i])) : (hist == 1 ? s_t[i] : 0);
    const int32_t r = hist >= 1 ? sat_sub_i32(q, p) : q;
    const int16_t c = fast::eb_code_bf(fast::q823_to_f32(r), scale);
    const int32_t d = fast::q823_from_f32((float)c * scale);
    const int32_t rc = hist >= 1 ? sat_add_i32(p, d) : d;
    codes[i] = c;
    recon[i] = rc;
    const float e = std::fabs(fast::q823_to_f32(q) - fast::q823_to_f32(rc));
    uint32_t eb;
    std::memcpy(&eb, &e, 4);
    maxbits = eb > maxbits ? eb : maxbits;
  }
  return maxbits;
}
}  // namespace detail

// examples/lammps_compress/src/main.rs:87-236: per step the LinearPredictor
// prediction, the residual's error-bounded codes in the chosen container,
// the reconstruction as the next history entry.
Bytes nz_compress(const float* data, size_t particles, size_t steps, int codec, float eps, NzStats* stats) {
  if (codec < 1 || codec > 4) throw std::runtime_error("unknown codec " + std::to_string(codec));
  Bytes out;
  out.insert(out.end(), {'N', 'Z', 'C', 'P'});
  out.push_back(1);
  out.push_back((uint8_t)codec);
  put_u32(out, (uint32_t)particles);
  put_u32(out, (uint32_t)steps);
  NzStats st;
  const float scale = 2.0f * eps;
  // the RLE quantizer reports scale 1.0 for an empty input (rle.rs)
  const float file_scale = (codec == kNzRLE && particles == 0) ? 1.0f : scale;
  std::vector<int16_t> codes(particles);
  Fixed hist_a(particles), hist_b(particles), hist_c(particles);
  Fixed *s_t = &hist_a, *s_tm1 = &hist_b, *next = &hist_c;
  int hist = 0;
  uint32_t maxbits = 0;
  for (size_t t = 0; t < steps; ++t) {
    st.total_raw += particles * 4;
    const uint32_t mb = detail::hpc_step(data + t * particles, s_t->data(), s_tm1->data(), hist, scale, particles,
                                         codes.data(), next->data());
    maxbits = std::max(maxbits, mb);
    Bytes q;
    switch (codec) {
      case kNzEB: q = eb_pack_codes(codes.data(), particles); break;
      case kNzRLE: q = rle_encode_i16(codes.data(), particles); break;
      case kNzBS: q = bs_pack_codes(codes.data(), particles); break;
      default: q = bsrle_pack_codes(codes.data(), particles); break;
    }
    st.total_comp += q.size() + 8;
    // history: s_{t-1} <- s_t, s_t <- recon
    Fixed* old = s_tm1;
    s_tm1 = s_t;
    s_t = next;
    next = old;
    hist = std::min(hist + 1, 2);
    put_f32(out, file_scale);
    put_u32(out, (uint32_t)q.size());
    out.insert(out.end(), q.begin(), q.end());
  }
  std::memcpy(&st.max_abs_err, &maxbits, 4);
  if (stats) *stats = st;
  return out;
}

NzHeader nz_read_header(const uint8_t* b, size_t n) {
  if (n < 4) throw std::runtime_error("read magic: unexpected end of file");
  if (std::memcmp(b, "NZCP", 4) != 0) throw std::runtime_error("bad magic");
  if (n < 14) throw std::runtime_error("read header: unexpected end of file");
  NzHeader h;
  h.version = b[4];
  h.codec = b[5];
  h.particles = get_u32(b + 6);
  h.steps = get_u32(b + 10);
  return h;
}

// main.rs:249-309 (add_back=false); add_back=true applies the closed loop.
Floats nz_decompress(const uint8_t* b, size_t n, bool add_back) {
  NzHeader h = nz_read_header(b, n);
  if (h.codec < 1 || h.codec > 4) throw std::runtime_error("unknown codec " + std::to_string(h.codec));
  size_t off = 14;
  Floats all;
  all.reserve((size_t)h.particles * h.steps);
  // The LinearPredictor closed loop in rotating buffers, with the checks of
  // its predict / add in the same order: with two snapshots the history's
  // sizes must agree (q823_sub), an empty prediction passes the decoded step
  // through, any other prediction must match its size (q823_add).
  Fixed s_t, s_tm1, next;
  int hist = 0;
  for (uint32_t t = 0; t < h.steps; ++t) {
    if (off + 8 > n) throw std::runtime_error("read scale/len: unexpected end of file");
    float scale = get_f32(b + off);
    uint32_t len = get_u32(b + off + 4);
    off += 8;
    if (off + len > n) throw std::runtime_error("read bytes: unexpected end of file");
    Fixed deq = nz_dequantize(h.codec, b + off, len, scale);
    off += len;
    const size_t m = deq.size();
    if (!add_back) {
      const size_t base = all.size();
      all.resize(base + m);
      for (size_t i = 0; i < m; ++i) all[base + i] = fast::q823_to_f32(deq[i]);
      continue;
    }
    if (hist >= 2 && s_t.size() != s_tm1.size()) throw ShapeMismatch(s_t.size(), s_tm1.size());
    const bool use_p = hist >= 1 && !s_t.empty();
    if (use_p && s_t.size() != m) throw ShapeMismatch(s_t.size(), m);
    const size_t base = all.size();
    all.resize(base + m);
    next.resize(m);
    for (size_t i = 0; i < m; ++i) {
      int32_t rc = deq[i];
      if (use_p) {
        const int32_t p = hist >= 2 ? sat_add_i32(s_t[i], sat_sub_i32(s_t[i], s_tm1[i])) : s_t[i];
        rc = sat_add_i32(p, deq[i]);
      }
      next[i] = rc;
      all[base + i] = fast::q823_to_f32(rc);
    }
    if (hist >= 1) s_tm1.swap(s_t);  // LinearPredictor::update
    s_t.swap(next);
    hist = std::min(hist + 1, 2);
  }
  return all;
}

// main.rs:311-322
Floats lammps_generate_synthetic(size_t particles, size_t steps) {
  Floats out;
  out.reserve(particles * steps);
  for (size_t t = 0; t < steps; ++t) {
    float tt = (float)t * 0.1f;
    for (size_t i = 0; i < particles; ++i) {
      float phase = tt + (float)i * 0.01f;
      float noise = (float)(i % 100) * 0.0001f;
      out.push_back(std::cos(phase) + noise);
    }
  }
  return out;
}

}  // namespace host
}  // namespace ngl
