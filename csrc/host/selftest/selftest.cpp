// Self-test driver of the host library for sanitizer builds (AddressSanitizer
// and UndefinedBehaviorSanitizer): every codec on random inputs (round trip
// within its bound), every decoder on random garbage and on truncations of
// valid streams (no out-of-bounds access, no undefined arithmetic), the NZCP
// container, TopologyMask bincode (including malformed input), the LAMMPS
// dump reader (valid, truncated and random text), the HDF5 writer and
// reader (round trip, every truncation and random byte flips of a written
// file), and the product-format oracle.  Exit status 0 and "selftest ok" on success.
//
//   g++ -std=c++17 -O1 -g -fsanitize=address,undefined -fno-sanitize-recover=all \
//       -fno-omit-frame-pointer -Icsrc csrc/host/codecs.cpp csrc/host/pipeline.cpp \
//       csrc/host/product.cpp csrc/host/lammps_io.cpp csrc/host/hdf5_io.cpp csrc/host/selftest/selftest.cpp \
//       -o selftest && ./selftest
#include <cmath>
#include <cstdio>
#include <cstdlib>
#include <random>
#include <string>

#include "../hdf5_io.hpp"
#include "../nangila_host.hpp"

using namespace ngl::host;

namespace {
std::mt19937_64 rng(12345);

#define CHECK(c)                                                          \
  do {                                                                    \
    if (!(c)) {                                                           \
      std::fprintf(stderr, "selftest failed at %s:%d: %s\n", __FILE__, __LINE__, #c); \
      std::exit(1);                                                       \
    }                                                                     \
  } while (0)

Floats randn(size_t n, float scale, float zero_frac) {
  std::normal_distribution<float> nd(0.0f, scale);
  std::uniform_real_distribution<float> u(0.0f, 1.0f);
  Floats x(n);
  for (auto& v : x) v = u(rng) < zero_frac ? 0.0f : nd(rng);
  return x;
}

// Random bytes; with `header`, the first 4 bytes are a small element count
// (decoders size their output from it, as the reference's do).
Bytes garbage(size_t n, bool header = false) {
  Bytes b(n);
  for (auto& v : b) v = (uint8_t)(rng() & 0xff);
  if (header && n >= 4) {
    const uint32_t c = (uint32_t)(rng() % 5000);
    for (int i = 0; i < 4; ++i) b[i] = (uint8_t)(c >> (8 * i));
  }
  return b;
}

template <class Q, class D>
void codec_roundtrip(Q quant, D dequant, float eps, float bound, bool header) {
  for (size_t n : {0, 1, 31, 32, 33, 255, 256, 257, 1000, 4097}) {
    for (float zf : {0.0f, 0.7f, 1.0f}) {
      Floats x = randn(n, 0.01f, zf);
      Fixed r = q823_from_f32(x.data(), n);
      QuantOut q = quant(r.data(), n, eps);
      Fixed d = dequant(q.bytes.data(), q.bytes.size(), q.scale);
      CHECK(d.size() >= n);
      Floats y = q823_to_f32(d.data(), n);
      Floats xr = q823_to_f32(r.data(), n);
      for (size_t i = 0; i < n; ++i) CHECK(std::fabs(y[i] - xr[i]) <= bound);
      for (size_t cut = 0; cut <= q.bytes.size(); cut += 1 + q.bytes.size() / 17)
        (void)dequant(q.bytes.data(), cut, q.scale);  // truncated: must not crash
    }
  }
  for (int t = 0; t < 200; ++t) {
    Bytes g = garbage((size_t)(rng() % 600), header);
    (void)dequant(g.data(), g.size(), 0.002f);  // garbage: must not crash
  }
}
}  // namespace

int main() {
  const float eps = 1e-3f;
  codec_roundtrip(eb_quantize, eb_dequantize, eps, 1.001f * eps, false);
  codec_roundtrip(rle_quantize, rle_dequantize, eps, 1.001f * eps, false);
  codec_roundtrip(bs_quantize, bs_dequantize, eps, 1.001f * eps, true);
  codec_roundtrip(bsrle_quantize, bsrle_dequantize, eps, 1.001f * eps, true);
  codec_roundtrip(unified_eb_quantize, unified_eb_dequantize, eps, 1.001f * eps, false);
  // stochastic INT4 / INT8 and top-k: garbage and truncation only (lossy by design)
  for (int bits : {4, 8, 3}) {
    uint64_t counter = 0;
    Floats x = randn(1001, 0.01f, 0.2f);
    Fixed r = q823_from_f32(x.data(), x.size());
    QuantOut q = stochastic_quantize(r.data(), r.size(), bits, 7, &counter);
    for (size_t cut = 0; cut <= q.bytes.size(); cut += 37) (void)stochastic_dequantize(q.bytes.data(), cut, q.scale, bits);
    Bytes g = garbage(333);
    (void)stochastic_dequantize(g.data(), g.size(), 0.01f, bits);
  }
  for (float k : {0.0f, 0.05f, 0.5f, 1.0f, 1.5f}) {
    Floats x = randn(5000, 1.0f, 0.3f);
    Fixed r = q823_from_f32(x.data(), x.size());
    QuantOut q = topk_quantize(r.data(), r.size(), k);
    Fixed d = topk_dequantize(q.bytes.data(), q.bytes.size(), q.scale);
    CHECK(d.size() == r.size());
    for (size_t cut = 0; cut <= q.bytes.size(); cut += 1 + q.bytes.size() / 13)
      (void)topk_dequantize(q.bytes.data(), cut, q.scale);
  }
  for (int t = 0; t < 200; ++t) {
    Bytes g = garbage((size_t)(rng() % 400), true);
    (void)topk_dequantize(g.data(), g.size(), 0.1f);
    (void)rle_decode_i16(g.data(), g.size());
  }
  // Q8.23 arithmetic on extreme values (saturation paths)
  {
    Floats x = {0.0f, 1e30f, -1e30f, 255.9f, -256.0f, NAN, INFINITY, -INFINITY, 6.26e16f, 1e-30f};
    Fixed a = q823_from_f32(x.data(), x.size());
    Fixed s = q823_add(a.data(), a.size(), a.data(), a.size());
    Fixed d = q823_sub(a.data(), a.size(), s.data(), s.size());
    for (float m : {0.5f, -3.0f, 1e20f, -1e20f, 0.0f}) (void)q823_mul_scalar(d.data(), d.size(), m);
    (void)fixedq_from_f32(x.data(), x.size());
    bool threw = false;
    try {
      (void)q823_add(a.data(), a.size(), a.data(), a.size() - 1);
    } catch (const ShapeMismatch&) {
      threw = true;
    }
    CHECK(threw);
  }
  // NZCP container: every codec, decode with and without add-back, truncations
  for (int codec = 1; codec <= 4; ++codec) {
    const size_t P = 3001, T = 5;
    Floats data = lammps_generate_synthetic(P, T);
    NzStats st;
    Bytes nz = nz_compress(data.data(), P, T, codec, eps, &st);
    Floats back = nz_decompress(nz.data(), nz.size(), true);
    CHECK(back.size() == P * T);
    for (size_t i = 0; i < P * T; ++i) CHECK(std::fabs(back[i] - data[i]) <= 1.01f * eps);
    for (size_t cut = 0; cut < nz.size(); cut += 1 + nz.size() / 11) {
      try {
        (void)nz_decompress(nz.data(), cut, true);
      } catch (const std::exception&) {
      }
    }
  }
  // TopologyMask bincode, malformed input must throw, not read out of bounds
  {
    Floats v = randn(12, 1.0f, 0.0f);
    for (auto& x : v) x = std::fabs(x);
    TopologyMask m = TopologyMask::from_variance_threshold(v.data(), v.size(), 0.3f);
    Bytes b = m.to_bytes();
    TopologyMask m2 = TopologyMask::from_bytes(b.data(), b.size());
    CHECK(m2.to_bytes() == b);
    for (size_t cut = 0; cut < b.size(); ++cut) {
      try {
        (void)TopologyMask::from_bytes(b.data(), cut);
      } catch (const std::exception&) {
      }
    }
    for (int t = 0; t < 100; ++t) {
      Bytes g = garbage((size_t)(rng() % 200));
      try {
        (void)TopologyMask::from_bytes(g.data(), g.size());
      } catch (const std::exception&) {
      }
    }
  }
  // LAMMPS dump reader: a valid dump, every truncation of it, random text
  {
    std::string d;
    for (int t = 0; t < 2; ++t) {
      d += "ITEM: TIMESTEP\n" + std::to_string(t) + "\nITEM: NUMBER OF ATOMS\n3\nITEM: BOX BOUNDS xx yy zz\n";
      d += "0 10\n0 10\n0 10\nITEM: ATOMS id type z y x\n";
      d += "1 1 0.5 -1e-3 inf\n2 1 +2. .25 1e40\n3 1 nan 7 -0\n";
    }
    std::vector<Floats> snaps = lammps_read_dump_text(d.data(), d.size());
    CHECK(snaps.size() == 2 && snaps[0].size() == 9 && snaps[0][2] == 0.5f && snaps[0][0] == INFINITY);
    for (size_t cut = 0; cut < d.size(); ++cut) {
      try {
        (void)lammps_read_dump_text(d.data(), cut);
      } catch (const std::exception&) {
      }
    }
    const char alphabet[] = "ITEM: TIMESTEPNUMBEROFATOMSBXyz0123456789.e+-\n \t";
    for (int t = 0; t < 300; ++t) {
      std::string g = t % 2 ? d.substr(0, (size_t)(rng() % d.size())) : std::string();
      const size_t extra = (size_t)(rng() % 400);
      for (size_t i = 0; i < extra; ++i) g += alphabet[rng() % (sizeof(alphabet) - 1)];
      try {
        (void)lammps_read_dump_text(g.data(), g.size());
      } catch (const std::exception&) {
      }
    }
  }
  // product-format oracle: encode/reduce and top-k on odd sizes, with
  // topology; 300000 (1172 blocks, the last one partial) splits every
  // block-parallel loop over several host threads
  for (size_t n : {1, 255, 257, 2049, 20000, 300000}) {
    Floats g = randn(n, 1e-3f, 0.1f), pred = randn(n, 1e-3f, 0.0f), e = randn(n, 1e-4f, 0.0f);
    ProductParams p;
    p.topo_a = 1;
    p.topo_b = 0;
    p.topo_ndrop = (int64_t)(product_wire_bytes(n, 0, 0) / 1056) / 3;
    TopoChunks t = product_topology(product_wire_bytes(n, 0, 0) / 1056, 0.3, 5, 1);
    p.topo_a = t.a;
    p.topo_b = t.b;
    p.topo_ndrop = t.ndrop;
    Bytes w(product_wire_bytes(n, 0, 0));
    Floats eo(n), avg(n);
    product_encode(g.data(), pred.data(), e.data(), n, p, w.data(), eo.data());
    const uint8_t* ws[2] = {w.data(), w.data()};
    product_reduce(ws, 2, n, 4, pred.data(), 0.5f, avg.data());
    product_reduce_twoshot(ws, 2, n, 4, pred.data(), 0.5f, avg.data());
    Bytes tk(product_wire_bytes(n, 2, 13));
    product_topk_encode(g.data(), pred.data(), e.data(), n, 13, true, tk.data(), eo.data(), t);
    const uint8_t* ts[1] = {tk.data()};
    product_topk_reduce(ts, 1, n, 13, pred.data(), 1.0f, avg.data());
    product_ema(pred.data(), avg.data(), n, 0.9f, false);
  }
  // HDF5: a tree with nested groups, more links than one symbol table node
  // holds, every element type and scalar / N-D / empty values; then every
  // truncation and random byte flips of the file must fail cleanly
  {
    namespace h5 = ngl::h5;
    auto val = [](char kind, int size, std::vector<uint64_t> shape) {
      h5::Value v;
      v.kind = kind;
      v.size = size;
      v.shape = shape;
      uint64_t n = 1;
      for (uint64_t d : shape) n *= d;
      v.bytes.resize(n * size);
      for (auto& c : v.bytes) c = (char)(rng() & 0x7f);
      return v;
    };
    std::vector<h5::Object> objs(1);
    objs[0].attrs.push_back({"root_attr", val('f', 8, {})});
    h5::Object g;
    g.name = "grp";
    g.parent = 0;
    g.attrs.push_back({"codec", val('S', 17, {})});
    g.attrs.push_back({"total_len", val('u', 8, {})});
    objs.push_back(g);
    for (int i = 0; i < 21; ++i) {
      h5::Object d;
      d.is_group = false;
      d.name = "d" + std::to_string(i);
      d.parent = i % 2 ? 1 : 0;
      const char kinds[] = {'u', 'i', 'f', 'S'};
      const char k = kinds[i % 4];
      const int size = k == 'f' ? (i % 8 < 4 ? 4 : 8) : (k == 'S' ? 5 : 1 << (i % 4));
      d.data = val(k, size, i % 5 == 0 ? std::vector<uint64_t>{} : std::vector<uint64_t>{(uint64_t)(i * 7 % 13), 3});
      d.attrs.push_back({"a", val('i', 4, {2})});
      objs.push_back(d);
    }
    h5::Object sub;
    sub.name = "sub";
    sub.parent = 1;
    objs.push_back(sub);
    const std::string file = h5::write_file(objs);
    const std::vector<h5::Object> back = h5::read_file(file);
    CHECK(back.size() == objs.size());
    size_t checked = 0;
    for (const auto& b : back)
      for (const auto& o : objs)
        if (o.name == b.name && !o.is_group && !b.is_group) {
          CHECK(o.data.bytes == b.data.bytes && o.data.shape == b.data.shape && o.data.kind == b.data.kind);
          ++checked;
        }
    CHECK(checked == 21);
    for (size_t cut = 0; cut < file.size(); cut += 1 + file.size() / 257) {
      try {
        (void)h5::read_file(file.substr(0, cut));
      } catch (const std::exception&) {
      }
    }
    for (int t = 0; t < 400; ++t) {
      std::string f = file;
      for (int k = 0; k < 1 + t % 4; ++k) f[rng() % f.size()] = (char)(rng() & 0xff);
      try {
        (void)h5::read_file(f);
      } catch (const std::exception&) {
      }
    }
  }
  std::printf("selftest ok\n");
  return 0;
}
