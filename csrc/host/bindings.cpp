// pybind11 bindings of the native host library (module mini_nangila_b200._host).
#include <pybind11/numpy.h>
#include <pybind11/pybind11.h>
#include <pybind11/stl.h>

#include <string>

#include "hdf5_io.hpp"
#include "nangila_host.hpp"

namespace py = pybind11;
using namespace ngl::host;

namespace {
template <typename T>
using carr = py::array_t<T, py::array::c_style | py::array::forcecast>;

// Hand a std::vector to numpy without a copy.
template <typename T>
py::array_t<T> to_np(std::vector<T>&& v) {
  auto* heap = new std::vector<T>(std::move(v));
  py::capsule owner(heap, [](void* p) { delete reinterpret_cast<std::vector<T>*>(p); });
  return py::array_t<T>({(py::ssize_t)heap->size()}, {(py::ssize_t)sizeof(T)}, heap->data(), owner);
}
template <typename T>
const T* ptr(const carr<T>& a) {
  return a.size() ? a.data() : nullptr;
}
py::tuple qout(QuantOut&& q) { return py::make_tuple(to_np(std::move(q.bytes)), q.scale); }
// An optional output array (None, or float32, C-contiguous, writable, n
// elements) that a call writes in place instead of returning a new one.
float* out_f32(const py::object& o, size_t n, const char* what) {
  if (o.is_none()) return nullptr;
  auto a = o.cast<py::array_t<float, py::array::c_style>>();
  // a converted copy would be written and lost: the caller's array must already conform
  if (a.ptr() != o.ptr()) throw std::runtime_error(std::string(what) + " must be a float32 C-contiguous array");
  if ((size_t)a.size() != n) throw std::runtime_error(std::string(what) + " size mismatch");
  if (!a.writeable()) throw std::runtime_error(std::string(what) + " is read-only");
  return a.mutable_data();
}
// HDF5 objects <-> Python: a value is (kind, size, shape, bytes); an object
// is (is_group, name, parent, value or None, [(attr name, value), ...]).
ngl::h5::Value h5_value(const py::tuple& t) {
  ngl::h5::Value v;
  const std::string kind = t[0].cast<std::string>();
  if (kind.size() != 1) throw std::runtime_error("HDF5 value kind must be one character");
  v.kind = kind[0];
  v.size = t[1].cast<int>();
  v.shape = t[2].cast<std::vector<uint64_t>>();
  v.bytes = t[3].cast<std::string>();
  return v;
}
py::tuple h5_tuple(const ngl::h5::Value& v) {
  return py::make_tuple(std::string(1, v.kind), v.size, v.shape, py::bytes(v.bytes));
}
}  // namespace

PYBIND11_MODULE(_host, m) {
  py::register_exception<ngl::h5::Error>(m, "H5Error", PyExc_ValueError);
  m.def("h5_write", [](const py::list& objs) {
    std::vector<ngl::h5::Object> v;
    for (const auto& it : objs) {
      const auto t = it.cast<py::tuple>();
      ngl::h5::Object o;
      o.is_group = t[0].cast<bool>();
      o.name = t[1].cast<std::string>();
      o.parent = t[2].cast<int>();
      if (!t[3].is_none()) o.data = h5_value(t[3].cast<py::tuple>());
      for (const auto& a : t[4].cast<py::list>()) {
        const auto at = a.cast<py::tuple>();
        o.attrs.push_back({at[0].cast<std::string>(), h5_value(at[1].cast<py::tuple>())});
      }
      v.push_back(std::move(o));
    }
    std::string out;
    {
      py::gil_scoped_release nogil;
      out = ngl::h5::write_file(v);
    }
    return py::bytes(out);
  }, py::arg("objects"), "HDF5 file bytes of a flat object list (objects[0] is the root group)");
  m.def("h5_read", [](const py::bytes& file) {
    const std::string f = file;
    std::vector<ngl::h5::Object> v;
    {
      py::gil_scoped_release nogil;
      v = ngl::h5::read_file(f);
    }
    py::list out;
    for (const auto& o : v) {
      py::list attrs;
      for (const auto& a : o.attrs) attrs.append(py::make_tuple(a.name, h5_tuple(a.value)));
      out.append(py::make_tuple(o.is_group, o.name, o.parent, o.is_group ? py::object(py::none())
                                                                           : py::object(h5_tuple(o.data)), attrs));
    }
    return out;
  }, py::arg("file"), "Flat object list of an HDF5 file image");
  m.doc() = "Native host library: bit-exact codecs, predictors, topology, NZCP, product-format oracle";
  py::register_exception<ShapeMismatch>(m, "ShapeMismatch", PyExc_ValueError);

  // nangila-math / nangila-edge
  m.def("q823_from_f32", [](carr<float> x) { return to_np(q823_from_f32(ptr(x), x.size())); });
  m.def("q823_to_f32", [](carr<int32_t> q) { return to_np(q823_to_f32(ptr(q), q.size())); });
  m.def("q823_add", [](carr<int32_t> a, carr<int32_t> b) { return to_np(q823_add(ptr(a), a.size(), ptr(b), b.size())); });
  m.def("q823_sub", [](carr<int32_t> a, carr<int32_t> b) { return to_np(q823_sub(ptr(a), a.size(), ptr(b), b.size())); });
  m.def("q823_mul_scalar", [](carr<int32_t> a, float s) { return to_np(q823_mul_scalar(ptr(a), a.size(), s)); });
  m.def("q823_momentum_update", [](carr<int32_t> state, carr<int32_t> obs, float beta, float one_minus_beta) {
    if (state.size() != obs.size()) throw ShapeMismatch(state.size(), obs.size());
    return to_np(q823_momentum_update(ptr(state), ptr(obs), state.size(), beta, one_minus_beta));
  });
  m.def("fixedq_from_f32", [](carr<float> x) { return to_np(fixedq_from_f32(ptr(x), x.size())); });
  m.def("fixedq_to_f32", [](carr<int32_t> q) { return to_np(fixedq_to_f32(ptr(q), q.size())); });

  // UnifiedQuantizer
  m.def("stochastic_quantize", [](carr<int32_t> r, int bits, uint64_t seed, uint64_t counter) {
    QuantOut q = stochastic_quantize(ptr(r), r.size(), bits, seed, &counter);
    return py::make_tuple(to_np(std::move(q.bytes)), q.scale, counter);
  });
  m.def("stochastic_dequantize", [](carr<uint8_t> b, float scale, int bits) {
    return to_np(stochastic_dequantize(ptr(b), b.size(), scale, bits));
  });
  m.def("topk_quantize", [](carr<int32_t> r, float k) { return qout(topk_quantize(ptr(r), r.size(), k)); });
  m.def("topk_dequantize", [](carr<uint8_t> b, float s) { return to_np(topk_dequantize(ptr(b), b.size(), s)); });
  m.def("topk_threshold", [](carr<float> x, float k) { return topk_threshold(ptr(x), x.size(), k); });

  // nangila-hpc
  m.def("eb_quantize", [](carr<int32_t> r, float eps) { return qout(eb_quantize(ptr(r), r.size(), eps)); });
  m.def("eb_dequantize", [](carr<uint8_t> b, float s) { return to_np(eb_dequantize(ptr(b), b.size(), s)); });
  m.def("rle_quantize", [](carr<int32_t> r, float eps) { return qout(rle_quantize(ptr(r), r.size(), eps)); });
  m.def("rle_dequantize", [](carr<uint8_t> b, float s) { return to_np(rle_dequantize(ptr(b), b.size(), s)); });
  m.def("bs_quantize", [](carr<int32_t> r, float eps) { return qout(bs_quantize(ptr(r), r.size(), eps)); });
  m.def("bs_dequantize", [](carr<uint8_t> b, float s) { return to_np(bs_dequantize(ptr(b), b.size(), s)); });
  m.def("bsrle_quantize", [](carr<int32_t> r, float eps) { return qout(bsrle_quantize(ptr(r), r.size(), eps)); });
  m.def("bsrle_dequantize", [](carr<uint8_t> b, float s) { return to_np(bsrle_dequantize(ptr(b), b.size(), s)); });
  m.def("rle_encode_i16", [](carr<int16_t> q) { return to_np(rle_encode_i16(ptr(q), q.size())); });
  m.def("rle_decode_i16", [](carr<uint8_t> b) { return to_np(rle_decode_i16(ptr(b), b.size())); });

  // Predictors
  py::class_<MomentumPredictor>(m, "MomentumPredictor")
      .def(py::init<float>())
      .def("predict", [](const MomentumPredictor& p) { return to_np(p.predict()); })
      .def("update", [](MomentumPredictor& p, carr<int32_t> o) { p.update(ptr(o), o.size()); })
      .def("reset", &MomentumPredictor::reset)
      .def_property_readonly("beta", &MomentumPredictor::beta)
      .def_property_readonly("has_state", &MomentumPredictor::has_state)
      .def("get_state", [](const MomentumPredictor& p) { return py::make_tuple(to_np(Fixed(p.state())), p.has_state()); })
      .def("set_state", [](MomentumPredictor& p, carr<int32_t> s, bool has) {
        p.set_state(Fixed(ptr(s), ptr(s) + s.size()), has);
      });
  py::class_<LinearPredictor>(m, "LinearPredictor")
      .def(py::init<>())
      .def("predict", [](const LinearPredictor& p) { return to_np(p.predict()); })
      .def("update", [](LinearPredictor& p, carr<int32_t> o) { p.update(ptr(o), o.size()); })
      .def("reset", &LinearPredictor::reset)
      .def_property_readonly("history", &LinearPredictor::history)
      .def("get_state", [](const LinearPredictor& p) {
        return py::make_tuple(to_np(Fixed(p.s_t())), to_np(Fixed(p.s_tm1())), p.history());
      })
      .def("set_state", [](LinearPredictor& p, carr<int32_t> st, carr<int32_t> stm1, int n) {
        p.set_history(Fixed(ptr(st), ptr(st) + st.size()), Fixed(ptr(stm1), ptr(stm1) + stm1.size()), n);
      });

  // TopologyMask
  py::class_<TopologyMask>(m, "TopologyMask")
      .def(py::init<>())
      .def_static("from_variance_threshold",
                  [](carr<float> v, float d) { return TopologyMask::from_variance_threshold(ptr(v), v.size(), d); })
      .def_static("all_drivers", &TopologyMask::all_drivers)
      .def_readwrite("driver_indices", &TopologyMask::driver_indices)
      .def_readwrite("passenger_indices", &TopologyMask::passenger_indices)
      .def_readwrite("threshold", &TopologyMask::threshold)
      .def_readwrite("total_layers", &TopologyMask::total_layers)
      .def("is_driver", &TopologyMask::is_driver)
      .def("is_passenger", &TopologyMask::is_passenger)
      .def("compression_factor", &TopologyMask::compression_factor)
      .def("passenger_percentage", &TopologyMask::passenger_percentage)
      .def("to_bytes", [](const TopologyMask& t) {
        Bytes b = t.to_bytes();
        return py::bytes(reinterpret_cast<const char*>(b.data()), b.size());
      })
      .def_static("from_bytes", [](py::bytes b) {
        std::string s = b;
        return TopologyMask::from_bytes(reinterpret_cast<const uint8_t*>(s.data()), s.size());
      });

  // NZCP
  m.def("nz_compress", [](carr<float> data, size_t particles, size_t steps, int codec, float eps) {
    if (particles * steps > (size_t)data.size()) throw std::runtime_error("data shorter than particles*steps");
    NzStats st;
    Bytes b;
    {
      py::gil_scoped_release nogil;
      b = nz_compress(ptr(data), particles, steps, codec, eps, &st);
    }
    py::dict stats;
    stats["total_raw"] = st.total_raw;
    stats["total_comp"] = st.total_comp;
    stats["max_abs_err"] = st.max_abs_err;
    return py::make_tuple(to_np(std::move(b)), stats);
  });
  m.def("nz_read_header", [](carr<uint8_t> b) {
    NzHeader h = nz_read_header(ptr(b), b.size());
    return py::make_tuple(h.version, h.codec, h.particles, h.steps);
  });
  m.def("nz_decompress", [](carr<uint8_t> b, bool add_back) {
    Floats f;
    {
      py::gil_scoped_release nogil;
      f = nz_decompress(ptr(b), b.size(), add_back);
    }
    return to_np(std::move(f));
  });
  m.def("lammps_generate_synthetic", [](size_t p, size_t s) { return to_np(lammps_generate_synthetic(p, s)); });
  m.def("lammps_read_dump", [](const std::string& path) {
    std::vector<Floats> snaps;
    {
      py::gil_scoped_release nogil;
      snaps = lammps_read_dump(path);
    }
    py::list out;
    for (auto& v : snaps) out.append(to_np(std::move(v)));
    return out;
  });
  m.def("lammps_read_dump_text", [](py::bytes text) {
    const std::string t = text;
    py::list out;
    for (auto& v : lammps_read_dump_text(t.data(), t.size())) out.append(to_np(std::move(v)));
    return out;
  });
  m.def("lammps_write_dump", [](const std::string& path, size_t atoms, size_t steps) {
    py::gil_scoped_release nogil;
    lammps_write_dump(path, atoms, steps);
  });

  // Product format oracle (chunked wire payloads)
  m.def("product_wire_bytes", &product_wire_bytes);
  m.def("product_topology", [](size_t nchunks, double drop, uint64_t seed, uint64_t stream) {
    const TopoChunks t = product_topology(nchunks, drop, seed, stream);
    return py::make_tuple(t.a, t.b, t.ndrop);
  });
  m.def("product_encode", [](carr<float> g, py::object pred, py::object e_in, int bits, bool stochastic, bool ef,
                             uint64_t seed, uint32_t rank, uint32_t bucket, uint64_t step, py::tuple topo,
                             py::object e_out_arr) {
    const size_t n = g.size();
    carr<float> pr = pred.is_none() ? carr<float>() : pred.cast<carr<float>>();
    carr<float> ei = e_in.is_none() ? carr<float>() : e_in.cast<carr<float>>();
    if (!pred.is_none() && (size_t)pr.size() != n) throw std::runtime_error("pred size mismatch");
    if (!e_in.is_none() && (size_t)ei.size() != n) throw std::runtime_error("e size mismatch");
    std::vector<uint8_t> wire(product_wire_bytes(n, bits == 4 ? 0 : 1, 0));
    float* e_dst = ef ? out_f32(e_out_arr, n, "e_out") : nullptr;
    std::vector<float> e_out(ef && !e_dst ? n : 0);
    if (ef && !e_dst) e_dst = e_out.data();
    ProductParams p;
    p.bits = bits;
    p.stochastic = stochastic;
    p.error_feedback = ef;
    p.seed = seed;
    p.rank = rank;
    p.bucket = bucket;
    p.step = step;
    if (topo.size() == 3) {
      p.topo_a = topo[0].cast<uint64_t>();
      p.topo_b = topo[1].cast<uint64_t>();
      p.topo_ndrop = topo[2].cast<int64_t>();
    }
    // e_out may be e_in itself: each block's residuals are read before its
    // error feedback is written, and blocks are disjoint
    product_encode(ptr(g), pred.is_none() ? nullptr : ptr(pr), e_in.is_none() ? nullptr : ptr(ei), n, p,
                   wire.data(), e_dst);
    py::object e_ret = (ef && !e_out_arr.is_none()) ? e_out_arr : py::object(to_np(std::move(e_out)));
    return py::make_tuple(to_np(std::move(wire)), e_ret);
  }, py::arg("g"), py::arg("pred"), py::arg("e_in"), py::arg("bits"), py::arg("stochastic"), py::arg("ef"),
     py::arg("seed"), py::arg("rank"), py::arg("bucket"), py::arg("step"), py::arg("topo") = py::tuple(),
     py::arg("e_out") = py::none());
  auto reduce_impl = [](bool twoshot) {
    return [twoshot](std::vector<carr<uint8_t>> wires, size_t n, int bits, py::object pred, float inv_world,
                     py::object out) -> py::object {
      const int W = (int)wires.size();
      std::vector<const uint8_t*> wp(W);
      for (int r = 0; r < W; ++r) wp[r] = ptr(wires[r]);
      carr<float> pr = pred.is_none() ? carr<float>() : pred.cast<carr<float>>();
      float* dst = out_f32(out, n, "out");
      std::vector<float> avg(dst ? 0 : n);
      if (!dst) dst = avg.data();
      if (twoshot)
        product_reduce_twoshot(wp.data(), W, n, bits, pred.is_none() ? nullptr : ptr(pr), inv_world, dst);
      else
        product_reduce(wp.data(), W, n, bits, pred.is_none() ? nullptr : ptr(pr), inv_world, dst);
      return out.is_none() ? py::object(to_np(std::move(avg))) : out;
    };
  };
  m.def("product_reduce", reduce_impl(false), py::arg("wires"), py::arg("n"), py::arg("bits"), py::arg("pred"),
        py::arg("inv_world"), py::arg("out") = py::none());
  m.def("product_reduce_twoshot", reduce_impl(true), py::arg("wires"), py::arg("n"), py::arg("bits"), py::arg("pred"),
        py::arg("inv_world"), py::arg("out") = py::none());
  m.def("product_ema", [](carr<float> state, carr<float> avg, float beta, bool first) {
    std::vector<float> s(state.data(), state.data() + state.size());
    product_ema(s.data(), ptr(avg), s.size(), beta, first);
    return to_np(std::move(s));
  });
  // In place on a float32 C-contiguous writable state array.
  m.def("product_ema_", [](py::object state, carr<float> avg, float beta, bool first) {
    const size_t n = (size_t)avg.size();
    float* s = out_f32(state, n, "state");
    if (!s) throw std::runtime_error("state is required");
    product_ema(s, ptr(avg), n, beta, first);
  });
  m.def("product_topk_encode", [](carr<float> g, py::object pred, py::object e_in, int k, bool ef, py::tuple topo) {
    TopoChunks t;
    if (topo.size() == 3) {
      t.a = topo[0].cast<uint64_t>();
      t.b = topo[1].cast<uint64_t>();
      t.ndrop = topo[2].cast<int64_t>();
    }
    const size_t n = g.size();
    carr<float> pr = pred.is_none() ? carr<float>() : pred.cast<carr<float>>();
    carr<float> ei = e_in.is_none() ? carr<float>() : e_in.cast<carr<float>>();
    std::vector<uint8_t> rec(product_wire_bytes(n, 2, k));
    std::vector<float> e_out(ef ? n : 0);
    product_topk_encode(ptr(g), pred.is_none() ? nullptr : ptr(pr), e_in.is_none() ? nullptr : ptr(ei), n, k, ef,
                        rec.data(), ef ? e_out.data() : nullptr, t);
    return py::make_tuple(to_np(std::move(rec)), to_np(std::move(e_out)));
  }, py::arg("g"), py::arg("pred"), py::arg("e_in"), py::arg("k"), py::arg("ef"), py::arg("topo") = py::tuple());
  m.def("product_topk_reduce", [](std::vector<carr<uint8_t>> recs, size_t n, int k, py::object pred, float inv_world) {
    const int W = (int)recs.size();
    std::vector<const uint8_t*> rp(W);
    for (int r = 0; r < W; ++r) rp[r] = ptr(recs[r]);
    carr<float> pr = pred.is_none() ? carr<float>() : pred.cast<carr<float>>();
    std::vector<float> avg(n);
    product_topk_reduce(rp.data(), W, n, k, pred.is_none() ? nullptr : ptr(pr), inv_world, avg.data());
    return to_np(std::move(avg));
  });
}
