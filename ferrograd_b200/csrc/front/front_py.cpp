// front_py.cpp -- Python binding of the C++ front end (module
// ferrograd_b200._front).  Names and argument meaning follow the reference's
// Rust API (src/tensor.rs, src/nn.rs, src/optim.rs); panics become
// RuntimeError.
#include <pybind11/numpy.h>
#include <pybind11/pybind11.h>
#include <pybind11/stl.h>

#include <cstring>

#include "front_internal.h"

namespace py = pybind11;
using namespace ferro;

namespace {

DType parse_dtype(const std::string &s) {
  if (s == "f32" || s == "float32") return DType::F32;
  if (s == "i32" || s == "int32") return DType::I32;
  if (s == "bool") return DType::Bool;
  throw Panic("unknown dtype '" + s + "'");
}

Shape to_shape(const py::sequence &seq) {
  Shape s;
  for (auto v : seq) s.push_back(v.cast<int64_t>());
  return s;
}

py::tuple shape_tuple(const Shape &s) {
  py::tuple t(s.size());
  for (size_t i = 0; i < s.size(); i++) t[i] = s[i];
  return t;
}

Tensor tensor_from_array(const py::array &arr) {
  Shape shape;
  for (py::ssize_t i = 0; i < arr.ndim(); i++) shape.push_back((int64_t)arr.shape(i));
  if (py::isinstance<py::array_t<float>>(arr)) {
    auto a = py::array_t<float, py::array::c_style | py::array::forcecast>::ensure(arr);
    return Tensor::from_f32(a.data(), shape);
  }
  if (py::isinstance<py::array_t<int32_t>>(arr)) {
    auto a = py::array_t<int32_t, py::array::c_style | py::array::forcecast>::ensure(arr);
    return Tensor::from_i32(a.data(), shape);
  }
  if (py::isinstance<py::array_t<bool>>(arr)) {
    auto a = py::array_t<uint8_t, py::array::c_style | py::array::forcecast>::ensure(arr);
    return Tensor::from_bool(a.data(), shape);
  }
  throw Panic("Tensor.new: unsupported element type (float32, int32 or bool)");
}

py::array tensor_to_numpy(const Tensor &t) {
  auto bytes = t.to_bytes();
  Shape s = t.shape();
  std::vector<py::ssize_t> shp(s.begin(), s.end());
  py::array out;
  switch (t.dtype()) {
    case DType::F32: out = py::array_t<float>(shp); break;
    case DType::I32: out = py::array_t<int32_t>(shp); break;
    case DType::Bool: out = py::array_t<bool>(shp); break;
  }
  if (!bytes.empty()) std::memcpy(out.mutable_data(), bytes.data(), bytes.size());
  return out;
}

py::list items_summary(const SchedulePlan &plan, bool with_source) {
  py::list items;
  for (const ScheduleItem &it : plan.items) {
    py::dict d;
    d["kind"] = it.store_dest ? "store" : "alloc";
    py::list ins;
    for (const KernelInput &in : it.inputs) {
      if (in.kind == KernelInput::Buffer)
        ins.append(py::make_tuple("buffer", in.buffer->id));
      else if (in.kind == KernelInput::I32)
        ins.append(py::make_tuple("i32", in.i));
      else if (in.kind == KernelInput::F32)
        ins.append(py::make_tuple("f32", in.f));
      else
        ins.append(py::make_tuple("bool", in.i));
    }
    d["inputs"] = ins;
    d["output"] = it.output ? py::cast(it.output->id) : py::none();
    d["out_shape"] = shape_tuple(it.out_shape);
    RoutePlan rp = plan_route(it);
    d["route"] = rp.route;
    d["steps"] = rp.steps;
    d["graph"] = dump(it.value);
    if (with_source) d["source"] = render_item_source(it);
    items.append(d);
  }
  return items;
}

// UOp-level handle for scheduler tests (the reference's schedule tests work
// on UOps directly, src/schedule.rs:367-571).
struct PyUOp {
  UOpP u;
};

}  // namespace

PYBIND11_MODULE(_front, m) {
  m.doc() = "ferrograd lazy Tensor front end on the B200 backend";

  py::class_<Tensor>(m, "Tensor")
      .def_static("new", &tensor_from_array, py::arg("data"),
                  "Tensor::new: a realized tensor holding a copy of `data`.")
      .def_static("zeros",
                  [](const py::sequence &s, const std::string &dt) {
                    return Tensor::zeros(to_shape(s), parse_dtype(dt));
                  },
                  py::arg("shape"), py::arg("dtype") = "f32")
      .def_static("ones",
                  [](const py::sequence &s, const std::string &dt) {
                    return Tensor::ones(to_shape(s), parse_dtype(dt));
                  },
                  py::arg("shape"), py::arg("dtype") = "f32")
      .def_static("full",
                  [](const py::sequence &s, float v) { return Tensor::full(to_shape(s), v); },
                  py::arg("shape"), py::arg("value"))
      .def_static("scalar", &Tensor::scalar, py::arg("value"))
      .def_static("empty",
                  [](const py::sequence &s, const std::string &dt) {
                    return Tensor::empty(to_shape(s), parse_dtype(dt));
                  },
                  py::arg("shape"), py::arg("dtype") = "f32")
      .def_static("from_u8",
                  [](const py::array_t<uint8_t, py::array::c_style | py::array::forcecast> &a,
                     float divisor) {
                    Shape shape;
                    for (py::ssize_t i = 0; i < a.ndim(); i++) shape.push_back((int64_t)a.shape(i));
                    return Tensor::from_u8_div(a.data(), shape, divisor);
                  },
                  py::arg("data"), py::arg("divisor") = 255.0f,
                  "Bytes uploaded once, converted on the device to (float)b / divisor.")
      .def_static("one_hot_u8",
                  [](const py::array_t<uint8_t, py::array::c_style | py::array::forcecast> &a,
                     int classes) { return Tensor::one_hot_u8(a.data(), (int64_t)a.size(), classes); },
                  py::arg("labels"), py::arg("classes"))
      .def_property_readonly("shape", [](const Tensor &t) { return shape_tuple(t.shape()); })
      .def_property_readonly("dtype", [](const Tensor &t) { return std::string(dtype_name(t.dtype())); })
      .def("numel", &Tensor::numel)
      .def("ndim", &Tensor::ndim)
      .def("is_realized", &Tensor::is_realized)
      .def("requires_grad", &Tensor::requires_grad)
      .def("with_requires_grad", &Tensor::with_requires_grad, py::arg("requires_grad") = true)
      .def("grad",
           [](const Tensor &t) -> py::object {
             Tensor g = t.grad();
             return g.defined() ? py::cast(g) : py::none();
           })
      .def("ptr_eq", &Tensor::ptr_eq)
      .def("detach", &Tensor::detach)
      .def("replace", &Tensor::replace)
      .def("assign", &Tensor::assign)
      .def("add", &Tensor::add)
      .def("mul", &Tensor::mul)
      .def("sub", &Tensor::sub)
      .def("neg", &Tensor::neg)
      .def("reciprocal", &Tensor::reciprocal)
      .def("exp2", &Tensor::exp2)
      .def("log2", &Tensor::log2)
      .def("sqrt", &Tensor::sqrt)
      .def("relu", &Tensor::relu)
      .def("exp", &Tensor::exp)
      .def("log", &Tensor::log)
      .def("reshape", [](const Tensor &t, const py::sequence &s) { return t.reshape(to_shape(s)); })
      .def("narrow", &Tensor::narrow, py::arg("dim"), py::arg("start"), py::arg("len"))
      .def("permute", [](const Tensor &t, const py::sequence &s) { return t.permute(to_shape(s)); })
      .def("contiguous", &Tensor::contiguous)
      .def("expand", [](const Tensor &t, const py::sequence &s) { return t.expand(to_shape(s)); })
      .def("sum", [](const Tensor &t, const py::sequence &a) { return t.sum(to_shape(a)); })
      .def("max", [](const Tensor &t, const py::sequence &a) { return t.max(to_shape(a)); })
      .def("log_softmax", &Tensor::log_softmax, py::arg("axis"))
      .def("cross_entropy", &Tensor::cross_entropy, py::arg("targets"))
      .def("matmul", &Tensor::matmul)
      .def("__add__", &Tensor::add)
      .def("__mul__", &Tensor::mul)
      .def("__sub__", &Tensor::sub)
      .def("__neg__", &Tensor::neg)
      .def("__matmul__", &Tensor::matmul)
      .def("realize", &Tensor::realize)
      .def_static("realize_many", &Tensor::realize_many)
      .def("to_vec", &Tensor::to_vec)
      .def("numpy", &tensor_to_numpy)
      .def("backward", &Tensor::backward)
      .def(
          "all_reduce_mean",
          [](const Tensor &t, uintptr_t comm) { t.all_reduce_mean(reinterpret_cast<fg_comm *>(comm)); },
          py::arg("comm"), "In place: realize, then the mean over the communicator's ranks.")
      .def("gradient", &Tensor::gradient)
      .def("_graph", [](const Tensor &t) { return dump(t.uop()); })
      .def("__repr__", [](const Tensor &t) {
        return "Tensor(shape=" + shape_str(t.shape()) + ", dtype=" + dtype_name(t.dtype()) +
               ", requires_grad=" + (t.requires_grad() ? "true" : "false") + ")";
      });

  py::class_<Linear>(m, "Linear")
      .def(py::init<int64_t, int64_t, bool>(), py::arg("in_features"), py::arg("out_features"),
           py::arg("bias") = true)
      .def_static("without_bias",
                  [](int64_t i, int64_t o) { return Linear(i, o, false); })
      .def_readonly("weight", &Linear::weight)
      .def_property_readonly("bias",
                             [](const Linear &l) -> py::object {
                               return l.bias.defined() ? py::cast(l.bias) : py::none();
                             })
      .def("forward", &Linear::forward)
      .def("__call__", &Linear::forward)
      .def("parameters", &Linear::parameters);

  py::class_<Sgd>(m, "Sgd")
      .def(py::init<const std::vector<Tensor> &, float>(), py::arg("params"), py::arg("lr"))
      .def_readonly("params", &Sgd::params)
      .def_readonly("lr", &Sgd::lr)
      .def("zero_grad", &Sgd::zero_grad)
      .def("step", &Sgd::step)
      .def(
          "set_comm",
          [](Sgd &s, uintptr_t comm) { s.comm = reinterpret_cast<fg_comm *>(comm); },
          py::arg("comm"),
          "Attach an fg_comm handle (0 detaches): step() then averages the gradients over "
          "the ranks first.")
      .def_property_readonly("comm", [](const Sgd &s) { return (uintptr_t)s.comm; });

  m.def("reset_init_seed", &reset_init_seed, py::arg("seed") = 42);
  m.def("init_seed", &init_seed);
  m.def("set_device", &set_device);
  m.def("synchronize", &synchronize);
  m.def(
      "stream",
      []() {
        void *st = nullptr;
        if (fg_device_stream(device(), &st) != FG_OK) throw Panic(fg_last_error());
        return (uintptr_t)st;
      },
      "CUDA stream (as an integer handle) the front end launches on.");
  m.def("exact_mode", &exact_mode);
  m.def(
      "parse_optimize_config",
      [](const std::string &raw) {
        OptimizeConfig c = parse_optimize_config(raw.c_str());
        py::dict d;
        d["symbolic"] = c.symbolic;
        d["upcast"] = c.upcast;
        d["unroll"] = c.unroll;
        return d;
      },
      "The reference's OPT parsing (src/optimize/mod.rs:80-108) of the given string.");
  m.def(
      "optimize_config",
      []() {
        const OptimizeConfig &c = optimize_config();
        py::dict d;
        d["symbolic"] = c.symbolic;
        d["upcast"] = c.upcast;
        d["unroll"] = c.unroll;
        return d;
      },
      "This process's OPT setting (read once, at first use).");
  m.def("last_source", []() { return last_source(); });
  m.def("reset_stats", &reset_stats);
  m.def("stats", []() {
    Stats &s = stats();
    py::dict d;
    d["kernels"] = s.kernels;
    d["gemm"] = s.gemm;
    d["hand_reduce"] = s.hand_reduce;
    d["xent"] = s.xent;
    d["xent_reused"] = s.xent_reused;
    d["sgd"] = s.sgd;
    d["gemm_bias"] = s.gemm_bias;
    d["gemm_mask"] = s.gemm_mask;
    d["rendered"] = s.rendered;
    d["compiled"] = s.compiled;
    d["cache_hits"] = s.cache_hits;
    d["schedule_hits"] = s.schedule_hits;
    d["schedule_s"] = s.schedule_s;
    d["run_s"] = s.run_s;
    d["rewrite_s"] = s.rewrite_s;
    return d;
  });
  m.def("interner_size", &interner_size);
  m.def(
      "schedule",
      [](const std::vector<Tensor> &ts, bool with_source) {
        std::vector<UOpP> roots;
        for (const Tensor &t : ts)
          if (!t.is_realized()) roots.push_back(t.uop());
        if (roots.empty()) return py::list();
        return items_summary(schedule_many(roots), with_source);
      },
      py::arg("tensors"), py::arg("with_source") = false,
      "Schedule (without running) the kernels that realize_many(tensors) would run.");

  py::class_<PyUOp>(m, "UOp")
      .def_static("buffer",
                  [](const py::sequence &s, const std::string &dt) {
                    Shape shape = to_shape(s);
                    auto b = std::make_shared<DeviceBuffer>(parse_dtype(dt), (size_t)numel(shape));
                    return PyUOp{make_reshape(make_buffer(b), shape)};
                  },
                  py::arg("shape"), py::arg("dtype") = "f32")
      .def_static("const_int", [](int64_t v) { return PyUOp{make_const((double)v, DType::I32)}; })
      .def_static("add", [](const PyUOp &a, const PyUOp &b) { return PyUOp{make_add(a.u, b.u)}; })
      .def_static("mul", [](const PyUOp &a, const PyUOp &b) { return PyUOp{make_mul(a.u, b.u)}; })
      .def_static("reshape",
                  [](const PyUOp &a, const py::sequence &s) {
                    return PyUOp{make_reshape(a.u, to_shape(s))};
                  })
      .def_static("permute",
                  [](const PyUOp &a, const py::sequence &s) {
                    return PyUOp{make_permute(a.u, to_shape(s))};
                  })
      .def_static("reduce",
                  [](const PyUOp &a, const std::string &op, const py::sequence &axes) {
                    return PyUOp{make_reduce(a.u, op == "max" ? Op::Max : Op::Add, to_shape(axes))};
                  })
      .def_static("shrink",
                  [](const PyUOp &a, const std::vector<PyUOp> &starts, const py::sequence &lens) {
                    std::vector<UOpP> st;
                    for (auto &s : starts) st.push_back(s.u);
                    return PyUOp{make_shrink(a.u, st, to_shape(lens))};
                  })
      .def_static("store",
                  [](const PyUOp &d, const PyUOp &v) { return PyUOp{make_store(d.u, v.u)}; })
      .def_static("after",
                  [](const PyUOp &v, const PyUOp &e) { return PyUOp{make_after(v.u, e.u)}; })
      .def("buffer_id",
           [](const PyUOp &p) -> py::object {
             const UOp *u = p.u.get();
             while (u->op != Op::Buffer && !u->src.empty()) u = u->src[0].get();
             return u->op == Op::Buffer ? py::cast(u->buf->id) : py::none();
           })
      .def("same", [](const PyUOp &a, const PyUOp &b) { return a.u == b.u; })
      .def("dump", [](const PyUOp &a) { return dump(a.u); });

  m.def(
      "schedule_uops",
      [](const std::vector<PyUOp> &roots, bool with_source) {
        std::vector<UOpP> r;
        for (auto &p : roots) r.push_back(p.u);
        return items_summary(schedule_many(r), with_source);
      },
      py::arg("roots"), py::arg("with_source") = false);
}
