// bridge.cpp -- the front end's scheduled proto-kernels lowered by the
// restated reference pipeline and executed as the reference's C (TEST
// INFRASTRUCTURE).  Python module `_lowering`, built against the front end
// of the host test device (tests/hostdev), where device memory is host
// memory, so the C kernels read and write the front end's buffers in place.
//
// Per scheduled item this follows Tensor::realize_many / execute_item
// (src/tensor.rs:781-898): the proto-kernel Sink(Store(Param(0), expr)) (or
// the in-place Sink(Store(dest, expr))) with buffers and Shrink starts as
// parameters (src/schedule.rs:88-200) -> rangeify -> optimize (the process's
// OPT) -> late_expand -> devectorize -> linearize -> the clang renderer
// (kernel_<n>) -> compile -> execute with the item's inputs.
#include <pybind11/pybind11.h>
#include <pybind11/stl.h>

#include <chrono>
#include <stdexcept>

#include "../../ferrograd_b200/csrc/front/ferro_front.h"
#include "../../ferrograd_b200/csrc/front/front_internal.h"
#include "kir.h"
#include "lowering.h"

namespace py = pybind11;

namespace {

kir::DType kdt(ferro::DType d) {
  switch (d) {
    case ferro::DType::F32: return kir::DType::f32();
    case ferro::DType::I32: return kir::DType::i32();
    case ferro::DType::Bool: return kir::DType::boolean();
  }
  return kir::DType::f32();
}

kir::Op kop(ferro::Op op) {
  switch (op) {
    case ferro::Op::Add: return kir::Op::Add;
    case ferro::Op::Mul: return kir::Op::Mul;
    case ferro::Op::Neg: return kir::Op::Neg;
    case ferro::Op::Reciprocal: return kir::Op::Reciprocal;
    case ferro::Op::Exp2: return kir::Op::Exp2;
    case ferro::Op::Log2: return kir::Op::Log2;
    case ferro::Op::Sqrt: return kir::Op::Sqrt;
    case ferro::Op::Max: return kir::Op::Max;
    case ferro::Op::CmpLt: return kir::Op::CmpLt;
    case ferro::Op::Where: return kir::Op::Where;
    default: throw std::runtime_error(std::string("no kernel op for ") + ferro::op_name(op));
  }
}

// The proto-kernel of one scheduled item in the reference's form.
struct Proto {
  kir::U sink;
  std::vector<ferro::KernelInput> inputs;  // by slot (slot 0 = output when allocating)
};

Proto to_proto(const ferro::ScheduleItem &item) {
  const bool in_place = item.store_dest != nullptr;
  ferro::UOpP root = in_place ? ferro::make_store(item.store_dest, item.value) : item.value;
  ferro::ParamSlots ps = ferro::collect_params(root, in_place ? 0 : 1);
  std::unordered_map<const ferro::UOp *, kir::U> conv;
  for (const ferro::UOpP &n : ferro::toposort(root)) {
    std::vector<kir::U> s;
    for (const ferro::UOpP &x : n->src) s.push_back(conv.at(x.get()));
    const kir::DType dt = kdt(n->dtype);
    kir::U k;
    switch (n->op) {
      case ferro::Op::Buffer:
        k = kir::param_buffer(ps.buffer_slot.at(n->buf.get()), dt, (int64_t)n->buf->count);
        break;
      case ferro::Op::Const:
        k = kir::const_float(n->value, dt);  // UOp::full's literal (const_float)
        break;
      case ferro::Op::Reshape:
        k = kir::make(kir::Op::Reshape, dt, s, kir::Arg::shape(n->arg));
        break;
      case ferro::Op::Expand:
        k = kir::make(kir::Op::Expand, dt, s, kir::Arg::shape(n->arg));
        break;
      case ferro::Op::Permute:
        k = kir::make(kir::Op::Permute, dt, s, kir::Arg::axes(n->arg));
        break;
      case ferro::Op::Shrink: {
        // starts: a parameter slot where the schedule made one, else the
        // literal as const_int (Tensor::narrow's starts)
        const std::vector<int> &slots = ps.shrink_slots.at(n.get());
        std::vector<kir::U> srcs{s[0]};
        for (size_t a = 0; a < slots.size(); a++) {
          const ferro::UOpP &start = n->src[a + 1];
          if (slots[a] >= 0)
            srcs.push_back(kir::param_scalar(slots[a], kdt(start->dtype)));
          else if (start->op == ferro::Op::Const)
            srcs.push_back(kir::const_int((int64_t)start->value, kdt(start->dtype)));
          else
            srcs.push_back(s[a + 1]);
        }
        k = kir::make(kir::Op::Shrink, dt, srcs, kir::Arg::bounds(n->arg));
        break;
      }
      case ferro::Op::Contiguous:
        k = kir::make(kir::Op::Contiguous, dt, s);
        break;
      case ferro::Op::ReduceAxis:
        k = kir::make(kir::Op::ReduceAxis, dt, s,
                      kir::Arg::reduce(n->reduce_op == ferro::Op::Max ? kir::Op::Max : kir::Op::Add,
                                       n->arg));
        break;
      case ferro::Op::Store:
        k = kir::store(s[0], s[1]);
        break;
      default:
        k = kir::make(kop(n->op), dt, s);
        break;
    }
    conv[n.get()] = k;
  }
  Proto p;
  p.inputs = ps.inputs;
  if (in_place) {
    p.sink = kir::sink({conv.at(root.get())});
  } else {
    const int64_t numel = ferro::numel(item.out_shape);
    kir::U out = kir::param_buffer(0, kdt(item.value->dtype), numel);
    p.sink = kir::sink({kir::store(out, conv.at(root.get()))});
  }
  return p;
}

kir::OptimizeConfig opt_config() {
  const ferro::OptimizeConfig &c = ferro::optimize_config();
  kir::OptimizeConfig k;
  k.symbolic = c.symbolic;
  k.upcast = c.upcast;
  k.unroll = c.unroll;
  return k;
}

uint64_t g_kernels = 0, g_launches = 0;
struct Traced {
  std::string code;
  std::vector<uint8_t> out;  // allocating kernels' output bytes
  double seconds;            // the C function's run time
};
std::vector<Traced> g_trace;
bool g_tracing = false;
double g_kernel_seconds = 0;  // time inside the kernels' C functions (and first compiles)

kir::U lower(const kir::U &sink) {
  kir::U r = kir::rangeify(sink);
  kir::U o = kir::optimize(r, opt_config());
  kir::U e = kir::late_expand(o);
  return kir::devectorize(e);
}

std::string lower_to_c(const kir::U &sink, const std::string &name) {
  return kir::render_c(kir::linearize(lower(sink)), name);
}

// Programs by lowered sink, as the reference's backend caches them
// (cached_program / insert_program, src/tensor.rs:838-890): the entry holds
// the sink, so an identical kernel of a later step interns to the same node;
// a hit skips linearize, render and compile and keeps the first name.
struct Program {
  kir::U sink;
  std::string code, name;
};
std::unordered_map<const kir::Node *, Program> &programs() {
  static std::unordered_map<const kir::Node *, Program> p;
  return p;
}

// Tensor::realize_many (src/tensor.rs:781-821) with every kernel lowered and
// run as the reference's C.
void realize(const std::vector<ferro::Tensor> &ts) {
  std::vector<ferro::UOpP> roots;
  for (const ferro::Tensor &t : ts)
    if (!t.is_realized()) roots.push_back(t.uop());
  if (roots.empty()) return;
  ferro::SchedulePlan plan = ferro::schedule_many(roots, true);
  for (const ferro::ScheduleItem &item : plan.items) {
    Proto p = to_proto(item);
    kir::U lowered = lower(p.sink);
    auto hit = programs().find(lowered.get());
    if (hit == programs().end()) {
      const std::string nm = "kernel_" + std::to_string(g_kernels++);
      hit = programs()
                .emplace(lowered.get(),
                         Program{lowered, kir::render_c(kir::linearize(lowered), nm), nm})
                .first;
    }
    const std::string &name = hit->second.name;
    const std::string &code = hit->second.code;
    std::vector<int32_t> i32(p.inputs.size() + 1);
    std::vector<float> f32(p.inputs.size() + 1);
    std::vector<uint8_t> b8(p.inputs.size() + 1);
    std::vector<void *> args;
    if (!item.store_dest) args.push_back(item.output->ptr());
    for (size_t i = 0; i < p.inputs.size(); i++) {
      const ferro::KernelInput &in = p.inputs[i];
      switch (in.kind) {
        case ferro::KernelInput::Buffer: args.push_back(in.buffer->ptr()); break;
        case ferro::KernelInput::I32: i32[i] = (int32_t)in.i; args.push_back(&i32[i]); break;
        case ferro::KernelInput::F32: f32[i] = (float)in.f; args.push_back(&f32[i]); break;
        case ferro::KernelInput::Bool: b8[i] = (uint8_t)in.i; args.push_back(&b8[i]); break;
      }
    }
    const auto k0 = std::chrono::steady_clock::now();
    kir::run_c(code, name, args);  // compiles on first use
    g_kernel_seconds +=
        std::chrono::duration<double>(std::chrono::steady_clock::now() - k0).count();
    double secs = 0;
    if (g_tracing) {  // a second, timed run (kernels are idempotent for their outputs
                      // unless in place; in-place ones are timed on the first run)
      if (!item.store_dest) {
        const auto t0 = std::chrono::steady_clock::now();
        kir::run_c(code, name, args);
        secs = std::chrono::duration<double>(std::chrono::steady_clock::now() - t0).count();
      }
    }
    g_launches++;
    if (g_tracing)
      g_trace.push_back({code, item.output ? item.output->to_host() : std::vector<uint8_t>{}, secs});
    if (item.store_dest) {
      const ferro::UOp *d = item.store_dest.get();
      while (d->op != ferro::Op::Buffer && !d->src.empty()) d = d->src[0].get();
      if (d->op == ferro::Op::Buffer) d->buf->version++;
    }
  }
  ferro::Tensor::apply_map_to_tensors(plan.replacements);
}

// The C of each kernel realize_many(ts) would run, without running them.
std::vector<std::string> sources(const std::vector<ferro::Tensor> &ts) {
  std::vector<ferro::UOpP> roots;
  for (const ferro::Tensor &t : ts)
    if (!t.is_realized()) roots.push_back(t.uop());
  std::vector<std::string> out;
  if (roots.empty()) return out;
  ferro::SchedulePlan plan = ferro::schedule_many(roots, true);
  for (size_t i = 0; i < plan.items.size(); i++)
    out.push_back(lower_to_c(to_proto(plan.items[i]).sink, "kernel_" + std::to_string(i)));
  return out;
}

}  // namespace

PYBIND11_MODULE(_lowering, m) {
  m.doc() = "The reference's CPU lowering restated (test infrastructure)";
  m.def("realize", &realize, py::arg("tensors"),
        "Realize tensors with every kernel lowered to the reference's C and run on the CPU.");
  m.def("sources", &sources, py::arg("tensors"),
        "The reference's C of each kernel realizing `tensors` would run.");
  m.def("set_repair", &kir::set_repair, py::arg("on"),
        "Keep tags across rebuilds and group reduce lanes by axis (not the reference's "
        "behaviour; see kir.h).");
  m.def("trace", [](bool on) {
          g_tracing = on;
          g_trace.clear();
        }, py::arg("on"),
        "Record each allocating kernel's C and output bytes from now on.");
  m.def("traced", []() {
    py::list l;
    for (auto &t : g_trace)
      l.append(py::make_tuple(t.code, py::bytes((const char *)t.out.data(), t.out.size()),
                              t.seconds));
    return l;
  });
  m.def("kernel_seconds", [](bool reset) {
          const double s = g_kernel_seconds;
          if (reset) g_kernel_seconds = 0;
          return s;
        }, py::arg("reset"),
        "Seconds spent in run_c (the kernels' C, and compiles on first use) since the last reset.");
  m.def("stats", []() {
    py::dict d;
    d["kernels"] = g_kernels;
    d["launches"] = g_launches;
    return d;
  });
  m.def("case_names", []() {
    std::vector<std::string> n;
    for (auto &c : kir::structure_cases()) n.push_back(c.name);
    return n;
  });
  m.def("run_case", [](const std::string &name) {
    for (auto &c : kir::structure_cases())
      if (c.name == name) {
        c.fn();
        return;
      }
    throw std::runtime_error("no case " + name);
  });
}
