// kir.cpp -- nodes, interning, walks and the rewrite engine of the kernel IR
// (TEST INFRASTRUCTURE).  Restates src/uop.rs and src/rewrite.rs of the
// reference.
#include "kir.h"

#include <cmath>
#include <cstring>
#include <sstream>
#include <stdexcept>
#include <unordered_set>

namespace kir {

const char *op_name(Op op) {
  static const char *names[] = {
      "Device", "DefineVar", "Bind", "Buffer", "Shrink", "Reshape", "Permute", "Expand",
      "Contiguous", "ReduceAxis", "ParamBuffer", "ParamScalar", "Range", "End", "Sink", "Index",
      "Load", "Store", "Vectorize", "Unroll", "Contract", "Const", "Neg", "Exp2", "Log2", "Sqrt",
      "Reciprocal", "Add", "Mul", "Max", "CmpLt", "Where", "Reduce", "After", "DefineAcc",
      "Assign", "Gep"};
  return names[(int)op];
}

bool is_alu(Op op) {
  switch (op) {
    case Op::Add: case Op::Mul: case Op::Max: case Op::CmpLt: case Op::Where: case Op::Neg:
    case Op::Exp2: case Op::Log2: case Op::Sqrt: case Op::Reciprocal:
      return true;
    default:
      return false;
  }
}

bool is_movement(Op op) {
  return op == Op::Shrink || op == Op::Reshape || op == Op::Permute || op == Op::Expand;
}

const char *DType::c_type() const {
  switch (kind) {
    case Kind::F32: return "float";
    case Kind::I32: return "int";
    case Kind::Bool: return "_Bool";
    case Kind::Void: return "void";
  }
  return "?";
}

bool Arg::operator==(const Arg &o) const {
  if (tag != o.tag) return false;
  switch (tag) {
    case None: return true;
    case Index: case ParamScalar: case Int: case Bool: return a == o.a;
    case Range: case ParamBuffer: return a == o.a && b == o.b;
    case Float: {
      uint64_t x, y;
      std::memcpy(&x, &f, 8);
      std::memcpy(&y, &o.f, 8);
      return x == y;  // to_bits() equality
    }
    case Bounds: case Shape: case Axes: return v == o.v;
    case Lanes: return lanes == o.lanes;
    case Reduce: return rop == o.rop && v == o.v;
  }
  return false;
}

std::string Arg::str() const {
  std::ostringstream o;
  auto list = [&o](const std::vector<int64_t> &x) {
    o << "[";
    for (size_t i = 0; i < x.size(); i++) o << (i ? ", " : "") << x[i];
    o << "]";
  };
  static const char *kinds[] = {"LOOP", "GLOBAL", "LOCAL", "REDUCE", "GROUP_REDUCE",
                                "UPCAST", "UNROLL", "THREAD"};
  switch (tag) {
    case None: break;
    case Index: o << a; break;
    case Range: o << a << ":" << kinds[b]; break;
    case ParamBuffer: o << "buf_slot=" << a << ",n=" << b; break;
    case ParamScalar: o << "scalar_slot=" << a; break;
    case Float: o << f; break;
    case Int: o << a; break;
    case Bool: o << (a ? "true" : "false"); break;
    case Bounds: case Shape: case Axes: list(v); break;
    case Lanes:
      o << "[";
      for (size_t i = 0; i < lanes.size(); i++)
        o << (i ? ", " : "") << "(" << lanes[i].first << ", " << lanes[i].second << ")";
      o << "]";
      break;
    case Reduce: o << op_name(rop) << "("; list(v); o << ")"; break;
  }
  return o.str();
}

// ---- interning ------------------------------------------------------------
namespace {

std::string node_key(Op op, DType dt, const std::vector<U> &src, const Arg &arg,
                     const std::optional<uint64_t> &tag) {
  std::string k;
  auto put = [&k](const void *p, size_t n) { k.append(static_cast<const char *>(p), n); };
  auto put64 = [&put](int64_t v) { put(&v, 8); };
  put64((int64_t)op | ((int64_t)dt.kind << 8) | ((int64_t)dt.vcount << 16));
  put64((int64_t)src.size());
  for (const U &s : src) {
    const Node *p = s.get();
    put(&p, sizeof(p));
  }
  put64((int64_t)arg.tag);
  put64(arg.a);
  put64(arg.b);
  put(&arg.f, 8);
  put64((int64_t)arg.rop);
  put64((int64_t)arg.v.size());
  for (int64_t x : arg.v) put64(x);
  put64((int64_t)arg.lanes.size());
  for (auto &l : arg.lanes) {
    put64(l.first);
    put64(l.second);
  }
  put64(tag ? 1 : 0);
  put64(tag ? (int64_t)*tag : 0);
  return k;
}

std::unordered_map<std::string, std::weak_ptr<const Node>> &interner() {
  static std::unordered_map<std::string, std::weak_ptr<const Node>> m;
  return m;
}

}  // namespace

U make(Op op, DType dt, std::vector<U> src, Arg arg, std::optional<uint64_t> tag) {
  auto &m = interner();
  std::string key = node_key(op, dt, src, arg, tag);
  auto it = m.find(key);
  if (it != m.end())
    if (U live = it->second.lock()) return live;
  auto n = std::make_shared<Node>();
  n->op = op;
  n->dtype = dt;
  n->src = std::move(src);
  n->arg = std::move(arg);
  n->tag = tag;
  U out = n;
  m[key] = out;
  if (m.size() > 4096 && m.size() % 4096 == 0) {
    for (auto i = m.begin(); i != m.end();) i = i->second.expired() ? m.erase(i) : std::next(i);
  }
  return out;
}

U device() { return make(Op::Device, DType::void_(), {}, Arg::none()); }
U param_buffer(int64_t slot, DType dt, int64_t numel) {
  return make(Op::ParamBuffer, dt, {device()}, Arg::param_buffer(slot, numel));
}
U param_scalar(int64_t slot, DType dt) {
  return make(Op::ParamScalar, dt, {device()}, Arg::param_scalar(slot));
}
U const_float(double v, DType dt) { return make(Op::Const, dt, {device()}, Arg::flt(v)); }
U const_int(int64_t v, DType dt) { return make(Op::Const, dt, {device()}, Arg::integer(v)); }
U const_bool(bool v, DType dt) { return make(Op::Const, dt, {device()}, Arg::boolean(v)); }
U add(const U &a, const U &b) { return make(Op::Add, a->dtype, {a, b}); }
U mul(const U &a, const U &b) { return make(Op::Mul, a->dtype, {a, b}); }
U neg(const U &a) { return make(Op::Neg, a->dtype, {a}); }
U store(const U &dest, const U &value) { return make(Op::Store, DType::void_(), {dest, value}); }
U after(const U &value, const U &effect) { return make(Op::After, value->dtype, {value, effect}); }
U sink(std::vector<U> srcs) { return make(Op::Sink, DType::void_(), std::move(srcs)); }
U gep(const U &x, size_t i) {
  if (x->op == Op::Vectorize) return x->src[i];
  return make(Op::Gep, x->dtype.scalar(), {x}, Arg::integer((int64_t)i));
}
U reshape(const U &s, std::vector<int64_t> shape) {
  return make(Op::Reshape, s->dtype, {s}, Arg::shape(std::move(shape)));
}
U reduce_axis(const U &s, Op rop, std::vector<int64_t> axes) {
  return make(Op::ReduceAxis, s->dtype, {s}, Arg::reduce(rop, std::move(axes)));
}

bool is_const(const U &u) { return u->op == Op::Const; }
bool is_zero(const U &u) {
  return u->op == Op::Const && (u->arg == Arg::flt(0.0) || u->arg == Arg::integer(0));
}
bool is_one(const U &u) {
  return u->op == Op::Const && (u->arg == Arg::flt(1.0) || u->arg == Arg::integer(1));
}
std::optional<int64_t> const_i32(const U &u) {
  if (u->arg.tag != Arg::Int || u->dtype != DType::i32()) return std::nullopt;
  return u->arg.a;
}

std::optional<std::vector<int64_t>> shape_of(const U &u) {
  switch (u->op) {
    case Op::ParamBuffer: return std::vector<int64_t>{u->arg.b};
    case Op::Shrink: case Op::Reshape: case Op::Expand: return u->arg.v;
    case Op::Permute: {
      auto s = shape_of(u->src[0]);
      if (!s) return std::nullopt;
      std::vector<int64_t> r;
      for (int64_t a : u->arg.v) r.push_back((*s)[(size_t)a]);
      return r;
    }
    case Op::ReduceAxis: {
      auto s = shape_of(u->src[0]);
      if (!s) return std::nullopt;
      for (int64_t a : u->arg.v) (*s)[(size_t)a] = 1;
      return s;
    }
    case Op::Const: return std::vector<int64_t>{1};
    case Op::Contiguous: case Op::After: return shape_of(u->src[0]);
    default:
      if (is_alu(u->op)) return shape_of(u->src[0]);
      return std::nullopt;
  }
}

std::vector<U> toposort(const U &root) {
  std::vector<U> out;
  std::unordered_set<const Node *> visited;
  std::vector<std::pair<U, bool>> stack{{root, false}};
  while (!stack.empty()) {
    auto [node, processed] = stack.back();
    stack.pop_back();
    if (visited.count(node.get())) continue;
    if (processed) {
      visited.insert(node.get());
      out.push_back(node);
      continue;
    }
    stack.push_back({node, true});
    if (node->op == Op::After) {
      for (const U &s : node->src)
        if (!visited.count(s.get())) stack.push_back({s, false});
    } else {
      for (auto it = node->src.rbegin(); it != node->src.rend(); ++it)
        if (!visited.count(it->get())) stack.push_back({*it, false});
    }
  }
  return out;
}

std::string dump(const U &root) {
  auto order = toposort(root);
  std::unordered_map<const Node *, size_t> id;
  std::ostringstream o;
  for (size_t i = 0; i < order.size(); i++) {
    const Node &n = *order[i];
    id[&n] = i;
    o << "  %" << i << " = " << op_name(n.op) << " ";
    static const char *kn[] = {"f32", "i32", "bool", "void"};
    o << kn[(int)n.dtype.kind];
    if (n.dtype.vcount != 1) o << "x" << n.dtype.vcount;
    if (!n.src.empty()) {
      o << " (";
      for (size_t j = 0; j < n.src.size(); j++) o << (j ? ", " : "") << "%" << id[n.src[j].get()];
      o << ")";
    }
    if (n.arg.tag != Arg::None) o << "  arg=" << n.arg.str();
    if (n.tag) o << "  tag=" << *n.tag;
    o << "\n";
  }
  return o.str();
}

std::vector<U> ended_ranges(const U &node) {
  if (node->op == Op::End && !node->src.empty()) return {node->src[0]};
  if (node->op == Op::After) {
    std::vector<U> r;
    for (size_t i = 1; i < node->src.size(); i++)
      for (const U &e : ended_ranges(node->src[i])) r.push_back(e);
    return r;
  }
  return {};
}

namespace {
bool g_repair = false;
}  // namespace
void set_repair(bool on) { g_repair = on; }
bool repair() { return g_repair; }
std::optional<uint64_t> rebuilt_tag(const Node &n) { return g_repair ? n.tag : std::nullopt; }

// ---- src/rewrite.rs ---------------------------------------------------------
U graph_rewrite(const U &root, const Rule &rule) {
  U current = root;
  for (;;) {
    auto order = toposort(current);
    std::unordered_map<const Node *, U> replace;
    bool changed = false;
    for (const U &node : order) {
      std::vector<U> srcs;
      srcs.reserve(node->src.size());
      bool srcs_changed = false;
      for (const U &s : node->src) {
        auto f = replace.find(s.get());
        U ns = f != replace.end() ? f->second : s;
        srcs_changed |= ns != s;
        srcs.push_back(ns);
      }
      // a rebuilt node carries no tag (UOp::new)
      U rebuilt = srcs_changed ? make(node->op, node->dtype, std::move(srcs), node->arg,
                                      rebuilt_tag(*node))
                               : node;
      if (U r = rule(rebuilt); r && r != rebuilt) {
        replace[node.get()] = r;
        changed = true;
        continue;
      }
      replace[node.get()] = rebuilt;
    }
    auto f = replace.find(current.get());
    if (f != replace.end()) current = f->second;
    if (!changed) return current;
  }
}

U substitute(const U &root, const std::unordered_map<const Node *, U> &repl) {
  auto order = toposort(root);
  std::unordered_map<const Node *, U> sub;
  for (const U &node : order) {
    if (auto r = repl.find(node.get()); r != repl.end()) {
      sub[node.get()] = r->second;
      continue;
    }
    std::vector<U> srcs;
    bool changed = false;
    for (const U &s : node->src) {
      auto f = sub.find(s.get());
      U ns = f != sub.end() ? f->second : s;
      changed |= ns != s;
      srcs.push_back(ns);
    }
    sub[node.get()] =
        changed ? make(node->op, node->dtype, std::move(srcs), node->arg, rebuilt_tag(*node)) : node;
  }
  auto f = sub.find(root.get());
  return f != sub.end() ? f->second : root;
}

U flatten_end_bodies(const U &node) {
  if (node->op != Op::End || node->src.size() < 2) return nullptr;
  bool changed = false;
  std::vector<U> srcs{node->src[0]};
  for (size_t i = 1; i < node->src.size(); i++) {
    const U &body = node->src[i];
    if (body->op == Op::Sink) {
      changed = true;
      srcs.insert(srcs.end(), body->src.begin(), body->src.end());
      continue;
    }
    srcs.push_back(body);
  }
  return changed ? make(Op::End, DType::void_(), std::move(srcs)) : nullptr;
}

U flatten_nested_sinks(const U &node) {
  if (node->op != Op::Sink) return nullptr;
  bool changed = false;
  std::vector<U> srcs;
  for (const U &s : node->src) {
    if (s->op == Op::Sink) {
      changed = true;
      srcs.insert(srcs.end(), s->src.begin(), s->src.end());
      continue;
    }
    srcs.push_back(s);
  }
  return changed ? sink(std::move(srcs)) : nullptr;
}

}  // namespace kir
