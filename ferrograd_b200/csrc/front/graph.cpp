// graph.cpp -- interned UOp graph nodes (src/uop.rs), reverse-mode gradient
// rules (src/gradient.rs) and the kernel scheduler (src/schedule.rs).
#include <algorithm>
#include <cstdlib>
#include <cstring>
#include <functional>
#include <sstream>
#include <stdexcept>
#include <unordered_map>
#include <unordered_set>

#include "ferro_front.h"
#include "front_internal.h"

namespace ferro {

int64_t numel(const Shape &s) {
  int64_t n = 1;
  for (int64_t d : s) n *= d;
  return n;
}

std::string shape_str(const Shape &s) {
  std::ostringstream o;
  o << "[";
  for (size_t i = 0; i < s.size(); i++) o << (i ? ", " : "") << s[i];
  o << "]";
  return o.str();
}

size_t dtype_size(DType d) { return d == DType::Bool ? 1 : 4; }

const char *dtype_name(DType d) {
  switch (d) {
    case DType::F32: return "f32";
    case DType::I32: return "i32";
    case DType::Bool: return "bool";
  }
  return "?";
}

const char *op_name(Op op) {
  static const char *names[] = {"Buffer", "Const", "Reshape", "Permute", "Expand", "Shrink",
                                "Contiguous", "Add", "Mul", "Neg", "Reciprocal", "Exp2", "Log2",
                                "Sqrt", "Max", "CmpLt", "Where", "ReduceAxis", "Store", "After",
                                "Sink", "XentLoss", "XentGrad"};
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

// ---------------------------------------------------------------------------
// Interning (src/uop.rs:536-570): a node is looked up by (op, dtype, source
// identities, arg, literal, buffer identity).  The table is an open-addressing
// set of live nodes (linear probing, power-of-two size, at most half full)
// keyed by the hash of those fields; a lookup compares the candidates' own
// fields, so it allocates nothing.  A node leaves the table in its destructor
// (backward-shift deletion, no tombstones), so the table holds live nodes
// only and its entries need no reference counts.  Sources of a live node are
// alive (the node owns them), so comparing source pointers is sound.
namespace {

uint64_t node_hash(Op op, DType dt, Op rop, uint64_t vbits, const DeviceBuffer *buf,
                   const std::vector<UOpP> &srcs, const std::vector<int64_t> &arg) {
  uint64_t h = 1469598103934665603ULL;
  auto mix = [&h](uint64_t v) { h = (h ^ v) * 1099511628211ULL; };
  mix((uint64_t)op);
  mix((uint64_t)dt);
  mix((uint64_t)(op == Op::ReduceAxis ? (int)rop : 0));
  mix(vbits);
  mix((uint64_t)(uintptr_t)buf);
  for (auto &p : srcs) mix((uint64_t)(uintptr_t)p.get());
  for (auto a : arg) mix((uint64_t)a);
  return h ^ (h >> 31);
}

bool same_node(const UOp &u, Op op, DType dt, Op rop, uint64_t vbits, const DeviceBuffer *buf,
               const std::vector<UOpP> &srcs, const std::vector<int64_t> &arg) {
  if (u.op != op || u.dtype != dt || u.buf.get() != buf || u.src.size() != srcs.size())
    return false;
  if (op == Op::ReduceAxis && u.reduce_op != rop) return false;
  uint64_t ub;
  std::memcpy(&ub, &u.value, sizeof(ub));
  if (ub != vbits) return false;
  for (size_t i = 0; i < srcs.size(); i++)
    if (u.src[i].get() != srcs[i].get()) return false;
  return u.arg == arg;
}

struct InternTable {
  struct Slot {
    uint64_t h;
    UOp *p;  // null: empty
  };
  std::vector<Slot> slots = std::vector<Slot>(1024, Slot{0, nullptr});
  size_t count = 0;

  size_t mask() const { return slots.size() - 1; }
  void place(uint64_t h, UOp *p) {
    size_t i = h & mask();
    while (slots[i].p) i = (i + 1) & mask();
    slots[i] = {h, p};
  }
  void insert(uint64_t h, UOp *p) {
    if (2 * (count + 1) > slots.size()) {
      std::vector<Slot> old(slots.size() * 2, Slot{0, nullptr});
      old.swap(slots);
      for (const Slot &s : old)
        if (s.p) place(s.h, s.p);
    }
    place(h, p);
    count++;
  }
  void erase(uint64_t h, const UOp *p) {
    size_t i = h & mask();
    while (slots[i].p != p) {
      if (!slots[i].p) return;
      i = (i + 1) & mask();
    }
    // backward shift: move later entries of the probe run into the hole
    // unless their home slot lies cyclically in (hole, entry]
    size_t j = i;
    for (;;) {
      j = (j + 1) & mask();
      if (!slots[j].p) break;
      const size_t k = slots[j].h & mask();
      const bool stays = i <= j ? (i < k && k <= j) : (i < k || k <= j);
      if (stays) continue;
      slots[i] = slots[j];
      i = j;
    }
    slots[i] = Slot{0, nullptr};
    count--;
  }
};

// Never destroyed: nodes held by other static objects may be destroyed
// after this file's statics at exit, and their destructors still use it.
InternTable &interner() {
  static InternTable *t = new InternTable;
  return *t;
}
uint64_t g_uid = 0;

void infer_shape(UOp &u) {
  switch (u.op) {
    case Op::Buffer:
      u.has_shape = true;
      u.shape = {(int64_t)u.buf->count};
      return;
    case Op::Shrink:
    case Op::Reshape:
    case Op::Expand:
      u.has_shape = true;
      u.shape = u.arg;
      return;
    case Op::Permute: {
      const UOp &s = *u.src[0];
      if (!s.has_shape) return;
      u.has_shape = true;
      for (int64_t a : u.arg) u.shape.push_back(s.shape[(size_t)a]);
      return;
    }
    case Op::ReduceAxis: {
      const UOp &s = *u.src[0];
      if (!s.has_shape) return;
      u.has_shape = true;
      u.shape = s.shape;
      for (int64_t a : u.arg) u.shape[(size_t)a] = 1;
      return;
    }
    case Op::Const:
      u.has_shape = true;
      u.shape = {1};
      return;
    case Op::Contiguous:
    case Op::After:
      u.has_shape = u.src[0]->has_shape;
      u.shape = u.src[0]->shape;
      return;
    case Op::Store:
    case Op::Sink:
      return;
    case Op::XentLoss:
      // the reference's loss keeps every axis as 1 ([1, 1] for rank-2 logits)
      u.has_shape = u.src[0]->has_shape;
      u.shape = Shape(u.src[0]->shape.size(), 1);
      return;
    case Op::XentGrad:
      u.has_shape = u.src[0]->has_shape;
      u.shape = u.src[0]->shape;
      return;
    default:
      if (is_alu(u.op)) {
        u.has_shape = u.src[0]->has_shape;
        u.shape = u.src[0]->shape;
      }
      return;
  }
}

const std::vector<int64_t> kNoArg;

UOpP intern(Op op, DType dt, std::vector<UOpP> srcs, const std::vector<int64_t> &arg = kNoArg,
            Op rop = Op::Add, double value = 0.0, const BufferP &buf = nullptr) {
  uint64_t vbits;
  std::memcpy(&vbits, &value, sizeof(double));
  const uint64_t h = node_hash(op, dt, rop, vbits, buf.get(), srcs, arg);
  InternTable &t = interner();
  for (size_t i = h & t.mask(); t.slots[i].p; i = (i + 1) & t.mask())
    if (t.slots[i].h == h && same_node(*t.slots[i].p, op, dt, rop, vbits, buf.get(), srcs, arg))
      return t.slots[i].p->shared_from_this();
  auto u = std::make_shared<UOp>();
  u->op = op;
  u->dtype = dt;
  u->src = std::move(srcs);
  u->arg = arg;
  u->reduce_op = op == Op::ReduceAxis ? rop : Op::Add;
  u->value = value;
  u->buf = buf;
  u->uid = g_uid++;
  infer_shape(*u);
  u->intern_hash = h;
  u->interned = true;
  t.insert(h, u.get());
  return u;
}

}  // namespace

UOp::~UOp() {
  if (interned) interner().erase(intern_hash, this);
}

size_t interner_size() { return interner().count; }

UOpP make_buffer(const BufferP &b) { return intern(Op::Buffer, b->dtype, {}, {}, Op::Add, 0.0, b); }
UOpP make_const(double v, DType dt) { return intern(Op::Const, dt, {}, {}, Op::Add, v); }
UOpP make_reshape(const UOpP &s, const Shape &shape) {
  // A reshape views the same elements: a count that differs would make every
  // kernel that reads the node index past its source.
  if (s->has_shape && numel(s->shape) != numel(shape))
    throw Panic("reshape: numel mismatch for " + shape_str(s->shape) + " -> " + shape_str(shape));
  return intern(Op::Reshape, s->dtype, {s}, shape);
}
UOpP make_permute(const UOpP &s, const std::vector<int64_t> &order) {
  return intern(Op::Permute, s->dtype, {s}, order);
}
UOpP make_expand(const UOpP &s, const Shape &shape) {
  return intern(Op::Expand, s->dtype, {s}, shape);
}
UOpP make_shrink(const UOpP &s, const std::vector<UOpP> &starts, const Shape &lengths) {
  std::vector<UOpP> srcs{s};
  srcs.insert(srcs.end(), starts.begin(), starts.end());
  return intern(Op::Shrink, s->dtype, std::move(srcs), lengths);
}
UOpP make_contiguous(const UOpP &s) { return intern(Op::Contiguous, s->dtype, {s}); }
UOpP make_alu(Op op, DType dt, std::vector<UOpP> srcs) { return intern(op, dt, std::move(srcs)); }
UOpP make_add(const UOpP &a, const UOpP &b) { return intern(Op::Add, a->dtype, {a, b}); }
UOpP make_mul(const UOpP &a, const UOpP &b) { return intern(Op::Mul, a->dtype, {a, b}); }
UOpP make_neg(const UOpP &a) { return intern(Op::Neg, a->dtype, {a}); }
UOpP make_reciprocal(const UOpP &a) { return intern(Op::Reciprocal, a->dtype, {a}); }
UOpP make_cmplt(const UOpP &a, const UOpP &b) { return intern(Op::CmpLt, DType::Bool, {a, b}); }
UOpP make_where(const UOpP &c, const UOpP &t, const UOpP &f) {
  return intern(Op::Where, t->dtype, {c, t, f});
}
UOpP make_reduce(const UOpP &s, Op rop, const std::vector<int64_t> &axes) {
  return intern(Op::ReduceAxis, s->dtype, {s}, axes, rop);
}
UOpP make_store(const UOpP &dest, const UOpP &value) {
  return intern(Op::Store, dest->dtype, {dest, value});
}
UOpP make_after(const UOpP &value, const UOpP &effect) {
  return intern(Op::After, value->dtype, {value, effect});
}
UOpP make_sink(const std::vector<UOpP> &srcs) { return intern(Op::Sink, DType::F32, srcs); }
UOpP make_xent_loss(const UOpP &logits, const UOpP &targets) {
  return intern(Op::XentLoss, DType::F32, {logits, targets});
}
UOpP make_xent_grad(const UOpP &logits, const UOpP &targets) {
  return intern(Op::XentGrad, DType::F32, {logits, targets});
}

UOpP make_full(const Shape &shape, DType dt, double value) {
  Shape base(shape.size(), 1);
  UOpP b = make_reshape(make_const(value, dt), base);
  bool all_one = std::all_of(shape.begin(), shape.end(), [](int64_t d) { return d == 1; });
  return all_one ? b : make_expand(b, shape);
}

bool has_buffer_identity(const UOp *u) {
  if (u->op == Op::Buffer) return true;
  if (u->op == Op::After || is_movement(u->op)) return has_buffer_identity(u->src[0].get());
  return false;
}

// A fresh walk number for the visited stamps (UOp::walk_mark), shared by
// every walker so two walks never use the same number.
static uint64_t new_walk() {
  static uint64_t walks = 0;
  return ++walks;
}

std::vector<UOpP> toposort(const UOpP &root) {
  // Iterative post-order DFS.  Sources are pushed in reverse so the first
  // source is finished first; After walks its effect last-pushed-first
  // (src/uop.rs:1044-1074).  The stack holds pointers to the handles inside
  // the (immutable) parents, so a node's handle is copied once, into `out`.
  const uint64_t mark = new_walk();
  auto visited = [mark](const UOp *n) { return n->walk_mark == mark; };
  std::vector<UOpP> out;
  out.reserve(64);
  // the stack's storage is kept across calls (no walk runs inside another)
  static std::vector<std::pair<const UOpP *, bool>> stack;
  stack.clear();
  stack.push_back({&root, false});
  while (!stack.empty()) {
    auto [hp, processed] = stack.back();
    stack.pop_back();
    const UOp *node = hp->get();
    if (visited(node)) continue;
    if (processed) {
      node->walk_mark = mark;
      out.push_back(*hp);
      continue;
    }
    stack.push_back({hp, true});
    if (node->op == Op::After) {
      for (auto &s : node->src)
        if (!visited(s.get())) stack.push_back({&s, false});
    } else {
      for (auto it = node->src.rbegin(); it != node->src.rend(); ++it)
        if (!visited(it->get())) stack.push_back({&*it, false});
    }
  }
  return out;
}

std::vector<const UOp *> toposort_nodes(const UOp *root) {
  // The same walk and order as toposort, over plain pointers: for walkers
  // that only read the nodes (no handle copies, no reference counting).
  const uint64_t mark = new_walk();
  std::vector<const UOp *> out;
  out.reserve(64);
  static std::vector<std::pair<const UOp *, bool>> stack;
  const size_t base = stack.size();  // callers may walk inside a walk's loop
  stack.push_back({root, false});
  while (stack.size() > base) {
    auto [node, processed] = stack.back();
    stack.pop_back();
    if (node->walk_mark == mark) continue;
    if (processed) {
      node->walk_mark = mark;
      out.push_back(node);
      continue;
    }
    stack.push_back({node, true});
    if (node->op == Op::After) {
      for (auto &s : node->src)
        if (s->walk_mark != mark) stack.push_back({s.get(), false});
    } else {
      for (auto it = node->src.rbegin(); it != node->src.rend(); ++it)
        if ((*it)->walk_mark != mark) stack.push_back({it->get(), false});
    }
  }
  return out;
}

std::string dump(const UOpP &root) {
  auto order = toposort(root);
  std::unordered_map<const UOp *, size_t> idx;
  std::ostringstream o;
  for (size_t i = 0; i < order.size(); i++) {
    const UOp *u = order[i].get();
    idx[u] = i;
    o << "%" << i << " = " << op_name(u->op) << " " << dtype_name(u->dtype);
    if (u->has_shape) o << " " << shape_str(u->shape);
    if (!u->src.empty()) {
      o << " (";
      for (size_t j = 0; j < u->src.size(); j++) o << (j ? ", " : "") << "%" << idx[u->src[j].get()];
      o << ")";
    }
    if (u->op == Op::Const) o << " value=" << u->value;
    if (u->op == Op::Buffer) o << " buf#" << u->buf->id << "[" << u->buf->count << "]";
    if (u->op == Op::ReduceAxis) o << " " << op_name(u->reduce_op) << shape_str(u->arg);
    if (u->op == Op::Permute || u->op == Op::Reshape || u->op == Op::Expand ||
        u->op == Op::Shrink)
      o << " arg=" << shape_str(u->arg);
    o << "\n";
  }
  return o.str();
}

// ---------------------------------------------------------------------------
// Gradient rules (src/gradient.rs:97-205).
namespace {

std::unordered_map<const UOp *, std::vector<const UOp *>> consumer_map(
    const std::vector<UOpP> &order) {
  std::unordered_map<const UOp *, std::vector<const UOp *>> m;
  m.reserve(order.size());
  for (auto &n : order)
    for (auto &s : n->src) m[s.get()].push_back(n.get());
  return m;
}

UOpP const_like(const UOp *node, double v) { return make_const(v, node->dtype); }

UOpP zero_like(const UOp *node) {
  Shape s = node->has_shape ? node->shape : Shape{1};
  return make_full(s, node->dtype, 0.0);
}

std::vector<UOpP> gradient_for_op(const UOpP &nodep, const UOpP &grad) {
  const UOp *node = nodep.get();
  switch (node->op) {
    case Op::Add:
      return {grad, grad};
    case Op::Mul:
      return {make_mul(node->src[1], grad), make_mul(node->src[0], grad)};
    case Op::Neg:
      return {make_neg(grad)};
    case Op::Reciprocal:
      return {make_mul(make_neg(grad), make_mul(nodep, nodep))};
    case Op::Exp2:
      return {make_mul(make_mul(nodep, const_like(node, 0.6931471805599453)), grad)};
    case Op::Log2:
      return {make_mul(grad, make_reciprocal(make_mul(node->src[0],
                                                      const_like(node, 0.6931471805599453))))};
    case Op::Sqrt:
      return {make_mul(grad, make_reciprocal(make_mul(const_like(node, 2.0), nodep)))};
    case Op::Max: {
      const UOpP &x = node->src[0], &y = node->src[1];
      UOpP zero = const_like(node, 0.0);
      UOpP half = make_mul(grad, const_like(node, 0.5));
      UOpP x_wins = make_cmplt(y, x), y_wins = make_cmplt(x, y);
      UOpP x_grad = make_where(x_wins, grad, make_where(y_wins, zero, half));
      UOpP y_grad = make_where(y_wins, grad, make_where(x_wins, zero, half));
      return {x_grad, y_grad};
    }
    case Op::CmpLt:
      return {nullptr, nullptr};
    case Op::Where: {
      UOpP zero = const_like(node, 0.0);
      return {nullptr, make_where(node->src[0], grad, zero), make_where(node->src[0], zero, grad)};
    }
    case Op::Reshape:
      return {make_reshape(grad, node->src[0]->shape)};
    case Op::Permute: {
      std::vector<int64_t> inv(node->arg.size());
      for (size_t i = 0; i < node->arg.size(); i++) inv[(size_t)node->arg[i]] = (int64_t)i;
      return {make_permute(grad, inv)};
    }
    case Op::Expand: {
      // Summed over the broadcast axes (src/gradient.rs:165-176).  The
      // reference's axis test (src/shape.rs:93-101) takes dst > 1; an axis of
      // 1 expanded to 0 is reduced here too (its gradient is the sum over
      // nothing, 0), because left out it would hand the Reshape rule below a
      // gradient with 0 elements to view as the source's shape, a kernel that
      // reads past the end of its buffer.
      const Shape &src = node->src[0]->shape;
      std::vector<int64_t> axes;
      for (size_t a = 0; a < src.size(); a++)
        if (src[a] == 1 && node->arg[a] != 1) axes.push_back((int64_t)a);
      if (axes.empty()) return {grad};
      return {make_reduce(grad, Op::Add, axes)};
    }
    case Op::Contiguous:
      return {grad};
    case Op::ReduceAxis: {
      const UOpP &src = node->src[0];
      const Shape &ss = src->shape;
      if (node->reduce_op == Op::Add) return {make_expand(grad, ss)};
      UOpP max_e = make_expand(nodep, ss);
      UOpP grad_e = make_expand(grad, ss);
      UOpP is_not_max = make_cmplt(src, max_e);
      UOpP mask = make_where(is_not_max, make_const(0.0, grad->dtype), make_const(1.0, grad->dtype));
      UOpP count = make_reduce(mask, Op::Add, node->arg);
      UOpP weighted = make_mul(mask, make_reciprocal(make_expand(count, ss)));
      return {make_mul(weighted, grad_e)};
    }
    case Op::XentLoss: {
      // d loss / d logits scaled by the incoming gradient (one value); the
      // plain loss.backward() seed 1.0 needs no scaling.  The targets get no
      // gradient: the front end fuses only when they do not require one.
      UOpP d = make_xent_grad(node->src[0], node->src[1]);
      const UOp *g = grad.get();
      while (g->op == Op::Reshape || g->op == Op::Expand) g = g->src[0].get();
      if (g->op == Op::Const && g->value == 1.0) return {d, nullptr};
      const Shape &ls = node->src[0]->shape;
      UOpP ge = make_expand(make_reshape(grad, Shape(ls.size(), 1)), ls);
      return {make_mul(d, ge), nullptr};
    }
    case Op::Buffer:
    case Op::Const:
      return {};
    default:
      throw Panic(std::string("gradient not implemented for ") + op_name(node->op));
  }
}

}  // namespace

std::map<const UOp *, UOpP> compute_gradient(const UOpP &root, const UOpP &root_grad,
                                             const std::vector<UOpP> &targets) {
  // Per-node state lives in vectors indexed by toposort position
  // (UOp::topo_pos), so the walk does no hash lookups.
  const std::vector<const UOp *> order = toposort_nodes(root.get());
  const size_t n = order.size();
  if (n == 0) throw Panic("compute_gradient: empty graph");
  for (size_t i = 0; i < n; i++) order[i]->topo_pos = (int64_t)i;
  auto pos_of = [&](const UOp *u) -> int64_t {
    const int64_t p = u->topo_pos;
    return p >= 0 && (size_t)p < n && order[(size_t)p] == u ? p : -1;
  };
  // needed_nodes (src/gradient.rs:64-81): the nodes on a path from a target
  // up to the root -- a node is needed when it is a target or one of its
  // sources is needed, decided in one pass in toposort order.
  std::vector<char> needed(n, 0);
  for (auto &t : targets)
    if (int64_t p = pos_of(t.get()); p >= 0) needed[(size_t)p] = 1;
  for (size_t i = 0; i < n; i++) {
    if (needed[i]) continue;
    for (const UOpP &s : order[i]->src)
      if (needed[(size_t)s->topo_pos]) {
        needed[i] = 1;
        break;
      }
  }
  needed[n - 1] = 1;  // the root

  std::vector<UOpP> grads(n);
  grads[n - 1] = root_grad;
  for (size_t k = n; k-- > 0;) {
    if (!needed[k] || !grads[k]) continue;
    const UOpP node = order[k]->shared_from_this();
    auto local = gradient_for_op(node, grads[k]);
    for (size_t i = 0; i < node->src.size() && i < local.size(); i++) {
      if (!local[i]) continue;
      const size_t sp = (size_t)node->src[i]->topo_pos;
      if (!needed[sp]) continue;
      grads[sp] = grads[sp] ? make_add(grads[sp], local[i]) : local[i];
    }
  }
  std::map<const UOp *, UOpP> result;
  for (auto &t : targets) {
    const int64_t p = pos_of(t.get());
    result[t.get()] = p >= 0 && grads[(size_t)p] ? grads[(size_t)p] : zero_like(t.get());
  }
  return result;
}

// ---------------------------------------------------------------------------
// Scheduling (src/schedule.rs:64-365).
namespace {

using ReplMap = std::map<const UOp *, UOpP>;

// Chained reductions: every node below a ReduceAxis (src/schedule.rs:264-272).
std::unordered_set<const UOp *> nested_reduce_inputs(const std::vector<UOpP> &order) {
  std::unordered_set<const UOp *> feeds;
  for (auto it = order.rbegin(); it != order.rend(); ++it) {
    const UOp *n = it->get();
    if (n->op == Op::ReduceAxis || feeds.count(n))
      for (auto &s : n->src) feeds.insert(s.get());
  }
  return feeds;
}

bool should_materialize(const UOp *node, const std::unordered_set<const UOp *> &roots,
                        const std::unordered_map<const UOp *, std::vector<const UOp *>> &consumers,
                        const std::unordered_set<const UOp *> &nested) {
  if (roots.count(node) || !node->has_shape) return false;
  switch (node->op) {
    case Op::Sink: case Op::Store: case Op::After: case Op::Buffer: case Op::Const:
      return false;
    default:
      break;
  }
  if (node->op == Op::Contiguous) {
    // Default mode: a contiguous() of what is already a contiguous view of a
    // buffer (Linear's W.permute().permute().contiguous() inside matmul,
    // src/tensor.rs:770-774) is that view; the copy would be bit-identical.
    if (!exact_mode()) {
      auto v = try_view(node->src[0].get());
      if (v) {
        int64_t st = 1;
        bool contig = true;
        for (size_t a = v->shape.size(); a-- > 0;) {
          if (v->shape[a] != 1 && v->strides[a] != st) contig = false;
          st *= v->shape[a];
        }
        if (contig) return false;
      }
    }
    return true;
  }
  // the fused cross-entropy ops are kernels of their own
  if (node->op == Op::XentLoss || node->op == Op::XentGrad) return true;
  if (is_movement(node->op)) return false;
  if (has_buffer_identity(node)) return false;
  auto it = consumers.find(node);
  if (it != consumers.end() && it->second.size() > 1) return true;
  // the fused cross-entropy reads its operands from memory: compute them in
  // kernels of their own (routed like any other: the logits' contraction
  // still reaches the GEMM)
  if (it != consumers.end() &&
      std::any_of(it->second.begin(), it->second.end(), [](const UOp *c) {
        return c->op == Op::XentLoss || c->op == Op::XentGrad;
      }))
    return true;
  if (node->op == Op::ReduceAxis && it != consumers.end() &&
      std::any_of(it->second.begin(), it->second.end(),
                  [](const UOp *c) { return is_alu(c->op); }))
    return true;
  return node->op == Op::ReduceAxis && nested.count(node);
}

// Default-mode fusion (not in the reference, which materialises every node
// with two or more consumers, src/schedule.rs:303-335): an elementwise node
// whose value involves no reduction, whose consumers are all elementwise ops
// at its own coordinates, and whose consumers all end up in the same kernel
// is recomputed inside that kernel instead of being written out and read
// back.  Its value is the same either way (one correctly rounded op per
// node), so only HBM traffic changes: relu(a*b+c) is one kernel, not two.
// Kernel membership is found from the roots down: a node that is not
// materialised belongs to the kernel of its consumers when they agree.
std::unordered_set<const UOp *> fusible_shared_nodes(
    const std::vector<UOpP> &order, const std::unordered_set<const UOp *> &roots,
    const std::unordered_map<const UOp *, std::vector<const UOp *>> &consumers,
    const std::unordered_set<const UOp *> &nested) {
  std::unordered_set<const UOp *> fused;
  if (exact_mode()) return fused;
  std::unordered_map<const UOp *, bool> has_reduce;
  for (auto &n : order) {
    bool r = n->op == Op::ReduceAxis;
    for (auto &s : n->src) r = r || has_reduce[s.get()];
    has_reduce[n.get()] = r;
  }
  // kernel[n]: the node whose kernel computes n (itself when materialised);
  // nullptr when its consumers lie in different kernels
  std::unordered_map<const UOp *, const UOp *> kernel;
  for (auto it = order.rbegin(); it != order.rend(); ++it) {
    const UOp *n = it->get();
    auto c = consumers.find(n);
    const std::vector<const UOp *> none;
    const std::vector<const UOp *> &cs = c != consumers.end() ? c->second : none;
    const UOp *common = nullptr;
    bool agree = !cs.empty();
    for (size_t i = 0; i < cs.size(); i++) {
      auto k = kernel.find(cs[i]);
      const UOp *kc = k != kernel.end() ? k->second : nullptr;
      if (!kc || (i > 0 && kc != common)) agree = false;
      common = kc;
    }
    bool mat = roots.count(n) || should_materialize(n, roots, consumers, nested);
    if (mat && cs.size() > 1 && agree && is_alu(n->op) && !has_reduce[n] && !roots.count(n) &&
        std::all_of(cs.begin(), cs.end(), [](const UOp *u) { return is_alu(u->op); })) {
      fused.insert(n);
      mat = false;
    }
    kernel[n] = mat || cs.empty() ? n : (agree ? common : nullptr);
  }
  return fused;
}

// Default-mode fusion of Linear::forward (src/nn.rs:97-104): the
// contraction of x.matmul(W^T) is materialised by the chained-reduction rule
// (its value feeds the next layer's reductions), and the bias add that
// consumes it becomes a second kernel.  When the contraction's only use is
// that add (through matmul's reshape) and the add is a kernel boundary
// itself, the contraction is computed inside the add's kernel instead (the
// GEMM's bias epilogue), the same values in one pass.
std::unordered_set<const UOp *> bias_fused_contractions(
    const std::vector<UOpP> &order, const std::unordered_set<const UOp *> &roots,
    const std::unordered_map<const UOp *, std::vector<const UOp *>> &consumers,
    const std::unordered_set<const UOp *> &nested) {
  std::unordered_set<const UOp *> fused;
  if (exact_mode()) return fused;
  auto only = [&](const UOp *n) -> const UOp * {
    auto it = consumers.find(n);
    return it != consumers.end() && it->second.size() == 1 ? it->second[0] : nullptr;
  };
  auto contraction_via = [&](const UOp *x, const UOp *a) -> const UOp * {
    if (x->op != Op::Reshape || only(x) != a) return nullptr;
    const UOp *r = x->src[0].get();
    if (r->op != Op::ReduceAxis || r->reduce_op != Op::Add || r->arg.size() != 1 ||
        r->src[0]->op != Op::Mul || r->shape.size() != 3 || only(r) != x)
      return nullptr;
    return r;
  };
  for (auto &np : order) {
    const UOp *a = np.get();
    // ReLU's gradient where(0 < z, dX, 0) keeps its dX contraction as well
    // (the GEMM's mask epilogue; the executor checks the literal zeros)
    if (a->op == Op::Where && a->dtype == DType::F32 && a->shape.size() == 2 &&
        a->src[0]->op == Op::CmpLt &&
        (roots.count(a) || should_materialize(a, roots, consumers, nested)))
      if (const UOp *r = contraction_via(a->src[1].get(), a)) fused.insert(r);
    if (a->op != Op::Add || a->dtype != DType::F32 || a->shape.size() != 2) continue;
    if (!roots.count(a) && !should_materialize(a, roots, consumers, nested)) continue;
    for (int side = 0; side < 2; side++) {
      const UOp *x = a->src[(size_t)side].get(), *b = a->src[(size_t)(1 - side)].get();
      if (x->op != Op::Reshape || only(x) != a) continue;
      const UOp *r = x->src[0].get();
      if (r->op != Op::ReduceAxis || r->reduce_op != Op::Add || r->arg != std::vector<int64_t>{2} ||
          r->src[0]->op != Op::Mul || r->shape.size() != 3 || only(r) != x)
        continue;
      auto bv = try_view(b);
      if (!bv || bv->strides.size() != 2 || (bv->shape[0] != 1 && bv->strides[0] != 0) ||
          (bv->shape[1] != 1 && bv->strides[1] != 1))
        continue;
      fused.insert(r);
    }
  }
  return fused;
}

}  // namespace

// Post-order walk that does not descend below nodes for which stop() holds
// (other than the root): a rewrite never needs what lies under a node it
// replaces or has already rewritten.
template <typename Stop>
static std::vector<UOpP> toposort_until(const UOpP &root, Stop stop) {
  const uint64_t mark = new_walk();
  auto visited = [mark](const UOp *n) { return n->walk_mark == mark; };
  std::vector<UOpP> out;
  std::vector<std::pair<const UOpP *, bool>> stack{{&root, false}};
  while (!stack.empty()) {
    auto [hp, processed] = stack.back();
    stack.pop_back();
    const UOp *node = hp->get();
    if (visited(node)) continue;
    if (processed || (node != root.get() && stop(node))) {
      node->walk_mark = mark;
      out.push_back(*hp);
      continue;
    }
    stack.push_back({hp, true});
    for (auto it = node->src.rbegin(); it != node->src.rend(); ++it)
      if (!visited(it->get())) stack.push_back({&*it, false});
  }
  return out;
}

UOpP substitute_materialized(const UOpP &root, const ReplMap &repl) {
  auto order = toposort_until(root, [&](const UOp *n) { return repl.count(n) > 0; });
  std::unordered_map<const UOp *, UOpP> sub;
  for (auto &node : order) {
    if (node != root) {
      auto r = repl.find(node.get());
      if (r != repl.end()) {
        sub[node.get()] = r->second;
        continue;
      }
    }
    bool changed = false;
    std::vector<UOpP> srcs;
    srcs.reserve(node->src.size());
    for (auto &s : node->src) {
      auto f = sub.find(s.get());
      UOpP ns = f != sub.end() ? f->second : s;
      changed |= ns != s;
      srcs.push_back(ns);
    }
    sub[node.get()] =
        changed ? intern(node->op, node->dtype, std::move(srcs), node->arg, node->reduce_op,
                         node->value, node->buf)
                : node;
  }
  return sub[root.get()];
}

namespace {
bool g_rewriter_live = false;
}  // namespace

Rewriter::Rewriter() {
  if (g_rewriter_live) throw Panic("Rewriter: another rewriter is live");
  g_rewriter_live = true;
  static uint64_t rewriters = 0;
  mark_ = ++rewriters;
}

Rewriter::~Rewriter() { g_rewriter_live = false; }

UOpP Rewriter::operator()(const UOpP &root) {
  // Iterative post-order DFS that stops at nodes already rewritten (or
  // replaced); a node is rebuilt once all its sources are done.
  if (done(root.get())) return vals_[root->memo_slot];
  std::vector<std::pair<const UOpP *, bool>> stack{{&root, false}};
  while (!stack.empty()) {
    auto [hp, processed] = stack.back();
    stack.pop_back();
    const UOp *node = hp->get();
    if (done(node)) continue;
    if (!processed) {
      stack.push_back({hp, true});
      for (auto it = node->src.rbegin(); it != node->src.rend(); ++it)
        if (!done(it->get())) stack.push_back({&*it, false});
      continue;
    }
    bool changed = false;
    for (const UOpP &s : node->src) changed |= vals_[s->memo_slot] != s;
    if (!changed) {
      remember(node, *hp);
      continue;
    }
    std::vector<UOpP> srcs;
    srcs.reserve(node->src.size());
    for (const UOpP &s : node->src) srcs.push_back(vals_[s->memo_slot]);
    remember(node, intern(node->op, node->dtype, std::move(srcs), node->arg, node->reduce_op,
                          node->value, node->buf));
  }
  return vals_[root->memo_slot];
}

ParamSlots collect_params(const UOpP &root, int slot_offset) {
  return collect_params_from(toposort_nodes(root.get()), slot_offset);
}

ParamSlots collect_params_from(const std::vector<const UOp *> &order, int slot_offset) {
  // parameterize_inputs (src/schedule.rs:176-245): buffers by first
  // appearance, one scalar per parameterised Shrink start.
  ParamSlots ps;
  for (auto &node : order) {
    if (node->op == Op::Buffer) {
      if (!ps.buffer_slot.count(node->buf.get())) {
        ps.buffer_slot[node->buf.get()] = (int)ps.inputs.size() + slot_offset;
        KernelInput in{KernelInput::Buffer, node->buf};
        ps.inputs.push_back(in);
      }
    } else if (node->op == Op::Shrink) {
      const Shape &ss = node->src[0]->shape;
      std::vector<int> slots(node->arg.size(), -1);
      for (size_t a = 0; a < node->arg.size(); a++) {
        const UOpP &start = node->src[a + 1];
        if (node->arg[a] != ss[a] && start->op == Op::Const) {
          slots[a] = (int)ps.inputs.size() + slot_offset;
          KernelInput in{KernelInput::I32, nullptr};
          in.i = (int64_t)start->value;
          ps.inputs.push_back(in);
        }
      }
      ps.shrink_slots[node] = slots;
    }
  }
  return ps;
}

namespace {

ScheduleItem parameterize(const UOpP &expr, bool with_inputs) {
  ScheduleItem it;
  it.value = expr;
  it.out_shape = expr->has_shape ? expr->shape : Shape{1};
  it.output = std::make_shared<DeviceBuffer>(expr->dtype, (size_t)numel(it.out_shape));
  if (with_inputs) it.inputs = collect_params(expr, 1).inputs;
  return it;
}

ScheduleItem parameterize_store(const UOpP &store, bool with_inputs) {
  ScheduleItem it;
  it.store_dest = store->src[0];
  it.value = store->src[1];
  it.out_shape = it.value->has_shape ? it.value->shape : Shape{1};
  if (with_inputs) it.inputs = collect_params(store, 0).inputs;
  return it;
}

UOpP buffer_replacement(const ScheduleItem &it) {
  return make_reshape(make_buffer(it.output), it.out_shape);
}

}  // namespace

SchedulePlan schedule_many(const std::vector<UOpP> &exprs, bool with_inputs) {
  if (exprs.empty()) throw Panic("schedule_many requires at least one root");
  UOpP uni = make_sink(exprs);
  auto order = toposort(uni);
  auto consumers = consumer_map(order);
  auto nested = nested_reduce_inputs(order);
  std::unordered_set<const UOp *> roots;
  for (auto &e : exprs) roots.insert(e.get());

  auto fused = fusible_shared_nodes(order, roots, consumers, nested);
  for (const UOp *r : bias_fused_contractions(order, roots, consumers, nested)) fused.insert(r);

  // Default mode: a comparison whose operands are all in memory (relu's
  // 0 < z once z is materialised, with its zeros buffer) is recomputed by
  // each consumer rather than written out as a bool tensor: the backward
  // where(0 < z, dX, 0) then reads z itself, which lets the dX GEMM apply
  // the mask in its epilogue.
  const bool exact = exact_mode();
  SchedulePlan plan;
  auto operand_ready = [&](const UOpP &x) {
    const UOp *n = x.get();
    while (is_movement(n->op)) n = n->src[0].get();
    return n->op == Op::Const || n->op == Op::Buffer || plan.replacements.count(n) > 0;
  };
  for (auto &node : order) {
    if (fused.count(node.get()) || !should_materialize(node.get(), roots, consumers, nested))
      continue;
    if (!exact && node->op == Op::CmpLt && !roots.count(node.get()) &&
        std::all_of(node->src.begin(), node->src.end(), operand_ready))
      continue;
    UOpP k = substitute_materialized(node, plan.replacements);
    ScheduleItem item = parameterize(k, with_inputs);
    plan.replacements[node.get()] = buffer_replacement(item);
    plan.keep.push_back(node);
    plan.items.push_back(std::move(item));
  }
  for (auto &e : exprs) {
    UOpP fin = substitute_materialized(e, plan.replacements);
    if (fin->op == Op::After && fin->src.size() == 2 && fin->src[1]->op == Op::Store) {
      plan.items.push_back(parameterize_store(fin->src[1], with_inputs));
      plan.replacements[e.get()] = fin->src[0];
    } else {
      ScheduleItem item = parameterize(fin, with_inputs);
      plan.replacements[e.get()] = buffer_replacement(item);
      plan.items.push_back(std::move(item));
    }
    plan.keep.push_back(e);
  }
  return plan;
}

// ---- structural schedule cache ----------------------------------------------
namespace {

// A schedule whose leaves (buffers, literals) are placeholders, stored as a
// flat program: the template's nodes in toposort order (sources first), each
// with what an instance puts in its place -- the keyed graph's leaf at a
// toposort position, an item's fresh output buffer, or the template node
// rebuilt over its sources' instances (the node itself when none changed).
// An instance is then one pass over a vector, with no hash lookups.
struct CachedSchedule {
  enum Kind : uint8_t { Interior, Leaf, Output };
  struct Node {
    UOpP t;
    Kind kind = Interior;
    int64_t ref = 0;           // Leaf: toposort position; Output: item index
    std::vector<int32_t> src;  // Interior: node indices of t's sources
  };
  struct Item {
    Shape out_shape;
    BufferP output;  // placeholder (dtype and count) or null for in-place items
    int32_t value = -1, store_dest = -1;
  };
  std::vector<Node> nodes;
  std::vector<Item> items;
  std::vector<std::pair<size_t, int32_t>> repl;  // (position of the replaced node, node)
};

std::unordered_map<std::string, CachedSchedule> &schedule_cache() {
  static std::unordered_map<std::string, CachedSchedule> c;
  return c;
}

bool schedule_cache_on() {
  static const bool on = [] {
    const char *e = std::getenv("FG_SCHEDULE_CACHE");
    return !(e && *e && std::strcmp(e, "0") == 0);
  }();
  return on;
}

// Everything schedule_many's decisions depend on: per node in toposort
// order its op, dtype, reduce op, args and source positions, a buffer's
// dtype and size; and the mode (exact mode schedules differently).
std::string structure_key(const std::vector<const UOp *> &order) {
  std::vector<int64_t> k;
  k.reserve(2 + order.size() * 8);
  auto put = [&k](int64_t v) { k.push_back(v); };
  put(exact_mode() ? 1 : 0);
  put((int64_t)order.size());
  for (size_t i = 0; i < order.size(); i++) {
    const UOp *n = order[i];
    n->topo_pos = (int64_t)i;
    put((int64_t)n->op | ((int64_t)n->dtype << 8) | ((int64_t)n->reduce_op << 16));
    put((int64_t)n->arg.size());
    for (int64_t a : n->arg) put(a);
    put((int64_t)n->src.size());
    for (auto &s : n->src) put(s->topo_pos);
    if (n->op == Op::Buffer) put((int64_t)n->buf->count);
  }
  return std::string(reinterpret_cast<const char *>(k.data()), k.size() * sizeof(int64_t));
}

}  // namespace

SchedulePlan schedule_cached(const std::vector<UOpP> &roots) {
  if (!schedule_cache_on()) return schedule_many(roots, false);
  if (roots.empty()) throw Panic("schedule_many requires at least one root");
  // the sink holds the whole graph; the walk's order is plain pointers
  UOpP sink = make_sink(roots);
  const std::vector<const UOp *> order = toposort_nodes(sink.get());
  std::string key = structure_key(order);
  auto &cache = schedule_cache();
  auto hit = cache.find(key);
  if (hit != cache.end()) {
    const CachedSchedule &cs = hit->second;
    SchedulePlan plan;
    plan.items.resize(cs.items.size());
    for (size_t i = 0; i < cs.items.size(); i++) {
      plan.items[i].out_shape = cs.items[i].out_shape;
      if (const BufferP &o = cs.items[i].output)
        plan.items[i].output = std::make_shared<DeviceBuffer>(o->dtype, o->count);
    }
    std::vector<UOpP> inst(cs.nodes.size());
    for (size_t i = 0; i < cs.nodes.size(); i++) {
      const CachedSchedule::Node &nd = cs.nodes[i];
      switch (nd.kind) {
        case CachedSchedule::Leaf:
          inst[i] = order[(size_t)nd.ref]->shared_from_this();
          break;
        case CachedSchedule::Output:
          inst[i] = make_buffer(plan.items[(size_t)nd.ref].output);
          break;
        case CachedSchedule::Interior: {
          const UOp &t = *nd.t;
          bool changed = false;
          std::vector<UOpP> srcs;
          srcs.reserve(nd.src.size());
          for (size_t j = 0; j < nd.src.size(); j++) {
            const UOpP &s = inst[(size_t)nd.src[j]];
            changed |= s != t.src[j];
            srcs.push_back(s);
          }
          inst[i] = changed ? intern(t.op, t.dtype, std::move(srcs), t.arg, t.reduce_op, t.value,
                                     t.buf)
                            : nd.t;
          break;
        }
      }
    }
    for (size_t i = 0; i < cs.items.size(); i++) {
      plan.items[i].value = inst[(size_t)cs.items[i].value];
      if (cs.items[i].store_dest >= 0)
        plan.items[i].store_dest = inst[(size_t)cs.items[i].store_dest];
    }
    for (auto &[pos, idx] : cs.repl) plan.replacements[order[pos]] = inst[(size_t)idx];
    plan.keep.push_back(std::move(sink));
    stats().schedule_hits++;
    return plan;
  }
  SchedulePlan plan = schedule_many(roots, false);
  // Template: every leaf and item output replaced by a placeholder that owns
  // no device memory, so the cache keeps no tensor alive.
  std::unordered_map<const UOp *, UOpP> m;
  std::unordered_map<const UOp *, std::pair<CachedSchedule::Kind, int64_t>> role;
  for (size_t i = 0; i < order.size(); i++) {
    const UOp *n = order[i];
    if (n->op == Op::Buffer) {
      UOpP ph = make_buffer(std::make_shared<DeviceBuffer>(n->buf->dtype, n->buf->count));
      m[n] = ph;
      role[ph.get()] = {CachedSchedule::Leaf, (int64_t)i};
    } else if (n->op == Op::Const) {
      role[n] = {CachedSchedule::Leaf, (int64_t)i};
    }
  }
  std::vector<BufferP> outputs;
  for (size_t i = 0; i < plan.items.size(); i++) {
    const ScheduleItem &it = plan.items[i];
    if (!it.output) {
      outputs.push_back(nullptr);
      continue;
    }
    outputs.push_back(std::make_shared<DeviceBuffer>(it.output->dtype, it.output->count));
    UOpP ph = make_buffer(outputs.back());
    m[make_buffer(it.output).get()] = ph;
    role[ph.get()] = {CachedSchedule::Output, (int64_t)i};
  }
  std::vector<UOpP> troots;
  std::vector<std::pair<UOpP, UOpP>> titems;
  Rewriter rewrite(m);
  for (const ScheduleItem &it : plan.items) {
    UOpP v = rewrite(it.value);
    UOpP d = it.store_dest ? rewrite(it.store_dest) : nullptr;
    troots.push_back(v);
    if (d) troots.push_back(d);
    titems.emplace_back(v, d);
  }
  std::vector<std::pair<size_t, UOpP>> trepl;
  for (auto &[node, rep] : plan.replacements) {
    trepl.emplace_back((size_t)node->topo_pos, rewrite(rep));
    troots.push_back(trepl.back().second);
  }
  CachedSchedule cs;
  std::unordered_map<const UOp *, int32_t> index;
  std::vector<UOpP> torder = toposort(make_sink(troots));
  torder.pop_back();  // the sink
  for (const UOpP &n : torder) {
    CachedSchedule::Node nd;
    nd.t = n;
    if (auto r = role.find(n.get()); r != role.end()) {
      nd.kind = r->second.first;
      nd.ref = r->second.second;
    } else {
      for (const UOpP &s : n->src) nd.src.push_back(index.at(s.get()));
    }
    index[n.get()] = (int32_t)cs.nodes.size();
    cs.nodes.push_back(std::move(nd));
  }
  for (size_t i = 0; i < plan.items.size(); i++) {
    CachedSchedule::Item t;
    t.out_shape = plan.items[i].out_shape;
    t.output = outputs[i];
    t.value = index.at(titems[i].first.get());
    if (titems[i].second) t.store_dest = index.at(titems[i].second.get());
    cs.items.push_back(std::move(t));
  }
  for (auto &[pos, rep] : trepl) cs.repl.emplace_back(pos, index.at(rep.get()));
  if (cache.size() >= 32) cache.clear();
  cache.emplace(std::move(key), std::move(cs));
  return plan;
}

}  // namespace ferro
