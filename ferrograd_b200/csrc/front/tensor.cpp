// tensor.cpp -- Tensor (src/tensor.rs), nn::Linear (src/nn.rs) and
// optim::Sgd (src/optim.rs) over the interned UOp graph.
#include <algorithm>
#include <chrono>
#include <cmath>
#include <cstring>
#include <unordered_set>

#include "front_internal.h"

namespace ferro {

// TensorInner (src/tensor.rs:84-97).
struct TensorInner {
  UOpP uop;
  bool requires_grad = false;
  std::shared_ptr<TensorInner> grad;
};

namespace {

// Weak references to every live tensor (src/tensor.rs:74-82): realization
// rewrites each handle whose graph references a realized subexpression.
std::vector<std::weak_ptr<TensorInner>> &live_list() {
  static std::vector<std::weak_ptr<TensorInner>> v;
  return v;
}

// Checks a precondition; the message (often built from shapes) is only
// formatted when the check fails.
#define require(ok, msg)         \
  do {                           \
    if (!(ok)) throw Panic(msg); \
  } while (0)

// Numpy-style broadcast target (src/shape.rs:66-89).
bool broadcast_shape(const Shape &a, const Shape &b, Shape *out) {
  size_t n = std::max(a.size(), b.size());
  Shape l(n - a.size(), 1), r(n - b.size(), 1);
  l.insert(l.end(), a.begin(), a.end());
  r.insert(r.end(), b.begin(), b.end());
  out->assign(n, 0);
  for (size_t i = 0; i < n; i++) {
    if (l[i] == r[i])
      (*out)[i] = l[i];
    else if (l[i] == 1)
      (*out)[i] = r[i];
    else if (r[i] == 1)
      (*out)[i] = l[i];
    else
      return false;
  }
  return true;
}

Shape pad_left(const Shape &s, size_t n) {
  Shape o(n - s.size(), 1);
  o.insert(o.end(), s.begin(), s.end());
  return o;
}

}  // namespace

Tensor Tensor::from_uop(UOpP u, bool requires_grad) {
  auto p = std::make_shared<TensorInner>();
  p->uop = std::move(u);
  p->requires_grad = requires_grad;
  auto &live = live_list();
  if (live.size() > 64 && live.size() % 64 == 0)
    live.erase(std::remove_if(live.begin(), live.end(),
                              [](const std::weak_ptr<TensorInner> &w) { return w.expired(); }),
               live.end());
  live.push_back(p);
  return Tensor(p);
}

UOpP Tensor::uop() const {
  require((bool)p_, "use of an undefined tensor");
  return p_->uop;
}
void Tensor::set_uop(UOpP u) const { p_->uop = std::move(u); }

UOpP Tensor::target_uop() const {
  UOpP cur = uop();
  if (cur->op == Op::After) return cur->src[0];
  return cur;
}

std::vector<Tensor> Tensor::live_tensors() {
  std::vector<Tensor> out;
  auto &live = live_list();
  std::vector<std::weak_ptr<TensorInner>> keep;
  keep.reserve(live.size());
  for (auto &w : live) {
    if (auto p = w.lock()) {
      out.push_back(Tensor(p));
      keep.push_back(w);
    }
  }
  live.swap(keep);
  return out;
}

void Tensor::apply_map_to_tensors(const std::map<const UOp *, UOpP> &replacements) {
  // src/tensor.rs:222-252: one combined substitution over all affected roots.
  if (replacements.empty()) return;
  // One memoised rewrite over all live tensors: shared subgraphs are walked
  // once, and a graph that reaches no replaced node comes back unchanged.
  Rewriter rewrite(replacements);
  for (Tensor &t : live_tensors()) {
    UOpP cur = t.uop();
    UOpP rewritten = rewrite(cur);
    if (rewritten != cur) t.set_uop(rewritten);
  }
}

Tensor Tensor::from_host(DType dt, const void *data, size_t bytes, const Shape &shape) {
  for (int64_t d : shape) require(d >= 0, "negative dimension in " + shape_str(shape));
  const size_t n = (size_t)ferro::numel(shape);
  require(bytes == n * dtype_size(dt), "data length " + std::to_string(bytes / dtype_size(dt)) +
                                           " doesn't match shape " + shape_str(shape));
  auto buf = std::make_shared<DeviceBuffer>(dt, n);
  if (bytes) {
    if (device_is_open())
      buf->upload(data, bytes);  // straight from the caller's memory
    else
      buf->pending.assign((const uint8_t *)data, (const uint8_t *)data + bytes);
  }
  return from_uop(make_reshape(make_buffer(buf), shape), false);
}

Tensor Tensor::from_f32(const float *data, const Shape &shape) {
  return from_host(DType::F32, data, (size_t)ferro::numel(shape) * 4, shape);
}
Tensor Tensor::from_i32(const int32_t *data, const Shape &shape) {
  return from_host(DType::I32, data, (size_t)ferro::numel(shape) * 4, shape);
}
Tensor Tensor::from_bool(const uint8_t *data, const Shape &shape) {
  std::vector<uint8_t> b((size_t)ferro::numel(shape));
  for (size_t i = 0; i < b.size(); i++) b[i] = data[i] ? 1 : 0;
  return from_host(DType::Bool, b.data(), b.size(), shape);
}

Tensor Tensor::zeros(const Shape &shape, DType dt) {
  auto buf = std::make_shared<DeviceBuffer>(dt, (size_t)ferro::numel(shape));
  buf->zero_init = true;
  return from_uop(make_reshape(make_buffer(buf), shape), false);
}

Tensor Tensor::empty(const Shape &shape, DType dt) { return zeros(shape, dt); }

Tensor Tensor::from_u8_div(const uint8_t *data, const Shape &shape, float divisor) {
  for (int64_t d : shape) require(d >= 0, "negative dimension in " + shape_str(shape));
  BufferP b = device_u8_to_f32(data, (size_t)ferro::numel(shape), divisor);
  return from_uop(make_reshape(make_buffer(b), shape), false);
}

Tensor Tensor::one_hot_u8(const uint8_t *labels, int64_t n, int classes) {
  require(n >= 0 && classes > 0, "one_hot: bad size");
  BufferP b = device_one_hot_u8(labels, (size_t)n, classes);
  return from_uop(make_reshape(make_buffer(b), {n, (int64_t)classes}), false);
}

Tensor Tensor::full(const Shape &shape, float value) {
  std::vector<float> v((size_t)ferro::numel(shape), value);
  return from_f32(v.data(), shape);
}

Tensor Tensor::ones(const Shape &shape, DType dt) {
  if (dt == DType::F32) return full(shape, 1.0f);
  if (dt == DType::I32) {
    std::vector<int32_t> v((size_t)ferro::numel(shape), 1);
    return from_i32(v.data(), shape);
  }
  std::vector<uint8_t> v((size_t)ferro::numel(shape), 1);
  return from_bool(v.data(), shape);
}

Tensor Tensor::scalar(float value) {
  // The value stays on the host until a kernel reads the buffer (the upload
  // is then part of its allocation, DeviceBuffer::ensure_allocated): the
  // routes that take it by value (the SGD step's lr) never allocate or copy
  // it, which saves Sgd::step one host-to-device copy per parameter.
  auto buf = std::make_shared<DeviceBuffer>(DType::F32, 1);
  const uint8_t *p = reinterpret_cast<const uint8_t *>(&value);
  buf->pending.assign(p, p + sizeof(float));
  buf->has_host_scalar = true;
  buf->host_scalar = value;
  return from_uop(make_reshape(make_buffer(buf), {1}), false);
}

const UOp &Tensor::node() const {
  require((bool)p_, "use of an undefined tensor");
  return *p_->uop;
}
const Shape &Tensor::shape_ref() const {
  const UOp &u = node();
  require(u.has_shape, "tensor must have shape");
  return u.shape;
}
Shape Tensor::shape() const { return shape_ref(); }
DType Tensor::dtype() const { return node().dtype; }
int64_t Tensor::numel() const { return ferro::numel(shape_ref()); }
int64_t Tensor::ndim() const { return (int64_t)shape_ref().size(); }

bool Tensor::is_realized() const {
  const UOp &u = node();
  return u.op == Op::Buffer || (u.op == Op::Reshape && u.src[0]->op == Op::Buffer);
}

bool Tensor::requires_grad() const { return p_->requires_grad; }
Tensor Tensor::with_requires_grad(bool r) const {
  p_->requires_grad = r;
  return *this;
}
Tensor Tensor::grad() const { return p_->grad ? Tensor(p_->grad) : Tensor(); }
void Tensor::clear_grad() const { p_->grad.reset(); }
Tensor Tensor::detach() const { return from_uop(uop(), false); }

Tensor Tensor::replace(const Tensor &other) const {
  require(shape() == other.shape(), "replace: shape mismatch " + shape_str(shape()) + " != " +
                                        shape_str(other.shape()));
  set_uop(other.uop());
  return *this;
}

Tensor Tensor::assign(const Tensor &other) const {
  require(shape() == other.shape(), "assign: shape mismatch " + shape_str(shape()) + " != " +
                                        shape_str(other.shape()));
  require(dtype() == other.dtype(), "assign: dtype mismatch");
  UOpP target = target_uop();
  require(has_buffer_identity(target.get()),
          "assign requires a tensor with concrete buffer identity");
  UOpP effect = make_store(target, other.uop());
  set_uop(make_after(target, effect));
  return *this;
}

Tensor Tensor::unary(Op op) const {
  return from_uop(make_alu(op, dtype(), {uop()}), requires_grad());
}

Tensor Tensor::binary(const Tensor &o, Op op, DType out) const {
  require(shape_ref() == o.shape_ref(), std::string("shape mismatch for ") + op_name(op));
  return from_uop(make_alu(op, out, {uop(), o.uop()}), requires_grad() || o.requires_grad());
}

Tensor Tensor::broadcasted(const Tensor &o, Op op, DType out) const {
  if (shape_ref() == o.shape_ref()) return binary(o, op, out);
  Shape target;
  require(broadcast_shape(shape_ref(), o.shape_ref(), &target),
          "broadcast: incompatible dims for " + shape_str(shape()) + " vs " + shape_str(o.shape()));
  Tensor l = reshape(pad_left(shape_ref(), target.size())).expand(target);
  Tensor r = o.reshape(pad_left(o.shape_ref(), target.size())).expand(target);
  return l.binary(r, op, out);
}

Tensor Tensor::add(const Tensor &o) const { return broadcasted(o, Op::Add, dtype()); }
Tensor Tensor::mul(const Tensor &o) const { return broadcasted(o, Op::Mul, dtype()); }
Tensor Tensor::neg() const { return unary(Op::Neg); }
Tensor Tensor::sub(const Tensor &o) const { return add(o.neg()); }
Tensor Tensor::reciprocal() const { return unary(Op::Reciprocal); }
Tensor Tensor::exp2() const { return unary(Op::Exp2); }
Tensor Tensor::log2() const { return unary(Op::Log2); }
Tensor Tensor::sqrt() const { return unary(Op::Sqrt); }

Tensor Tensor::relu() const {
  // where(0 < x, x, zeros) with a real zero buffer (src/tensor.rs:519-531).
  Tensor zero = zeros(shape_ref(), dtype());
  Tensor cond = zero.binary(*this, Op::CmpLt, DType::Bool);
  return from_uop(make_alu(Op::Where, dtype(), {cond.uop(), uop(), zero.uop()}), requires_grad());
}

Tensor Tensor::reshape(const Shape &s) const {
  if (shape_ref() == s) return *this;
  require(numel() == ferro::numel(s),
          "reshape: numel mismatch for " + shape_str(shape()) + " -> " + shape_str(s));
  return from_uop(make_reshape(uop(), s), requires_grad());
}

Tensor Tensor::narrow(int64_t dim, int64_t start, int64_t len) const {
  Shape s = shape();
  require(dim >= 0 && dim < (int64_t)s.size(), "narrow: dim " + std::to_string(dim) +
                                                   " out of range");
  require(start >= 0 && len >= 0 && start + len <= s[(size_t)dim],
          "narrow: range [" + std::to_string(start) + ", " + std::to_string(start + len) +
              ") out of bounds for axis " + std::to_string(dim) + " with size " +
              std::to_string(s[(size_t)dim]));
  if (start == 0 && len == s[(size_t)dim]) return *this;
  std::vector<UOpP> starts;
  Shape lengths = s;
  for (size_t a = 0; a < s.size(); a++)
    starts.push_back(make_const((int64_t)a == dim ? (double)start : 0.0, DType::I32));
  lengths[(size_t)dim] = len;
  return from_uop(make_shrink(uop(), starts, lengths), requires_grad());
}

Tensor Tensor::permute(const std::vector<int64_t> &order) const {
  const int64_t n = ndim();
  require((int64_t)order.size() == n, "permute: wrong number of axes");
  std::vector<bool> seen((size_t)n, false);
  for (int64_t a : order) {
    require(a >= 0 && a < n, "permute: axis " + std::to_string(a) + " out of range");
    require(!seen[(size_t)a], "permute: axis " + std::to_string(a) + " duplicated");
    seen[(size_t)a] = true;
  }
  return from_uop(make_permute(uop(), order), requires_grad());
}

Tensor Tensor::contiguous() const {
  if (is_realized()) return *this;
  return from_uop(make_contiguous(uop()), requires_grad());
}

Tensor Tensor::expand(const Shape &s) const {
  const Shape &src = shape_ref();
  if (src == s) return *this;
  require(src.size() == s.size(),
          "expand: rank mismatch for " + shape_str(src) + " -> " + shape_str(s));
  for (size_t a = 0; a < s.size(); a++)
    require(src[a] == s[a] || src[a] == 1,
            "expand: incompatible source shape " + shape_str(src) + " -> " + shape_str(s));
  return from_uop(make_expand(uop(), s), requires_grad());
}

Tensor Tensor::sum(const std::vector<int64_t> &axes) const {
  const int64_t n = ndim();
  for (int64_t a : axes) require(a >= 0 && a < n, "sum: axes out of range for ndim " +
                                                      std::to_string(n));
  return from_uop(make_reduce(uop(), Op::Add, axes), requires_grad());
}

Tensor Tensor::max(const std::vector<int64_t> &axes) const {
  const int64_t n = ndim();
  for (int64_t a : axes) require(a >= 0 && a < n, "max: axes out of range for ndim " +
                                                      std::to_string(n));
  return from_uop(make_reduce(uop(), Op::Max, axes), requires_grad());
}

Tensor Tensor::exp() const { return mul(scalar(1.44269504088896340736f)).exp2(); }
Tensor Tensor::log() const { return log2().mul(scalar(0.693147180559945309417f)); }

Tensor Tensor::log_softmax(int64_t axis) const {
  require(axis >= 0 && axis < ndim(), "log_softmax: axis " + std::to_string(axis) +
                                          " out of range");
  Tensor max_x = max({axis});
  Tensor shifted = sub(max_x);
  Tensor sum_exp = shifted.exp().sum({axis});
  return shifted.sub(sum_exp.log());
}

Tensor Tensor::cross_entropy(const Tensor &targets) const {
  require(shape() == targets.shape(), "cross_entropy: target shape " +
                                          shape_str(targets.shape()) +
                                          " must match logits shape " + shape_str(shape()));
  const int64_t classes_axis = ndim() != 1 ? 1 : 0;
  // Default mode: one fused op, run as a single fg_xent_fwd_bwd pass that
  // also yields d loss / d logits for backward().  Exact mode (and targets
  // that need a gradient, other ranks/dtypes, or empty logits, which the
  // fused kernel rejects) build the reference graph.
  if (!exact_mode() && (ndim() == 1 || ndim() == 2) && dtype() == DType::F32 &&
      targets.dtype() == DType::F32 && !targets.requires_grad() && numel() > 0)
    return from_uop(make_xent_loss(uop(), targets.uop()), requires_grad());
  Tensor log_probs = log_softmax(classes_axis);
  Tensor per_sample = targets.mul(log_probs).sum({classes_axis}).neg();
  std::vector<int64_t> axes;
  for (int64_t a = 0; a < per_sample.ndim(); a++) axes.push_back(a);
  Tensor scale = scalar(1.0f / (float)per_sample.numel());
  return per_sample.sum(axes).mul(scale);
}

Tensor Tensor::matmul(const Tensor &o) const {
  require(ndim() == 2, "matmul: lhs must be 2D");
  require(o.ndim() == 2, "matmul: rhs must be 2D");
  const int64_t m = shape()[0], k = shape()[1], k2 = o.shape()[0], n = o.shape()[1];
  require(k == k2, "matmul: inner dim mismatch (" + std::to_string(k) + " vs " +
                       std::to_string(k2) + ")");
  Tensor a = reshape({m, 1, k}).expand({m, n, k});
  Tensor b = o.permute({1, 0}).contiguous().reshape({1, n, k}).expand({m, n, k});
  return a.mul(b).sum({2}).reshape({m, n});
}

void Tensor::realize_many(const std::vector<Tensor> &ts) {
  // src/tensor.rs:781-811.
  std::vector<UOpP> roots;
  std::unordered_set<const UOp *> seen;
  for (const Tensor &t : ts) {
    if (t.is_realized()) continue;
    UOpP r = t.uop();
    if (seen.insert(r.get()).second) roots.push_back(r);
  }
  if (roots.empty()) return;
  ExactModeScope mode;
  using clk = std::chrono::steady_clock;
  auto secs = [](clk::time_point a, clk::time_point b) {
    return std::chrono::duration<double>(b - a).count();
  };
  const auto t0 = clk::now();
  SchedulePlan plan = schedule_cached(roots);
  const auto t1 = clk::now();
  for (const ScheduleItem &item : plan.items) run_item(item);
  end_realize();
  const auto t2 = clk::now();
  apply_map_to_tensors(plan.replacements);
  Stats &st = stats();
  st.schedule_s += secs(t0, t1);
  st.run_s += secs(t1, t2);
  st.rewrite_s += secs(t2, clk::now());
}

Tensor Tensor::realize() const {
  realize_many({*this});
  return *this;
}

std::vector<uint8_t> Tensor::to_bytes() const {
  realize();
  UOpP u = uop();
  const UOp *b = u->op == Op::Buffer ? u.get() : u->src[0].get();
  require(b->op == Op::Buffer, "realized tensor must point at a buffer");
  return b->buf->to_host();
}

std::vector<float> Tensor::to_vec() const {
  require(dtype() == DType::F32, "to_vec requires F32 tensor data");
  auto bytes = to_bytes();
  std::vector<float> out(bytes.size() / 4);
  if (!out.empty()) std::memcpy(out.data(), bytes.data(), bytes.size());
  return out;
}

std::vector<Tensor> Tensor::gradient(const std::vector<Tensor> &targets) const {
  // src/tensor.rs:943-971.
  UOpP root_grad = make_full(shape(), DType::F32, 1.0);
  std::vector<UOpP> tu;
  for (const Tensor &t : targets)
    if (t.requires_grad()) tu.push_back(t.uop());
  auto gm = compute_gradient(uop(), root_grad, tu);
  std::vector<Tensor> out;
  for (const Tensor &t : targets) {
    auto it = gm.find(t.uop().get());
    if (it != gm.end())
      out.push_back(from_uop(it->second, false));
    else
      out.push_back(from_uop(make_full(t.shape(), DType::F32, 0.0), false));
  }
  return out;
}

void Tensor::backward() const {
  // src/tensor.rs:973-998.
  require(numel() == 1, "backward requires a scalar loss");
  // graph membership by toposort position (UOp::topo_pos), not a hash set
  const UOpP root = uop();
  const std::vector<const UOp *> all = toposort_nodes(root.get());
  for (size_t i = 0; i < all.size(); i++) all[i]->topo_pos = (int64_t)i;
  auto in_graph = [&all](const UOp *u) {
    return u->topo_pos >= 0 && (size_t)u->topo_pos < all.size() && all[(size_t)u->topo_pos] == u;
  };
  std::vector<Tensor> targets;
  for (Tensor &t : live_tensors())
    if (t.requires_grad() && in_graph(t.uop().get())) targets.push_back(t);
  if (targets.empty()) return;
  std::vector<UOpP> tu;
  for (auto &t : targets) tu.push_back(t.uop());
  UOpP root_grad = make_full(shape(), DType::F32, 1.0);
  auto grads = compute_gradient(uop(), root_grad, tu);
  for (Tensor &t : targets) {
    auto it = grads.find(t.uop().get());
    UOpP g = it != grads.end() ? it->second : make_full(t.shape(), DType::F32, 0.0);
    Tensor gt = from_uop(g, false);
    Tensor acc = t.p_->grad ? Tensor(t.p_->grad).add(gt) : gt;
    t.p_->grad = acc.p_;
  }
}

// ---- nn::Linear (src/nn.rs:12-104) -----------------------------------------
namespace {
uint64_t g_init_seed = 42;  // INIT_SEED (src/nn.rs:12-14)
}  // namespace

void reset_init_seed(uint64_t seed) { g_init_seed = seed; }
uint64_t init_seed() { return g_init_seed; }

static Tensor kaiming_normal(const Shape &shape, int64_t fan_in) {
  // The host draw is the C ABI's fg_kaiming_normal (the reference's LCG and
  // Box-Muller pairs); the seed state is carried here across layers.
  std::vector<float> data((size_t)numel(shape));
  uint64_t st = g_init_seed;
  if (fg_kaiming_normal(data.data(), data.size(), (size_t)fan_in, &st) != FG_OK)
    throw Panic(std::string("kaiming_normal: ") + fg_last_error());
  g_init_seed = st;
  return Tensor::from_f32(data.data(), shape);
}

Linear::Linear(int64_t in_features, int64_t out_features, bool with_bias) {
  weight = kaiming_normal({out_features, in_features}, in_features).with_requires_grad(true);
  if (with_bias) bias = Tensor::zeros({out_features}, DType::F32).with_requires_grad(true);
}

Tensor Linear::forward(const Tensor &x) const {
  Tensor w = weight.permute({1, 0});
  Tensor logits = x.matmul(w);
  return bias.defined() ? logits.add(bias) : logits;
}

std::vector<Tensor> Linear::parameters() const {
  std::vector<Tensor> p{weight};
  if (bias.defined()) p.push_back(bias);
  return p;
}

// ---- optim::Sgd (src/optim.rs:29-71) ----------------------------------------
Sgd::Sgd(const std::vector<Tensor> &ps, float lr_) : lr(lr_) {
  if (ps.empty()) throw Panic("optimizer must have at least one parameter");
  for (const Tensor &p : ps) {
    bool dup = std::any_of(params.begin(), params.end(),
                           [&](const Tensor &q) { return q.ptr_eq(p); });
    if (!dup) params.push_back(p);
  }
}

void Sgd::zero_grad() const {
  for (const Tensor &p : params) p.clear_grad();
}

void Tensor::all_reduce_mean(fg_comm *comm) const {
  require(comm != nullptr, "all_reduce_mean: no communicator");
  require(dtype() == DType::F32, "all_reduce_mean: f32 tensors only");
  realize();
  // a realized tensor is its buffer, or a reshape of all of it
  const UOp &u = node();
  const UOp *b = u.op == Op::Reshape ? u.src[0].get() : &u;
  require(b->op == Op::Buffer, "all_reduce_mean: tensor is not a whole buffer");
  all_reduce_mean_buffer(b->buf, comm);
}

void Sgd::step() const {
  if (comm) {
    std::vector<Tensor> grads;
    for (const Tensor &p : params) {
      Tensor g = p.grad();
      if (!g.defined()) throw Panic("optimizer step requires parameter gradients");
      grads.push_back(g);
    }
    Tensor::realize_many(grads);
    for (const Tensor &g : grads) g.all_reduce_mean(comm);
  }
  for (const Tensor &p : params) {
    Tensor lr_t = Tensor::scalar(lr);
    Tensor g = p.grad();
    if (!g.defined()) throw Panic("optimizer step requires parameter gradients");
    Tensor update = p.detach().sub(g.mul(lr_t));
    p.assign(update);
  }
  Tensor::realize_many(params);
}

}  // namespace ferro
