// ferro_front.h -- the lazy Tensor front end of ferrograd, restated in C++ on
// top of the B200 backend's C ABI (include/ferro_cuda.h).
//
// It mirrors the reference crate's user surface and its host-side compiler
// stages for the MLP training path:
//   UOp graph (src/uop.rs)             interned nodes, shape inference, toposort
//   Tensor (src/tensor.rs)             lazy graph handles, realize, backward
//   gradient (src/gradient.rs)         reverse-mode rules that build more graph
//   schedule (src/schedule.rs)         should_materialize kernel boundaries
//   Linear / Sgd (src/nn.rs, src/optim.rs)
// The reference's rangeify/optimize/expand/devectorize/linearize/clang stages
// are replaced by a CUDA router (exec.cpp): each scheduled proto-kernel either
// goes to a hand-written building block (the reduce-of-broadcast-mul
// contraction to the 3xTF32 tensor-core GEMM, large f32 row/column sums to
// the HBM reduction kernels) or is rendered to CUDA C with the reference's op
// semantics and reduction order (render.cpp) and compiled by NVRTC.
//
// Threading: like the reference (Rc/RefCell/thread_local), the front end is
// single-threaded; callers serialise access (the Python binding holds the GIL).
#pragma once
#include <cstdint>
#include <map>
#include <memory>
#include <string>
#include <vector>

#include "../../../include/ferro_cuda.h"

namespace ferro {

using Shape = std::vector<int64_t>;
int64_t numel(const Shape &s);
std::string shape_str(const Shape &s);

// src/dtype.rs:19-58
enum class DType : int { F32 = 0, I32 = 1, Bool = 2 };
size_t dtype_size(DType d);
const char *dtype_name(DType d);

// The subset of src/uop.rs:26-310 that tensor-level graphs use.
enum class Op : int {
  Buffer,
  Const,
  Reshape,
  Permute,
  Expand,
  Shrink,
  Contiguous,
  Add,
  Mul,
  Neg,
  Reciprocal,
  Exp2,
  Log2,
  Sqrt,
  Max,
  CmpLt,
  Where,
  ReduceAxis,
  Store,
  After,
  Sink,
  // Fused cross-entropy (default mode only; no counterpart op in the
  // reference, whose Tensor::cross_entropy builds the decomposed graph of
  // src/tensor.rs:715-752): XentLoss(logits [B,C], targets [B,C]) is the
  // loss (every axis 1, as the reference's); XentGrad(logits, targets)
  // [B,C] is d loss / d logits as src/gradient.rs:97-205 builds it for that
  // graph.  Either runs as one fg_xent_fwd_bwd pass, which yields both.
  XentLoss,
  XentGrad
};
const char *op_name(Op op);
bool is_alu(Op op);       // src/uop.rs:315-330
bool is_movement(Op op);  // src/uop.rs:333-338

// Device storage behind a Buffer UOp (src/device.rs:95-214).  Storage is
// acquired lazily (ensure_allocated); data given at construction is kept on
// the host until then, so graphs can be built and scheduled without a GPU.
struct DeviceBuffer {
  DType dtype;
  size_t count;
  uint64_t id;
  fg_buffer *h = nullptr;
  std::vector<uint8_t> pending;  // host bytes to upload on allocation
  bool zero_init = false;        // Tensor::zeros: must read as zeros (no data given)
  // Writes into an existing buffer (in-place stores) bump the version; the
  // TF32 residual of the contents is cached for the version it was made for.
  uint64_t version = 0;
  std::shared_ptr<DeviceBuffer> lo;
  uint64_t lo_version = ~0ull;
  // Tensor::scalar buffers keep their value on the host as well, so a kernel
  // that takes it as a by-value argument (the SGD step's lr) needs no read
  // back; valid while version == 0.
  bool has_host_scalar = false;
  float host_scalar = 0.0f;
  DeviceBuffer(DType dt, size_t n);
  ~DeviceBuffer();
  DeviceBuffer(const DeviceBuffer &) = delete;
  DeviceBuffer &operator=(const DeviceBuffer &) = delete;
  bool is_allocated() const { return h != nullptr; }
  // Zero-filled at creation and never written since (Tensor::zeros): kernels
  // may use the value 0 instead of reading it.
  bool known_zero() const { return zero_init && pending.empty() && version == 0; }
  void ensure_allocated();
  // Allocates and copies `bytes` from host memory now (Device::copy_from_host).
  void upload(const void *data, size_t bytes);
  void *ptr();
  std::vector<uint8_t> to_host();
};
using BufferP = std::shared_ptr<DeviceBuffer>;

struct UOp;
using UOpP = std::shared_ptr<const UOp>;

struct UOp : std::enable_shared_from_this<UOp> {
  Op op;
  DType dtype;
  std::vector<UOpP> src;
  std::vector<int64_t> arg;  // Reshape/Expand: shape, Permute: order,
                             // ReduceAxis: axes, Shrink: lengths
  Op reduce_op = Op::Add;    // ReduceAxis: Add or Max
  double value = 0.0;        // Const
  BufferP buf;               // Buffer
  bool has_shape = false;
  Shape shape;               // inferred as src/uop.rs:806-866
  uint64_t uid = 0;          // creation order (debug output only)
  // Graph walks mark a node visited by stamping their own walk number here
  // (toposort); the front end is single-threaded, so no two walks overlap.
  mutable uint64_t walk_mark = 0;
  // Scratch for the structural keys (schedule cache, program lookup): the
  // node's position in the toposort of the graph being keyed (valid only
  // inside that computation).
  mutable int64_t topo_pos = -1;
  // A Rewriter's memo: the node's rewritten form is slot memo_slot of the
  // rewriter whose number is memo_mark (one rewriter is live at a time).
  mutable uint64_t memo_mark = 0;
  mutable uint32_t memo_slot = 0;
  // The interner's entry: the node's structural hash; the node leaves the
  // table when it is destroyed.
  uint64_t intern_hash = 0;
  bool interned = false;
  UOp() = default;
  UOp(const UOp &) = delete;
  UOp &operator=(const UOp &) = delete;
  ~UOp();
};

// Interned constructors (src/uop.rs:536-760, 926-1040): structurally equal
// nodes are the same object, so pointer identity is value identity.
UOpP make_buffer(const BufferP &b);
UOpP make_const(double v, DType dt);
UOpP make_reshape(const UOpP &s, const Shape &shape);
UOpP make_permute(const UOpP &s, const std::vector<int64_t> &order);
UOpP make_expand(const UOpP &s, const Shape &shape);
UOpP make_shrink(const UOpP &s, const std::vector<UOpP> &starts, const Shape &lengths);
UOpP make_contiguous(const UOpP &s);
UOpP make_alu(Op op, DType dt, std::vector<UOpP> srcs);
UOpP make_add(const UOpP &a, const UOpP &b);
UOpP make_mul(const UOpP &a, const UOpP &b);
UOpP make_neg(const UOpP &a);
UOpP make_reciprocal(const UOpP &a);
UOpP make_cmplt(const UOpP &a, const UOpP &b);
UOpP make_where(const UOpP &c, const UOpP &t, const UOpP &f);
UOpP make_reduce(const UOpP &s, Op rop, const std::vector<int64_t> &axes);
UOpP make_store(const UOpP &dest, const UOpP &value);
UOpP make_after(const UOpP &value, const UOpP &effect);
UOpP make_sink(const std::vector<UOpP> &srcs);
UOpP make_xent_loss(const UOpP &logits, const UOpP &targets);
UOpP make_xent_grad(const UOpP &logits, const UOpP &targets);
// UOp::full (src/uop.rs:734-744): Expand(Reshape(Const, [1..1]), shape).
UOpP make_full(const Shape &shape, DType dt, double value);

bool has_buffer_identity(const UOp *u);  // src/uop.rs:870-877
std::vector<UOpP> toposort(const UOpP &root);  // src/uop.rs:1044-1074
// The same order as plain node pointers, for walks that only read the nodes.
std::vector<const UOp *> toposort_nodes(const UOp *root);
std::string dump(const UOpP &root);
size_t interner_size();

// gradient::compute_gradient (src/gradient.rs:20-58); keys are UOp pointers.
std::map<const UOp *, UOpP> compute_gradient(const UOpP &root, const UOpP &root_grad,
                                             const std::vector<UOpP> &targets);

// ---- scheduling (src/schedule.rs:30-126) ----------------------------------
struct KernelInput {
  enum Kind { Buffer, I32, F32, Bool } kind;
  BufferP buffer;
  int64_t i = 0;
  double f = 0.0;
};
struct ScheduleItem {
  // Allocating kernel: out = value (shape out_shape).  In-place kernel:
  // store_dest (a view of a buffer) <- value.
  UOpP value;
  UOpP store_dest;   // null for allocating kernels
  BufferP output;    // allocating kernels: reserved output buffer
  Shape out_shape;
  std::vector<KernelInput> inputs;  // reference slot order (slot 0 = output)
};
struct SchedulePlan {
  std::vector<ScheduleItem> items;
  std::map<const UOp *, UOpP> replacements;
  std::vector<UOpP> keep;  // keeps replaced keys alive while the plan lives
};
// with_inputs = false skips each item's slot list (ScheduleItem::inputs),
// which only schedule summaries read; execution derives slots itself.
SchedulePlan schedule_many(const std::vector<UOpP> &roots, bool with_inputs = true);
// schedule_many through a cache keyed by the graph's structure (ops, dtypes,
// shapes, args, edges, buffer sizes; not buffer identities or literal
// values): a graph shaped like an earlier one -- the next step of a training
// loop -- reuses that schedule with its buffers and literals renamed instead
// of re-deriving kernel boundaries.  Items come without `inputs`.
// FG_SCHEDULE_CACHE=0 turns it off.
SchedulePlan schedule_cached(const std::vector<UOpP> &roots);

// ---- Tensor (src/tensor.rs) ------------------------------------------------
struct TensorInner;

class Tensor {
 public:
  Tensor() = default;
  // Tensor::new (src/tensor.rs:255-270) for the three element types.
  static Tensor from_f32(const float *data, const Shape &shape);
  static Tensor from_i32(const int32_t *data, const Shape &shape);
  static Tensor from_bool(const uint8_t *data, const Shape &shape);
  static Tensor zeros(const Shape &shape, DType dt = DType::F32);
  static Tensor ones(const Shape &shape, DType dt = DType::F32);
  static Tensor full(const Shape &shape, float value);
  static Tensor scalar(float value);
  // A tensor over a reserved (not yet written) buffer, for graph building and
  // scheduling tests; reading it before a kernel writes it gives zeros.
  static Tensor empty(const Shape &shape, DType dt = DType::F32);
  // Dataset path (src/dataset.rs:116-140, examples/mnist.rs:7-14): bytes
  // uploaded once and converted on the device into realized f32 tensors --
  // pixels as (float)b / divisor, labels as dense one-hot rows.
  static Tensor from_u8_div(const uint8_t *data, const Shape &shape, float divisor);
  static Tensor one_hot_u8(const uint8_t *labels, int64_t n, int classes);

  bool defined() const { return (bool)p_; }
  Shape shape() const;
  DType dtype() const;
  int64_t numel() const;
  int64_t ndim() const;
  bool is_realized() const;
  bool requires_grad() const;
  Tensor with_requires_grad(bool r) const;
  Tensor grad() const;  // undefined Tensor when there is none
  bool ptr_eq(const Tensor &o) const { return p_ == o.p_; }
  void clear_grad() const;
  Tensor detach() const;
  Tensor replace(const Tensor &other) const;
  Tensor assign(const Tensor &other) const;

  Tensor add(const Tensor &o) const;
  Tensor mul(const Tensor &o) const;
  Tensor sub(const Tensor &o) const;
  Tensor neg() const;
  Tensor reciprocal() const;
  Tensor exp2() const;
  Tensor log2() const;
  Tensor sqrt() const;
  Tensor relu() const;
  Tensor exp() const;
  Tensor log() const;
  Tensor reshape(const Shape &s) const;
  Tensor narrow(int64_t dim, int64_t start, int64_t len) const;
  Tensor permute(const std::vector<int64_t> &order) const;
  Tensor contiguous() const;
  Tensor expand(const Shape &s) const;
  Tensor sum(const std::vector<int64_t> &axes) const;
  Tensor max(const std::vector<int64_t> &axes) const;
  Tensor log_softmax(int64_t axis) const;
  Tensor cross_entropy(const Tensor &targets) const;
  Tensor matmul(const Tensor &o) const;

  static void realize_many(const std::vector<Tensor> &ts);
  Tensor realize() const;
  std::vector<float> to_vec() const;
  std::vector<uint8_t> to_bytes() const;  // raw bytes of the realized buffer
  std::vector<Tensor> gradient(const std::vector<Tensor> &targets) const;
  void backward() const;
  // In place, on the device stream: realizes this f32 tensor and replaces
  // its contents by their mean over the communicator's ranks (every rank
  // calls it, in the same order).  No reference counterpart.
  void all_reduce_mean(fg_comm *comm) const;

  UOpP uop() const;
  // Tensor::apply_map_to_tensors (src/tensor.rs:222-252): every live
  // tensor's graph rewritten with a schedule's replacements (realized nodes
  // -> their buffers).  Public so that another executor of a SchedulePlan
  // (the restated CPU lowering under tests/lowering) can finish a realize.
  static void apply_map_to_tensors(const std::map<const UOp *, UOpP> &repl);

 private:
  explicit Tensor(std::shared_ptr<TensorInner> p) : p_(std::move(p)) {}
  static Tensor from_uop(UOpP u, bool requires_grad);
  static Tensor from_host(DType dt, const void *data, size_t bytes, const Shape &shape);
  void set_uop(UOpP u) const;
  // The node and its shape without copying the handle or the shape (valid
  // until the tensor's node is replaced).
  const UOp &node() const;
  const Shape &shape_ref() const;
  UOpP target_uop() const;
  Tensor unary(Op op) const;
  Tensor binary(const Tensor &o, Op op, DType out) const;
  Tensor broadcasted(const Tensor &o, Op op, DType out) const;
  static std::vector<Tensor> live_tensors();
  std::shared_ptr<TensorInner> p_;
};

// nn::Linear (src/nn.rs:67-104) with the thread-local Kaiming-normal init
// (src/nn.rs:12-47).
struct Linear {
  Tensor weight;
  Tensor bias;  // undefined for without_bias
  Linear(int64_t in_features, int64_t out_features, bool with_bias = true);
  Tensor forward(const Tensor &x) const;
  std::vector<Tensor> parameters() const;
};
void reset_init_seed(uint64_t seed = 42);
uint64_t init_seed();

// optim::Sgd (src/optim.rs:29-71).
struct Sgd {
  std::vector<Tensor> params;
  float lr;
  // Data parallelism (no reference counterpart: the reference is
  // single-device): with a communicator attached, step() first realizes every
  // parameter's gradient and replaces it by its mean over the ranks
  // (Tensor::all_reduce_mean), then applies the update as always.  Every rank
  // runs the same step on its own shard of the batch from the same
  // parameters, so the parameters stay identical across ranks.
  fg_comm *comm = nullptr;
  Sgd(const std::vector<Tensor> &params, float lr);
  void zero_grad() const;
  void step() const;
};

// ---- execution (exec.cpp) ---------------------------------------------------
// Device the front end runs on: cuda:0, or FG_DEVICE=cuda:N, or set_device.
void set_device(int ordinal);
fg_device *device();
bool device_is_open();
void synchronize();
// Drops per-realize caches (staged GEMM operands); called after a realize.
void end_realize();
// fg_allreduce_mean_f32 over a whole f32 buffer on the device stream; the
// buffer's contents change, so its version moves on (cached residuals and
// cross-entropy losses of the old contents are not reused).
void all_reduce_mean_buffer(const std::shared_ptr<DeviceBuffer> &buf, fg_comm *comm);

// Per-kernel routing decision for an item, without running it.
struct RoutePlan {
  std::string route;              // "gemm", "reduce_rows", "reduce_cols", "rendered", "alias"
  std::vector<std::string> steps;  // sub-steps (extracted contractions, etc.)
};
RoutePlan plan_route(const ScheduleItem &item);
void run_item(const ScheduleItem &item);

struct Stats {
  uint64_t kernels = 0;      // schedule items executed
  uint64_t gemm = 0;         // contractions run on the tensor-core GEMM
  uint64_t hand_reduce = 0;  // reductions run on the hand-written HBM kernels
  uint64_t xent = 0;         // fused cross-entropy passes (fg_xent_fwd_bwd)
  uint64_t xent_reused = 0;  // losses taken from an earlier XentGrad pass
  uint64_t sgd = 0;          // parameter stores run on the fused SGD kernel
  uint64_t gemm_bias = 0;    // GEMMs with the bias epilogue (Linear::forward)
  uint64_t gemm_mask = 0;    // GEMMs with the ReLU-mask epilogue (relu's gradient)
  uint64_t rendered = 0;     // launches of NVRTC-rendered kernels
  uint64_t compiled = 0;     // NVRTC compilations (program cache misses)
  uint64_t cache_hits = 0;
  uint64_t schedule_hits = 0;  // realizes that reused a cached schedule
  // host time inside realize_many, seconds: scheduling, enqueueing the
  // items (routing, program lookup, launches) and the live-tensor rewrite
  double schedule_s = 0, run_s = 0, rewrite_s = 0;
};
Stats &stats();
void reset_stats();
// Source of the most recently rendered kernel.
const std::string &last_source();
// Render an item's generic kernel without compiling it (tests, DEBUG=4).
std::string render_item_source(const ScheduleItem &item);

}  // namespace ferro
