// front_internal.h -- declarations shared by the front end's translation units.
#pragma once
#include <map>
#include <optional>
#include <stdexcept>
#include <string>
#include <unordered_map>
#include <vector>

#include "ferro_front.h"

namespace ferro {

// The reference panics on misuse (assert!/expect); the front end throws.
struct Panic : std::runtime_error {
  using std::runtime_error::runtime_error;
};

// Slot assignment of a kernel's inputs (src/schedule.rs:176-245).
struct ParamSlots {
  std::vector<KernelInput> inputs;  // in slot order, starting at slot_offset
  std::unordered_map<const DeviceBuffer *, int> buffer_slot;
  // For each Shrink node: per-axis scalar slot of its start, or -1 when the
  // start stays a literal (full-length axis).
  std::unordered_map<const UOp *, std::vector<int>> shrink_slots;
};
ParamSlots collect_params(const UOpP &root, int slot_offset);
// The same over an existing toposort of the kernel's root.
ParamSlots collect_params_from(const std::vector<const UOp *> &order, int slot_offset);

// A node's value as a strided view of one buffer: element (c0..cn) of the
// node is buf[offset + sum_a c_a * strides[a]].
struct View {
  BufferP buf;
  int64_t offset = 0;
  Shape shape;
  std::vector<int64_t> strides;
};
// The view of a movement chain (Reshape/Permute/Expand/Shrink with literal
// starts) over a Buffer, or nothing when some step is not a strided view.
std::optional<View> try_view(const UOp *n);

UOpP substitute_materialized(const UOpP &root, const std::map<const UOp *, UOpP> &repl);

// Rewrites graphs under one replacement map: every node at or above a
// replaced node is rebuilt (interned) over its sources' rewritten forms, and
// the rest come back unchanged.  Each node's result is remembered in the node
// itself (UOp::memo_mark / memo_slot) instead of a hash map, so the subgraphs
// shared by all graphs given to one Rewriter are rewritten once.  Only one
// Rewriter may be live at a time (a second one throws).
class Rewriter {
 public:
  template <typename Map>
  explicit Rewriter(const Map &repl) : Rewriter() {
    for (auto &[node, with] : repl) remember(node, with);
  }
  ~Rewriter();
  Rewriter(const Rewriter &) = delete;
  Rewriter &operator=(const Rewriter &) = delete;
  // Adds a replacement (for a node this rewriter has not met yet).
  void replace(const UOp *node, const UOpP &with) { remember(node, with); }
  UOpP operator()(const UOpP &root);

 private:
  Rewriter();
  bool done(const UOp *n) const { return n->memo_mark == mark_; }
  void remember(const UOp *n, UOpP v) {
    n->memo_mark = mark_;
    n->memo_slot = (uint32_t)vals_.size();
    vals_.push_back(std::move(v));
  }
  uint64_t mark_;
  std::vector<UOpP> vals_;
};

// ---- CUDA C renderer (render.cpp) -----------------------------------------
// One rendered kernel: thread t of the grid evaluates `value` at the domain
// coordinates of element(s) t and stores the result.
struct RenderSpec {
  UOpP value;
  Shape domain;                    // iteration shape (row-major element order)
  // Index expression per axis of value's shape in terms of the domain
  // coordinates c0..c{n-1}; empty means value's shape == domain.
  std::vector<std::string> value_ctx;
  enum Store { Contig, Pitched, View } store = Contig;
  int64_t pitch = 0;  // Pitched: out[c0 * pitch + c1] over a 2-D domain
  UOpP dest;          // View: movement chain over the destination buffer
  DType out_dtype = DType::F32;
  int unroll = 1;     // elements per thread
  // Thread mapping of a kernel with reductions.  Thread: one thread per
  // output element, each reduction walked sequentially in the reference's
  // order.  Warp: one warp per output element; the lanes split the
  // reduction's innermost reduced axis and fold their partials with a
  // shuffle tree.  Block: 32 output elements per 1024-thread block, one per
  // lane; the 32 warps split the reduced axis and fold through shared memory.
  // Warp and Block change the summation order, so only the default mode
  // (not FG_FRONT_EXACT) picks them (choose_thread_mapping).
  enum Coop { Thread, Warp, Block } coop = Thread;
  // f32 stores only: the kernel takes one more argument after its inputs,
  // plo, and stores there the TF32 residual of each value (v minus v with its
  // low 13 mantissa bits cleared, as fg_split_lo), a GEMM operand's `lo`.
  bool with_lo = false;
};

// Picks spec.coop from the kernel's reductions: Warp when the longest
// reduced axis (>= 32 elements) is its source's innermost axis, Block when it
// is an outer axis and the kernel has few outputs, else Thread.
void choose_thread_mapping(RenderSpec &spec);

struct RenderedKernel {
  std::string source;
  uint32_t grid = 1, block = 256;
  // Arguments in slot order: slot 0 is the output for Contig/Pitched stores.
  bool has_out_slot = true;
  std::vector<KernelInput> params;  // slots after the output slot
};
RenderedKernel render_kernel(const RenderSpec &spec);

// Float literal as the reference prints constants: from the f64 value with
// an f suffix (src/codegen/clang.rs).
std::string float_literal(double v);

// Environment flag: FG_FRONT_EXACT=1 renders every kernel (no GEMM or
// hand-written reductions), reproducing the reference's arithmetic order.
bool exact_mode();
// Inside a realize the flag is read once, at its start: every kernel of one
// realize runs in the same mode, and the per-kernel lookups cost nothing.
struct ExactModeScope {
  ExactModeScope();
  ~ExactModeScope();
  int prev;
};
int debug_level();
// The reference's OPT environment variable (src/optimize/mod.rs:80-112),
// read once per process: "0"/"off"/"none" disables every pass, "1"/"on"/
// "all" or unset enables every pass, otherwise a comma list of "symbolic",
// "upcast", "unroll".  unroll decides the reduction order (4-lane blocks)
// and symbolic the constant folds of rendered kernels; upcast, as the
// reference's passes intend it, only changes the loop structure (as they are
// written it also changes values in some kernels -- the restated lowering in
// tests/lowering/kir.h lists where -- which the front end does not copy).
struct OptimizeConfig {
  bool symbolic = true, upcast = true, unroll = true;
};
OptimizeConfig parse_optimize_config(const char *raw);
const OptimizeConfig &optimize_config();

// Device-side conversions behind Tensor::from_u8_div / one_hot_u8.
BufferP device_u8_to_f32(const uint8_t *data, size_t n, float divisor);
BufferP device_one_hot_u8(const uint8_t *labels, size_t n, int classes);

}  // namespace ferro
