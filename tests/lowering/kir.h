// kir.h -- kernel-level IR of the reference's CPU lowering (TEST
// INFRASTRUCTURE: a second oracle; nothing in the product links it).
//
// A restatement of the reference's UOp as its lowering passes see it
// (src/uop.rs:12-170, 263-330): the op set including the kernel-level ops
// (Range, End, Index, Load, Reduce, DefineAcc, Assign, Vectorize, Unroll,
// Contract, Gep), dtypes with a lane count (src/dtype.rs), the Arg variants,
// an optional tag, and hash-consing so that structurally equal nodes are the
// same object (pointer identity is value identity, as UOp's PartialEq).
#pragma once
#include <cstdint>
#include <functional>
#include <memory>
#include <optional>
#include <string>
#include <unordered_map>
#include <utility>
#include <vector>

namespace kir {

enum class Op : uint8_t {
  Device, DefineVar, Bind, Buffer, Shrink, Reshape, Permute, Expand, Contiguous, ReduceAxis,
  ParamBuffer, ParamScalar, Range, End, Sink, Index, Load, Store, Vectorize, Unroll, Contract,
  Const, Neg, Exp2, Log2, Sqrt, Reciprocal, Add, Mul, Max, CmpLt, Where, Reduce, After, DefineAcc,
  Assign, Gep,
};
const char *op_name(Op op);
bool is_alu(Op op);
bool is_movement(Op op);

enum class Kind : uint8_t { F32, I32, Bool, Void };
struct DType {
  Kind kind = Kind::F32;
  uint16_t vcount = 1;
  static DType f32() { return {Kind::F32, 1}; }
  static DType i32() { return {Kind::I32, 1}; }
  static DType boolean() { return {Kind::Bool, 1}; }
  static DType void_() { return {Kind::Void, 1}; }
  DType vec(uint16_t n) const { return {kind, n}; }
  DType scalar() const { return {kind, 1}; }
  bool is_scalar() const { return vcount == 1; }
  const char *c_type() const;
  bool operator==(const DType &o) const { return kind == o.kind && vcount == o.vcount; }
  bool operator!=(const DType &o) const { return !(*this == o); }
};

enum class Axis : uint8_t { Loop, Global, Local, Reduce, GroupReduce, Upcast, Unroll, Thread };

struct Arg {
  enum Tag : uint8_t {
    None, Index, Range, ParamBuffer, ParamScalar, Float, Int, Bool, Bounds, Shape, Axes, Lanes,
    Reduce
  };
  Tag tag = None;
  int64_t a = 0, b = 0;  // Index(a); Range(axis a, kind b); ParamBuffer(slot a, numel b);
                         // ParamScalar(a); Int(a); Bool(a)
  double f = 0.0;        // Float
  std::vector<int64_t> v;                         // Bounds / Shape / Axes / Reduce axes
  std::vector<std::pair<int64_t, int64_t>> lanes;  // Lanes
  Op rop = Op::Add;                               // Reduce

  static Arg none() { return {}; }
  static Arg index(int64_t i) { Arg r; r.tag = Index; r.a = i; return r; }
  static Arg range(int64_t axis, Axis k) { Arg r; r.tag = Range; r.a = axis; r.b = (int64_t)k; return r; }
  static Arg param_buffer(int64_t slot, int64_t n) { Arg r; r.tag = ParamBuffer; r.a = slot; r.b = n; return r; }
  static Arg param_scalar(int64_t slot) { Arg r; r.tag = ParamScalar; r.a = slot; return r; }
  static Arg flt(double x) { Arg r; r.tag = Float; r.f = x; return r; }
  static Arg integer(int64_t x) { Arg r; r.tag = Int; r.a = x; return r; }
  static Arg boolean(bool x) { Arg r; r.tag = Bool; r.a = x; return r; }
  static Arg bounds(std::vector<int64_t> x) { Arg r; r.tag = Bounds; r.v = std::move(x); return r; }
  static Arg shape(std::vector<int64_t> x) { Arg r; r.tag = Shape; r.v = std::move(x); return r; }
  static Arg axes(std::vector<int64_t> x) { Arg r; r.tag = Axes; r.v = std::move(x); return r; }
  static Arg lanes_of(std::vector<std::pair<int64_t, int64_t>> x) { Arg r; r.tag = Lanes; r.lanes = std::move(x); return r; }
  static Arg reduce(Op op, std::vector<int64_t> ax) { Arg r; r.tag = Reduce; r.rop = op; r.v = std::move(ax); return r; }

  bool is_range(Axis k) const { return tag == Range && b == (int64_t)k; }
  Axis axis_kind() const { return (Axis)b; }
  bool operator==(const Arg &o) const;
  bool operator!=(const Arg &o) const { return !(*this == o); }
  std::string str() const;
};

struct Node;
using U = std::shared_ptr<const Node>;

struct Node {
  Op op;
  DType dtype;
  std::vector<U> src;
  Arg arg;
  std::optional<uint64_t> tag;
};

// Hash-consed constructor (intern_uop, src/uop.rs:285-310).
U make(Op op, DType dt, std::vector<U> src, Arg arg = Arg::none(),
       std::optional<uint64_t> tag = std::nullopt);

// Leaves and helpers of src/uop.rs:330-700.
U device();
U param_buffer(int64_t slot, DType dt, int64_t numel);
U param_scalar(int64_t slot, DType dt);
U const_float(double v, DType dt);
U const_int(int64_t v, DType dt);
U const_bool(bool v, DType dt);
U add(const U &a, const U &b);
U mul(const U &a, const U &b);
U neg(const U &a);
U store(const U &dest, const U &value);
U after(const U &value, const U &effect);
U sink(std::vector<U> srcs);
U gep(const U &x, size_t i);
U reshape(const U &s, std::vector<int64_t> shape);
U reduce_axis(const U &s, Op rop, std::vector<int64_t> axes);

bool is_const(const U &u);
bool is_zero(const U &u);
bool is_one(const U &u);
std::optional<int64_t> const_i32(const U &u);  // optimize/mod.rs const_i32
// The tensor-level shape (src/uop.rs:436-505), or nothing.
std::optional<std::vector<int64_t>> shape_of(const U &u);

// Sources before consumers; After walks its sources first-pushed-first
// (src/uop.rs:704-732).
std::vector<U> toposort(const U &root);
std::string dump(const U &root);
// Ranges a node closes: End -> its range, After -> those of its effects.
std::vector<U> ended_ranges(const U &node);

// Two behaviours of the reference's lowering that change results once the
// upcast pass has split an output loop, restated as read:
//  * a node whose sources changed is rebuilt with UOp::new, which carries no
//    tag (src/rewrite.rs:54 and :104, src/devectorize.rs:432), so the lane
//    accumulators of one reduction -- DefineAccs told apart only by their
//    tags (src/devectorize.rs:292-320) -- become one node when linearize's
//    control-flow edges (src/linearize.rs:204-290) rebuild a range they
//    depend on, i.e. whenever the reduction sits in a nested output loop;
//  * reduce_lane_groups (src/devectorize.rs:147-180, the flat index at :171)
//    takes the contracted (unrolled reduce) lanes as the fastest-varying
//    ones, which they are not when the reduced axis is numbered before the
//    upcast output axis (lanes are sorted by axis, src/expand.rs:282);
//  * lanes are identified by axis number (src/expand.rs:88-117), and output
//    axes (numbered over the stored value's shape) and reduce axes (over the
//    reduced source's shape) are numbered independently, so an upcast lane
//    and an unroll lane can carry the same id and be merged as one.
// And one that needs no upcast: a reduction whose value does not depend on
// its reduce range (a constant broadcast and summed, as a gradient of sum
// builds) gets an update that the linearizer is free to hoist out of the
// loop (src/devectorize.rs:274-330 with src/linearize.rs:79-100 priorities),
// so it is applied once; with the range unrolled the Contract of a
// lane-invariant value is never lowered and rendering stops
// (src/devectorize.rs:147-150, src/codegen/clang.rs:260).
// set_repair(true) keeps tags across rebuilds, groups lanes by their axes,
// gives upcast lanes ids of their own, makes the update depend on the reduce
// ranges and expands a lane-invariant contracted value to its lanes (not
// the reference; used to show that these are the only differences).
void set_repair(bool on);
bool repair();
std::optional<uint64_t> rebuilt_tag(const Node &n);

// src/rewrite.rs: fixed-point rewrite, map substitution, End/Sink flattening.
using Rule = std::function<U(const U &)>;
U graph_rewrite(const U &root, const Rule &rule);
U substitute(const U &root, const std::unordered_map<const Node *, U> &repl);
U flatten_end_bodies(const U &node);
U flatten_nested_sinks(const U &node);

// ---- passes (passes.cpp) ------------------------------------------------
U rangeify(const U &sink);                      // src/schedule/rangeify.rs
U upcast_loops(const U &root);                  // src/optimize/upcast.rs
U unroll_reduce_loops(const U &root);           // src/optimize/unroll.rs
U symbolic_simple(const U &node);               // src/optimize/symbolic.rs
struct OptimizeConfig { bool symbolic = true, upcast = true, unroll = true; };
U optimize(const U &kernel, const OptimizeConfig &c);  // src/optimize/mod.rs
U late_expand(const U &root);                   // src/expand.rs
U devectorize(const U &root);                   // src/devectorize.rs
std::vector<U> linearize(const U &root);        // src/linearize.rs
std::string render_c(const std::vector<U> &uops, const std::string &name);  // src/codegen/clang.rs

// The Const literal as the reference's renderer prints it.
std::string c_literal(const Node &n);

}  // namespace kir
