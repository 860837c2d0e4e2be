// cases.cpp -- the reference's own unit tests of its lowering passes,
// restated over the kernel IR (TEST INFRASTRUCTURE).  Each case names the
// reference test it follows; the assertions are the reference's.
#include <algorithm>
#include <cmath>
#include <functional>
#include <stdexcept>
#include <string>
#include <vector>

#include "kir.h"
#include "lowering.h"

namespace kir {
namespace {

struct CaseFail : std::runtime_error {
  using std::runtime_error::runtime_error;
};
#define CHECK(cond)                                                                    \
  do {                                                                                 \
    if (!(cond)) throw CaseFail(std::string("check failed: ") + #cond + " (line " + \
                                std::to_string(__LINE__) + ")");                       \
  } while (0)

U range_(int64_t n, int64_t axis, Axis k) {
  return make(Op::Range, DType::i32(), {const_int(n, DType::i32())}, Arg::range(axis, k));
}
U index_(const U &buf, const U &i) { return make(Op::Index, buf->dtype, {buf, i}); }
U load_(const U &idx) { return make(Op::Load, DType::f32(), {idx}); }
U end_(std::vector<U> s) { return make(Op::End, DType::void_(), std::move(s)); }
int64_t bound(const U &r) { return r->src.at(0)->arg.a; }

std::vector<U> filter(const std::vector<U> &order, const std::function<bool(const U &)> &f) {
  std::vector<U> r;
  for (const U &n : order)
    if (f(n)) r.push_back(n);
  return r;
}
bool any_of(const std::vector<U> &order, const std::function<bool(const U &)> &f) {
  return std::any_of(order.begin(), order.end(), f);
}
std::vector<U> ranges_of(const std::vector<U> &order) {
  return filter(order, [](const U &n) { return n->op == Op::Range; });
}

// src/optimize/upcast.rs tests: build_add_graph
U build_add_graph(int64_t n) {
  U out = param_buffer(0, DType::f32(), n), a = param_buffer(1, DType::f32(), n);
  U idx = range_(n, 0, Axis::Loop);
  U sum = add(load_(index_(a, idx)), const_float(1.0, DType::f32()));
  U st = store(index_(out, idx), sum);
  return sink({end_({idx, st})});
}

U build_matmul_like_kernel(int64_t m, int64_t n, int64_t k) {
  U out = param_buffer(0, DType::f32(), m * n), lhs = param_buffer(1, DType::f32(), m * k),
    rhs = param_buffer(2, DType::f32(), n * k);
  U mr = range_(m, 0, Axis::Loop), nr = range_(n, 1, Axis::Loop), kr = range_(k, 2, Axis::Reduce);
  U oi = index_(out, add(mul(mr, const_int(n, DType::i32())), nr));
  U li = index_(lhs, add(mul(mr, const_int(k, DType::i32())), kr));
  U ri = index_(rhs, add(mul(nr, const_int(k, DType::i32())), kr));
  U value = mul(load_(li), load_(ri));
  U red = make(Op::Reduce, DType::f32(), {value, kr}, Arg::reduce(Op::Add, {}));
  U st = store(oi, red);
  return sink({end_({mr, end_({nr, st})})});
}

U build_scaled_plane_reduce_graph(int64_t depth, int64_t rows, int64_t cols) {
  U out = param_buffer(0, DType::f32(), rows * cols);
  U base = param_buffer(1, DType::f32(), rows * cols);
  U input = param_buffer(2, DType::f32(), depth * rows * cols);
  U scale = param_buffer(3, DType::f32(), 1);
  U reduced = reduce_axis(reshape(input, {depth, rows, cols}), Op::Add, {0});
  reduced = reshape(reduced, {rows, cols});
  U b = reshape(base, {rows, cols});
  U sc = make(Op::Expand, DType::f32(), {reshape(scale, {1, 1})}, Arg::shape({rows, cols}));
  U updated = add(b, neg(mul(reduced, sc)));
  return sink({store(out, updated)});
}

U build_reduce_graph(int64_t n) {
  U out = param_buffer(0, DType::f32(), 1), in = param_buffer(1, DType::f32(), n);
  return sink({store(out, reduce_axis(reshape(in, {n}), Op::Add, {0}))});
}

U build_row_reduce_graph(int64_t rows, int64_t cols) {
  U out = param_buffer(0, DType::f32(), rows), in = param_buffer(1, DType::f32(), rows * cols);
  return sink({store(out, reduce_axis(reshape(in, {rows, cols}), Op::Add, {1}))});
}

std::vector<Case> build_cases() {
  std::vector<Case> c;
  // ---- src/schedule/rangeify.rs ----
  c.push_back({"rangeify::singleton_output_axis_flattens_from_full_rank_indices", [] {
    U out = param_buffer(0, DType::f32(), 3), in = param_buffer(1, DType::f32(), 6);
    U narrowed = make(Op::Shrink, DType::f32(),
                      {reshape(in, {2, 3}), const_int(1, DType::i32()), const_int(0, DType::i32())},
                      Arg::bounds({1, 3}));
    U s = sink({make(Op::Store, DType::void_(), {out, narrowed})});
    U simplified = graph_rewrite(rangeify(s), symbolic_simple);
    auto order = toposort(simplified);
    auto ranges = ranges_of(order);
    CHECK(ranges.size() == 1);
    auto st = filter(order, [](const U &n) { return n->op == Op::Store; });
    CHECK(!st.empty());
    const U &oi = st[0]->src[0];
    CHECK(oi->op == Op::Index);
    CHECK(oi->src[1] == ranges[0]);
  }});
  c.push_back({"rangeify::marks_output_and_reduce_axes", [] {
    U out = param_buffer(0, DType::f32(), 2), in = param_buffer(1, DType::f32(), 6);
    U s = sink({make(Op::Store, DType::void_(),
                     {out, reduce_axis(reshape(in, {2, 3}), Op::Add, {1})})});
    auto ranges = ranges_of(toposort(rangeify(s)));
    CHECK(ranges.size() == 2);
    CHECK(any_of(ranges, [](const U &r) { return r->arg == Arg::range(0, Axis::Loop); }));
    CHECK(any_of(ranges, [](const U &r) { return r->arg == Arg::range(1, Axis::Reduce); }));
  }});
  // ---- src/optimize/upcast.rs ----
  c.push_back({"upcast::splits_innermost_loop_by_four", [] {
    auto order = toposort(upcast_loops(build_add_graph(8)));
    auto ranges = ranges_of(order);
    CHECK(ranges.size() == 2);
    CHECK(ranges[0]->arg == Arg::range(0, Axis::Global));
    CHECK(bound(ranges[0]) == 2);
    CHECK(ranges[1]->arg == Arg::range(0, Axis::Upcast));
    CHECK(bound(ranges[1]) == 4);
    CHECK(filter(order, [](const U &n) { return n->op == Op::Store; }).size() == 1);
  }});
  c.push_back({"upcast::skips_reduction_bodies", [] {
    U out = param_buffer(0, DType::f32(), 1), in = param_buffer(1, DType::f32(), 8);
    U s = sink({store(out, reduce_axis(reshape(in, {2, 4}), Op::Add, {1}))});
    U r = rangeify(s);
    CHECK(upcast_loops(r) == r);
  }});
  c.push_back({"upcast::targets_trailing_matmul_output_axis", [] {
    auto order = toposort(upcast_loops(build_matmul_like_kernel(8, 8, 8)));
    CHECK(any_of(order, [](const U &n) { return n->arg == Arg::range(1, Axis::Upcast); }));
    CHECK(any_of(order, [](const U &n) { return n->arg == Arg::range(0, Axis::Loop); }));
    CHECK(!any_of(order, [](const U &n) { return n->arg == Arg::range(0, Axis::Upcast); }));
  }});
  c.push_back({"upcast::skips_post_reduce_store_alu", [] {
    U r = rangeify(build_scaled_plane_reduce_graph(8, 8, 8));
    CHECK(upcast_loops(r) == r);
  }});
  // ---- src/optimize/unroll.rs ----
  auto reduce_ranges = [](const U &root) {
    auto order = toposort(root);
    return std::make_pair(ranges_of(order),
                          filter(order, [](const U &n) { return n->op == Op::Reduce; }));
  };
  c.push_back({"unroll::splits_constant_reduce_by_four", [reduce_ranges] {
    auto [ranges, reds] = reduce_ranges(unroll_reduce_loops(rangeify(build_reduce_graph(8))));
    CHECK(ranges.size() == 2);
    CHECK(ranges[0]->arg == Arg::range(0, Axis::Reduce));
    CHECK(bound(ranges[0]) == 2);
    CHECK(ranges[1]->arg == Arg::range(0, Axis::Unroll));
    CHECK(bound(ranges[1]) == 4);
    CHECK(reds.size() == 1);
    CHECK(reds[0]->src[1] == ranges[0]);
    CHECK(reds[0]->src[2] == ranges[1]);
  }});
  c.push_back({"unroll::skips_non_divisible_reduce", [reduce_ranges] {
    auto [ranges, reds] = reduce_ranges(unroll_reduce_loops(rangeify(build_reduce_graph(6))));
    CHECK(ranges.size() == 1);
    CHECK(ranges[0]->arg == Arg::range(0, Axis::Reduce));
    CHECK(bound(ranges[0]) == 6);
    CHECK(reds.size() == 1);
  }});
  c.push_back({"unroll::does_not_resplit_outer_reduce", [reduce_ranges] {
    auto [ranges, reds] = reduce_ranges(unroll_reduce_loops(rangeify(build_reduce_graph(64))));
    CHECK(ranges.size() == 2);
    CHECK(ranges[0]->arg == Arg::range(0, Axis::Reduce));
    CHECK(bound(ranges[0]) == 16);
    CHECK(ranges[1]->arg == Arg::range(0, Axis::Unroll));
    CHECK(bound(ranges[1]) == 4);
    CHECK(reds.size() == 1);
  }});
  c.push_back({"unroll::composes_with_upcast", [] {
    auto order = toposort(unroll_reduce_loops(upcast_loops(rangeify(build_row_reduce_graph(8, 8)))));
    CHECK(any_of(order, [](const U &n) { return n->arg.is_range(Axis::Unroll); }));
  }});
  // ---- src/optimize/symbolic.rs ----
  c.push_back({"symbolic::add_zero_eliminated", [] {
    U r = graph_rewrite(add(const_float(5.0, DType::f32()), const_float(0.0, DType::f32())),
                        symbolic_simple);
    CHECK(r->op == Op::Const && r->arg == Arg::flt(5.0));
  }});
  c.push_back({"symbolic::zero_plus_x_eliminated", [] {
    U r = graph_rewrite(add(const_float(0.0, DType::f32()), const_float(5.0, DType::f32())),
                        symbolic_simple);
    CHECK(r->op == Op::Const && r->arg == Arg::flt(5.0));
  }});
  c.push_back({"symbolic::constant_folding_add", [] {
    U r = graph_rewrite(add(const_float(2.0, DType::f32()), const_float(3.0, DType::f32())),
                        symbolic_simple);
    CHECK(r->op == Op::Const && r->arg == Arg::flt(5.0));
  }});
  c.push_back({"symbolic::fixed_point_chains_identities", [] {
    U x = add(const_float(7.0, DType::f32()), const_float(0.0, DType::f32()));
    U r = graph_rewrite(mul(x, const_float(1.0, DType::f32())), symbolic_simple);
    CHECK(r->op == Op::Const && r->arg == Arg::flt(7.0));
  }});
  c.push_back({"symbolic::mul_zero", [] {
    U r = graph_rewrite(mul(const_float(42.0, DType::f32()), const_float(0.0, DType::f32())),
                        symbolic_simple);
    CHECK(r->op == Op::Const && r->arg == Arg::flt(0.0));
  }});
  // ---- src/expand.rs ----
  c.push_back({"expand::late_expand_materializes_upcast_lanes", [] {
    auto order = toposort(late_expand(upcast_loops(build_add_graph(8))));
    CHECK(!any_of(order, [](const U &n) { return n->arg.is_range(Axis::Upcast); }));
    CHECK(any_of(order, [](const U &n) { return n->op == Op::Unroll; }));
  }});
  c.push_back({"expand::late_expand_rewrites_reduce_unroll_to_contract", [] {
    auto order = toposort(late_expand(unroll_reduce_loops(rangeify(build_reduce_graph(8)))));
    CHECK(any_of(order, [](const U &n) { return n->op == Op::Contract; }));
    CHECK(!any_of(order, [](const U &n) { return n->arg.is_range(Axis::Unroll); }));
  }});
  c.push_back({"expand::late_expand_keeps_reduce_lane_aware_under_upcast", [] {
    U opt = unroll_reduce_loops(upcast_loops(rangeify(build_row_reduce_graph(8, 8))));
    auto order = toposort(late_expand(opt));
    CHECK(any_of(order, [](const U &n) { return n->op == Op::Reduce; }));
    CHECK(any_of(order, [](const U &n) { return n->op == Op::Contract; }));
    CHECK(any_of(order, [](const U &n) { return n->op == Op::Unroll; }));
  }});
  // ---- src/devectorize.rs ----
  c.push_back({"devectorize::lowers_scalar_reduce_to_accumulator_loop", [] {
    auto order = toposort(devectorize(late_expand(rangeify(build_reduce_graph(8)))));
    CHECK(any_of(order, [](const U &n) { return n->op == Op::DefineAcc; }));
    CHECK(any_of(order, [](const U &n) { return n->op == Op::Assign; }));
    CHECK(!any_of(order, [](const U &n) { return n->op == Op::Reduce; }));
  }});
  c.push_back({"devectorize::lowers_upcast_unroll_reduce_to_multiple_accumulators", [] {
    U opt = unroll_reduce_loops(upcast_loops(rangeify(build_row_reduce_graph(8, 8))));
    auto order = toposort(devectorize(late_expand(opt)));
    CHECK(!any_of(order, [](const U &n) { return n->op == Op::Reduce || n->op == Op::Contract; }));
    CHECK(!any_of(order, [](const U &n) { return n->arg.is_range(Axis::Unroll); }));
    CHECK(filter(order, [](const U &n) { return n->op == Op::DefineAcc; }).size() == 4);
  }});
  // ---- src/linearize.rs ----
  c.push_back({"linearize::closes_first_loop_before_second_opens", [] {
    U out = param_buffer(0, DType::f32(), 2);
    U n = const_int(1, DType::i32());
    U i0 = make(Op::Range, DType::i32(), {n}, Arg::range(0, Axis::Loop));
    U e0 = end_({i0, store(index_(out, i0), const_float(1.0, DType::f32()))});
    U i1 = make(Op::Range, DType::i32(), {n}, Arg::range(1, Axis::Loop));
    U e1 = end_({i1, store(index_(out, const_int(1, DType::i32())), const_float(2.0, DType::f32()))});
    auto lin = linearize(sink({e0, e1}));
    auto find = [&lin](Op op, const Arg &a) {
      for (size_t i = 0; i < lin.size(); i++)
        if (lin[i]->op == op && lin[i]->arg == a) return i;
      throw CaseFail("node should exist in linearized output");
    };
    size_t r0 = find(Op::Range, Arg::range(0, Axis::Loop)), r1 = find(Op::Range, Arg::range(1, Axis::Loop));
    std::vector<size_t> ends;
    for (size_t i = 0; i < lin.size(); i++)
      if (lin[i]->op == Op::End) ends.push_back(i);
    CHECK(ends.size() >= 1);
    CHECK(r0 < ends[0]);
    CHECK(ends[0] < r1);
  }});
  c.push_back({"linearize::places_accumulator_before_reduce_loop", [] {
    U out = param_buffer(0, DType::f32(), 1), in = param_buffer(1, DType::f32(), 4);
    U outer = range_(1, 0, Axis::Loop), red = range_(4, 1, Axis::Reduce);
    U val = load_(index_(in, red));
    U acc = make(Op::DefineAcc, DType::f32(), {const_float(0.0, DType::f32())});
    U upd = make(Op::Assign, DType::f32(), {acc, make(Op::Add, DType::f32(), {acc, val})});
    U rend = end_({red, upd});
    U st = store(index_(out, outer), after(acc, rend));
    auto lin = linearize(sink({end_({outer, st})}));
    auto pos = [&lin](const std::function<bool(const U &)> &f) {
      for (size_t i = 0; i < lin.size(); i++)
        if (f(lin[i])) return i;
      throw CaseFail("node should exist");
    };
    CHECK(pos([](const U &n) { return n->op == Op::DefineAcc; }) <
          pos([](const U &n) { return n->arg.is_range(Axis::Reduce); }));
  }});
  // ---- src/codegen/clang.rs ----
  auto build_clang_add = [](int64_t n) {
    U out = param_buffer(0, DType::f32(), 3), a = param_buffer(1, DType::f32(), 3),
      b = param_buffer(2, DType::f32(), 3);
    U idx = range_(n, 0, Axis::Loop);
    U sum = add(load_(index_(a, idx)), load_(index_(b, idx)));
    U st = store(index_(out, idx), sum);
    return sink({st, end_({idx, st})});
  };
  auto contains = [](const std::string &s, const std::string &x) {
    return s.find(x) != std::string::npos;
  };
  c.push_back({"clang::render_add_kernel_structure", [build_clang_add, contains] {
    std::string code = render_c(linearize(build_clang_add(3)), "add");
    CHECK(contains(code, "void add("));
    CHECK(contains(code, "float* restrict data0"));
    CHECK(contains(code, "float* restrict data1"));
    CHECK(contains(code, "float* restrict data2"));
    CHECK(contains(code, "for (int idx0 = 0; idx0 < 3; idx0++)"));
    CHECK(contains(code, "float val"));
    CHECK(contains(code, "float alu"));
  }});
  c.push_back({"clang::render_add_kernel_compiles_and_runs", [build_clang_add] {
    std::string code = render_c(linearize(build_clang_add(3)), "add");
    std::vector<float> out(3), a{1, 2, 3}, b{4, 5, 6};
    run_c(code, "add", {out.data(), a.data(), b.data()});
    CHECK(out == (std::vector<float>{5, 7, 9}));
  }});
  c.push_back({"clang::render_negate_kernel", [] {
    U out = param_buffer(0, DType::f32(), 3), a = param_buffer(1, DType::f32(), 3);
    U idx = range_(3, 0, Axis::Loop);
    U st = store(index_(out, idx), neg(load_(index_(a, idx))));
    std::string code = render_c(linearize(sink({st, end_({idx, st})})), "negate");
    std::vector<float> o(3), x{1, -2, 3};
    run_c(code, "negate", {o.data(), x.data()});
    CHECK(o == (std::vector<float>{-1, 2, -3}));
  }});
  c.push_back({"clang::render_relu_kernel", [] {
    U out = param_buffer(0, DType::f32(), 4), a = param_buffer(1, DType::f32(), 4);
    U zero = const_float(0.0, DType::f32());
    U idx = range_(4, 0, Axis::Loop);
    U v = load_(index_(a, idx));
    U relu = make(Op::Where, DType::f32(), {make(Op::CmpLt, DType::boolean(), {zero, v}), v, zero});
    U st = store(index_(out, idx), relu);
    std::string code = render_c(linearize(sink({st, end_({idx, st})})), "relu");
    std::vector<float> o(4), x{1, -2, 3, -4};
    run_c(code, "relu", {o.data(), x.data()});
    CHECK(o == (std::vector<float>{1, 0, 3, 0}));
  }});
  c.push_back({"clang::render_reduce_range_uses_same_loop_codegen", [contains] {
    U red = range_(4, 1, Axis::Reduce);
    std::string code = render_c(linearize(sink({end_({red})})), "noop_reduce");
    CHECK(contains(code, "for (int ridx1 = 0; ridx1 < 4; ridx1++)"));
  }});
  c.push_back({"clang::render_loop_and_reduce_axes_use_distinct_names", [contains] {
    U lr = range_(3, 0, Axis::Loop), rr = range_(2, 0, Axis::Reduce);
    std::string code = render_c(linearize(sink({end_({lr, end_({rr})})})), "nested_ranges");
    CHECK(contains(code, "for (int idx0 = 0; idx0 < 3; idx0++)"));
    CHECK(contains(code, "for (int ridx0 = 0; ridx0 < 2; ridx0++)"));
  }});
  auto build_shared_reduce = [] {
    U ob = param_buffer(0, DType::f32(), 2), ib = param_buffer(1, DType::f32(), 6);
    U width = const_int(2, DType::i32()), rb = const_int(3, DType::i32());
    U ninf = const_float(-INFINITY, DType::f32());
    U outer = make(Op::Range, DType::i32(), {const_int(1, DType::i32())}, Arg::range(0, Axis::Loop));
    U red = make(Op::Range, DType::i32(), {rb}, Arg::range(1, Axis::Reduce));
    U base = mul(outer, width);
    U l0 = add(base, const_int(0, DType::i32())), l1 = add(base, const_int(1, DType::i32()));
    U v0 = load_(index_(ib, add(mul(l0, rb), red))), v1 = load_(index_(ib, add(mul(l1, rb), red)));
    U a0 = make(Op::DefineAcc, DType::f32(), {ninf}, Arg::none(), 1);
    U a1 = make(Op::DefineAcc, DType::f32(), {ninf}, Arg::none(), 2);
    U u0 = make(Op::Assign, DType::f32(), {a0, make(Op::Max, DType::f32(), {a0, v0})});
    U u1 = make(Op::Assign, DType::f32(), {a1, make(Op::Max, DType::f32(), {a1, v1})});
    U rend = end_({red, u0, u1});
    U s0 = store(index_(ob, l0), after(a0, rend)), s1 = store(index_(ob, l1), after(a1, rend));
    return sink({end_({outer, s0, s1})});
  };
  c.push_back({"clang::render_shared_reduce_multi_acc_declares_accumulators_before_loop",
               [build_shared_reduce] {
    std::string code = render_c(linearize(build_shared_reduce()), "shared_reduce");
    size_t loop = code.find("for (int ridx1 = 0; ridx1 < 3; ridx1++)");
    CHECK(loop != std::string::npos);
    size_t accs = 0, start = 0;
    while (start < code.size()) {
      size_t e = code.find('\n', start);
      if (e == std::string::npos) e = code.size();
      std::string line = code.substr(start, e - start);
      if (line.find("float acc") != std::string::npos && line.find("(-INFINITY);") != std::string::npos) {
        accs++;
        CHECK(code.find(line) < loop);
      }
      start = e + 1;
    }
    CHECK(accs >= 2);
  }});
  c.push_back({"clang::render_shared_reduce_multi_acc_compiles_and_runs", [build_shared_reduce] {
    std::string code = render_c(linearize(build_shared_reduce()), "shared_reduce");
    std::vector<float> o(2), x{1, 5, 3, -1, 0, 7};
    run_c(code, "shared_reduce", {o.data(), x.data()});
    CHECK(o == (std::vector<float>{5, 7}));
  }});
  return c;
}

}  // namespace

std::vector<Case> structure_cases() { return build_cases(); }

}  // namespace kir
