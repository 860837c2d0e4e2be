// passes.cpp -- the reference's CPU lowering restated pass by pass (TEST
// INFRASTRUCTURE: a second oracle that emits the reference's C for a
// proto-kernel).  Each function names the reference code it follows.
#include <algorithm>
#include <charconv>
#include <cmath>
#include <map>
#include <queue>
#include <set>
#include <sstream>
#include <stdexcept>
#include <unordered_set>

#include "kir.h"

namespace kir {

namespace {

[[noreturn]] void fail(const std::string &m) { throw std::runtime_error("lowering: " + m); }

using Map = std::unordered_map<const Node *, U>;

// ---- src/schedule/indexing.rs -------------------------------------------
std::vector<int64_t> contiguous_strides(const std::vector<int64_t> &shape) {
  std::vector<int64_t> s(shape.size());
  int64_t acc = 1;
  for (size_t i = shape.size(); i-- > 0;) {
    s[i] = acc;
    acc *= shape[i];
  }
  return s;
}

U flat_index(const std::vector<U> &idxs, const std::vector<int64_t> &strides) {
  if (idxs.size() != strides.size()) fail("flat_index: rank mismatch");
  if (idxs.empty()) fail("flat_index requires at least one index");
  U acc;
  for (size_t i = 0; i < idxs.size(); i++) {
    if (strides[i] == 0) continue;
    U term = strides[i] == 1 ? idxs[i] : mul(idxs[i], const_int(strides[i], DType::i32()));
    acc = acc ? add(acc, term) : term;
  }
  return acc ? acc : const_int(0, DType::i32());
}

U index_wrap(const U &src, const std::vector<U> &idxs) {
  std::vector<U> s{src};
  s.insert(s.end(), idxs.begin(), idxs.end());
  return make(Op::Index, src->dtype, std::move(s));
}

bool same_squeezed_dims(const std::vector<int64_t> &a, const std::vector<int64_t> &b) {
  std::vector<int64_t> x, y;
  for (int64_t d : a)
    if (d != 1) x.push_back(d);
  for (int64_t d : b)
    if (d != 1) y.push_back(d);
  return x == y;
}

U rewrite_index_alu(const U &inner, const std::vector<U> &idxs) {
  std::vector<U> s;
  for (const U &src : inner->src) s.push_back(index_wrap(src, idxs));
  return make(inner->op, inner->dtype, std::move(s), inner->arg);
}

U rewrite_index_movement(const U &inner, const std::vector<U> &idxs) {
  const U &src = inner->src[0];
  std::vector<U> out;
  switch (inner->op) {
    case Op::Shrink:
      for (size_t i = 0; i < idxs.size() && i < inner->arg.v.size(); i++) {
        const U &start = inner->src[i + 1];
        out.push_back(is_zero(start) ? idxs[i] : add(idxs[i], start));
      }
      break;
    case Op::Expand: {
      auto ss = shape_of(src);
      if (!ss) return nullptr;
      const auto &ex = inner->arg.v;
      for (size_t a = 0; a < idxs.size(); a++)
        out.push_back((*ss)[a] == 1 && ex[a] > 1 ? const_int(0, DType::i32()) : idxs[a]);
      break;
    }
    case Op::Permute: {
      const auto &order = inner->arg.v;
      std::vector<size_t> inverse(order.size());
      for (size_t i = 0; i < order.size(); i++) inverse[(size_t)order[i]] = i;
      for (size_t a : inverse) {
        if (a >= idxs.size()) fail("permute index out of range");
        out.push_back(idxs[a]);
      }
      break;
    }
    case Op::Reshape: {
      auto ss = shape_of(src);
      if (!ss) return nullptr;
      const auto &shape = inner->arg.v;
      if (same_squeezed_dims(*ss, shape)) {
        std::vector<U> non1;
        for (size_t a = 0; a < idxs.size() && a < shape.size(); a++)
          if (shape[a] != 1) non1.push_back(idxs[a]);
        size_t next = 0;
        for (int64_t d : *ss) {
          if (d == 1) {
            out.push_back(const_int(0, DType::i32()));
          } else {
            if (next >= non1.size()) fail("reshape index out of range");
            out.push_back(non1[next++]);
          }
        }
      } else {
        out.push_back(flat_index(idxs, contiguous_strides(shape)));
      }
      break;
    }
    case Op::Contiguous:
      out = idxs;
      break;
    default:
      fail("rangeify only sends movement ops here");
  }
  return index_wrap(src, out);
}

U rewrite_index_reduce(const U &inner, const std::vector<U> &idxs) {
  const U &src = inner->src[0];
  auto ss = shape_of(src);
  if (!ss) return nullptr;
  if (idxs.size() != ss->size()) fail("idxs should match source ndim");
  const auto &axes = inner->arg.v;
  std::vector<U> full, ranges;
  for (size_t a = 0; a < ss->size(); a++) {
    if (std::find(axes.begin(), axes.end(), (int64_t)a) != axes.end()) {
      U r = make(Op::Range, DType::i32(), {const_int((*ss)[a], DType::i32())},
                 Arg::range((int64_t)a, Axis::Reduce));
      full.push_back(r);
      ranges.push_back(r);
    } else {
      full.push_back(idxs[a]);
    }
  }
  std::vector<U> s{index_wrap(src, full)};
  s.insert(s.end(), ranges.begin(), ranges.end());
  return make(Op::Reduce, inner->dtype, std::move(s), Arg::reduce(inner->arg.rop, {}));
}

U rewrite_index_param(const U &inner, const std::vector<U> &idxs) {
  if (idxs.size() != 1) fail("Param should have exactly one flat index");
  U index = make(Op::Index, inner->dtype, {inner, idxs[0]}, Arg::index(0));
  return make(Op::Load, inner->dtype, {index});
}

// ---- src/schedule/rangeify.rs -------------------------------------------
U new_range(size_t axis, int64_t size) {
  if (size == 1) return const_int(0, DType::i32());
  return make(Op::Range, DType::i32(), {const_int(size, DType::i32())},
              Arg::range((int64_t)axis, Axis::Loop));
}

U chain_ends(const std::vector<U> &ranges, const U &body) {
  U cur = body;
  for (size_t i = ranges.size(); i-- > 0;) cur = make(Op::End, DType::void_(), {ranges[i], cur});
  return cur;
}

U store_output_index(const U &dest, const std::vector<U> &idxs) {
  if (dest->op == Op::ParamBuffer || dest->op == Op::Buffer) {
    if (idxs.size() != 1) fail("store destination must be flattened");
    return make(Op::Index, dest->dtype, {dest, idxs[0]}, Arg::index(0));
  }
  if (is_movement(dest->op)) {
    U moved = rewrite_index_movement(dest, idxs);
    if (!moved) return nullptr;
    return store_output_index(moved->src[0],
                              std::vector<U>(moved->src.begin() + 1, moved->src.end()));
  }
  return nullptr;
}

U rewrite_store_add_ranges(const U &store) {
  if (store->src.size() != 2) return nullptr;
  const U &out_param = store->src[0];
  const U &expr = store->src[1];
  auto shape = shape_of(expr);
  if (!shape) return nullptr;
  std::vector<U> axis_indices;
  for (size_t a = 0; a < shape->size(); a++) axis_indices.push_back(new_range(a, (*shape)[a]));
  U indexed = index_wrap(expr, axis_indices);
  U out_flat = flat_index(axis_indices, contiguous_strides(*shape));
  std::vector<U> out_ranges;
  for (const U &i : axis_indices)
    if (i->op == Op::Range) out_ranges.push_back(i);
  U out_idx = out_param->op == Op::ParamBuffer
                  ? make(Op::Index, out_param->dtype, {out_param, out_flat}, Arg::index(0))
                  : store_output_index(out_param, axis_indices);
  if (!out_idx) return nullptr;
  U st = make(Op::Store, DType::void_(), {out_idx, indexed});
  return chain_ends(out_ranges, st);
}

U rangeify_rule(const U &node) {
  if (node->op == Op::Store) return rewrite_store_add_ranges(node);
  if (node->op == Op::Index && node->arg.tag == Arg::None) {
    const U &inner = node->src[0];
    std::vector<U> idxs(node->src.begin() + 1, node->src.end());
    if (is_alu(inner->op)) return rewrite_index_alu(inner, idxs);
    switch (inner->op) {
      case Op::Expand: case Op::Permute: case Op::Reshape: case Op::Shrink: case Op::Contiguous:
        return rewrite_index_movement(inner, idxs);
      case Op::ReduceAxis: return rewrite_index_reduce(inner, idxs);
      case Op::Const: case Op::ParamScalar: return inner;
      case Op::ParamBuffer: return rewrite_index_param(inner, idxs);
      default: return nullptr;
    }
  }
  return nullptr;
}

// ---- src/optimize/upcast.rs ---------------------------------------------
constexpr int64_t kLoopUpcast = 4;
constexpr int64_t kReduceUnroll = 4;

bool output_kind(const Arg &a) {
  return a.tag == Arg::Range && (a.is_range(Axis::Loop) || a.is_range(Axis::Global) ||
                                 a.is_range(Axis::Local) || a.is_range(Axis::Thread));
}

std::vector<U> ordered_output_ranges(const U &root) {
  std::vector<U> r;
  for (const U &n : toposort(root))
    if (output_kind(n->arg)) r.push_back(n);
  std::stable_sort(r.begin(), r.end(), [](const U &a, const U &b) { return a->arg.a < b->arg.a; });
  r.erase(std::unique(r.begin(), r.end()), r.end());
  return r;
}

bool has_post_reduce_store_alu(const U &root) {
  for (const U &n : toposort(root)) {
    if (n->op != Op::Store || n->src.size() != 2) continue;
    const U &v = n->src[1];
    if (v->op == Op::Reduce) continue;
    for (const U &m : toposort(v))
      if (m->op == Op::Reduce) return true;
  }
  return false;
}

U select_upcast_range(const U &root) {
  for (const U &n : toposort(root))
    if (n->arg.is_range(Axis::Upcast)) return nullptr;
  if (has_post_reduce_store_alu(root)) return nullptr;
  auto ranges = ordered_output_ranges(root);
  if (ranges.empty()) return nullptr;
  U range = ranges.back();
  if (!range->arg.is_range(Axis::Loop) || range->src.size() != 1) return nullptr;
  auto size = const_i32(range->src[0]);
  if (!size || *size <= kLoopUpcast || *size % kLoopUpcast != 0) return nullptr;
  return range;
}

U split_loop_upcast(const U &end, const U &target) {
  if (end->op != Op::End || end->src.size() < 2) return nullptr;
  const U &range = end->src[0];
  if (range != target || !range->arg.is_range(Axis::Loop) || range->src.size() != 1) return nullptr;
  auto size = const_i32(range->src[0]);
  if (!size || *size <= kLoopUpcast || *size % kLoopUpcast != 0) return nullptr;
  const int64_t axis = range->arg.a;
  U outer = make(Op::Range, DType::i32(), {const_int(*size / kLoopUpcast, DType::i32())},
                 Arg::range(axis, Axis::Global));
  U inner = make(Op::Range, DType::i32(), {const_int(kLoopUpcast, DType::i32())},
                 Arg::range(axis, Axis::Upcast));
  U expanded = add(mul(outer, const_int(kLoopUpcast, DType::i32())), inner);
  Map repl{{range.get(), expanded}};
  std::vector<U> srcs{inner};
  for (size_t i = 1; i < end->src.size(); i++) srcs.push_back(substitute(end->src[i], repl));
  U upcasted = make(Op::End, DType::void_(), std::move(srcs));
  return make(Op::End, DType::void_(), {outer, upcasted});
}

// ---- src/optimize/unroll.rs ---------------------------------------------
U split_reduce_unroll(const U &reduce) {
  if (reduce->op != Op::Reduce || reduce->src.size() < 2) return nullptr;
  for (size_t i = 1; i < reduce->src.size(); i++)
    if (reduce->src[i]->arg.is_range(Axis::Unroll)) return nullptr;
  size_t range_idx = 0;
  for (size_t i = reduce->src.size(); i-- > 1;)
    if (reduce->src[i]->arg.is_range(Axis::Reduce)) {
      range_idx = i;
      break;
    }
  if (!range_idx) return nullptr;
  const U &range = reduce->src[range_idx];
  if (range->src.size() != 1) return nullptr;
  auto size = const_i32(range->src[0]);
  if (!size || *size <= kReduceUnroll || *size % kReduceUnroll != 0) return nullptr;
  const int64_t axis = range->arg.a;
  U outer = make(Op::Range, DType::i32(), {const_int(*size / kReduceUnroll, DType::i32())},
                 Arg::range(axis, Axis::Reduce));
  U inner = make(Op::Range, DType::i32(), {const_int(kReduceUnroll, DType::i32())},
                 Arg::range(axis, Axis::Unroll));
  U expanded = add(mul(outer, const_int(kReduceUnroll, DType::i32())), inner);
  U value = substitute(reduce->src[0], Map{{range.get(), expanded}});
  std::vector<U> srcs{value};
  for (size_t i = 1; i < reduce->src.size(); i++) {
    if (i == range_idx) {
      srcs.push_back(outer);
      srcs.push_back(inner);
    } else {
      srcs.push_back(reduce->src[i]);
    }
  }
  return make(Op::Reduce, reduce->dtype, std::move(srcs), reduce->arg);
}

// ---- src/expand.rs ----------------------------------------------------------
using Lanes = std::vector<std::pair<int64_t, int64_t>>;

U lane_pack_for_range(const U &range) {
  if (range->arg.tag != Arg::Range) return nullptr;
  if (!range->arg.is_range(Axis::Upcast) && !range->arg.is_range(Axis::Unroll)) return nullptr;
  if (range->src.size() != 1 || range->src[0]->arg.tag != Arg::Int) return nullptr;
  const int64_t n = range->src[0]->arg.a;
  std::vector<U> lanes;
  for (int64_t i = 0; i < n; i++) lanes.push_back(const_int(i, DType::i32()));
  U vec = make(Op::Vectorize, DType::i32().vec((uint16_t)n), std::move(lanes));
  // the lane id is the range's axis number; output and reduce axes are
  // numbered independently, so an upcast and an unroll lane can share an id
  // (repair: upcast lanes get ids of their own)
  const int64_t id =
      repair() && range->arg.is_range(Axis::Upcast) ? range->arg.a + (int64_t(1) << 20) : range->arg.a;
  return make(Op::Unroll, DType::i32(), {vec}, Arg::lanes_of({{id, n}}));
}

U expand_upcast_end(const U &end) {
  if (end->op != Op::End || end->src.size() < 2) return nullptr;
  const U &range = end->src[0];
  if (!range->arg.is_range(Axis::Upcast)) return nullptr;
  U lane = lane_pack_for_range(range);
  if (!lane) return nullptr;
  Map repl{{range.get(), lane}};
  std::vector<U> effects;
  for (size_t i = 1; i < end->src.size(); i++) effects.push_back(substitute(end->src[i], repl));
  return sink(std::move(effects));
}

U rewrite_scheduled_range(const U &node) {
  if (node->op != Op::Range) return nullptr;
  return lane_pack_for_range(node);
}

U fix_reduce_unroll(const U &node) {
  if (node->op != Op::Reduce || node->src.size() < 2) return nullptr;
  Lanes axes;
  std::vector<U> ranges;
  for (size_t i = 1; i < node->src.size(); i++) {
    const U &s = node->src[i];
    if (s->op == Op::Unroll) {
      if (s->arg.tag != Arg::Lanes) return nullptr;
      axes.insert(axes.end(), s->arg.lanes.begin(), s->arg.lanes.end());
    } else if (s->op == Op::Range) {
      ranges.push_back(s);
    } else {
      return nullptr;
    }
  }
  if (axes.empty()) return nullptr;
  U contracted = make(Op::Contract, node->src[0]->dtype, {node->src[0]}, Arg::lanes_of(axes));
  std::vector<U> srcs{contracted};
  srcs.insert(srcs.end(), ranges.begin(), ranges.end());
  return make(Op::Reduce, node->dtype, std::move(srcs), node->arg);
}

std::vector<size_t> swizzle_indices(const Lanes &src_meta, const Lanes &merged) {
  size_t total = 1;
  for (auto &m : merged) total *= (size_t)m.second;
  std::vector<size_t> out(total);
  if (src_meta == merged) {
    for (size_t i = 0; i < total; i++) out[i] = i;
    return out;
  }
  std::vector<size_t> ss(src_meta.size(), 1), ms(merged.size(), 1);
  for (size_t i = src_meta.size(); i-- > 1;) ss[i - 1] = ss[i] * (size_t)src_meta[i].second;
  for (size_t i = merged.size(); i-- > 1;) ms[i - 1] = ms[i] * (size_t)merged[i].second;
  std::map<int64_t, size_t> pos;
  for (size_t i = 0; i < merged.size(); i++) pos[merged[i].first] = i;
  for (size_t flat = 0; flat < total; flat++) {
    size_t s = 0;
    for (size_t p = 0; p < src_meta.size(); p++) {
      const size_t mp = pos.at(src_meta[p].first);
      const size_t coord = (flat / ms[mp]) % (size_t)merged[mp].second;
      s += coord * ss[p];
    }
    out[flat] = s;
  }
  return out;
}

U expand_lane_expr(const U &node) {
  if (!is_alu(node->op) && node->op != Op::Index && node->op != Op::Load) return nullptr;
  Lanes merged;
  bool any = false;
  for (const U &s : node->src) {
    if (s->op != Op::Unroll || s->arg.tag != Arg::Lanes) continue;
    any = true;
    for (auto &l : s->arg.lanes)
      if (std::none_of(merged.begin(), merged.end(), [&](auto &m) { return m.first == l.first; }))
        merged.push_back(l);
  }
  if (!any) return nullptr;
  std::stable_sort(merged.begin(), merged.end(),
                   [](auto &a, auto &b) { return a.first < b.first; });
  size_t n = 1;
  for (auto &m : merged) n *= (size_t)m.second;
  std::vector<U> lanes;
  for (size_t lane = 0; lane < n; lane++) {
    std::vector<U> srcs;
    for (const U &s : node->src) {
      if (s->op == Op::Unroll && s->arg.tag == Arg::Lanes) {
        auto sw = swizzle_indices(s->arg.lanes, merged);
        srcs.push_back(gep(s->src[0], sw[lane]));
      } else {
        srcs.push_back(s);
      }
    }
    lanes.push_back(make(node->op, node->dtype, std::move(srcs), node->arg));
  }
  U vec = make(Op::Vectorize, node->dtype.vec((uint16_t)n), std::move(lanes));
  return make(Op::Unroll, node->dtype, {vec}, Arg::lanes_of(merged));
}

U merge_shared_range_ends(const U &root) {
  auto order = toposort(root);
  std::vector<const Node *> range_order;
  std::unordered_map<const Node *, std::vector<U>> ends;
  for (const U &n : order) {
    if (n->op != Op::End || n->src.empty()) continue;
    auto &v = ends[n->src[0].get()];
    if (v.empty()) range_order.push_back(n->src[0].get());
    v.push_back(n);
  }
  Map repl;
  for (const Node *r : range_order) {
    auto &es = ends[r];
    if (es.size() < 2) continue;
    std::vector<U> srcs{es[0]->src[0]};
    std::unordered_set<const Node *> seen;
    for (const U &e : es)
      for (size_t i = 1; i < e->src.size(); i++) {
        const U &body = e->src[i];
        std::vector<U> bodies = body->op == Op::Sink ? body->src : std::vector<U>{body};
        for (const U &b : bodies)
          if (seen.insert(b.get()).second) srcs.push_back(b);
      }
    U merged = make(Op::End, DType::void_(), std::move(srcs));
    for (const U &e : es) repl[e.get()] = merged;
  }
  if (repl.empty()) return root;
  return substitute(root, repl);
}

// ---- src/devectorize.rs -----------------------------------------------------
U no_vectorized_alu(const U &node) {
  if (node->dtype.is_scalar()) return nullptr;
  if (!is_alu(node->op) && node->op != Op::Index && node->op != Op::Load &&
      node->op != Op::After)
    return nullptr;
  const size_t n = node->dtype.vcount;
  std::vector<U> lanes;
  for (size_t i = 0; i < n; i++) {
    std::vector<U> srcs;
    for (const U &s : node->src) srcs.push_back(s->dtype.is_scalar() ? s : gep(s, i));
    lanes.push_back(make(node->op, node->dtype.scalar(), std::move(srcs), node->arg));
  }
  return make(Op::Vectorize, node->dtype, std::move(lanes));
}

bool unwrap_unroll(const U &node, U *vec, Lanes *meta) {
  if (node->op != Op::Unroll || node->src.size() != 1 || node->arg.tag != Arg::Lanes) return false;
  if (node->src[0]->op != Op::Vectorize) return false;
  *vec = node->src[0];
  *meta = node->arg.lanes;
  return true;
}

bool reduce_lane_groups(const U &value, std::vector<std::vector<U>> *groups, Lanes *meta) {
  if (value->op == Op::Contract) {
    if (value->arg.tag != Arg::Lanes) return false;
    const Lanes &contract = value->arg.lanes;
    U vec;
    Lanes full;
    if (!unwrap_unroll(value->src[0], &vec, &full)) {
      if (!repair()) return false;
      // a lane-invariant value (a constant reduced over an unrolled axis):
      // each unrolled lane contributes it once
      size_t csize = 1;
      for (auto &c : contract) csize *= (size_t)c.second;
      *groups = {std::vector<U>(csize, value->src[0])};
      meta->clear();
      return true;
    }
    Lanes remaining;
    for (auto &l : full)
      if (std::none_of(contract.begin(), contract.end(),
                       [&](auto &c) { return c.first == l.first; }))
        remaining.push_back(l);
    size_t csize = 1, rsize = 1;
    for (auto &c : contract) csize *= (size_t)c.second;
    for (auto &r : remaining) rsize *= (size_t)r.second;
    const size_t total = vec->src.size();
    // lane strides of the full lane layout (row-major over `full`)
    std::map<int64_t, size_t> stride;
    for (size_t i = full.size(), st = 1; i-- > 0;) {
      stride[full[i].first] = st;
      st *= (size_t)full[i].second;
    }
    auto flat_of = [&](const Lanes &axes, size_t k) {  // k row-major over `axes`
      size_t f = 0;
      for (size_t i = axes.size(); i-- > 0;) {
        f += (k % (size_t)axes[i].second) * stride.at(axes[i].first);
        k /= (size_t)axes[i].second;
      }
      return f;
    };
    groups->clear();
    for (size_t o = 0; o < rsize; o++) {
      std::vector<U> g;
      for (size_t c = 0; c < csize; c++) {
        const size_t flat = repair() ? flat_of(remaining, o) + flat_of(contract, c) : o * csize + c;
        if (flat >= total) fail("lane index out of bounds");
        g.push_back(gep(vec, flat));
      }
      groups->push_back(std::move(g));
    }
    *meta = remaining;
    return true;
  }
  U vec;
  if (!unwrap_unroll(value, &vec, meta)) return false;
  groups->clear();
  for (size_t i = 0; i < vec->src.size(); i++) groups->push_back({gep(vec, i)});
  return true;
}

U horizontal_reduce(const std::vector<U> &values, Op op) {
  if (values.empty()) fail("horizontal reduction requires at least one value");
  U acc = values[0];
  for (size_t i = 1; i < values.size(); i++) acc = make(op, acc->dtype, {acc, values[i]});
  return acc;
}

U chain_reduce_ends(const std::vector<U> &ranges, std::vector<U> inner) {
  if (ranges.empty()) return sink(std::move(inner));
  std::vector<U> srcs{ranges.back()};
  srcs.insert(srcs.end(), inner.begin(), inner.end());
  U cur = make(Op::End, DType::void_(), std::move(srcs));
  for (size_t i = ranges.size() - 1; i-- > 0;) cur = make(Op::End, DType::void_(), {ranges[i], cur});
  return cur;
}

U lower_reduce(const U &node) {
  if (node->op != Op::Reduce || node->src.size() < 2) return nullptr;
  const Op rop = node->arg.rop;
  const U &value = node->src[0];
  std::vector<U> rranges(node->src.begin() + 1, node->src.end());
  std::unordered_set<const Node *> rset;
  for (const U &r : rranges) rset.insert(r.get());
  std::vector<U> outer;
  for (const U &n : toposort(value))
    if (n->op == Op::Range && !rset.count(n.get())) outer.push_back(n);
  std::vector<std::vector<U>> groups;
  Lanes meta;
  if (!reduce_lane_groups(value, &groups, &meta)) {
    groups = {{value}};
    meta.clear();
  }
  U init;
  if (rop == Op::Add)
    init = const_float(0.0, node->dtype);
  else if (rop == Op::Max)
    init = const_float(-INFINITY, node->dtype);
  else
    fail("unsupported reduce op");
  std::vector<U> accs, assigns;
  for (size_t i = 0; i < groups.size(); i++) {
    const uint64_t tag = (uint64_t)i + 1;
    std::vector<U> asrc{init};
    asrc.insert(asrc.end(), outer.begin(), outer.end());
    U acc = make(Op::DefineAcc, node->dtype, std::move(asrc), Arg::none(), tag << 32);
    U red = horizontal_reduce(groups[i], rop);
    std::vector<U> usrc{acc, red};
    // repair: the update depends on the reduce ranges even when the reduced
    // value does not (a constant), so the linearizer keeps it in the loop
    // (the renderer reads only the first two sources of an ALU node)
    if (repair()) usrc.insert(usrc.end(), rranges.begin(), rranges.end());
    U upd = make(rop, node->dtype, std::move(usrc));
    assigns.push_back(make(Op::Assign, node->dtype, {acc, upd}, Arg::none(), (tag << 32) | 1));
    accs.push_back(acc);
  }
  U rend = chain_reduce_ends(rranges, assigns);
  std::vector<U> afters;
  for (const U &a : accs) afters.push_back(after(a, rend));
  if (meta.empty()) {
    if (afters.size() != 1) fail("scalar reduction should produce one accumulator");
    return afters[0];
  }
  U vec = make(Op::Vectorize, node->dtype.vec((uint16_t)afters.size()), afters);
  return make(Op::Unroll, node->dtype, {vec}, Arg::lanes_of(meta));
}

U scalarize_lane_store(const U &node) {
  if (node->op != Op::Store || node->src.size() != 2) return nullptr;
  const U &idx = node->src[0], &val = node->src[1];
  if (idx->op != Op::Unroll && val->op != Op::Unroll) return nullptr;
  const size_t n = idx->op == Op::Unroll ? idx->src[0]->src.size() : val->src[0]->src.size();
  std::vector<U> stores;
  for (size_t i = 0; i < n; i++) {
    U li = idx->op == Op::Unroll ? gep(idx->src[0], i) : idx;
    U lv = val->op == Op::Unroll ? gep(val->src[0], i) : val;
    stores.push_back(make(Op::Store, DType::void_(), {li, lv}));
  }
  return sink(std::move(stores));
}

U single_after_effect(const U &root) {
  U effect;
  for (const U &n : toposort(root)) {
    if (n->op != Op::After || n->src.size() != 2) continue;
    const U &end = n->src[1];
    if (effect && effect != end) return nullptr;
    if (!effect) effect = end;
  }
  return effect;
}

U strip_after_effect(const U &root, const U &effect) {
  Map rw;
  for (const U &n : toposort(root)) {
    U nn;
    if (n->op == Op::After && n->src.size() == 2 && n->src[1] == effect) {
      auto f = rw.find(n->src[0].get());
      nn = f != rw.end() ? f->second : n->src[0];
    } else {
      std::vector<U> srcs;
      bool changed = false;
      for (const U &s : n->src) {
        auto f = rw.find(s.get());
        U ns = f != rw.end() ? f->second : s;
        changed |= ns != s;
        srcs.push_back(ns);
      }
      nn = changed ? make(n->op, n->dtype, std::move(srcs), n->arg, rebuilt_tag(*n)) : n;
    }
    rw[n.get()] = nn;
  }
  auto f = rw.find(root.get());
  return f != rw.end() ? f->second : root;
}

U lift_after_in_store(const U &node) {
  if (node->op != Op::Store || node->src.size() != 2) return nullptr;
  const U &idx = node->src[0], &value = node->src[1];
  U effect = single_after_effect(value);
  if (!effect) return nullptr;
  U stripped = strip_after_effect(value, effect);
  U li = idx->op == Op::After && idx->src.size() == 2 && idx->src[1] == effect ? idx
                                                                              : after(idx, effect);
  U lv = after(stripped, effect);
  if (li == idx && lv == value) return nullptr;
  return make(Op::Store, DType::void_(), {li, lv});
}

// ---- src/linearize.rs ---------------------------------------------------------
using NodeSet = std::set<const Node *>;

int64_t range_extent(const U &r) {
  if (r->src.empty()) return 1;
  const Arg &a = r->src[0]->arg;
  return a.tag == Arg::Int && a.a > 0 ? a.a : 1;
}

const NodeSet &active_ranges(const U &n, std::unordered_map<const Node *, NodeSet> &cache,
                             std::unordered_map<const Node *, U> &keep) {
  auto it = cache.find(n.get());
  if (it != cache.end()) return it->second;
  NodeSet r;
  for (const U &s : n->src) {
    const NodeSet &x = active_ranges(s, cache, keep);
    r.insert(x.begin(), x.end());
  }
  for (const U &e : ended_ranges(n)) {
    if (e->op == Op::Range) {
      r.erase(e.get());
      continue;
    }
    for (const Node *x : active_ranges(e, cache, keep)) r.erase(x);
  }
  if (n->op == Op::Range) {
    r.insert(n.get());
    keep[n.get()] = n;
  }
  return cache[n.get()] = std::move(r);
}

struct PKey {
  int64_t run, prio, extra;
  size_t idx;
  bool operator<(const PKey &o) const {
    return std::tie(run, prio, extra, idx) < std::tie(o.run, o.prio, o.extra, o.idx);
  }
};

PKey priority_key(const U &n, size_t idx, std::unordered_map<const Node *, U> &ranges_by_ptr) {
  std::unordered_map<const Node *, NodeSet> cache;  // a fresh cache per node, as run_count
  int64_t run = 1;
  for (const Node *r : active_ranges(n, cache, ranges_by_ptr)) {
    const int64_t e = range_extent(ranges_by_ptr.at(r));
    run = (run > 0 && e > INT64_MAX / run) ? INT64_MAX : run * e;
  }
  int64_t prio = 0, extra = 0;
  switch (n->op) {
    case Op::ParamBuffer: case Op::ParamScalar: prio = -20; extra = n->arg.a; break;
    case Op::DefineVar: prio = -19; break;
    case Op::DefineAcc: prio = -17; break;
    case Op::Load: prio = -1; break;
    case Op::Store: prio = 1; break;
    case Op::Range: prio = 5; break;
    case Op::End: prio = -5; break;
    default: break;
  }
  return {run, prio, extra, idx};
}

U inject_control_flow(const U &root) {
  auto order = toposort(root);
  std::unordered_map<const Node *, NodeSet> deps;
  std::unordered_map<const Node *, U> nesting;
  for (const U &n : order) {
    NodeSet nd;
    for (const U &s : n->src) {
      auto f = deps.find(s.get());
      if (f != deps.end()) nd.insert(f->second.begin(), f->second.end());
    }
    if (n->op == Op::End || n->op == Op::Sink) {
      for (const Node *d : nd) {
        if (d->op != Op::End || nesting.count(d)) continue;
        bool nested = n->op == Op::Sink || deps[d].count(n->src[0].get());
        if (nested) nesting[d] = n;
      }
    }
    if (n->op == Op::Range || n->op == Op::End) nd.insert(n.get());
    deps[n.get()] = std::move(nd);
  }
  // siblings per parent, in toposort order of the children
  std::vector<const Node *> parents;
  std::unordered_map<const Node *, std::vector<U>> siblings;
  std::unordered_map<const Node *, U> parent_node;
  for (const U &n : order) {
    auto f = nesting.find(n.get());
    if (f == nesting.end()) continue;
    const Node *p = f->second.get();
    if (!siblings.count(p)) parents.push_back(p);
    siblings[p].push_back(n);
    parent_node[p] = f->second;
  }
  std::unordered_map<const Node *, std::vector<U>> edges;
  auto push_edge = [&edges](const U &node, const U &pred) {
    auto &v = edges[node.get()];
    if (std::find(v.begin(), v.end(), pred) == v.end()) v.push_back(pred);
  };
  for (const Node *p : parents) {
    std::vector<U> ordered = siblings[p];
    std::unordered_map<const Node *, size_t> count;
    for (const U &e : ordered) {
      size_t c = 0;
      for (const U &cand : ordered)
        if (deps[e.get()].count(cand.get())) c++;
      count[e.get()] = c;
    }
    std::stable_sort(ordered.begin(), ordered.end(),
                     [&](const U &a, const U &b) { return count[a.get()] < count[b.get()]; });
    const U &parent = parent_node[p];
    if (parent->op == Op::Sink) {
      for (size_t i = 1; i < ordered.size(); i++) {
        const U &prev = ordered[i - 1];
        const U &next_range = ordered[i]->src[0];
        if (deps[prev.get()].count(next_range.get()))
          fail("linearize: control-flow cycle between sibling loops");
        push_edge(next_range, prev);
      }
      continue;
    }
    U pred = parent->src[0];
    for (const U &e : ordered) {
      const U &next_range = e->src[0];
      if (deps[pred.get()].count(next_range.get())) fail("linearize: nested control-flow cycle");
      push_edge(next_range, pred);
      pred = e;
    }
  }
  if (edges.empty()) return root;
  return graph_rewrite(root, [&edges](const U &node) -> U {
    auto f = edges.find(node.get());
    if (f == edges.end()) return nullptr;
    std::vector<U> srcs = node->src;
    srcs.insert(srcs.end(), f->second.begin(), f->second.end());
    return make(node->op, node->dtype, std::move(srcs), node->arg);
  });
}

}  // namespace

U rangeify(const U &sink) { return graph_rewrite(sink, rangeify_rule); }

U upcast_loops(const U &root) {
  U target = select_upcast_range(root);
  if (!target) return root;
  return graph_rewrite(root, [&target](const U &n) { return split_loop_upcast(n, target); });
}

U unroll_reduce_loops(const U &root) { return graph_rewrite(root, split_reduce_unroll); }

U symbolic_simple(const U &node) {
  // src/optimize/symbolic.rs
  if ((node->op == Op::Add || node->op == Op::Mul) && node->src.size() == 2) {
    const U &x = node->src[0], &y = node->src[1];
    if (is_const(x) && is_const(y)) {
      const Arg &a = x->arg, &b = y->arg;
      if (a.tag == Arg::Float && b.tag == Arg::Float)
        return const_float(node->op == Op::Add ? a.f + b.f : a.f * b.f, x->dtype);
      if (a.tag == Arg::Int && b.tag == Arg::Int)
        return const_int(node->op == Op::Add ? a.a + b.a : a.a * b.a, x->dtype);
      return nullptr;
    }
    if (node->op == Op::Add) {
      if (is_zero(y)) return x;
      if (is_zero(x)) return y;
    } else {
      if (is_one(y)) return x;
      if (is_one(x)) return y;
      if (is_zero(y)) return y;
      if (is_zero(x)) return x;
    }
  }
  return nullptr;
}

U optimize(const U &kernel, const OptimizeConfig &c) {
  U cur = kernel;
  if (c.upcast) cur = upcast_loops(cur);
  if (c.unroll) cur = unroll_reduce_loops(cur);
  if (c.symbolic) cur = graph_rewrite(cur, symbolic_simple);
  return cur;
}

U late_expand(const U &root) {
  U a = graph_rewrite(root, expand_upcast_end);
  U b = graph_rewrite(a, rewrite_scheduled_range);
  U c = graph_rewrite(b, fix_reduce_unroll);
  U d = graph_rewrite(c, expand_lane_expr);
  U e = graph_rewrite(d, flatten_end_bodies);
  U f = merge_shared_range_ends(e);
  return graph_rewrite(f, flatten_nested_sinks);
}

U devectorize(const U &root) {
  U a = graph_rewrite(root, lower_reduce);
  U b = graph_rewrite(a, no_vectorized_alu);
  U c = graph_rewrite(b, scalarize_lane_store);
  U d = graph_rewrite(c, flatten_end_bodies);
  U e = graph_rewrite(d, lift_after_in_store);
  return graph_rewrite(e, flatten_nested_sinks);
}

std::vector<U> linearize(const U &root_in) {
  if (root_in->op != Op::Sink) fail("linearize: root must be a Sink node");
  U root = inject_control_flow(root_in);
  auto order = toposort(root);
  std::unordered_map<const Node *, size_t> idx_of;
  for (size_t i = 0; i < order.size(); i++) idx_of[order[i].get()] = i;
  std::vector<size_t> out_degree(order.size(), 0);
  for (size_t i = order.size(); i-- > 0;)
    for (const U &s : order[i]->src) out_degree[idx_of.at(s.get())]++;
  std::unordered_map<const Node *, U> ranges_by_ptr;
  std::vector<std::pair<PKey, size_t>> ranked;
  for (size_t i = 0; i < order.size(); i++)
    ranked.push_back({priority_key(order[i], i, ranges_by_ptr), i});
  std::stable_sort(ranked.begin(), ranked.end(),
                   [](auto &a, auto &b) { return a.first < b.first; });
  std::vector<size_t> nkey(order.size());
  for (size_t r = 0; r < ranked.size(); r++) nkey[ranked[r].second] = r;
  std::priority_queue<std::pair<size_t, size_t>> heap;  // max-heap, as BinaryHeap
  const size_t root_idx = idx_of.at(root.get());
  heap.push({nkey[root_idx], root_idx});
  std::vector<char> visited(order.size(), 0);
  std::vector<U> linear;
  while (!heap.empty()) {
    const size_t i = heap.top().second;
    heap.pop();
    if (visited[i]) continue;
    visited[i] = 1;
    linear.push_back(order[i]);
    for (const U &s : order[i]->src) {
      const size_t si = idx_of.at(s.get());
      if (--out_degree[si] == 0) heap.push({nkey[si], si});
    }
  }
  if (linear.size() != order.size()) fail("linearize: failed to order the full kernel graph");
  std::reverse(linear.begin(), linear.end());
  std::vector<U> out;
  for (const U &n : linear)
    if (n->op != Op::Sink) out.push_back(n);
  return out;
}

std::string c_literal(const Node &n) {
  const Arg &a = n.arg;
  if (a.tag == Arg::Int) return std::to_string(a.a);
  if (a.tag == Arg::Bool) return a.a ? "1" : "0";
  if (a.tag != Arg::Float) fail("Const with unexpected arg");
  const double v = a.f;
  if (std::isinf(v)) return v > 0 ? "INFINITY" : "(-INFINITY)";
  if (std::isnan(v)) return "NAN";
  // Rust's Display for f64: the shortest digits that round-trip, in plain
  // (never exponent) notation; "{:.1}" when the value is integral.
  char buf[512];
  std::to_chars_result r;
  if (v == std::trunc(v))
    r = std::to_chars(buf, buf + sizeof(buf), v, std::chars_format::fixed, 1);
  else
    r = std::to_chars(buf, buf + sizeof(buf), v, std::chars_format::fixed);
  std::string s(buf, r.ptr);
  if (n.dtype == DType::f32()) s += "f";
  return s;
}

std::string render_c(const std::vector<U> &uops, const std::string &name) {
  // src/codegen/clang.rs:12-281
  struct P {
    int64_t slot;
    DType dt;
    bool buffer;
  };
  std::vector<P> params;
  for (const U &n : uops) {
    if (n->op == Op::ParamBuffer) params.push_back({n->arg.a, n->dtype, true});
    if (n->op == Op::ParamScalar) params.push_back({n->arg.a, n->dtype, false});
  }
  std::stable_sort(params.begin(), params.end(),
                   [](const P &a, const P &b) { return a.slot < b.slot; });
  std::ostringstream out;
  out << "#include <math.h>\nvoid " << name << "(";
  for (size_t i = 0; i < params.size(); i++) {
    if (i) out << ", ";
    out << params[i].dt.c_type() << (params[i].buffer ? "* restrict data" : " data")
        << params[i].slot;
  }
  out << ") {\n";
  std::unordered_map<const Node *, std::string> names;
  size_t depth = 1, vals = 0, alus = 0;
  auto ind = [&depth]() { return std::string(2 * depth, ' '); };
  auto name_of = [&names](const U &u) -> const std::string & {
    auto f = names.find(u.get());
    if (f == names.end())
      fail(std::string("node referenced before being rendered: op=") + op_name(u->op));
    return f->second;
  };
  for (const U &n : uops) {
    switch (n->op) {
      case Op::Device: case Op::DefineVar: names[n.get()] = ""; break;
      case Op::ParamBuffer: case Op::ParamScalar:
        names[n.get()] = "data" + std::to_string(n->arg.a);
        break;
      case Op::Const: names[n.get()] = c_literal(*n); break;
      default: break;
    }
  }
  for (const U &n : uops) {
    switch (n->op) {
      case Op::Sink: case Op::Device: case Op::DefineVar: case Op::ParamBuffer:
      case Op::ParamScalar: case Op::Const:
        continue;
      case Op::End:
        depth--;
        out << ind() << "}\n";
        continue;
      case Op::Store:
        out << ind() << "*" << name_of(n->src[0]) << " = " << name_of(n->src[1]) << ";\n";
        continue;
      case Op::After:
        names[n.get()] = name_of(n->src[0]);
        continue;
      case Op::Range: {
        static const char *pre[] = {"idx", "idx", "lidx", "ridx", "ridx", "uidx", "uidx", "tidx"};
        const std::string var = std::string(pre[n->arg.b]) + std::to_string(n->arg.a);
        out << ind() << "for (int " << var << " = 0; " << var << " < " << name_of(n->src[0])
            << "; " << var << "++) {\n";
        names[n.get()] = var;
        depth++;
        continue;
      }
      case Op::Buffer: fail("Buffer is a tensor-level op");
      default: break;
    }
    std::vector<std::string> s;
    for (const U &x : n->src) s.push_back(name_of(x));
    switch (n->op) {
      case Op::Index: names[n.get()] = "(" + s[0] + "+" + s[1] + ")"; break;
      case Op::Load: {
        const std::string var = "val" + std::to_string(vals++);
        out << ind() << n->dtype.c_type() << " " << var << " = *" << s[0] << ";\n";
        names[n.get()] = var;
        break;
      }
      case Op::Neg: case Op::Exp2: case Op::Log2: case Op::Sqrt: case Op::Reciprocal:
      case Op::Add: case Op::Mul: case Op::Max: case Op::CmpLt: case Op::Where:
      case Op::DefineAcc: {
        std::string prefix = "alu", expr;
        switch (n->op) {
          case Op::Neg: expr = "(-" + s[0] + ")"; break;
          case Op::Exp2: expr = "exp2(" + s[0] + ")"; break;
          case Op::Log2: expr = "log2(" + s[0] + ")"; break;
          case Op::Sqrt: expr = "__builtin_sqrtf(" + s[0] + ")"; break;
          case Op::Reciprocal: expr = "(1/" + s[0] + ")"; break;
          case Op::Add: expr = "(" + s[0] + "+" + s[1] + ")"; break;
          case Op::Mul: expr = "(" + s[0] + "*" + s[1] + ")"; break;
          case Op::Max: expr = "((" + s[0] + ">" + s[1] + ")?" + s[0] + ":" + s[1] + ")"; break;
          case Op::CmpLt: expr = "(" + s[0] + "<" + s[1] + ")"; break;
          case Op::Where: expr = "(" + s[0] + "?" + s[1] + ":" + s[2] + ")"; break;
          default: prefix = "acc"; expr = s[0]; break;
        }
        const std::string var = prefix + std::to_string(alus++);
        out << ind() << n->dtype.c_type() << " " << var << " = " << expr << ";\n";
        names[n.get()] = var;
        break;
      }
      case Op::Assign:
        out << ind() << s[0] << " = " << s[1] << ";\n";
        names[n.get()] = s[0];
        break;
      default:
        fail(std::string(op_name(n->op)) + " should be lowered before codegen");
    }
  }
  out << "}\n";
  return out.str();
}

}  // namespace kir
