// render.cpp -- CUDA C renderer for scheduled proto-kernels.
//
// Replaces the reference's rangeify -> optimize -> late_expand ->
// devectorize -> linearize -> ClangRenderer chain (src/schedule/rangeify.rs,
// src/optimize/*.rs, src/expand.rs, src/devectorize.rs, src/linearize.rs,
// src/codegen/clang.rs) with a direct walk of the tensor-level expression.
// The arithmetic is the reference's, op for op:
//   * every ALU op is one correctly rounded operation; Add/Mul use
//     __fadd_rn/__fmul_rn so nvcc never contracts them into an FMA (the
//     reference emits one op per C statement, clang.rs:216-229);
//   * exp2/log2 are double-precision calls on the float argument, rounded to
//     float; sqrt and reciprocal are correctly rounded; max is (a>b)?a:b;
//   * a reduction walks its axes in order with one accumulator; when the
//     last reduced axis has size R > 4 and R % 4 == 0 it is split into
//     blocks of four lanes folded left to right, acc = acc op (((v0 op v1)
//     op v2) op v3) (src/optimize/unroll.rs:41-113,
//     src/devectorize.rs:206-347); the identity is 0 or -inf (INT_MIN for
//     i32);
//   * symbolic_simple (src/optimize/symbolic.rs:42-56) folds ALU ops on
//     literal constants: const op const in f64, x+0, 0+x, x*1, 1*x -> x,
//     x*0, 0*x -> 0.
// Both the 4-lane reduction blocks and the folds follow the reference's OPT
// setting (optimize_config(): without "unroll" every reduction is
// sequential, without "symbolic" nothing is folded).
// The thread mapping is the B200's: elementwise kernels give each thread
// groups of 4 consecutive elements (one 128-bit access per operand where the
// layout allows, several groups with all loads issued before the stores);
// reductions run one thread per output in exact mode, and in the default
// mode a warp per output (reduced axis innermost) or 32 outputs per
// 1024-thread block (reduced axis outer), with 8 independent partials per
// thread folded in a fixed order (choose_thread_mapping).
#include <algorithm>
#include <charconv>
#include <functional>
#include <unordered_set>
#include <cmath>
#include <cstring>
#include <sstream>

#include "front_internal.h"

namespace ferro {

std::string float_literal(double v) {
  if (std::isinf(v)) return v > 0 ? "INFINITY" : "(-INFINITY)";
  if (std::isnan(v)) return "NAN";
  char buf[64];
  auto r = std::to_chars(buf, buf + sizeof(buf), v);
  std::string s(buf, r.ptr);
  if (s.find_first_of(".eEn") == std::string::npos) s += ".0";
  return s + "f";
}

namespace {

const char *ctype(DType d) {
  switch (d) {
    case DType::F32: return "float";
    case DType::I32: return "int";
    case DType::Bool: return "bool";
  }
  return "float";
}
const char *storage_type(DType d) {
  switch (d) {
    case DType::F32: return "float";
    case DType::I32: return "int";
    case DType::Bool: return "unsigned char";
  }
  return "float";
}

bool is_int_literal(const std::string &s) {
  if (s.empty()) return false;
  size_t i = s[0] == '-' ? 1 : 0;
  if (i == s.size()) return false;
  for (; i < s.size(); i++)
    if (s[i] < '0' || s[i] > '9') return false;
  return true;
}

struct Val {
  std::string expr;
  DType dt = DType::F32;
  bool is_const = false;
  double c = 0.0;
};

std::string literal_of(double v, DType dt) {
  if (dt == DType::F32) return float_literal(v);
  if (dt == DType::Bool) return v != 0.0 ? "true" : "false";
  if (std::isinf(v)) return v > 0 ? "2147483647" : "(-2147483647 - 1)";
  char buf[32];
  snprintf(buf, sizeof(buf), "%lld", (long long)v);
  return buf;
}

bool bits_equal(double a, double b) {
  uint64_t x, y;
  std::memcpy(&x, &a, 8);
  std::memcpy(&y, &b, 8);
  return x == y;
}

// A view whose 4 consecutive elements along `axis` are 4 consecutive
// buffer elements on a 16-byte boundary (4-byte for bool) whenever that
// axis's coordinate is a multiple of 4.
bool vec_along(const View &v, size_t axis) {
  if (axis >= v.strides.size() || v.strides[axis] != 1 || v.offset % 4 != 0) return false;
  for (size_t a = 0; a < v.strides.size(); a++)
    if (a != axis && v.shape[a] != 1 && v.strides[a] % 4 != 0) return false;
  return true;
}

// The chain tops (Buffer or a movement chain over one) of an elementwise
// expression; false when it holds anything else (a reduction).
bool chain_tops(const UOp *n, std::vector<const UOp *> &tops,
                std::unordered_set<const UOp *> &seen) {
  if (!seen.insert(n).second || n->op == Op::Const) return true;
  if (n->op == Op::Contiguous || n->op == Op::After) return chain_tops(n->src[0].get(), tops, seen);
  if (is_alu(n->op)) {
    for (auto &c : n->src)
      if (!chain_tops(c.get(), tops, seen)) return false;
    return true;
  }
  if (n->op == Op::Buffer || is_movement(n->op)) {
    tops.push_back(n);
    return true;
  }
  return false;
}

const char *vec4_type(DType d) {
  switch (d) {
    case DType::F32: return "float4";
    case DType::I32: return "int4";
    case DType::Bool: return "uchar4";
  }
  return "float4";
}

class Emitter {
 public:
  explicit Emitter(const ParamSlots &ps) : ps_(ps) { scopes_.emplace_back(); }

  std::ostringstream body;
  int indent = 2;

  void line(const std::string &s) { body << std::string((size_t)indent, ' ') << s << "\n"; }
  std::string fresh(const char *p) { return std::string(p) + std::to_string(tmp_++); }
  void open(const std::string &head) {
    line(head + " {");
    indent += 2;
    scopes_.emplace_back();
  }
  void close() {
    indent -= 2;
    line("}");
    scopes_.pop_back();
  }
  // A brace block that starts a fresh memo scope.
  void open_block() { open(""); }

  // Index expression variables: literals stay literal, others get a name.
  std::string idx(const std::string &expr) {
    if (is_int_literal(expr)) return expr;
    for (auto s = scopes_.rbegin(); s != scopes_.rend(); ++s) {
      auto f = s->idx.find(expr);
      if (f != s->idx.end()) return f->second;
    }
    std::string v = fresh("i");
    line("const long long " + v + " = " + expr + ";");
    scopes_.back().idx[expr] = v;
    return v;
  }

  Val value(const UOp *n, const std::vector<std::string> &ctx);

  // Index into the buffer at the bottom of a movement chain.
  std::string view_index(const UOp *n, const std::vector<std::string> &ctx,
                         const DeviceBuffer **buf);

 private:
  struct Scope {
    std::unordered_map<std::string, Val> vals;
    std::unordered_map<std::string, std::string> idx;
  };

  Val lookup(const std::string &key) {
    for (auto s = scopes_.rbegin(); s != scopes_.rend(); ++s) {
      auto f = s->vals.find(key);
      if (f != s->vals.end()) return f->second;
    }
    return Val{};
  }

  std::vector<std::string> src_ctx(const UOp *n, const std::vector<std::string> &ctx);
  Val emit_alu(Op op, DType dt, const std::vector<Val> &a);
  Val emit_reduce(const UOp *n, const std::vector<std::string> &ctx);
  Val bind(const std::string &expr, DType dt) {
    std::string v = fresh("v");
    line(std::string("const ") + ctype(dt) + " " + v + " = " + expr + ";");
    return Val{v, dt};
  }

  const ParamSlots &ps_;
  std::vector<Scope> scopes_;
  int tmp_ = 0;

 public:
  // Thread mapping of the kernel's reductions (RenderSpec::coop).
  RenderSpec::Coop coop = RenderSpec::Thread;
  // Block mapping: which shared-memory fold arrays the kernel declares.
  bool smem_f = false, smem_i = false;
  // 128-bit path: the value of a vector-loaded leaf at lane `lane` is a
  // component of the loaded vector; keyed by the leaf node and the lane's
  // coordinate key.
  std::unordered_map<std::string, std::string> vec_vals;
  static std::string vec_key(const UOp *n, const std::vector<std::string> &ctx) {
    std::string k = std::to_string((uintptr_t)n);
    for (auto &c : ctx) k += "," + c;
    return k;
  }
};

// Block mapping: 32 output elements per block (one per lane), the reduced
// axis split over kBlockWarps warps (1024 threads, so enough loads are in
// flight when the kernel has few outputs).
constexpr int kBlockWarps = 32;

std::string mul_idx(const std::string &a, int64_t k) {
  if (a == "0" || k == 0) return "0";
  if (k == 1) return a;
  return a + " * " + std::to_string(k) + "LL";
}

std::vector<std::string> Emitter::src_ctx(const UOp *n, const std::vector<std::string> &ctx) {
  const UOp *s = n->src[0].get();
  const Shape &ss = s->shape;
  std::vector<std::string> out(ss.size(), "0");
  switch (n->op) {
    case Op::Reshape: {
      const Shape &ds = n->shape;
      if (numel(ss) == 1) return out;
      if (ctx.size() != ds.size())
        throw Panic("render: reshape index rank " + std::to_string(ctx.size()) + " != shape " +
                    shape_str(ds));
      std::vector<size_t> dn, sn;
      for (size_t a = 0; a < ds.size(); a++)
        if (ds[a] != 1) dn.push_back(a);
      for (size_t a = 0; a < ss.size(); a++)
        if (ss[a] != 1) sn.push_back(a);
      bool same = dn.size() == sn.size();
      for (size_t i = 0; same && i < dn.size(); i++) same = ds[dn[i]] == ss[sn[i]];
      if (same) {
        for (size_t i = 0; i < dn.size(); i++) out[sn[i]] = ctx[dn[i]];
        return out;
      }
      // General reshape: row-major linear index, unflattened into the source.
      std::string lin;
      int64_t stride = 1;
      for (size_t a = ds.size(); a-- > 0;) {
        if (ds[a] != 1 && ctx[a] != "0") {
          std::string t = mul_idx(ctx[a], stride);
          lin = lin.empty() ? t : t + " + " + lin;
        }
        stride *= ds[a];
      }
      if (lin.empty()) return out;
      std::string l = idx(lin);
      int64_t sstride = 1;
      std::vector<int64_t> strides(ss.size());
      for (size_t a = ss.size(); a-- > 0;) {
        strides[a] = sstride;
        sstride *= ss[a];
      }
      bool first = true;
      for (size_t a = 0; a < ss.size(); a++) {
        if (ss[a] == 1) continue;
        std::string e = strides[a] == 1 ? l : "(" + l + " / " + std::to_string(strides[a]) + "LL)";
        if (!first) e = "(" + e + " % " + std::to_string(ss[a]) + "LL)";
        first = false;
        out[a] = idx(e);
      }
      return out;
    }
    case Op::Permute:
      for (size_t i = 0; i < n->arg.size(); i++) out[(size_t)n->arg[i]] = ctx.at(i);
      return out;
    case Op::Expand:
      for (size_t a = 0; a < ss.size(); a++) out[a] = ss[a] == 1 ? "0" : ctx.at(a);
      return out;
    case Op::Shrink: {
      auto it = ps_.shrink_slots.find(n);
      for (size_t a = 0; a < ss.size(); a++) {
        int slot = it != ps_.shrink_slots.end() ? it->second[a] : -1;
        std::string start;
        if (slot >= 0)
          start = "(long long)s" + std::to_string(slot);
        else
          start = std::to_string((long long)n->src[a + 1]->value);
        if (start == "0")
          out[a] = ctx.at(a);
        else if (ctx.at(a) == "0")
          out[a] = idx(start);
        else
          out[a] = idx(ctx.at(a) + " + " + start);
      }
      return out;
    }
    default:
      return ctx;
  }
}

std::string Emitter::view_index(const UOp *n, const std::vector<std::string> &ctx,
                                const DeviceBuffer **buf) {
  if (n->op == Op::Buffer) {
    *buf = n->buf.get();
    return ctx.empty() ? "0" : ctx[0];
  }
  if (is_movement(n->op) || n->op == Op::After || n->op == Op::Contiguous) {
    if (n->op == Op::After || n->op == Op::Contiguous) return view_index(n->src[0].get(), ctx, buf);
    return view_index(n->src[0].get(), src_ctx(n, ctx), buf);
  }
  throw Panic(std::string("render: store destination must be a view of a buffer, got ") +
              op_name(n->op));
}

Val Emitter::emit_alu(Op op, DType dt, const std::vector<Val> &a) {
  // symbolic_simple folds (src/optimize/symbolic.rs:42-56).
  if ((op == Op::Add || op == Op::Mul) && a.size() == 2 && optimize_config().symbolic) {
    const Val &x = a[0], &y = a[1];
    if (x.is_const && y.is_const) {
      double r = op == Op::Add ? x.c + y.c : x.c * y.c;
      if (dt == DType::I32) r = (double)(op == Op::Add ? (long long)x.c + (long long)y.c
                                                       : (long long)x.c * (long long)y.c);
      return Val{literal_of(r, dt), dt, true, r};
    }
    if (op == Op::Add && y.is_const && bits_equal(y.c, 0.0)) return x;
    if (op == Op::Add && x.is_const && bits_equal(x.c, 0.0)) return y;
    if (op == Op::Mul && y.is_const && bits_equal(y.c, 1.0)) return x;
    if (op == Op::Mul && x.is_const && bits_equal(x.c, 1.0)) return y;
    if (op == Op::Mul && y.is_const && bits_equal(y.c, 0.0)) return y;
    if (op == Op::Mul && x.is_const && bits_equal(x.c, 0.0)) return x;
  }
  const bool f = dt == DType::F32;
  std::string e;
  switch (op) {
    case Op::Add:
      e = f ? "__fadd_rn(" + a[0].expr + ", " + a[1].expr + ")"
            : "(int)((unsigned)(" + a[0].expr + ") + (unsigned)(" + a[1].expr + "))";
      break;
    case Op::Mul:
      e = f ? "__fmul_rn(" + a[0].expr + ", " + a[1].expr + ")"
            : "(int)((unsigned)(" + a[0].expr + ") * (unsigned)(" + a[1].expr + "))";
      break;
    case Op::Neg:
      e = f ? "(-" + a[0].expr + ")" : "(int)(0u - (unsigned)(" + a[0].expr + "))";
      break;
    case Op::Reciprocal:
      e = f ? "__frcp_rn(" + a[0].expr + ")" : "(1 / (" + a[0].expr + "))";
      break;
    case Op::Exp2:
      e = "(float)exp2((double)" + a[0].expr + ")";
      break;
    case Op::Log2:
      e = "(float)log2((double)" + a[0].expr + ")";
      break;
    case Op::Sqrt:
      e = "__fsqrt_rn(" + a[0].expr + ")";
      break;
    case Op::Max:
      e = "((" + a[0].expr + " > " + a[1].expr + ") ? " + a[0].expr + " : " + a[1].expr + ")";
      break;
    case Op::CmpLt:
      e = "(" + a[0].expr + " < " + a[1].expr + ")";
      break;
    case Op::Where:
      e = "(" + a[0].expr + " ? " + a[1].expr + " : " + a[2].expr + ")";
      break;
    default:
      throw Panic(std::string("render: not an ALU op: ") + op_name(op));
  }
  return bind(e, dt);
}

Val Emitter::emit_reduce(const UOp *n, const std::vector<std::string> &ctx) {
  const UOp *s = n->src[0].get();
  const Shape &ss = s->shape;
  std::vector<int64_t> axes = n->arg;
  std::sort(axes.begin(), axes.end());
  axes.erase(std::unique(axes.begin(), axes.end()), axes.end());
  const DType dt = n->dtype;
  const Op rop = n->reduce_op;
  std::string init = rop == Op::Add ? literal_of(0.0, dt) : literal_of(-INFINITY, dt);
  std::string acc = fresh("acc");
  line(std::string(ctype(dt)) + " " + acc + " = " + init + ";");
  // An empty reduced axis leaves the identity: no element is read.
  for (int64_t a : axes)
    if (ss[(size_t)a] == 0) return Val{acc, dt};
  std::vector<std::string> sc = ctx;
  sc.resize(ss.size(), "0");
  size_t opened = 0;
  auto combine = [&](const Val &x, const Val &y) {
    // Reduce combination is built after symbolic folding in the reference,
    // so it is never folded.
    Val nx = x, ny = y;
    nx.is_const = ny.is_const = false;
    return emit_alu(rop, dt, {nx, ny});
  };
  // Warp / Block mapping: the last reduced axis longer than 1 is split over
  // the lanes (Warp) or the warps (Block) of the threads sharing an output
  // element; the other reduced axes are walked in order by every thread.
  int64_t split = -1;
  for (int64_t a : axes)
    if (ss[(size_t)a] > 1) split = a;
  if (coop != RenderSpec::Thread && split >= 0) {
    const bool warp = coop == RenderSpec::Warp;
    // kPar independent partial accumulators per thread, so kPar loads are in
    // flight at once; folded pairwise after the loops (a fixed order)
    constexpr int kPar = 8;
    const int64_t R = ss[(size_t)split];
    const int64_t step = warp ? 32 : kBlockWarps;
    std::vector<std::string> part(kPar);
    for (int u = 0; u < kPar; u++) {
      part[u] = fresh("acc");
      line(std::string(ctype(dt)) + " " + part[u] + " = " + init + ";");
    }
    for (int64_t a : axes) {
      if (a == split) continue;
      if (ss[(size_t)a] == 1) {
        sc[(size_t)a] = "0";
        continue;
      }
      std::string r = fresh("r");
      open("for (long long " + r + " = 0; " + r + " < " + std::to_string(ss[(size_t)a]) +
           "LL; ++" + r + ")");
      opened++;
      sc[(size_t)a] = r;
    }
    // Warp mapping over a split axis that every operand reads contiguously:
    // each lane takes 4 consecutive elements per access (one 128-bit load
    // per operand), 4 partials of 4 elements each per iteration.
    std::vector<const UOp *> vleaves;
    if (warp && R % 4 == 0 && R >= 128) {
      std::vector<const UOp *> tops;
      std::unordered_set<const UOp *> seen;
      if (chain_tops(s, tops, seen))
        for (const UOp *t : tops) {
          if (t->shape != ss) continue;
          auto v = try_view(t);
          if (v && !v->buf->known_zero() && vec_along(*v, (size_t)split)) vleaves.push_back(t);
        }
    }
    if (!vleaves.empty()) {
      constexpr int kParV = 4;
      std::string r = fresh("r");
      open("for (long long " + r + " = fg_lane * 4LL; " + r + " < " + std::to_string(R) + "LL; " + r +
           " += " + std::to_string(128 * kParV) + "LL)");
      opened++;
      static const char *comp[4] = {".x", ".y", ".z", ".w"};
      for (int u = 0; u < kParV; u++) {
        std::string ru = u == 0 ? r : idx(r + " + " + std::to_string(128 * u) + "LL");
        if (u > 0) open("if (" + ru + " < " + std::to_string(R) + "LL)");
        std::vector<std::vector<std::string>> lc(4, sc);
        lc[0][(size_t)split] = ru;
        for (int j = 1; j < 4; j++) lc[j][(size_t)split] = idx(ru + " + " + std::to_string(j) + "LL");
        for (const UOp *leaf : vleaves) {
          const DeviceBuffer *db = nullptr;
          std::string at = view_index(leaf, lc[0], &db);
          std::string q = fresh("q");
          line(std::string("const ") + vec4_type(leaf->dtype) + " " + q +
               " = *reinterpret_cast<const " + vec4_type(leaf->dtype) + " *>(p" +
               std::to_string(ps_.buffer_slot.at(db)) + " + " + at + ");");
          for (int j = 0; j < 4; j++) {
            std::string xv = q + comp[j];
            if (leaf->dtype == DType::Bool) xv = "(" + xv + " != 0)";
            vec_vals[vec_key(leaf, lc[j])] = xv;
          }
        }
        for (int j = 0; j < 4; j++) {
          Val v = value(s, lc[j]);
          Val upd = combine(Val{part[u], dt}, v);
          line(part[u] + " = " + upd.expr + ";");
        }
        vec_vals.clear();
        if (u > 0) close();
      }
      while (opened--) close();
      for (int w = kParV / 2; w >= 1; w /= 2)
        for (int u = 0; u < w; u++) {
          Val f = combine(Val{part[u], dt}, Val{part[u + w], dt});
          line(part[u] + " = " + f.expr + ";");
        }
      line(acc + " = " + part[0] + ";");
      for (int off = 16; off >= 1; off >>= 1) {
        open_block();
        std::string t = fresh("t");
        line(std::string("const ") + ctype(dt) + " " + t + " = __shfl_xor_sync(0xffffffffu, " +
             acc + ", " + std::to_string(off) + ");");
        Val u = combine(Val{acc, dt}, Val{t, dt});
        line(acc + " = " + u.expr + ";");
        close();
      }
      return Val{acc, dt};
    }
    std::string r = fresh("r");
    open(std::string("for (long long ") + r + " = " + (warp ? "fg_lane" : "fg_warp") + "; " + r +
         " < " + std::to_string(R) + "LL; " + r + " += " + std::to_string(step * kPar) + "LL)");
    opened++;
    for (int u = 0; u < kPar; u++) {
      std::string ru = u == 0 ? r : idx(r + " + " + std::to_string(step * u) + "LL");
      if (u > 0) open("if (" + ru + " < " + std::to_string(R) + "LL)");
      sc[(size_t)split] = ru;
      Val v = value(s, sc);
      Val upd = combine(Val{part[u], dt}, v);
      line(part[u] + " = " + upd.expr + ";");
      if (u > 0) close();
    }
    while (opened--) close();
    for (int w = kPar / 2; w >= 1; w /= 2)
      for (int u = 0; u < w; u++) {
        Val f = combine(Val{part[u], dt}, Val{part[u + w], dt});
        line(part[u] + " = " + f.expr + ";");
      }
    line(acc + " = " + part[0] + ";");
    if (warp) {
      // xor-shuffle tree: every lane ends with the fold of all 32 partials
      for (int off = 16; off >= 1; off >>= 1) {
        open_block();
        std::string t = fresh("t");
        line(std::string("const ") + ctype(dt) + " " + t + " = __shfl_xor_sync(0xffffffffu, " +
             acc + ", " + std::to_string(off) + ");");
        Val u = combine(Val{acc, dt}, Val{t, dt});
        line(acc + " = " + u.expr + ";");
        close();
      }
    } else {
      // warp w's partial goes to sm[w*32 + lane]; warp 0 folds the partials
      // in warp order and every warp reads the result back
      const std::string sm = dt == DType::I32 ? "fg_sm_i" : "fg_sm_f";
      (dt == DType::I32 ? smem_i : smem_f) = true;
      line(sm + "[threadIdx.x] = " + acc + ";");
      line("__syncthreads();");
      open("if (fg_warp == 0)");
      for (int w = 1; w < kBlockWarps; w++) {
        Val u = combine(Val{acc, dt}, Val{sm + "[" + std::to_string(32 * w) + " + fg_lane]", dt});
        line(acc + " = " + u.expr + ";");
      }
      line(sm + "[fg_lane] = " + acc + ";");
      close();
      line("__syncthreads();");
      line(acc + " = " + sm + "[fg_lane];");
      line("__syncthreads();");
    }
    return Val{acc, dt};
  }
  for (size_t i = 0; i + 1 < axes.size(); i++) {
    size_t a = (size_t)axes[i];
    std::string r = fresh("r");
    open("for (long long " + r + " = 0; " + r + " < " + std::to_string(ss[a]) + "LL; ++" + r +
         ")");
    opened++;
    sc[a] = r;
  }
  size_t last = axes.empty() ? 0 : (size_t)axes.back();
  int64_t R = axes.empty() ? 1 : ss[last];
  if (!axes.empty() && R > 4 && R % 4 == 0 && optimize_config().unroll) {
    std::string r = fresh("r");
    if (R / 4 > 8) line("#pragma unroll 4");
    open("for (long long " + r + " = 0; " + r + " < " + std::to_string(R / 4) + "LL; ++" + r + ")");
    opened++;
    Val lanes[4];
    for (int u = 0; u < 4; u++) {
      sc[last] = idx(r + " * 4LL + " + std::to_string(u));
      lanes[u] = value(s, sc);
    }
    Val h = combine(combine(combine(lanes[0], lanes[1]), lanes[2]), lanes[3]);
    Val acc_v{acc, dt};
    Val upd = combine(acc_v, h);
    line(acc + " = " + upd.expr + ";");
  } else if (!axes.empty() && R > 1) {
    std::string r = fresh("r");
    if (R > 8) line("#pragma unroll 4");
    open("for (long long " + r + " = 0; " + r + " < " + std::to_string(R) + "LL; ++" + r + ")");
    opened++;
    sc[last] = r;
    Val v = value(s, sc);
    Val upd = combine(Val{acc, dt}, v);
    line(acc + " = " + upd.expr + ";");
  } else {
    if (!axes.empty()) sc[last] = "0";
    open_block();
    opened++;
    Val v = value(s, sc);
    Val upd = combine(Val{acc, dt}, v);
    line(acc + " = " + upd.expr + ";");
  }
  while (opened--) close();
  return Val{acc, dt};
}

Val Emitter::value(const UOp *n, const std::vector<std::string> &ctx) {
  if (n->op == Op::Const) return Val{literal_of(n->value, n->dtype), n->dtype, true, n->value};
  std::string key = vec_key(n, ctx);
  if (!vec_vals.empty()) {
    auto f = vec_vals.find(key);
    if (f != vec_vals.end()) return Val{f->second, n->dtype};
  }
  Val m = lookup(key);
  if (!m.expr.empty()) return m;
  Val out;
  switch (n->op) {
    case Op::Buffer: {
      if (n->buf->known_zero()) {
        // a never-written zeros buffer: the loaded value is 0 (not folded
        // as a literal: the reference loads it)
        out = Val{literal_of(0.0, n->dtype), n->dtype};
        break;
      }
      int slot = ps_.buffer_slot.at(n->buf.get());
      std::string i = ctx.empty() ? "0" : ctx[0];
      std::string ld = "p" + std::to_string(slot) + "[" + i + "]";
      if (n->dtype == DType::Bool) ld = "(" + ld + " != 0)";
      out = bind(ld, n->dtype);
      break;
    }
    case Op::Reshape:
    case Op::Permute:
    case Op::Expand:
    case Op::Shrink:
      out = value(n->src[0].get(), src_ctx(n, ctx));
      break;
    case Op::Contiguous:
    case Op::After:
      out = value(n->src[0].get(), ctx);
      break;
    case Op::ReduceAxis:
      out = emit_reduce(n, ctx);
      break;
    default: {
      if (!is_alu(n->op)) throw Panic(std::string("render: unsupported op ") + op_name(n->op));
      std::vector<Val> a;
      for (auto &s : n->src) a.push_back(value(s.get(), ctx));
      out = emit_alu(n->op, n->dtype, a);
      break;
    }
  }
  if (!out.is_const) scopes_.back().vals[key] = out;
  return out;
}

bool contains_reduce(const UOpP &root) {
  for (const UOp *n : toposort_nodes(root.get()))
    if (n->op == Op::ReduceAxis) return true;
  return false;
}

const char *vec_type(DType d) {
  switch (d) {
    case DType::F32: return "float4";
    case DType::I32: return "int4";
    case DType::Bool: return "uchar4";
  }
  return "float4";
}

// A view whose 4 consecutive elements along the innermost axis are 4
// consecutive, 16-byte aligned (4-byte for bool) elements of its buffer,
// given that the innermost coordinate is a multiple of 4.
bool vec_view(const View &v) {
  const size_t r = v.strides.size();
  if (r == 0 || v.strides[r - 1] != 1 || v.offset % 4 != 0) return false;
  for (size_t a = 0; a + 1 < r; a++)
    if (v.shape[a] != 1 && v.strides[a] % 4 != 0) return false;
  return true;
}

// 128-bit path of an elementwise kernel: the leaves (maximal movement chains
// over a buffer, at the domain's shape) whose 4 consecutive elements can be
// one vector load.  Empty when the kernel does not qualify.
struct VecPlan {
  bool ok = false;
  std::vector<const UOp *> leaves;  // vector-loaded chain tops
  bool vec_store = false;
  size_t axis = 0;  // the value's axis that the domain's last coordinate walks
};

VecPlan plan_vec4(const RenderSpec &spec) {
  VecPlan vp;
  const Shape &D = spec.domain;
  if (D.empty() || D.back() % 4 != 0 || numel(D) == 0) return vp;
  const Shape &VS = spec.value->shape;
  if (spec.value_ctx.empty()) {
    if (VS != D) return vp;
    vp.axis = VS.size() - 1;
  } else {
    // a staging copy: exactly one value axis is walked by the last domain
    // coordinate, and no other axis depends on it
    const std::string last = "c" + std::to_string(D.size() - 1);
    int found = -1;
    for (size_t a = 0; a < spec.value_ctx.size(); a++) {
      if (spec.value_ctx[a] == last) {
        if (found >= 0) return vp;
        found = (int)a;
      } else if (spec.value_ctx[a].find(last) != std::string::npos) {
        return vp;
      }
    }
    if (found < 0) return vp;
    vp.axis = (size_t)found;
  }
  if (spec.store == RenderSpec::Pitched && (D.size() != 2 || spec.pitch % 4 != 0)) return vp;
  bool ok = true;
  std::unordered_set<const UOp *> seen;
  std::function<void(const UOp *)> visit = [&](const UOp *n) {
    if (!ok || !seen.insert(n).second) return;
    if (n->op == Op::Const) return;
    if (n->op == Op::Contiguous || n->op == Op::After) return visit(n->src[0].get());
    if (is_alu(n->op)) {
      for (auto &c : n->src) visit(c.get());
      return;
    }
    if (n->op == Op::Buffer || is_movement(n->op)) {
      if (n->shape != VS) return;  // read element by element
      auto v = try_view(n);
      if (v && !v->buf->known_zero() && vec_along(*v, vp.axis)) vp.leaves.push_back(n);
      return;
    }
    ok = false;  // a reduction or an op the 128-bit path does not cover
  };
  visit(spec.value.get());
  if (!ok) return vp;
  if (spec.store == RenderSpec::View) {
    auto v = try_view(spec.dest.get());
    vp.vec_store = v && spec.dest->shape == D && vec_view(*v);
  } else {
    vp.vec_store = true;  // contiguous, or pitched rows with pitch % 4 == 0
  }
  vp.ok = vp.vec_store || !vp.leaves.empty();
  return vp;
}

}  // namespace

void choose_thread_mapping(RenderSpec &spec) {
  spec.coop = RenderSpec::Thread;
  if (exact_mode() || spec.store == RenderSpec::Pitched) return;
  const int64_t outputs = numel(spec.domain);
  if (outputs <= 0) return;
  int64_t best = 0;
  bool inner = false;
  int reduces = 0;
  const auto order = toposort_nodes(spec.value.get());
  for (const UOp *n : order) {
    if (n->op != Op::ReduceAxis) continue;
    reduces++;
    if (n->dtype == DType::Bool) return;
    const Shape &ss = n->src[0]->shape;
    int64_t split = -1;
    for (int64_t a : n->arg)
      if (ss[(size_t)a] > 1 && a > split) split = a;
    if (split < 0) continue;
    if (ss[(size_t)split] > best) {
      best = ss[(size_t)split];
      inner = true;
      for (size_t b = (size_t)split + 1; b < ss.size(); b++)
        if (ss[b] != 1) inner = false;
    }
  }
  // A reduction inside another's source (the scheduler materialises those;
  // kept as a guard) stays on the sequential mapping.
  if (reduces > 1)
    for (const UOp *n : order)
      if (n->op == Op::ReduceAxis)
        for (const UOp *m : toposort_nodes(n->src[0].get()))
          if (m->op == Op::ReduceAxis) return;
  if (best < 32) return;
  if (inner)
    spec.coop = RenderSpec::Warp;
  else if (outputs < (int64_t(1) << 17))
    spec.coop = RenderSpec::Block;
}

RenderedKernel render_kernel(const RenderSpec &spec) {
  const bool store_view = spec.store == RenderSpec::View;
  // Slot assignment as the reference parameterises (slot 0 = output for
  // allocating kernels; the destination is a regular input for stores).
  ParamSlots ps = store_view ? collect_params(make_store(spec.dest, spec.value), 0)
                             : collect_params(spec.value, 1);
  Emitter em(ps);
  const Shape &D = spec.domain;
  const int64_t N = numel(D);
  const bool has_reduce = contains_reduce(spec.value);
  const RenderSpec::Coop coop = has_reduce && N > 0 ? spec.coop : RenderSpec::Thread;
  em.coop = coop;
  const VecPlan vp = has_reduce ? VecPlan{} : plan_vec4(spec);
  // elements per thread: `U` groups (of 4 consecutive elements on the
  // 128-bit path, of one element otherwise) 256 * group apart
  const int V = vp.ok ? 4 : 1;
  const int U = coop != RenderSpec::Thread ? 1 : vp.ok ? 2 : has_reduce ? 1 : std::max(1, spec.unroll);
  int dest_slot = -1;
  if (store_view) {
    const DeviceBuffer *db = nullptr;
    std::vector<std::string> dummy(spec.dest->shape.size(), "0");
    Emitter probe(ps);
    probe.view_index(spec.dest.get(), dummy, &db);
    dest_slot = ps.buffer_slot.at(db);
  }

  std::vector<int64_t> strides(D.size());
  int64_t st = 1;
  for (size_t a = D.size(); a-- > 0;) {
    strides[a] = st;
    st *= D[a];
  }
  const DType odt = store_view ? spec.dest->dtype : spec.out_dtype;
  const DType vdt = spec.value->dtype;
  const std::string Ns = std::to_string(N) + "LL";
  int64_t per_block = 256LL * U * V;
  if (coop == RenderSpec::Warp) {
    em.line("const int fg_lane = threadIdx.x & 31;");
    em.line("const long long e0 = (long long)blockIdx.x * 8LL + (threadIdx.x >> 5);");
    per_block = 8;
  } else if (coop == RenderSpec::Block) {
    // every thread takes part in the block's folds, so an out-of-range lane
    // evaluates the last element and does not store
    em.line("const int fg_lane = threadIdx.x & 31, fg_warp = threadIdx.x >> 5;");
    em.line("const bool fg_in = (long long)blockIdx.x * 32LL + fg_lane < " + Ns + ";");
    em.line("const long long e0 = fg_in ? (long long)blockIdx.x * 32LL + fg_lane : " + Ns +
            " - 1LL;");
    per_block = 32;
  } else if (vp.ok) {
    em.line("const long long e0 = ((long long)blockIdx.x * " + std::to_string(256 * U) +
            "LL + threadIdx.x) * 4LL;");
  } else {
    em.line("const long long e0 = (long long)blockIdx.x * " + std::to_string(256 * U) +
            "LL + threadIdx.x;");
  }
  // res[u][j]: value of lane j of group u; sidx[u]: its store index (lane 0
  // of the group on the 128-bit path), -1 when out of range
  std::vector<std::vector<std::string>> res(U, std::vector<std::string>(V));
  std::vector<std::string> sidx(U);
  std::vector<std::vector<std::string>> lane_sidx(U, std::vector<std::string>(V));
  const bool scalar_stores = vp.ok && !vp.vec_store;
  for (int u = 0; u < U; u++) {
    for (int j = 0; j < V; j++) {
      res[u][j] = "res" + std::to_string(u) + (V > 1 ? "_" + std::to_string(j) : "");
      em.line(std::string(ctype(vdt)) + " " + res[u][j] + " = " + literal_of(0.0, vdt) + ";");
      if (scalar_stores) {
        lane_sidx[u][j] = "st" + std::to_string(u) + "_" + std::to_string(j);
        em.line("long long " + lane_sidx[u][j] + " = -1;");
      }
    }
    sidx[u] = "st" + std::to_string(u);
    em.line("long long " + sidx[u] + " = -1;");
  }
  for (int u = 0; u < U; u++) {
    std::string e = u == 0 ? "e0" : "(e0 + " + std::to_string(256 * V * u) + "LL)";
    if (coop == RenderSpec::Block)
      em.open_block();
    else
      em.open("if (" + e + " < " + Ns + ")");
    std::string ev = em.idx(e);
    std::vector<std::string> c(D.size(), "0");
    bool first = true;
    for (size_t a = 0; a < D.size(); a++) {
      if (D[a] == 1) continue;
      std::string x = strides[a] == 1 ? ev : "(" + ev + " / " + std::to_string(strides[a]) + "LL)";
      if (!first) x = "(" + x + " % " + std::to_string(D[a]) + "LL)";
      first = false;
      c[a] = em.idx(x);
    }
    std::vector<std::string> vctx = c;
    if (!spec.value_ctx.empty()) {
      vctx.clear();
      for (const std::string &t : spec.value_ctx) {
        std::string x = t;
        for (size_t a = D.size(); a-- > 0;) {
          std::string name = "c" + std::to_string(a);
          size_t pos;
          while ((pos = x.find(name)) != std::string::npos) x.replace(pos, name.size(), c[a]);
        }
        vctx.push_back(em.idx(x));
      }
    }
    // lane j's coordinates: the walked axis' one + j
    std::vector<std::vector<std::string>> lctx(V, vctx);
    for (int j = 1; j < V; j++)
      lctx[j][vp.axis] = em.idx(vctx[vp.axis] + " + " + std::to_string(j) + "LL");
    if (vp.ok) {
      // one 128-bit load per vector leaf; its lanes stand for the leaf's
      // value at the group's 4 elements
      em.vec_vals.clear();
      for (const UOp *leaf : vp.leaves) {
        const DeviceBuffer *db = nullptr;
        std::string at = em.view_index(leaf, vctx, &db);
        std::string q = em.fresh("q");
        const int slot = ps.buffer_slot.at(db);
        em.line(std::string("const ") + vec_type(leaf->dtype) + " " + q + " = *reinterpret_cast<const " +
                vec_type(leaf->dtype) + " *>(p" + std::to_string(slot) + " + " + at + ");");
        static const char *comp[4] = {".x", ".y", ".z", ".w"};
        for (int j = 0; j < V; j++) {
          std::string x = q + comp[j];
          if (leaf->dtype == DType::Bool) x = "(" + x + " != 0)";
          em.vec_vals[Emitter::vec_key(leaf, lctx[j])] = x;
        }
      }
    }
    for (int j = 0; j < V; j++) {
      Val v = em.value(spec.value.get(), lctx[j]);
      em.line(res[u][j] + " = " + v.expr + ";");
    }
    em.vec_vals.clear();
    std::string s;
    if (store_view) {
      const DeviceBuffer *db = nullptr;
      if (scalar_stores) {
        for (int j = 0; j < V; j++) {
          std::vector<std::string> cj = c;
          cj.back() = lctx[j].back();
          em.line(lane_sidx[u][j] + " = " + em.view_index(spec.dest.get(), cj, &db) + ";");
        }
      }
      s = em.view_index(spec.dest.get(), c, &db);
    } else if (spec.store == RenderSpec::Pitched) {
      s = c.size() == 2 ? em.idx(mul_idx(c[0], spec.pitch) + " + " + c[1]) : ev;
    } else {
      s = ev;
    }
    em.line(sidx[u] + " = " + s + ";");
    em.close();
  }
  const int out_slot = store_view ? dest_slot : 0;
  const std::string out = "p" + std::to_string(out_slot);
  std::string guard = coop == RenderSpec::Warp    ? "fg_lane == 0 && "
                      : coop == RenderSpec::Block ? "fg_warp == 0 && fg_in && "
                                                  : "";
  auto cast = [&](const std::string &r) {
    return odt == DType::Bool ? "(unsigned char)(" + r + ")" : r;
  };
  const bool with_lo = spec.with_lo && odt == DType::F32 && coop == RenderSpec::Thread;
  auto lo_of = [](const std::string &r) {
    return "__fsub_rn(" + r + ", __uint_as_float(__float_as_uint(" + r + ") & 0xffffe000u))";
  };
  for (int u = 0; u < U; u++) {
    if (vp.ok && vp.vec_store) {
      const char *mk = odt == DType::F32 ? "make_float4" : odt == DType::I32 ? "make_int4"
                                                                            : "make_uchar4";
      em.line("if (" + sidx[u] + " >= 0) *reinterpret_cast<" + vec_type(odt) + " *>(" + out +
              " + " + sidx[u] + ") = " + mk + "(" + cast(res[u][0]) + ", " + cast(res[u][1]) +
              ", " + cast(res[u][2]) + ", " + cast(res[u][3]) + ");");
      if (with_lo)
        em.line("if (" + sidx[u] + " >= 0) *reinterpret_cast<float4 *>(plo + " + sidx[u] +
                ") = make_float4(" + lo_of(res[u][0]) + ", " + lo_of(res[u][1]) + ", " +
                lo_of(res[u][2]) + ", " + lo_of(res[u][3]) + ");");
    } else if (scalar_stores) {
      for (int j = 0; j < V; j++) {
        em.line("if (" + sidx[u] + " >= 0) " + out + "[" + lane_sidx[u][j] + "] = " +
                cast(res[u][j]) + ";");
        if (with_lo)
          em.line("if (" + sidx[u] + " >= 0) plo[" + lane_sidx[u][j] + "] = " + lo_of(res[u][j]) +
                  ";");
      }
    } else {
      em.line("if (" + guard + sidx[u] + " >= 0) " + out + "[" + sidx[u] + "] = " +
              cast(res[u][0]) + ";");
      if (with_lo)
        em.line("if (" + sidx[u] + " >= 0) plo[" + sidx[u] + "] = " + lo_of(res[u][0]) + ";");
    }
  }

  std::ostringstream src;
  src << "// rendered by the ferrograd_b200 front end\n";
  src << "#ifndef INFINITY\n#define INFINITY __int_as_float(0x7f800000)\n#endif\n"
         "#ifndef NAN\n#define NAN __int_as_float(0x7fffffff)\n#endif\n";
  const int threads = coop == RenderSpec::Block ? 32 * kBlockWarps : 256;
  src << "extern \"C\" __global__ void __launch_bounds__(" << threads << ") fg_kernel(";
  std::vector<std::string> params;
  if (!store_view) params.push_back(std::string(storage_type(spec.out_dtype)) + "* __restrict__ p0");
  const int off = store_view ? 0 : 1;
  for (size_t i = 0; i < ps.inputs.size(); i++) {
    const KernelInput &in = ps.inputs[i];
    int slot = (int)i + off;
    if (in.kind == KernelInput::Buffer) {
      bool written = slot == out_slot;
      params.push_back(std::string(written ? "" : "const ") + storage_type(in.buffer->dtype) +
                       "* __restrict__ p" + std::to_string(slot));
    } else {
      params.push_back("int s" + std::to_string(slot));
    }
  }
  if (with_lo) params.push_back("float* __restrict__ plo");
  for (size_t i = 0; i < params.size(); i++) src << (i ? ", " : "") << params[i];
  src << ") {\n";
  if (em.smem_f) src << "  __shared__ float fg_sm_f[" << threads << "];\n";
  if (em.smem_i) src << "  __shared__ int fg_sm_i[" << threads << "];\n";
  src << em.body.str() << "}\n";

  RenderedKernel rk;
  rk.source = src.str();
  rk.block = (uint32_t)threads;
  int64_t blocks = (N + per_block - 1) / per_block;
  rk.grid = (uint32_t)std::max<int64_t>(1, blocks);
  rk.has_out_slot = !store_view;
  rk.params = ps.inputs;
  return rk;
}

}  // namespace ferro
