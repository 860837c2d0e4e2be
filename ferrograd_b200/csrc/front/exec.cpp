// exec.cpp -- runs scheduled proto-kernels on the B200 through the C ABI.
//
// Replaces Tensor::execute_item / run_kernel (src/tensor.rs:813-898,
// 1018-1028) and CpuDevice::{compile,execute} (src/device/cpu.rs:151-208,
// 318-380).  Per item the router
//   1. extracts every reduce-of-broadcast-mul contraction (Tensor::matmul,
//      src/tensor.rs:762-778, and the two contractions its gradient builds,
//      src/gradient.rs:100-106,165-176) large enough for the tensor cores and
//      runs it on fg_gemm_3xtf32, operands passed in place when they are
//      strided views of a buffer and staged into a K-major copy otherwise;
//   2. extracts large f32 ReduceAxis over a contiguous view and runs it on
//      the HBM reduction kernels (fg_reduce_rows / fg_reduce_cols);
//   3. renders what is left (render.cpp) and launches it with fg_execute,
//      compiling with fg_compile on a program-cache miss.
// Steps 1-2 change the summation order of those reductions (fp32 tree /
// tensor-core order instead of the reference's sequential one); with
// FG_FRONT_EXACT=1 every kernel is rendered and the arithmetic is the
// reference's.
#include <algorithm>
#include <chrono>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <optional>
#include <unordered_map>

#include "front_internal.h"

namespace ferro {

namespace {

fg_device *g_dev = nullptr;
int g_ordinal = -1;
uint64_t g_buffer_ids = 0;
Stats g_stats;
std::string g_last_source;
uint64_t g_kernel_count = 0;

void check(int rc, const char *what) {
  if (rc != FG_OK) throw Panic(std::string(what) + ": " + fg_last_error());
}

int env_ordinal() {
  const char *e = std::getenv("FG_DEVICE");
  if (!e || !*e) return 0;
  const char *p = std::strncmp(e, "cuda:", 5) == 0 ? e + 5 : e;
  return std::atoi(p);
}

std::unordered_map<std::string, fg_program *> &program_cache() {
  static std::unordered_map<std::string, fg_program *> c;
  return c;
}

}  // namespace

namespace {
bool exact_env() {
  const char *e = std::getenv("FG_FRONT_EXACT");
  return e && *e && std::strcmp(e, "0") != 0;
}
int g_exact_scope = -1;  // the flag as read at the current realize's start
}  // namespace

bool exact_mode() { return g_exact_scope >= 0 ? g_exact_scope != 0 : exact_env(); }

ExactModeScope::ExactModeScope() : prev(g_exact_scope) { g_exact_scope = exact_env() ? 1 : 0; }
ExactModeScope::~ExactModeScope() { g_exact_scope = prev; }

int debug_level() {
  static const int level = [] {
    const char *e = std::getenv("DEBUG");
    return e ? std::atoi(e) : 0;
  }();
  return level;
}

// DEBUG >= 2 prints each launch's execution time (src/tensor.rs:1017-1028,
// which times the reference's synchronous Device::execute): the device is
// synchronised before the launch and after it, and the wall time between is
// printed.  At lower levels this costs nothing.
struct ExecTimer {
  bool on;
  std::chrono::steady_clock::time_point t0;
  ExecTimer() : on(debug_level() >= 2) {
    if (on) {
      synchronize();
      t0 = std::chrono::steady_clock::now();
    }
  }
  ~ExecTimer() {
    if (!on) return;
    synchronize();
    const double ms =
        std::chrono::duration<double, std::milli>(std::chrono::steady_clock::now() - t0).count();
    fprintf(stderr, "              exec time=%.3fms\n", ms);
  }
};

OptimizeConfig parse_optimize_config(const char *raw) {
  // parse_optimize_config (src/optimize/mod.rs:80-108)
  OptimizeConfig all;
  if (!raw) return all;
  std::string s(raw);
  auto trim = [](std::string t) {
    const char *ws = " \t\n\r\f\v";
    const size_t b = t.find_first_not_of(ws);
    if (b == std::string::npos) return std::string();
    return t.substr(b, t.find_last_not_of(ws) - b + 1);
  };
  s = trim(s);
  if (s.empty() || s == "1" || s == "on" || s == "all") return all;
  OptimizeConfig c;
  c.symbolic = c.upcast = c.unroll = false;
  if (s == "0" || s == "off" || s == "none") return c;
  size_t pos = 0;
  while (pos <= s.size()) {
    size_t comma = s.find(',', pos);
    if (comma == std::string::npos) comma = s.size();
    const std::string pass = trim(s.substr(pos, comma - pos));
    if (pass == "symbolic") c.symbolic = true;
    if (pass == "upcast") c.upcast = true;
    if (pass == "unroll") c.unroll = true;
    pos = comma + 1;
  }
  return c;
}

const OptimizeConfig &optimize_config() {
  static const OptimizeConfig c = parse_optimize_config(std::getenv("OPT"));
  return c;
}

Stats &stats() { return g_stats; }
void reset_stats() { g_stats = Stats{}; }
const std::string &last_source() { return g_last_source; }

void set_device(int ordinal) {
  if (g_dev && ordinal == g_ordinal) return;
  if (g_dev) throw Panic("set_device: the front end's device is already open");
  g_ordinal = ordinal;
}

fg_device *device() {
  if (!g_dev) {
    int ord = g_ordinal >= 0 ? g_ordinal : env_ordinal();
    check(fg_device_open(ord, &g_dev), "open CUDA device");
    g_ordinal = ord;
  }
  return g_dev;
}

void synchronize() {
  if (g_dev) check(fg_device_sync(g_dev), "synchronize");
}

bool device_is_open() { return g_dev != nullptr; }

// ---- DeviceBuffer (src/device.rs:95-214) ----------------------------------
// Storage of dropped buffers is kept, per (dtype, count), and handed to the
// next buffer of the same size that a kernel or an upload will overwrite, so
// a training loop's per-step intermediates and temporaries are neither
// reallocated nor zero-filled.  Reuse is safe in stream order: every launch
// and copy of the front end is on its device's stream.  Buffers that must
// read as zeros (Tensor::zeros) still get fresh zero-filled storage.
namespace {
std::unordered_multimap<uint64_t, fg_buffer *> &storage_pool() {
  static std::unordered_multimap<uint64_t, fg_buffer *> p;
  return p;
}
size_t g_pooled_bytes = 0;
constexpr size_t kPoolCapBytes = size_t(16) << 30;
uint64_t pool_key(DType dt, size_t n) { return ((uint64_t)n << 2) | (uint64_t)dt; }
}  // namespace

DeviceBuffer::DeviceBuffer(DType dt, size_t n) : dtype(dt), count(n), id(g_buffer_ids++) {}

DeviceBuffer::~DeviceBuffer() {
  if (!h) return;
  const size_t bytes = count * dtype_size(dtype);
  if (count && g_pooled_bytes + bytes <= kPoolCapBytes) {
    storage_pool().emplace(pool_key(dtype, count), h);
    g_pooled_bytes += bytes;
  } else {
    fg_free(h);
  }
}

void DeviceBuffer::ensure_allocated() {
  if (h) return;
  const bool must_zero = zero_init && pending.empty();
  auto &pool = storage_pool();
  auto it = must_zero || !count ? pool.end() : pool.find(pool_key(dtype, count));
  if (it != pool.end()) {
    h = it->second;
    pool.erase(it);
    g_pooled_bytes -= count * dtype_size(dtype);
  } else {
    check(fg_alloc(device(), (int)dtype, count, &h), "allocate");
  }
  if (!pending.empty()) {
    int rc = fg_copy_h2d(h, pending.data(), pending.size());
    check(rc, "copy_from_host");
    std::vector<uint8_t>().swap(pending);
  }
}

void DeviceBuffer::upload(const void *data, size_t bytes) {
  ensure_allocated();
  check(fg_copy_h2d(h, data, bytes), "copy_from_host");
}

void *DeviceBuffer::ptr() {
  ensure_allocated();
  void *p = nullptr;
  check(fg_buffer_info(h, &p, nullptr, nullptr), "buffer_info");
  return p;
}

BufferP device_u8_to_f32(const uint8_t *data, size_t n, float divisor) {
  auto src = std::make_shared<DeviceBuffer>(DType::Bool, n);
  if (n) src->pending.assign(data, data + n);
  auto dst = std::make_shared<DeviceBuffer>(DType::F32, n);
  void *st = nullptr;
  check(fg_device_stream(device(), &st), "device stream");
  check(fg_u8_to_f32_div(static_cast<const uint8_t *>(src->ptr()), static_cast<float *>(dst->ptr()),
                         n, divisor, st),
        "u8_to_f32_div");
  return dst;  // src is released stream-ordered after the conversion
}

BufferP device_one_hot_u8(const uint8_t *labels, size_t n, int classes) {
  for (size_t i = 0; i < n; i++)
    if (labels[i] >= classes)
      throw Panic("one_hot: label " + std::to_string(labels[i]) + " out of range for " +
                  std::to_string(classes) + " classes");
  auto src = std::make_shared<DeviceBuffer>(DType::Bool, n);
  if (n) src->pending.assign(labels, labels + n);
  auto dst = std::make_shared<DeviceBuffer>(DType::F32, n * (size_t)classes);
  void *st = nullptr;
  check(fg_device_stream(device(), &st), "device stream");
  check(fg_one_hot_u8(static_cast<const uint8_t *>(src->ptr()), static_cast<float *>(dst->ptr()), n,
                      classes, st),
        "one_hot_u8");
  return dst;
}

std::vector<uint8_t> DeviceBuffer::to_host() {
  ensure_allocated();
  std::vector<uint8_t> out(count * dtype_size(dtype));
  check(fg_copy_d2h(h, out.data(), out.size()), "copy_to_host");
  return out;
}

namespace {

void *stream() {
  void *s = nullptr;
  check(fg_device_stream(device(), &s), "device stream");
  return s;
}

float *fptr(const BufferP &b, int64_t offset = 0) {
  return static_cast<float *>(b->ptr()) + offset;
}

}  // namespace

// ---- strided views --------------------------------------------------------
// Strides of `nd` over the same memory as (od, os), or nothing when the
// reshape is not expressible as a strided view.
std::optional<std::vector<int64_t>> reshape_strides(const Shape &od, const std::vector<int64_t> &os,
                                                    const Shape &nd) {
  std::vector<int64_t> ns(nd.size(), 0);
  if (numel(od) == 0 || od.empty()) {
    int64_t s = 1;
    for (size_t a = nd.size(); a-- > 0;) {
      ns[a] = s;
      s *= nd[a];
    }
    return ns;
  }
  // Walk old dimensions from the innermost, grouping runs that are
  // contiguous with each other; each run must be covered exactly by a run
  // of new dimensions.
  long vd = (long)nd.size() - 1;
  int64_t base = os.back(), run = 1, vrun = 1;
  for (long td = (long)od.size() - 1; td >= 0; td--) {
    run *= od[(size_t)td];
    bool run_ends = td == 0 || (od[(size_t)td - 1] != 1 && os[(size_t)td - 1] != run * base);
    if (!run_ends) continue;
    while (vd >= 0 && (vrun < run || nd[(size_t)vd] == 1)) {
      ns[(size_t)vd] = vrun * base;
      vrun *= nd[(size_t)vd];
      vd--;
    }
    if (vrun != run) return std::nullopt;
    if (td > 0) {
      base = os[(size_t)td - 1];
      run = 1;
      vrun = 1;
    }
  }
  if (vd != -1) return std::nullopt;
  return ns;
}

std::optional<View> try_view(const UOp *n) {
  switch (n->op) {
    case Op::Contiguous:
      return try_view(n->src[0].get());
    case Op::Buffer: {
      View v;
      v.buf = n->buf;
      v.shape = {(int64_t)n->buf->count};
      v.strides = {1};
      return v;
    }
    case Op::Reshape: {
      auto v = try_view(n->src[0].get());
      if (!v) return std::nullopt;
      auto ns = reshape_strides(v->shape, v->strides, n->shape);
      if (!ns) return std::nullopt;
      v->shape = n->shape;
      v->strides = *ns;
      return v;
    }
    case Op::Permute: {
      auto v = try_view(n->src[0].get());
      if (!v) return std::nullopt;
      View o = *v;
      for (size_t i = 0; i < n->arg.size(); i++) {
        o.shape[i] = v->shape[(size_t)n->arg[i]];
        o.strides[i] = v->strides[(size_t)n->arg[i]];
      }
      return o;
    }
    case Op::Expand: {
      auto v = try_view(n->src[0].get());
      if (!v) return std::nullopt;
      for (size_t a = 0; a < n->shape.size(); a++)
        if (v->shape[a] == 1 && n->shape[a] != 1) v->strides[a] = 0;
      v->shape = n->shape;
      return v;
    }
    case Op::Shrink: {
      auto v = try_view(n->src[0].get());
      if (!v) return std::nullopt;
      for (size_t a = 0; a < n->arg.size(); a++) {
        const UOp *s = n->src[a + 1].get();
        if (s->op != Op::Const) return std::nullopt;
        v->offset += (int64_t)s->value * v->strides[a];
      }
      v->shape = n->shape;
      return v;
    }
    default:
      return std::nullopt;
  }
}

namespace {

// Which axes of a node's value vary (used to classify contraction operands):
// bit a of `bits` for axis a; `all` marks every axis (set conservatively for
// an axis past 63, which no contraction operand has).
struct AxisSet {
  size_t rank = 0;
  uint64_t bits = 0;
  bool all = false;
  bool test(size_t a) const { return all || (a < 64 && ((bits >> a) & 1)); }
  void set(size_t a) {
    if (a < 64)
      bits |= uint64_t(1) << a;
    else
      all = true;
  }
  bool any() const { return all || bits != 0; }
};

AxisSet deps(const UOp *n) {
  AxisSet d;
  d.rank = n->has_shape ? n->shape.size() : 0;
  const size_t r = d.rank;
  switch (n->op) {
    case Op::Const:
      return d;
    case Op::Buffer:
      if (r && n->buf->count > 1) d.set(0);
      return d;
    case Op::Reshape: {
      const AxisSet sd = deps(n->src[0].get());
      const Shape &ss = n->src[0]->shape, &ds = n->shape;
      // the non-unit axes of both shapes, paired in order when they agree
      size_t dn[64], sn[64], nd = 0, ns = 0;
      bool same = true;
      for (size_t a = 0; a < ds.size(); a++)
        if (ds[a] != 1) {
          if (nd == 64) { same = false; break; }
          dn[nd++] = a;
        }
      for (size_t a = 0; same && a < ss.size(); a++)
        if (ss[a] != 1) {
          if (ns == 64) { same = false; break; }
          sn[ns++] = a;
        }
      same = same && nd == ns;
      for (size_t i = 0; same && i < nd; i++) same = ds[dn[i]] == ss[sn[i]];
      if (same) {
        for (size_t i = 0; i < nd; i++)
          if (sd.test(sn[i])) d.set(dn[i]);
      } else if (sd.any()) {
        for (size_t a = 0; a < ds.size(); a++)
          if (ds[a] != 1) d.set(a);
      }
      return d;
    }
    case Op::Permute: {
      const AxisSet sd = deps(n->src[0].get());
      for (size_t i = 0; i < r; i++)
        if (sd.test((size_t)n->arg[i])) d.set(i);
      return d;
    }
    case Op::Expand:
    case Op::Shrink: {
      const AxisSet sd = deps(n->src[0].get());
      for (size_t a = 0; a < r && a < sd.rank; a++)
        if (sd.test(a) && n->shape[a] != 1) d.set(a);
      return d;
    }
    case Op::ReduceAxis: {
      const AxisSet sd = deps(n->src[0].get());
      for (size_t a = 0; a < r; a++)
        if (sd.test(a) && std::find(n->arg.begin(), n->arg.end(), (int64_t)a) == n->arg.end())
          d.set(a);
      return d;
    }
    default: {
      for (auto &s : n->src) {
        if (s->op == Op::Const) continue;
        const AxisSet sd = deps(s.get());
        if (sd.rank != r) {
          d.all = true;
          return d;
        }
        d.bits |= sd.bits;
        d.all = d.all || sd.all;
      }
      return d;
    }
  }
}

// ---- program cache and generic launches -----------------------------------
void launch_args(fg_program *prog, bool has_out_slot, const std::vector<KernelInput> &params,
                 const BufferP &out, const DeviceBuffer *written = nullptr,
                 const BufferP &lo_out = nullptr);

// A one-element buffer passed in the slot of a known-zero input (never in
// the slot the kernel writes).
fg_buffer *placeholder_buffer() {
  static fg_buffer *b = nullptr;
  if (!b) check(fg_alloc(device(), FG_F32, 1, &b), "allocate");
  return b;
}

void launch_rendered(const RenderedKernel &rk, const BufferP &out,
                     const DeviceBuffer *written = nullptr, const BufferP &lo_out = nullptr) {
  auto &cache = program_cache();
  fg_program *prog = nullptr;
  auto it = cache.find(rk.source);
  int nargs = (int)rk.params.size() + (rk.has_out_slot ? 1 : 0) + (lo_out ? 1 : 0);
  const uint64_t kid = g_kernel_count++;
  if (it != cache.end()) {
    prog = it->second;
    g_stats.cache_hits++;
    if (debug_level() >= 1) fprintf(stderr, "*** CUDA %4llu  (cached)         arg %2d\n",
                                    (unsigned long long)kid, nargs);
  } else {
    uint32_t grid[3] = {rk.grid, 1, 1}, block[3] = {rk.block, 1, 1};
    check(fg_compile(device(), rk.source.c_str(), "fg_kernel", nargs, grid, block, &prog),
          "compile");
    cache.emplace(rk.source, prog);
    g_stats.compiled++;
    if (debug_level() >= 4) fprintf(stderr, "%s\n", rk.source.c_str());
    // src/tensor.rs:870-874: "(compiled)" from DEBUG=2 on
    if (debug_level() >= 1)
      fprintf(stderr, "*** CUDA %4llu  kernel_%-9llu arg %2d%s\n", (unsigned long long)kid,
              (unsigned long long)kid, nargs, debug_level() >= 2 ? "  (compiled)" : "");
  }
  g_last_source = rk.source;
  launch_args(prog, rk.has_out_slot, rk.params, out, written, lo_out);
}

void launch_args(fg_program *prog, bool has_out_slot, const std::vector<KernelInput> &params,
                 const BufferP &out, const DeviceBuffer *written, const BufferP &lo_out) {
  const int nargs = (int)params.size() + (has_out_slot ? 1 : 0) + (lo_out ? 1 : 0);
  std::vector<fg_kernel_arg> args;
  args.reserve((size_t)nargs);
  if (has_out_slot) {
    out->ensure_allocated();
    fg_kernel_arg a{};
    a.kind = FG_ARG_BUFFER;
    a.v.buffer = out->h;
    args.push_back(a);
  }
  for (const KernelInput &in : params) {
    fg_kernel_arg a{};
    switch (in.kind) {
      case KernelInput::Buffer:
        a.kind = FG_ARG_BUFFER;
        if (in.buffer->known_zero() && !in.buffer->is_allocated() && in.buffer.get() != written) {
          a.v.buffer = placeholder_buffer();  // the kernel never reads it
        } else {
          in.buffer->ensure_allocated();
          a.v.buffer = in.buffer->h;
        }
        break;
      case KernelInput::I32:
        a.kind = FG_ARG_I32;
        a.v.i32 = (int32_t)in.i;
        break;
      case KernelInput::F32:
        a.kind = FG_ARG_F32;
        a.v.f32 = (float)in.f;
        break;
      case KernelInput::Bool:
        a.kind = FG_ARG_BOOL;
        a.v.b = (uint8_t)in.i;
        break;
    }
    args.push_back(a);
  }
  if (lo_out) {  // the residual output of a staging kernel (RenderSpec::with_lo)
    lo_out->ensure_allocated();
    fg_kernel_arg a{};
    a.kind = FG_ARG_BUFFER;
    a.v.buffer = lo_out->h;
    args.push_back(a);
  }
  {
    ExecTimer timer;
    check(fg_execute(prog, args.data(), nargs), "execute");
  }
  g_stats.rendered++;
}

// Structural key of a render request: everything the rendered source
// depends on (ops, dtypes, shapes, args, literals, reduce ops, the graph's
// shape, buffer slots and Shrink parameter slots, the domain and the store),
// but not which buffers fill the slots.  Encoding it costs a walk of the
// expression; rendering costs ~60 us per kernel, so steady-state steps look
// programs up by this key and render only on a miss.
// Words collected in a vector (an inlined push_back each) and hashed as
// they are added; the vector itself is the map key (moved in, not copied).
struct KeyBuf {
  std::vector<int64_t> w;
  uint64_t h = 1469598103934665603ULL;
  void put(int64_t v) {
    w.push_back(v);
    h = (h ^ (uint64_t)v) * 1099511628211ULL;
  }
  void put_str(const std::string &t) {
    put((int64_t)t.size());
    for (size_t i = 0; i < t.size(); i += 8) {
      int64_t v = 0;
      std::memcpy(&v, t.data() + i, std::min<size_t>(8, t.size() - i));
      put(v);
    }
  }
  bool operator==(const KeyBuf &o) const { return h == o.h && w == o.w; }
};

struct KeyBufHash {
  size_t operator()(const KeyBuf &k) const { return (size_t)(k.h ^ (k.h >> 29)); }
};

KeyBuf spec_key(const RenderSpec &spec, const ParamSlots &ps,
                     const std::vector<const UOp *> &order) {
  KeyBuf k;
  k.w.reserve(16 + order.size() * 12);
  k.put((int64_t)spec.store);
  k.put(spec.pitch);
  k.put((int64_t)spec.out_dtype);
  k.put(spec.unroll);
  k.put((int64_t)spec.coop);
  k.put(spec.with_lo ? 1 : 0);
  k.put((int64_t)spec.domain.size());
  for (int64_t d : spec.domain) k.put(d);
  k.put((int64_t)spec.value_ctx.size());
  for (auto &c : spec.value_ctx) k.put_str(c);
  int64_t next = 0;
  for (auto &n : order) {
    n->topo_pos = next++;  // sources come first in `order`
    k.put((int64_t)n->op);
    k.put((int64_t)n->dtype);
    k.put((int64_t)n->reduce_op);
    int64_t vb;
    std::memcpy(&vb, &n->value, sizeof(vb));
    k.put(vb);
    k.put((int64_t)n->shape.size());
    for (int64_t d : n->shape) k.put(d);
    k.put((int64_t)n->arg.size());
    for (int64_t a : n->arg) k.put(a);
    k.put((int64_t)n->src.size());
    for (auto &src : n->src) k.put(src->topo_pos);
    if (n->op == Op::Buffer) {
      k.put(ps.buffer_slot.at(n->buf.get()));
      k.put((int64_t)n->buf->count);
      k.put(n->buf->known_zero() ? 1 : 0);
    } else if (n->op == Op::Shrink) {
      for (int sl : ps.shrink_slots.at(n)) k.put(sl);
    }
  }
  k.put(spec.store == RenderSpec::View ? 1 : 0);
  return k;
}

struct CachedKernel {
  fg_program *prog;
  bool has_out_slot;
};

std::unordered_map<KeyBuf, CachedKernel, KeyBufHash> &spec_cache() {
  static std::unordered_map<KeyBuf, CachedKernel, KeyBufHash> c;
  return c;
}

// Render (on a miss) and launch one generic kernel.
void launch_spec(const RenderSpec &spec, const BufferP &out, const BufferP &lo_out = nullptr) {
  const bool view = spec.store == RenderSpec::View;
  const DeviceBuffer *written = nullptr;  // an in-place store's destination
  if (view) {
    const UOp *d = spec.dest.get();
    while (d->op != Op::Buffer && !d->src.empty()) d = d->src[0].get();
    if (d->op == Op::Buffer) written = d->buf.get();
  }
  // one walk of the kernel's graph gives both its parameter slots and its
  // structural key
  const UOpP root = view ? make_store(spec.dest, spec.value) : spec.value;
  const std::vector<const UOp *> order = toposort_nodes(root.get());
  ParamSlots ps = collect_params_from(order, view ? 0 : 1);
  KeyBuf key = spec_key(spec, ps, order);
  auto &cache = spec_cache();
  auto it = cache.find(key);
  if (it == cache.end()) {
    RenderedKernel rk = render_kernel(spec);
    launch_rendered(rk, out, written, lo_out);
    auto pit = program_cache().find(rk.source);
    if (pit != program_cache().end())
      cache.emplace(std::move(key), CachedKernel{pit->second, rk.has_out_slot});
    return;
  }
  g_stats.cache_hits++;
  if (debug_level() >= 1)
    fprintf(stderr, "*** CUDA %4llu  (cached)         arg %2d\n",
            (unsigned long long)g_kernel_count++,
            (int)ps.inputs.size() + (it->second.has_out_slot ? 1 : 0));
  launch_args(it->second.prog, it->second.has_out_slot, ps.inputs, out, written, lo_out);
}

BufferP temp_buffer(DType dt, int64_t n) {
  auto b = std::make_shared<DeviceBuffer>(dt, (size_t)n);
  b->ensure_allocated();
  return b;
}

// ---- contraction matching ---------------------------------------------------
struct Contraction {
  const UOp *reduce;
  UOpP a, b;           // operand expressions over the 3-D domain
  size_t ai, bj, r;    // row axis (A), column axis (B), reduced axis
  int64_t M, N, K;
};

constexpr int64_t kGemmMinWork = int64_t(1) << 22;
constexpr int64_t kHandReduceMin = int64_t(1) << 20;

std::optional<Contraction> match_contraction(const UOp *n) {
  if (n->op != Op::ReduceAxis || n->reduce_op != Op::Add || n->dtype != DType::F32) return {};
  if (n->arg.size() != 1) return {};
  const UOp *m = n->src[0].get();
  if (m->op != Op::Mul || !m->has_shape || m->shape.size() != 3) return {};
  const size_t r = (size_t)n->arg[0];
  size_t i = r == 0 ? 1 : 0, j = r == 2 ? 1 : 2;
  const Shape &s = m->shape;
  if (s[i] * s[j] * s[r] < kGemmMinWork) return {};
  // Shorter than one 32-deep k-block, a contraction is an HBM pass over its
  // output (the 10-class layer's dX: K = 10); the tensor-core tile pipeline
  // only adds overhead there, so it is rendered (~7x faster measured).
  if (s[r] < 32) return {};
  const AxisSet dp = deps(m->src[0].get()), dq = deps(m->src[1].get());
  if (dp.rank != 3 || dq.rank != 3) return {};
  Contraction c;
  c.reduce = n;
  c.r = r;
  if (!dp.test(j) && !dq.test(i) && (dp.test(i) || dq.test(j))) {
    c.a = m->src[0];
    c.b = m->src[1];
    c.ai = i;
    c.bj = j;
  } else if (!dq.test(j) && !dp.test(i) && (dq.test(i) || dp.test(j))) {
    c.a = m->src[1];
    c.b = m->src[0];
    c.ai = i;
    c.bj = j;
  } else {
    return {};
  }
  c.M = s[i];
  c.N = s[j];
  c.K = s[r];
  return c;
}

struct Operand {
  BufferP hold;  // staged copy (if any)
  BufferP lo;    // TF32 residual
  const float *ptr = nullptr;
  const float *lo_ptr = nullptr;
  int ld = 0;
  bool mn_major = false;
};

// A staged operand is keyed by the expression and the two domain axes that
// index its rows and columns, so the forward GEMM (the ReLU output as A,
// K-major) and the dW GEMM (the same matrix as B, MN-major) share one copy.
struct StageKey {
  const UOp *x;
  size_t outer_axis, inner_axis;
  int64_t outer, inner;
  bool operator==(const StageKey &o) const {
    return x == o.x && outer_axis == o.outer_axis && inner_axis == o.inner_axis &&
           outer == o.outer && inner == o.inner;
  }
};
struct StageKeyHash {
  size_t operator()(const StageKey &k) const {
    return std::hash<const void *>()(k.x) ^ (size_t)(k.outer * 1000003 + k.inner * 31) ^
           (k.outer_axis << 7) ^ (k.inner_axis << 11);
  }
};
struct Staged {
  BufferP hold, lo;
  int64_t ld = 0;
  std::vector<std::pair<BufferP, uint64_t>> reads;  // buffers read, at their versions
  UOpP keep;
  bool valid() const {
    for (auto &r : reads)
      if (r.first->version != r.second) return false;
    return true;
  }
};
std::unordered_map<StageKey, Staged, StageKeyHash> &staged_cache() {
  static std::unordered_map<StageKey, Staged, StageKeyHash> c;
  return c;
}

Operand prepare_operand(const UOpP &x, size_t row_axis, size_t red_axis, size_t bcast_axis,
                        int64_t rows, int64_t K) {
  Operand op;
  auto v = x->dtype == DType::F32 ? try_view(x.get()) : std::nullopt;
  if (v && (v->strides[bcast_axis] == 0 || v->shape[bcast_axis] == 1) &&
      (v->offset * 4) % 16 == 0) {
    const int64_t sr = v->strides[row_axis], sk = v->strides[red_axis];
    const int64_t extent = (rows - 1) * sr + (K - 1) * sk + 1;
    bool kmaj = (sk == 1 || K == 1) && sr % 4 == 0 && sr >= K && sr <= INT32_MAX;
    bool mnmaj = !kmaj && (sr == 1 || rows == 1) && sk % 4 == 0 && sk >= rows && sk <= INT32_MAX;
    if (rows == 1 && (sk == 1 || K == 1)) {
      kmaj = true;
    }
    if (kmaj || mnmaj) {
      op.ptr = fptr(v->buf, v->offset);
      op.ld = kmaj ? (int)std::max<int64_t>(sr, (K + 3) / 4 * 4) : (int)sk;
      if (kmaj && rows == 1) op.ld = (int)((K + 3) / 4 * 4);
      op.mn_major = mnmaj;
      (void)extent;
      // The residual of the whole buffer, made once per version of its
      // contents (a weight read by the forward and the dX GEMM, an input
      // read by the forward and the dW GEMM).
      DeviceBuffer &b = *v->buf;
      if (!b.lo || b.lo_version != b.version) {
        b.lo = temp_buffer(DType::F32, (int64_t)b.count);
        check(fg_split_lo(fptr(v->buf), fptr(b.lo), b.count, stream()), "split_lo");
        b.lo_version = b.version;
      }
      op.lo = b.lo;
      op.lo_ptr = fptr(b.lo, v->offset);
      return op;
    }
  }
  // A lazy operand (the ReLU output) is staged once per realize, in a copy
  // whose contiguous axis is the operand's higher-numbered domain axis (its
  // natural row-major order, so the staging pass reads coalesced): K-major
  // out[row][k] when the reduced axis is inner, else MN-major out[k][row].
  // The broadcast axis is read at 0.  The staging kernel writes the TF32
  // residual in the same pass.
  const bool kmaj = red_axis > row_axis;
  const size_t outer_axis = kmaj ? row_axis : red_axis, inner_axis = kmaj ? red_axis : row_axis;
  const int64_t outer = kmaj ? rows : K, inner = kmaj ? K : rows;
  StageKey key{x.get(), outer_axis, inner_axis, outer, inner};
  auto &stage = staged_cache();
  auto sit = stage.find(key);
  if (sit == stage.end() || !sit->second.valid()) {
    Staged st;
    st.ld = (inner + 3) / 4 * 4;
    st.hold = temp_buffer(DType::F32, outer * st.ld);
    st.lo = temp_buffer(DType::F32, outer * st.ld);
    RenderSpec spec;
    spec.value = x;
    spec.domain = {outer, inner};
    spec.value_ctx.assign(3, "0");
    spec.value_ctx[outer_axis] = "c0";
    spec.value_ctx[inner_axis] = "c1";
    // When x only broadcasts a 2-D expression y whose axes are the copy's
    // rows and columns in order (matmul's reshape + expand of the ReLU
    // output), the copy is y itself: render y over its own shape, so its
    // loads see y's layout (128-bit accesses where it is contiguous).
    {
      const UOp *y = x.get();
      while (y->op == Op::Expand || y->op == Op::Reshape) y = y->src[0].get();
      const UOp *r = x->op == Op::Expand ? x->src[0].get() : nullptr;
      if (r && r->op == Op::Reshape && r->src[0].get() == y && y->shape.size() == 2 &&
          y->shape[0] == outer && y->shape[1] == inner) {
        std::vector<size_t> live;  // axes of the reshape that carry y's axes
        for (size_t a = 0; a < r->shape.size(); a++)
          if (r->shape[a] != 1) live.push_back(a);
        if (live.size() == 2 && live[0] == outer_axis && live[1] == inner_axis && outer > 1 &&
            inner > 1) {
          spec.value = r->src[0];
          spec.value_ctx.clear();
        }
      }
    }
    spec.store = RenderSpec::Pitched;
    spec.pitch = st.ld;
    spec.out_dtype = DType::F32;
    spec.unroll = 4;
    spec.with_lo = true;
    launch_spec(spec, st.hold, st.lo);
    st.keep = x;
    for (const UOp *n : toposort_nodes(x.get()))
      if (n->op == Op::Buffer) st.reads.emplace_back(n->buf, n->buf->version);
    sit = stage.insert_or_assign(key, std::move(st)).first;
  }
  const Staged &st = sit->second;
  op.hold = st.hold;
  op.lo = st.lo;
  op.ptr = fptr(st.hold);
  op.lo_ptr = fptr(st.lo);
  op.ld = (int)st.ld;
  op.mn_major = !kmaj;
  return op;
}

void run_contraction(const Contraction &c, const UOpP &a, const UOpP &b, const BufferP &out,
                     int epilogue = FG_EPI_NONE, const float *bias = nullptr,
                     const float *mask = nullptr, int ldmask = 0) {
  const size_t bc_a = c.bj, bc_b = c.ai;
  Operand A = prepare_operand(a, c.ai, c.r, bc_a, c.M, c.K);
  Operand B = prepare_operand(b, c.bj, c.r, bc_b, c.N, c.K);
  int flags = (A.mn_major ? FG_GEMM_A_MN_MAJOR : 0) | (B.mn_major ? FG_GEMM_B_MN_MAJOR : 0);
  if (debug_level() >= 1)
    fprintf(stderr, "*** CUDA %4llu  gemm3xtf32 %lldx%lldx%lld%s%s%s\n",
            (unsigned long long)g_kernel_count++, (long long)c.M, (long long)c.N,
            (long long)c.K, A.mn_major ? " A:mn" : "", B.mn_major ? " B:mn" : "",
            epilogue == FG_EPI_BIAS ? " +bias" : epilogue == FG_EPI_RELU_MASK ? " +relu-mask" : "");
  ExecTimer timer;
  check(fg_gemm_3xtf32((int)c.M, (int)c.N, (int)c.K, A.ptr, A.lo_ptr, A.ld, B.ptr, B.lo_ptr, B.ld,
                       fptr(out), nullptr, (int)c.N, flags, epilogue, bias, mask, ldmask,
                       stream()),
        "gemm");
  g_stats.gemm++;
}

// ---- hand-written reductions ------------------------------------------------
struct HandReduce {
  const UOp *reduce;
  View v;
  bool rows;  // reduce over the innermost extent (else over the outer one)
  int64_t outer, extent, inner;
};

std::optional<HandReduce> match_hand_reduce(const UOp *n) {
  if (n->op != Op::ReduceAxis || (n->dtype != DType::F32 && n->dtype != DType::I32)) return {};
  auto v = try_view(n->src[0].get());
  if (!v || numel(v->shape) < kHandReduceMin) return {};
  // The view must be contiguous row-major.
  int64_t s = 1;
  for (size_t a = v->shape.size(); a-- > 0;) {
    if (v->shape[a] != 1 && v->strides[a] != s) return {};
    s *= v->shape[a];
  }
  if ((v->offset * 4) % 16 != 0) return {};
  std::vector<int64_t> axes = n->arg;
  std::sort(axes.begin(), axes.end());
  const Shape &sh = v->shape;
  // Reduced axes (ignoring size-1 ones) must form one contiguous block.
  std::vector<int64_t> red;
  for (int64_t a : axes)
    if (sh[(size_t)a] != 1) red.push_back(a);
  if (red.empty()) return {};
  for (size_t i = 1; i < red.size(); i++)
    if (red[i] != red[i - 1] + 1) return {};
  HandReduce h;
  h.reduce = n;
  h.v = *v;
  h.outer = h.extent = h.inner = 1;
  for (size_t a = 0; a < sh.size(); a++) {
    if ((int64_t)a < red.front())
      h.outer *= sh[a];
    else if ((int64_t)a <= red.back())
      h.extent *= sh[a];
    else
      h.inner *= sh[a];
  }
  if (h.inner == 1) {
    h.rows = true;
  } else if (h.outer == 1) {
    h.rows = false;
  } else {
    return {};
  }
  return h;
}

void run_hand_reduce(const HandReduce &h, const BufferP &out) {
  int op = h.reduce->reduce_op == Op::Add ? FG_REDUCE_SUM : FG_REDUCE_MAX;
  const int dt = h.reduce->dtype == DType::I32 ? FG_I32 : FG_F32;
  // i32 and f32 elements are both 4 bytes
  const float *x = fptr(h.v.buf, h.v.offset);
  float *y = fptr(out);
  if (debug_level() >= 1)
    fprintf(stderr, "*** CUDA %4llu  reduce_%s %lldx%lld\n", (unsigned long long)g_kernel_count++,
            h.rows ? "rows" : "cols", (long long)(h.rows ? h.outer : h.extent),
            (long long)(h.rows ? h.extent : h.inner));
  ExecTimer timer;
  if (h.rows)
    check(fg_reduce_rows(dt, op, x, y, (size_t)h.outer, (size_t)h.extent, stream()),
          "reduce_rows");
  else
    check(fg_reduce_cols(dt, op, x, y, (size_t)h.extent, (size_t)h.inner, stream()),
          "reduce_cols");
  g_stats.hand_reduce++;
}

// Root of an allocating item, looking through a same-size Reshape.
const UOp *root_reduce(const UOpP &value) {
  const UOp *v = value.get();
  while (v->op == Op::Reshape) v = v->src[0].get();
  return v;
}

// ---- fused cross-entropy ------------------------------------------------------
bool contiguous_view(const View &v) {
  int64_t s = 1;
  for (size_t a = v.shape.size(); a-- > 0;) {
    if (v.shape[a] != 1 && v.strides[a] != s) return false;
    s *= v.shape[a];
  }
  return true;
}

// x as contiguous f32 memory: in place when it is a contiguous view of a
// buffer (*view set), else a rendered copy held in *hold.
const float *contiguous_operand(const UOpP &x, BufferP *hold, std::optional<View> *view) {
  auto v = try_view(x.get());
  if (v && contiguous_view(*v)) {
    *view = v;
    return fptr(v->buf, v->offset);
  }
  *hold = temp_buffer(DType::F32, numel(x->shape));
  RenderSpec spec;
  spec.value = x;
  spec.domain = x->shape;
  spec.out_dtype = DType::F32;
  spec.unroll = 4;
  choose_thread_mapping(spec);
  launch_spec(spec, *hold);
  return fptr(*hold);
}

// Losses computed by an XentGrad pass, kept until the XentLoss of the same
// logits and targets (same buffers, offsets and contents versions) is
// realized -- in a training step backward's pass runs in Sgd::step's realize
// and loss.to_vec() comes after it.
struct XentDone {
  BufferP logits, targets;
  int64_t loff, toff;
  uint64_t lver, tver;
  BufferP loss;
};
std::vector<XentDone> &xent_done() {
  static std::vector<XentDone> v;
  return v;
}

void run_xent(const ScheduleItem &item, const UOp *node) {
  const UOpP &lg = node->src[0], &tg = node->src[1];
  const Shape &ls = lg->shape;
  const size_t rows = ls.size() == 2 ? (size_t)ls[0] : 1, cols = (size_t)ls.back();
  BufferP hl, ht;
  std::optional<View> vl, vt;
  const float *L = contiguous_operand(lg, &hl, &vl);
  const float *T = contiguous_operand(tg, &ht, &vt);
  auto &done = xent_done();
  const bool keyed = vl && vt;
  auto same = [&](const XentDone &d) {
    return d.logits == vl->buf && d.targets == vt->buf && d.loff == vl->offset &&
           d.toff == vt->offset && d.lver == vl->buf->version && d.tver == vt->buf->version;
  };
  if (node->op == Op::XentLoss && keyed) {
    for (auto it = done.begin(); it != done.end(); ++it) {
      if (!same(*it)) continue;
      // the loss is already on the device: hand its storage to this item
      std::swap(item.output->h, it->loss->h);
      done.erase(it);
      g_stats.xent_reused++;
      if (debug_level() >= 1)
        fprintf(stderr, "*** CUDA %4llu  xent loss (from the gradient pass)\n",
                (unsigned long long)g_kernel_count++);
      return;
    }
  }
  if (debug_level() >= 1)
    fprintf(stderr, "*** CUDA %4llu  xent_fwd_bwd %zux%zu%s\n", (unsigned long long)g_kernel_count++,
            rows, cols, node->op == Op::XentGrad ? " +grad" : "");
  ExecTimer timer;
  if (node->op == Op::XentLoss) {
    check(fg_xent_fwd_bwd(L, T, rows, cols, fptr(item.output), nullptr, 1.0f, stream()), "xent");
  } else {
    BufferP loss = temp_buffer(DType::F32, 1);
    check(fg_xent_fwd_bwd(L, T, rows, cols, fptr(loss), fptr(item.output), 1.0f, stream()),
          "xent");
    if (keyed) {
      done.push_back({vl->buf, vt->buf, vl->offset, vt->offset, vl->buf->version,
                      vt->buf->version, loss});
      // bounded: an entry keeps its logits and targets alive until its loss
      // is read or it is evicted
      if (done.size() > 4) done.erase(done.begin());
    }
  }
  g_stats.xent++;
}

// ---- fused SGD store ------------------------------------------------------------
// Sgd::step's store (src/optim.rs:60-71): P <- P + (-(G * lr)) with P the
// destination view, G a contiguous view (a routed contraction's result or a
// realized gradient) and lr a Tensor::scalar buffer, runs on fg_sgd -- the
// same single-rounded ops -- which also rewrites the TF32 residual that the
// parameter keeps as a GEMM operand.  Returns false when the store does not
// have that form; *wrote_lo tells the caller the residual is current.
bool try_sgd(const ScheduleItem &item, const UOpP &value, bool *wrote_lo) {
  *wrote_lo = false;
  const UOp *v = value.get();
  if (v->op != Op::Add || v->dtype != DType::F32 || v->src[0] != item.store_dest) return false;
  const UOp *ng = v->src[1].get();
  if (ng->op != Op::Neg) return false;
  const UOp *m = ng->src[0].get();
  if (m->op != Op::Mul) return false;
  auto scalar_of = [](const UOp *x) -> const DeviceBuffer * {
    while (x->op == Op::Expand || x->op == Op::Reshape) x = x->src[0].get();
    if (x->op != Op::Buffer) return nullptr;
    const DeviceBuffer *b = x->buf.get();
    return b->count == 1 && b->has_host_scalar && b->version == 0 ? b : nullptr;
  };
  const DeviceBuffer *lr = scalar_of(m->src[1].get());
  const UOp *g = m->src[0].get();
  if (!lr) {
    lr = scalar_of(m->src[0].get());
    g = m->src[1].get();
  }
  if (!lr) return false;
  auto pv = try_view(item.store_dest.get());
  auto gv = try_view(g);
  if (!pv || !gv || !contiguous_view(*pv) || !contiguous_view(*gv)) return false;
  if (pv->buf->dtype != DType::F32 || gv->buf->dtype != DType::F32) return false;
  if (pv->buf.get() == gv->buf.get()) return false;
  const int64_t n = numel(pv->shape);
  if (n != numel(gv->shape)) return false;
  DeviceBuffer &pb = *pv->buf;
  float *lo = nullptr;
  if (pv->offset == 0 && n == (int64_t)pb.count && pb.lo && pb.lo->count == pb.count)
    lo = fptr(pb.lo);
  if (debug_level() >= 1)
    fprintf(stderr, "*** CUDA %4llu  sgd %lld%s\n", (unsigned long long)g_kernel_count++,
            (long long)n, lo ? " +lo" : "");
  ExecTimer timer;
  check(fg_sgd(fptr(pv->buf, pv->offset), fptr(gv->buf, gv->offset), (size_t)n, lr->host_scalar, lo,
               stream()),
        "sgd");
  g_stats.sgd++;
  *wrote_lo = lo != nullptr;
  return true;
}

// Linear::forward's x.matmul(W^T).add(bias) (src/nn.rs:97-104): an item
// whose value is a routed contraction [M,N] plus a row-broadcast bias vector
// runs as one GEMM with the bias epilogue (acc + bias[n], one rounding, as
// the rendered add), writing the item's output directly.
bool try_gemm_bias(const ScheduleItem &item) {
  const UOp *v = item.value.get();
  if (v->op != Op::Add || v->dtype != DType::F32 || v->shape.size() != 2) return false;
  for (int side = 0; side < 2; side++) {
    const UOp *x = v->src[(size_t)side].get(), *bsrc = v->src[(size_t)(1 - side)].get();
    if (x->op != Op::Reshape) continue;
    auto c = match_contraction(x->src[0].get());
    if (!c || c->r != 2 || c->ai != 0 || c->bj != 1) continue;
    auto bv = try_view(bsrc);
    if (!bv || bv->buf->dtype != DType::F32 || bv->strides.size() != 2 || bv->shape != v->shape)
      continue;
    if ((bv->shape[0] != 1 && bv->strides[0] != 0) || (bv->shape[1] != 1 && bv->strides[1] != 1))
      continue;
    if (bv->buf->known_zero() && !bv->buf->is_allocated()) {
      // a never-written zero bias (Linear::new): the plain product
      run_contraction(*c, c->a, c->b, item.output);
    } else {
      run_contraction(*c, c->a, c->b, item.output, FG_EPI_BIAS, fptr(bv->buf, bv->offset));
      g_stats.gemm_bias++;
    }
    return true;
  }
  return false;
}

// ReLU's gradient where(0 < z, dX, 0) (src/gradient.rs:145-153 on
// src/tensor.rs:519-531) over a routed contraction dX [M,N] and a
// materialised z: one GEMM with the ReLU-mask epilogue
// (C = z > 0 ? acc : 0, the same selection), writing the item's output.
bool is_zero_value(const UOp *n) {
  while (n->op == Op::Expand || n->op == Op::Reshape) n = n->src[0].get();
  if (n->op == Op::Const) return n->value == 0.0;
  return n->op == Op::Buffer && n->buf->known_zero();
}

bool try_gemm_relu_mask(const ScheduleItem &item) {
  const UOp *v = item.value.get();
  if (v->op != Op::Where || v->dtype != DType::F32 || v->shape.size() != 2) return false;
  const UOp *cond = v->src[0].get(), *x = v->src[1].get();
  if (cond->op != Op::CmpLt || !is_zero_value(cond->src[0].get()) ||
      !is_zero_value(v->src[2].get()) || x->op != Op::Reshape)
    return false;
  auto zv = try_view(cond->src[1].get());
  if (!zv || zv->buf->dtype != DType::F32 || !contiguous_view(*zv) || zv->shape != v->shape ||
      (zv->offset * 4) % 16 != 0 || v->shape[1] % 4 != 0)
    return false;
  auto c = match_contraction(x->src[0].get());
  if (!c || c->ai > c->bj) return false;
  // output [M, N] row-major: rows along the contraction's A axis
  if (c->M != v->shape[0] || c->N != v->shape[1]) return false;
  run_contraction(*c, c->a, c->b, item.output, FG_EPI_RELU_MASK, nullptr,
                  fptr(zv->buf, zv->offset), (int)v->shape[1]);
  g_stats.gemm_mask++;
  return true;
}

const UOp *xent_root(const UOpP &value) {
  const UOp *v = value.get();
  while (v->op == Op::Reshape) v = v->src[0].get();
  return v->op == Op::XentLoss || v->op == Op::XentGrad ? v : nullptr;
}

}  // namespace

RoutePlan plan_route(const ScheduleItem &item) {
  RoutePlan p;
  p.route = "rendered";
  if (!item.store_dest && xent_root(item.value)) {
    p.route = "xent";
    return p;
  }
  if (exact_mode()) return p;
  {
    const UOp *v = item.value.get();
    if (!item.store_dest && v->op == Op::Add && v->shape.size() == 2)
      for (auto &sv : v->src)
        if (sv->op == Op::Reshape)
          if (auto c = match_contraction(sv->src[0].get()))
            if (c->r == 2 && c->ai == 0 && c->bj == 1 && try_view(v->src[&sv == &v->src[0] ? 1 : 0].get())) {
              char buf[128];
              snprintf(buf, sizeof(buf), "gemm %lldx%lldx%lld +bias", (long long)c->M,
                       (long long)c->N, (long long)c->K);
              p.route = "gemm";
              p.steps.push_back(buf);
              return p;
            }
  }
  bool root_handled = false;
  for (const UOp *n : toposort_nodes(item.value.get())) {
    if (auto c = match_contraction(n)) {
      char buf[128];
      snprintf(buf, sizeof(buf), "gemm %lldx%lldx%lld", (long long)c->M, (long long)c->N,
               (long long)c->K);
      p.steps.push_back(buf);
      if (!item.store_dest && root_reduce(item.value) == n) root_handled = true;
    } else if (auto h = match_hand_reduce(n)) {
      p.steps.push_back(h->rows ? "reduce_rows" : "reduce_cols");
      if (!item.store_dest && root_reduce(item.value) == n) root_handled = true;
    }
  }
  if (root_handled && p.steps.size() == 1)
    p.route = p.steps[0].substr(0, p.steps[0].find(' '));
  else if (!p.steps.empty())
    p.route = "mixed";
  return p;
}

std::string render_item_source(const ScheduleItem &item) {
  if (!item.store_dest && xent_root(item.value))
    return "// fused cross-entropy: fg_xent_fwd_bwd (no rendered source)\n";
  RenderSpec spec;
  spec.value = item.value;
  spec.domain = item.out_shape;
  spec.unroll = 4;
  if (item.store_dest) {
    spec.store = RenderSpec::View;
    spec.dest = item.store_dest;
  } else {
    spec.out_dtype = item.value->dtype;
  }
  choose_thread_mapping(spec);
  return render_kernel(spec).source;
}

void end_realize() { staged_cache().clear(); }

void all_reduce_mean_buffer(const BufferP &buf, fg_comm *comm) {
  if (buf->dtype != DType::F32) throw Panic("all_reduce_mean: f32 buffers only");
  if (debug_level() >= 1)
    fprintf(stderr, "*** CUDA %4llu  all-reduce mean %zu\n", (unsigned long long)g_kernel_count++,
            buf->count);
  check(fg_allreduce_mean_f32(comm, fptr(buf), buf->count, stream()), "all-reduce");
  buf->version++;
}

void run_item(const ScheduleItem &item) {
  g_stats.kernels++;
  // DEBUG >= 3 dumps each kernel's graph (src/tensor.rs:855-869,900-904);
  // the proto-kernel as scheduled is the one stage this front end has
  if (debug_level() >= 3)
    fprintf(stderr, "\u2501\u2501\u2501 kernel_%llu [schedule] \u2501\u2501\u2501\n%s\n",
            (unsigned long long)g_kernel_count,
            dump(item.store_dest ? make_store(item.store_dest, item.value) : item.value).c_str());
  if (!item.store_dest) {
    if (const UOp *x = xent_root(item.value)) {
      run_xent(item, x);
      return;
    }
  }
  if (!item.store_dest && !exact_mode() && (try_gemm_bias(item) || try_gemm_relu_mask(item)))
    return;
  UOpP value = item.value;
  if (!exact_mode()) {
    // Extract routed reductions bottom-up, substituting each result.
    std::unordered_map<const UOp *, UOpP> repl;
    std::vector<UOpP> hold;
    for (const UOp *n : toposort_nodes(item.value.get())) {
      if (n->op != Op::ReduceAxis) continue;
      auto c = match_contraction(n);
      std::optional<HandReduce> h;
      if (!c) h = match_hand_reduce(n);
      if (!c && !h) continue;
      const bool is_root = !item.store_dest && root_reduce(item.value) == n;
      BufferP out = is_root ? item.output : temp_buffer(n->dtype, numel(n->shape));
      if (c) {
        UOpP a = c->a, b = c->b;
        if (!repl.empty()) {
          Rewriter rewrite(repl);
          a = rewrite(c->a);
          b = rewrite(c->b);
        }
        run_contraction(*c, a, b, out);
      } else {
        run_hand_reduce(*h, out);
      }
      if (is_root) return;
      UOpP sub = make_reshape(make_buffer(out), n->shape);
      hold.push_back(sub);
      repl[n] = sub;
    }
    if (!repl.empty()) {
      value = Rewriter(repl)(item.value);
    }
  }
  bool wrote_lo = false;
  if (!(item.store_dest && !exact_mode() && try_sgd(item, value, &wrote_lo))) {
    RenderSpec spec;
    spec.value = value;
    spec.domain = item.out_shape;
    spec.unroll = 4;
    if (item.store_dest) {
      spec.store = RenderSpec::View;
      spec.dest = item.store_dest;
    } else {
      spec.out_dtype = item.value->dtype;
    }
    choose_thread_mapping(spec);
    launch_spec(spec, item.output);
  }
  if (item.store_dest) {
    // the destination's contents changed: cached residuals and staged
    // operands that read it are stale (unless the SGD pass rewrote the
    // residual with the new contents)
    const UOp *d = item.store_dest.get();
    while (d->op != Op::Buffer && !d->src.empty()) d = d->src[0].get();
    if (d->op == Op::Buffer) {
      d->buf->version++;
      if (wrote_lo) d->buf->lo_version = d->buf->version;
    }
  }
}

}  // namespace ferro
