// hostdev.cpp -- TEST INFRASTRUCTURE ONLY: a host implementation of the
// device part of include/ferro_cuda.h, so the C++ front end can be linked
// against it and run on a machine without a GPU.
//
// fg_compile takes the CUDA C the front end renders, compiles it with g++
// (-ffp-contract=off, one rounding per op like the reference's clang C)
// behind a small prelude that maps the CUDA spellings to C++ (blockIdx /
// threadIdx become globals the launcher sets, __fadd_rn is a float add,
// exp2((double)x) is libm's), and fg_execute runs the kernel over its grid.
// That makes an independent CPU execution of the front end's schedule and
// rendered arithmetic -- a second oracle for exact mode (FG_FRONT_EXACT=1).
// The building blocks the default mode routes to (3xTF32 GEMM, HBM
// reductions, TF32 split) are restated on the CPU from their C-ABI
// contracts, so the front end's routing (contraction matching, operand
// layouts, staged operands, residual caching) runs here as well, held to
// tolerance.  Nothing in the product loads this library.
#include <dlfcn.h>
#include <stdarg.h>
#include <unistd.h>

#include <cmath>
#include <cstdint>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <fstream>
#include <functional>
#include <regex>
#include <string>
#include <vector>

// FG_HOSTDEV_NOEXEC: every compute entry point returns before computing, so
// the front end's host work (graph building, scheduling, routing, launch
// preparation) can be timed alone (tests/hostdev/host_time.py).
#ifdef FG_HOSTDEV_NOEXEC
#define FG_HOSTDEV_SKIP_COMPUTE() return FG_OK
#else
#define FG_HOSTDEV_SKIP_COMPUTE() (void)0
#endif

#include "ferro_cuda.h"

namespace fg {
static thread_local std::string g_err;
int set_error(int code, const char *fmt, ...) {
  char buf[4096];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  g_err = buf;
  return code;
}
}  // namespace fg

struct fg_device {
  int ordinal;
};
struct fg_buffer {
  void *p;
  int dtype;
  size_t numel;
};
struct fg_program {
  std::string source;
  void *so;
  void (*launch)(void **args, unsigned grid, unsigned block);
  int num_args;
  unsigned grid, block;
};

static size_t esize(int dt) { return dt == FG_BOOL ? 1 : 4; }

// Prelude that lets the rendered CUDA C compile as host C++.
static const char *kPrelude = R"(
#include <barrier>
#include <cmath>
#include <cstring>
#include <memory>
#include <thread>
#include <vector>
struct fg_dim3 { unsigned x, y, z; };
static thread_local fg_dim3 blockIdx, threadIdx;
#define __global__
#define __launch_bounds__(x)
#define __restrict__ __restrict
#define __shared__ static
struct float4 { float x, y, z, w; };
struct int4 { int x, y, z, w; };
struct uchar4 { unsigned char x, y, z, w; };
static inline float4 make_float4(float a, float b, float c, float d) { return {a, b, c, d}; }
static inline int4 make_int4(int a, int b, int c, int d) { return {a, b, c, d}; }
static inline uchar4 make_uchar4(unsigned char a, unsigned char b, unsigned char c,
                                 unsigned char d) { return {a, b, c, d}; }
// Cooperative kernels (warp shuffles, __syncthreads) run with one host
// thread per CUDA thread of a block: a barrier per warp and one per block.
static std::unique_ptr<std::barrier<>> fg_block_bar;
static std::vector<std::unique_ptr<std::barrier<>>> fg_warp_bar;
static double fg_xch[1024];
static inline void __syncthreads() { fg_block_bar->arrive_and_wait(); }
template <class T>
static inline T __shfl_xor_sync(unsigned, T v, int off) {
  const unsigned t = threadIdx.x;
  std::barrier<> &b = *fg_warp_bar[t >> 5];
  std::memcpy(&fg_xch[t], &v, sizeof(T));
  b.arrive_and_wait();
  T r;
  std::memcpy(&r, &fg_xch[t ^ (unsigned)off], sizeof(T));
  b.arrive_and_wait();
  return r;
}
static inline float __fadd_rn(float a, float b) { return a + b; }
static inline float __fmul_rn(float a, float b) { return a * b; }
static inline float __frcp_rn(float a) { return 1.0f / a; }
static inline float __fsqrt_rn(float a) { return std::sqrt(a); }
static inline float __int_as_float(int i) { float f; std::memcpy(&f, &i, 4); return f; }
static inline float __uint_as_float(unsigned i) { float f; std::memcpy(&f, &i, 4); return f; }
static inline unsigned __float_as_uint(float f) { unsigned i; std::memcpy(&i, &f, 4); return i; }
static inline float __fsub_rn(float a, float b) { return a - b; }
using std::exp2;
using std::log2;
)";

extern "C" {

const char *fg_last_error(void) { return fg::g_err.c_str(); }

int fg_device_open(int ordinal, fg_device **out) {
  *out = new fg_device{ordinal};
  return FG_OK;
}
int fg_device_close(fg_device *dev) {
  delete dev;
  return FG_OK;
}
int fg_device_stream(fg_device *, void **stream) {
  *stream = nullptr;
  return FG_OK;
}
int fg_device_sync(fg_device *) { return FG_OK; }

// Every allocation carries a guard band after its data; fg_execute checks
// the bands of its buffer arguments after each kernel, so an out-of-bounds
// write by a rendered kernel is reported with the kernel that made it.
constexpr size_t kGuard = 256;
constexpr unsigned char kGuardByte = 0xA7;

int fg_alloc(fg_device *, int dtype, size_t numel, fg_buffer **out) {
  void *p = nullptr;
  if (numel) {
    p = calloc(numel * esize(dtype) + kGuard, 1);
    memset(static_cast<char *>(p) + numel * esize(dtype), kGuardByte, kGuard);
  }
  *out = new fg_buffer{p, dtype, numel};
  return FG_OK;
}
int fg_free(fg_buffer *b) {
  if (b) free(b->p);
  delete b;
  return FG_OK;
}
static bool guard_ok(const fg_buffer *b) {
  if (!b->p) return true;
  const unsigned char *g = static_cast<const unsigned char *>(b->p) + b->numel * esize(b->dtype);
  for (size_t i = 0; i < kGuard; i++)
    if (g[i] != kGuardByte) return false;
  return true;
}
int fg_buffer_info(const fg_buffer *b, void **p, int *dtype, size_t *numel) {
  if (p) *p = b->p;
  if (dtype) *dtype = b->dtype;
  if (numel) *numel = b->numel;
  return FG_OK;
}
int fg_copy_h2d(fg_buffer *b, const void *src, size_t n) {
  if (n != b->numel * esize(b->dtype))
    return fg::set_error(FG_ERR_INVALID, "copy_from_host: expected %zu bytes, got %zu",
                         b->numel * esize(b->dtype), n);
  if (n) memcpy(b->p, src, n);
  return FG_OK;
}
int fg_copy_d2h(const fg_buffer *b, void *dst, size_t n) {
  if (n != b->numel * esize(b->dtype))
    return fg::set_error(FG_ERR_INVALID, "copy_to_host: expected %zu bytes, got %zu",
                         b->numel * esize(b->dtype), n);
  if (n) memcpy(dst, b->p, n);
  return FG_OK;
}

int fg_compile(fg_device *, const char *source, const char *func_name, int num_args,
               const uint32_t grid[3], const uint32_t block[3], fg_program **out) {
  // The launcher needs the parameter types: read them off the signature.
  std::string src(source);
  std::smatch m;
  std::regex sig(std::string(func_name) + R"(\(([^)]*)\))");
  if (!std::regex_search(src, m, sig)) return fg::set_error(FG_ERR_COMPILE, "no signature");
  std::vector<std::string> types;
  std::string params = m[1].str();
  size_t pos = 0;
  while (pos <= params.size()) {
    size_t c = params.find(',', pos);
    std::string p = params.substr(pos, c == std::string::npos ? std::string::npos : c - pos);
    size_t last = p.find_last_of(" *");
    std::string t = p.substr(0, last + 1);
    size_t r = t.find("__restrict__");
    if (r != std::string::npos) t.erase(r, 12);
    types.push_back(t);
    if (c == std::string::npos) break;
    pos = c + 1;
  }
  std::string call = std::string(func_name) + "(";
  for (size_t i = 0; i < types.size(); i++)
    call += (i ? ", " : "") + std::string("*(") + types[i] + "*)a[" + std::to_string(i) + "]";
  call += ");";
  const bool coop = src.find("__syncthreads") != std::string::npos ||
                    src.find("__shfl_xor_sync") != std::string::npos;
  std::string launcher;
  if (!coop) {
    launcher = "\nextern \"C\" void fg_host_launch(void **a, unsigned grid, unsigned block) {\n"
               "  for (unsigned b = 0; b < grid; b++) for (unsigned t = 0; t < block; t++) {\n"
               "    blockIdx.x = b; threadIdx.x = t;\n    " + call + "\n  }\n}\n";
  } else {
    // one host thread per CUDA thread; the block's threads finish block b
    // together (block barrier) before any starts block b + 1
    launcher = "\nextern \"C\" void fg_host_launch(void **a, unsigned grid, unsigned block) {\n"
               "  fg_block_bar.reset(new std::barrier<>(block));\n"
               "  fg_warp_bar.clear();\n"
               "  for (unsigned w = 0; w < (block + 31) / 32; w++)\n"
               "    fg_warp_bar.emplace_back(new std::barrier<>(block - 32 * w < 32 ? block - 32 * w : 32));\n"
               "  std::vector<std::thread> team;\n"
               "  for (unsigned t = 0; t < block; t++) team.emplace_back([=] {\n"
               "    threadIdx.x = t;\n"
               "    for (unsigned b = 0; b < grid; b++) {\n"
               "      blockIdx.x = b;\n      " + call + "\n"
               "      fg_block_bar->arrive_and_wait();\n"
               "    }\n"
               "  });\n"
               "  for (auto &th : team) th.join();\n"
               "}\n";
  }
  // Compiled kernels are cached on disk (FG_HOSTDEV_CACHE) by a hash of the
  // full source; the stored source is compared before reuse.
  const std::string full = std::string(kPrelude) + src + launcher;
  const char *cache_dir = getenv("FG_HOSTDEV_CACHE");
  std::string cached_so, cached_src;
  if (cache_dir && *cache_dir) {
    char name[64];
    snprintf(name, sizeof(name), "/k%016zx", std::hash<std::string>()(full));
    cached_so = std::string(cache_dir) + name + ".so";
    cached_src = std::string(cache_dir) + name + ".cpp";
    std::ifstream cf(cached_src);
    std::string prev((std::istreambuf_iterator<char>(cf)), std::istreambuf_iterator<char>());
    if (prev == full && access(cached_so.c_str(), R_OK) == 0) {
      void *h = dlopen(cached_so.c_str(), RTLD_NOW | RTLD_LOCAL);
      auto fn = h ? (void (*)(void **, unsigned, unsigned))dlsym(h, "fg_host_launch") : nullptr;
      if (fn) {
        *out = new fg_program{src, h, fn, num_args, grid[0] ? grid[0] : 1, block[0] ? block[0] : 1};
        return FG_OK;
      }
    }
  }
  char dir[] = "/tmp/fg_hostdev_XXXXXX";
  if (!mkdtemp(dir)) return fg::set_error(FG_ERR_COMPILE, "mkdtemp failed");
  std::string cpp = std::string(dir) + "/k.cpp", so = std::string(dir) + "/k.so";
  {
    std::ofstream f(cpp);
    f << full;
  }
  std::string cmd = "g++ -O1 -std=c++20 -pthread -shared -fPIC -ffp-contract=off -fno-fast-math -w -o " +
                    so + " " + cpp + " 2>" + std::string(dir) + "/log.txt";
  if (system(cmd.c_str()) != 0) {
    std::ifstream lf(std::string(dir) + "/log.txt");
    std::string log((std::istreambuf_iterator<char>(lf)), std::istreambuf_iterator<char>());
    return fg::set_error(FG_ERR_COMPILE, "g++ failed:\n%s", log.c_str());
  }
  if (!cached_so.empty()) {
    std::string cp = "cp " + so + " " + cached_so + " && cp " + cpp + " " + cached_src;
    if (system(cp.c_str()) != 0) unlink(cached_so.c_str());
  }
  void *h = dlopen(so.c_str(), RTLD_NOW | RTLD_LOCAL);
  unlink(cpp.c_str());
  unlink(so.c_str());
  unlink((std::string(dir) + "/log.txt").c_str());
  rmdir(dir);
  if (!h) return fg::set_error(FG_ERR_COMPILE, "dlopen: %s", dlerror());
  auto fn = (void (*)(void **, unsigned, unsigned))dlsym(h, "fg_host_launch");
  if (!fn) return fg::set_error(FG_ERR_COMPILE, "launcher missing");
  *out = new fg_program{src, h, fn, num_args, grid[0] ? grid[0] : 1, block[0] ? block[0] : 1};
  return FG_OK;
}

int fg_program_free(fg_program *p) {
  if (p) dlclose(p->so);
  delete p;
  return FG_OK;
}

int fg_execute(fg_program *prog, const fg_kernel_arg *args, int nargs) {
  if (nargs != prog->num_args)
    return fg::set_error(FG_ERR_INVALID, "expected %d kernel args, got %d", prog->num_args, nargs);
  std::vector<void *> ptrs(nargs), slots(nargs);
  std::vector<int32_t> ints(nargs);
  std::vector<float> floats(nargs);
  for (int i = 0; i < nargs; i++) {
    switch (args[i].kind) {
      case FG_ARG_BUFFER:
        ptrs[i] = args[i].v.buffer->p;
        slots[i] = &ptrs[i];
        break;
      case FG_ARG_I32:
        ints[i] = args[i].v.i32;
        slots[i] = &ints[i];
        break;
      case FG_ARG_F32:
        floats[i] = args[i].v.f32;
        slots[i] = &floats[i];
        break;
      default:
        ints[i] = args[i].v.b;
        slots[i] = &ints[i];
        break;
    }
  }
#ifndef FG_HOSTDEV_NOEXEC
  prog->launch(slots.data(), prog->grid, prog->block);
#endif
  for (int i = 0; i < nargs; i++)
    if (args[i].kind == FG_ARG_BUFFER && !guard_ok(args[i].v.buffer))
      return fg::set_error(FG_ERR_DEVICE,
                           "kernel wrote past the end of argument %d (%zu elements):\n%s", i,
                           args[i].v.buffer->numel, prog->source.c_str());
  return FG_OK;
}

// The building blocks the front end routes to (tensor-core GEMM, HBM
// reductions, TF32 residual split), on the CPU with the GPU kernels'
// contracts (include/ferro_cuda.h), so the routed (default) mode of the
// front end runs here too.  Sums are taken in double and rounded once: the
// routed mode is held to tolerance against the oracle, not to bits.  The
// GEMM forms the three products of the 3xTF32 split from the truncated
// operands and the residuals the caller passes (as the tensor cores do), so
// a residual that does not belong to its operand shows up here as well.
static float tf32_hi(float v) {
  uint32_t u;
  std::memcpy(&u, &v, 4);
  u &= 0xffffe000u;
  float h;
  std::memcpy(&h, &u, 4);
  return h;
}

int fg_gemm_3xtf32(int M, int N, int K, const float *a, const float *a_lo, int lda, const float *b,
                   const float *b_lo, int ldb, float *c, float *c_lo, int ldc, int flags,
                   int epilogue, const float *bias, const float *mask, int ldmask, void *) {
  FG_HOSTDEV_SKIP_COMPUTE();
  if (M <= 0 || N <= 0 || K <= 0)
    return fg::set_error(FG_ERR_INVALID, "gemm: M, N, K must be positive (got %d, %d, %d)", M, N, K);
  if (!a || !b || !c) return fg::set_error(FG_ERR_INVALID, "gemm: null operand");
  const bool a_mn = flags & FG_GEMM_A_MN_MAJOR, b_mn = flags & FG_GEMM_B_MN_MAJOR;
  const bool one = flags & FG_GEMM_1XTF32;
  if (!one && (!a_lo || !b_lo)) return fg::set_error(FG_ERR_INVALID, "gemm: residuals required");
  auto at = [&](const float *p, int ld, bool mn, int i, int k) {
    return mn ? p[(size_t)k * ld + i] : p[(size_t)i * ld + k];
  };
  for (int m = 0; m < M; m++)
    for (int n = 0; n < N; n++) {
      double acc = 0.0;
      for (int k = 0; k < K; k++) {
        const double ah = tf32_hi(at(a, lda, a_mn, m, k)), bh = tf32_hi(at(b, ldb, b_mn, n, k));
        acc += ah * bh;
        if (!one) acc += ah * (double)at(b_lo, ldb, b_mn, n, k) + (double)at(a_lo, lda, a_mn, m, k) * bh;
      }
      float v = (float)acc;
      switch (epilogue) {
        case FG_EPI_BIAS: v = v + bias[n]; break;
        case FG_EPI_BIAS_RELU: v = v + bias[n]; v = v > 0.f ? v : 0.f; break;
        case FG_EPI_RELU_MASK: v = mask[(size_t)m * ldmask + n] > 0.f ? v : 0.f; break;
        default: break;
      }
      c[(size_t)m * ldc + n] = v;
      if (c_lo) c_lo[(size_t)m * ldc + n] = v - tf32_hi(v);
    }
  return FG_OK;
}

int fg_split_lo(const float *x, float *lo, size_t n, void *) {
  FG_HOSTDEV_SKIP_COMPUTE();
  for (size_t i = 0; i < n; i++) lo[i] = x[i] - tf32_hi(x[i]);
  return FG_OK;
}

}  // extern "C"

template <typename T>
static int host_reduce(int op, const T *x, T *out, size_t outer, size_t extent, size_t inner) {
  // out[o, i] = op over e of x[o, e, i]
  for (size_t o = 0; o < outer; o++)
    for (size_t i = 0; i < inner; i++) {
      const T *p = x + o * extent * inner + i;
      if (op == FG_REDUCE_MAX) {
        T m = p[0];
        for (size_t e = 1; e < extent; e++) m = p[e * inner] > m ? p[e * inner] : m;
        out[o * inner + i] = extent ? m : T(0);
      } else {
        double acc = 0.0;
        for (size_t e = 0; e < extent; e++) acc += (double)p[e * inner];
        out[o * inner + i] = (T)acc;
      }
    }
  return FG_OK;
}

extern "C" {

int fg_reduce_rows(int dtype, int op, const void *x, void *out, size_t rows, size_t cols, void *) {
  FG_HOSTDEV_SKIP_COMPUTE();
  if (dtype == FG_F32)
    return host_reduce(op, (const float *)x, (float *)out, rows, cols, 1);
  if (dtype == FG_I32)
    return host_reduce(op, (const int32_t *)x, (int32_t *)out, rows, cols, 1);
  return fg::set_error(FG_ERR_INVALID, "fg_reduce_rows: dtype must be F32 or I32");
}

int fg_reduce_cols(int dtype, int op, const void *x, void *out, size_t rows, size_t cols, void *) {
  FG_HOSTDEV_SKIP_COMPUTE();
  if (dtype == FG_F32)
    return host_reduce(op, (const float *)x, (float *)out, 1, rows, cols);
  if (dtype == FG_I32)
    return host_reduce(op, (const int32_t *)x, (int32_t *)out, 1, rows, cols);
  return fg::set_error(FG_ERR_INVALID, "fg_reduce_cols: dtype must be F32 or I32");
}

int fg_u8_to_f32_div(const uint8_t *src, float *dst, size_t n, float divisor, void *) {
  for (size_t i = 0; i < n; i++) dst[i] = (float)src[i] / divisor;
  return FG_OK;
}
// The fused cross-entropy and SGD building blocks, restated from their
// C-ABI contracts (include/ferro_cuda.h): the loss is the mean over rows of
// -sum_c t * log_softmax(x) and dx = (softmax(x) * sum_c t - t) / rows *
// grad_scale, each evaluated in double and rounded once (held to the GPU
// tests' tolerance, not bit-exactness); the SGD step is p + (-(g * lr)) with
// one rounding per op, as the reference's store, plus the new residual.
int fg_xent_fwd_bwd(const float *x, const float *t, size_t rows, size_t cols, float *loss,
                    float *dx, float grad_scale, void *) {
  FG_HOSTDEV_SKIP_COMPUTE();
  if (rows == 0 || cols == 0) return fg::set_error(FG_ERR_INVALID, "cross_entropy: empty logits");
  if (!x || !t || !loss) return fg::set_error(FG_ERR_INVALID, "fg_xent_fwd_bwd: null pointer");
  double total = 0.0;
  for (size_t r = 0; r < rows; r++) {
    const float *xr = x + r * cols, *tr = t + r * cols;
    double m = -INFINITY, se = 0.0, ts = 0.0, row = 0.0;
    for (size_t c = 0; c < cols; c++) m = xr[c] > m ? xr[c] : m;
    for (size_t c = 0; c < cols; c++) se += std::exp((double)xr[c] - m);
    const double lse = m + std::log(se);
    for (size_t c = 0; c < cols; c++) {
      ts += tr[c];
      row += tr[c] * ((double)xr[c] - lse);
    }
    total -= row;
    if (dx)
      for (size_t c = 0; c < cols; c++)
        dx[r * cols + c] =
            (float)((std::exp((double)xr[c] - lse) * ts - tr[c]) / (double)rows * grad_scale);
  }
  loss[0] = (float)(total / (double)rows);
  return FG_OK;
}

int fg_sgd(float *p, const float *g, size_t n, float lr, float *lo, void *) {
  FG_HOSTDEV_SKIP_COMPUTE();
  for (size_t i = 0; i < n; i++) {
    const float d = g[i] * lr;
    p[i] = p[i] + (-d);
    if (lo) lo[i] = p[i] - tf32_hi(p[i]);
  }
  return FG_OK;
}

int fg_one_hot_u8(const uint8_t *labels, float *out, size_t n, int classes, void *) {
  for (size_t i = 0; i < n; i++)
    for (int c = 0; c < classes; c++) out[i * classes + c] = (int)labels[i] == c ? 1.0f : 0.0f;
  return FG_OK;
}

// Communicator: the ranks are processes on this machine, and the transport
// is a callback the test registers (fg_hostdev_set_allreduce), which sums a
// host buffer over the ranks in place -- a gloo all-reduce in the tests.  The
// mean is that sum times 1/nranks; NCCL's order of additions differs, so
// results through it are held to a tolerance, not to bits.
}  // extern "C"
struct fg_comm {
  int rank, nranks;
};
static int (*g_allreduce_sum)(float *, size_t) = nullptr;
extern "C" {
void fg_hostdev_set_allreduce(int (*fn)(float *, size_t)) { g_allreduce_sum = fn; }
int fg_comm_unique_id(char out[FG_UNIQUE_ID_BYTES]) {
  memset(out, 0, FG_UNIQUE_ID_BYTES);
  return FG_OK;
}
int fg_comm_init(int rank, int nranks, const char *, int, fg_comm **out) {
  if (nranks < 1 || rank < 0 || rank >= nranks)
    return fg::set_error(FG_ERR_INVALID, "fg_comm_init: bad rank %d of %d", rank, nranks);
  *out = new fg_comm{rank, nranks};
  return FG_OK;
}
int fg_comm_destroy(fg_comm *comm) {
  delete comm;
  return FG_OK;
}
int fg_comm_abort(fg_comm *comm) { return fg_comm_destroy(comm); }
int fg_allreduce_mean_f32(fg_comm *comm, float *buf, size_t count, void *) {
  if (!comm || (count && !buf)) return fg::set_error(FG_ERR_INVALID, "fg_allreduce_mean_f32: null argument");
  FG_HOSTDEV_SKIP_COMPUTE();
  if (comm->nranks == 1 || count == 0) return FG_OK;
  if (!g_allreduce_sum) return fg::set_error(FG_ERR_INVALID, "hostdev: no all-reduce transport registered");
  if (g_allreduce_sum(buf, count)) return fg::set_error(FG_ERR_NCCL, "hostdev: all-reduce transport failed");
  const float inv = 1.0f / (float)comm->nranks;
  for (size_t i = 0; i < count; i++) buf[i] *= inv;
  return FG_OK;
}

}  // extern "C"
