// Device, buffer, copy and NVRTC program entry points of the C ABI: the
// CUDA side of ferrograd's Device trait (src/device.rs:275-332).
#include <cuda.h>
#include <cudaTypedefs.h>
#include <nvrtc.h>

#include <math.h>

#include <atomic>
#include <mutex>
#include <string>
#include <vector>

#include "fg_internal.h"

namespace fg {

static thread_local std::string g_last_error;
static std::atomic<uint64_t> g_launches{0};

int set_error(int code, const char *fmt, ...) {
  char buf[4096];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  g_last_error = buf;
  return code;
}

void clear_error() { g_last_error.clear(); }

void count_launch(int n) { g_launches.fetch_add((uint64_t)n, std::memory_order_relaxed); }

static std::mutex g_ctx_mu;
static DevCtx g_ctx[64];

DevCtx *ctx_current() {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return nullptr;
  std::lock_guard<std::mutex> lock(g_ctx_mu);
  DevCtx &c = g_ctx[dev];
  if (c.ordinal < 0) {
    if (cudaMalloc(&c.d_err, sizeof(unsigned int)) != cudaSuccess) return nullptr;
    if (cudaMemset(c.d_err, 0, sizeof(unsigned int)) != cudaSuccess) return nullptr;
    cudaDeviceGetAttribute(&c.num_sms, cudaDevAttrMultiProcessorCount, dev);
    // fg_alloc/fg_free are stream-ordered (cudaMallocAsync/cudaFreeAsync)
    // from the device's default pool; keep freed blocks in the pool instead
    // of returning them to the driver at every synchronisation, so a
    // training loop reuses its per-step buffers.  This is a property of this
    // process's pool, not of the GPU.
    cudaMemPool_t pool;
    if (cudaDeviceGetDefaultMemPool(&pool, dev) == cudaSuccess) {
      uint64_t keep = UINT64_MAX;
      cudaMemPoolSetAttribute(pool, cudaMemPoolAttrReleaseThreshold, &keep);
    }
    cudaGetLastError();
    c.ordinal = dev;
  }
  return &c;
}

void *workspace(size_t bytes, int *status) {
  DevCtx *c = ctx_current();
  if (!c) {
    *status = set_error(FG_ERR_CUDA, "no CUDA device context");
    return nullptr;
  }
  if (bytes <= c->ws_bytes) {
    *status = FG_OK;
    return c->workspace;
  }
  if (c->workspace) {
    cudaDeviceSynchronize();
    cudaFree(c->workspace);
    c->workspace = nullptr;
    c->ws_bytes = 0;
  }
  size_t want = bytes < (1u << 20) ? (1u << 20) : bytes;
  if (cudaMalloc(&c->workspace, want) != cudaSuccess) {
    *status = set_error(FG_ERR_CUDA, "workspace allocation of %zu bytes failed", want);
    return nullptr;
  }
  c->ws_bytes = want;
  *status = FG_OK;
  return c->workspace;
}

// ---- driver API entry points, resolved through the runtime --------------
struct Driver {
  PFN_cuModuleLoadData_v2000 moduleLoadData = nullptr;
  PFN_cuModuleGetFunction_v2000 moduleGetFunction = nullptr;
  PFN_cuModuleUnload_v2000 moduleUnload = nullptr;
  PFN_cuLaunchKernel_v4000 launchKernel = nullptr;
  bool ok = false;
};

static Driver *driver() {
  static Driver d;
  static std::once_flag once;
  std::call_once(once, [] {
    cudaDriverEntryPointQueryResult q;
    bool ok = true;
    ok &= cudaGetDriverEntryPoint("cuModuleLoadData", (void **)&d.moduleLoadData,
                                  cudaEnableDefault, &q) == cudaSuccess && d.moduleLoadData;
    ok &= cudaGetDriverEntryPoint("cuModuleGetFunction", (void **)&d.moduleGetFunction,
                                  cudaEnableDefault, &q) == cudaSuccess && d.moduleGetFunction;
    ok &= cudaGetDriverEntryPoint("cuModuleUnload", (void **)&d.moduleUnload,
                                  cudaEnableDefault, &q) == cudaSuccess && d.moduleUnload;
    ok &= cudaGetDriverEntryPoint("cuLaunchKernel", (void **)&d.launchKernel,
                                  cudaEnableDefault, &q) == cudaSuccess && d.launchKernel;
    d.ok = ok;
  });
  return &d;
}

}  // namespace fg

struct fg_buffer {
  fg_device *dev;
  void *dptr;
  int dtype;
  size_t numel;
};

struct fg_program {
  fg_device *dev;
  CUmodule module;
  CUfunction func;
  int num_args;
  uint32_t grid[3];
  uint32_t block[3];
};

static size_t dtype_size(int dtype) {
  switch (dtype) {
    case FG_F32: return 4;
    case FG_I32: return 4;
    case FG_BOOL: return 1;
    default: return 0;
  }
}

extern "C" {

const char *fg_last_error(void) { return fg::g_last_error.c_str(); }

uint64_t fg_kernel_launches(void) { return fg::g_launches.load(); }

int fg_check_device_error(void) {
  fg::DevCtx *c = fg::ctx_current();
  if (!c) return fg::set_error(FG_ERR_CUDA, "no CUDA device context");
  unsigned int v = 0;
  FG_CUDA_TRY(cudaMemcpy(&v, c->d_err, sizeof(v), cudaMemcpyDeviceToHost));
  if (v) {
    FG_CUDA_TRY(cudaMemset(c->d_err, 0, sizeof(unsigned int)));
    return fg::set_error(FG_ERR_DEVICE,
                         "kernel error word 0x%x: a bounded wait expired (code %u, stage %u)", v,
                         v >> 16, v & 0xffff);
  }
  return FG_OK;
}

int fg_device_open(int ordinal, fg_device **out) {
  FG_REQUIRE(out, "fg_device_open: out is null");
  int n = 0;
  FG_CUDA_TRY(cudaGetDeviceCount(&n));
  FG_REQUIRE(ordinal >= 0 && ordinal < n, "fg_device_open: ordinal %d out of range (%d devices)",
             ordinal, n);
  FG_CUDA_TRY(cudaSetDevice(ordinal));
  if (!fg::ctx_current()) return fg::set_error(FG_ERR_CUDA, "device context init failed");
  // Buffers come from the device's stream-ordered pool (cudaMallocAsync).
  // With the pool's default release threshold (0) every synchronisation
  // hands freed memory back to the driver, and the next allocation maps it
  // again; keeping it in this process's pool makes a training loop's
  // per-step allocations cheap.  (A pool attribute of this process only.)
  {
    cudaMemPool_t pool;
    if (cudaDeviceGetDefaultMemPool(&pool, ordinal) == cudaSuccess) {
      uint64_t keep = UINT64_MAX;
      cudaMemPoolSetAttribute(pool, cudaMemPoolAttrReleaseThreshold, &keep);
    }
    cudaGetLastError();
  }
  fg_device *d = new fg_device;
  d->ordinal = ordinal;
  cudaError_t e = cudaStreamCreateWithFlags(&d->stream, cudaStreamNonBlocking);
  if (e != cudaSuccess) {
    delete d;
    return fg::set_error(FG_ERR_CUDA, "cudaStreamCreate: %s", cudaGetErrorString(e));
  }
  *out = d;
  return FG_OK;
}

int fg_device_close(fg_device *dev) {
  if (!dev) return FG_OK;
  cudaSetDevice(dev->ordinal);
  cudaStreamSynchronize(dev->stream);
  cudaStreamDestroy(dev->stream);
  delete dev;
  return FG_OK;
}

int fg_device_stream(fg_device *dev, void **stream) {
  FG_REQUIRE(dev && stream, "fg_device_stream: null argument");
  *stream = (void *)dev->stream;
  return FG_OK;
}

int fg_device_sync(fg_device *dev) {
  FG_REQUIRE(dev, "fg_device_sync: null device");
  FG_CUDA_TRY(cudaSetDevice(dev->ordinal));
  FG_CUDA_TRY(cudaStreamSynchronize(dev->stream));
  return fg_check_device_error();
}

// ---- device-side timing ----------------------------------------------------
struct fg_event {
  int ordinal;
  cudaEvent_t ev;
  cudaStream_t stream;  // the device's stream (used when record gets NULL)
};

int fg_event_create(fg_device *dev, fg_event **out) {
  FG_REQUIRE(dev && out, "fg_event_create: null argument");
  FG_CUDA_TRY(cudaSetDevice(dev->ordinal));
  cudaEvent_t e = nullptr;
  FG_CUDA_TRY(cudaEventCreate(&e));
  *out = new fg_event{dev->ordinal, e, dev->stream};
  return FG_OK;
}

int fg_event_record(fg_event *ev, void *stream) {
  FG_REQUIRE(ev, "fg_event_record: null event");
  FG_CUDA_TRY(cudaSetDevice(ev->ordinal));
  FG_CUDA_TRY(cudaEventRecord(ev->ev, stream ? (cudaStream_t)stream : ev->stream));
  return FG_OK;
}

int fg_event_elapsed_ms(fg_event *start, fg_event *end, float *ms) {
  FG_REQUIRE(start && end && ms, "fg_event_elapsed_ms: null argument");
  FG_REQUIRE(start->ordinal == end->ordinal, "fg_event_elapsed_ms: events of devices %d and %d",
             start->ordinal, end->ordinal);
  FG_CUDA_TRY(cudaSetDevice(start->ordinal));
  FG_CUDA_TRY(cudaEventSynchronize(end->ev));
  FG_CUDA_TRY(cudaEventElapsedTime(ms, start->ev, end->ev));
  return FG_OK;
}

int fg_event_destroy(fg_event *ev) {
  if (!ev) return FG_OK;
  cudaSetDevice(ev->ordinal);
  cudaEventDestroy(ev->ev);
  delete ev;
  return FG_OK;
}

int fg_alloc(fg_device *dev, int dtype, size_t numel, fg_buffer **out) {
  FG_REQUIRE(dev && out, "fg_alloc: null argument");
  size_t es = dtype_size(dtype);
  FG_REQUIRE(es > 0, "fg_alloc: unknown dtype %d", dtype);
  FG_CUDA_TRY(cudaSetDevice(dev->ordinal));
  void *p = nullptr;
  size_t nbytes = es * numel;
  if (nbytes) {
    FG_CUDA_TRY(cudaMallocAsync(&p, nbytes, dev->stream));
    FG_CUDA_TRY(cudaMemsetAsync(p, 0, nbytes, dev->stream));
  }
  fg_buffer *b = new fg_buffer{dev, p, dtype, numel};
  *out = b;
  return FG_OK;
}

int fg_free(fg_buffer *buf) {
  if (!buf) return FG_OK;
  if (buf->dptr) {
    cudaSetDevice(buf->dev->ordinal);
    cudaFreeAsync(buf->dptr, buf->dev->stream);
  }
  delete buf;
  return FG_OK;
}

int fg_buffer_info(const fg_buffer *buf, void **d_ptr, int *dtype, size_t *numel) {
  FG_REQUIRE(buf, "fg_buffer_info: null buffer");
  if (d_ptr) *d_ptr = buf->dptr;
  if (dtype) *dtype = buf->dtype;
  if (numel) *numel = buf->numel;
  return FG_OK;
}

int fg_copy_h2d(fg_buffer *buf, const void *h_src, size_t nbytes) {
  FG_REQUIRE(buf, "copy_from_host: null buffer");
  size_t want = dtype_size(buf->dtype) * buf->numel;
  FG_REQUIRE(nbytes == want, "copy_from_host: expected %zu bytes, got %zu", want, nbytes);
  if (!nbytes) return FG_OK;
  FG_REQUIRE(h_src, "copy_from_host: null source");
  FG_CUDA_TRY(cudaSetDevice(buf->dev->ordinal));
  // The reference copies synchronously from a borrowed slice, so the source
  // may be released as soon as this returns.  From pageable memory
  // cudaMemcpyAsync returns once the bytes are staged, which already gives
  // that; only a page-locked source needs the stream drained.
  cudaPointerAttributes attr;
  bool pinned = cudaPointerGetAttributes(&attr, h_src) == cudaSuccess &&
                attr.type == cudaMemoryTypeHost;
  cudaGetLastError();
  FG_CUDA_TRY(cudaMemcpyAsync(buf->dptr, h_src, nbytes, cudaMemcpyHostToDevice, buf->dev->stream));
  if (pinned) FG_CUDA_TRY(cudaStreamSynchronize(buf->dev->stream));
  return FG_OK;
}

int fg_copy_d2h(const fg_buffer *buf, void *h_dst, size_t nbytes) {
  FG_REQUIRE(buf, "copy_to_host: null buffer");
  size_t want = dtype_size(buf->dtype) * buf->numel;
  FG_REQUIRE(nbytes == want, "copy_to_host: expected %zu bytes, got %zu", want, nbytes);
  if (!nbytes) return FG_OK;
  FG_REQUIRE(h_dst, "copy_to_host: null destination");
  FG_CUDA_TRY(cudaSetDevice(buf->dev->ordinal));
  FG_CUDA_TRY(cudaMemcpyAsync(h_dst, buf->dptr, nbytes, cudaMemcpyDeviceToHost, buf->dev->stream));
  FG_CUDA_TRY(cudaStreamSynchronize(buf->dev->stream));
  return fg_check_device_error();
}

int fg_compile(fg_device *dev, const char *source, const char *func_name, int num_args,
               const uint32_t grid[3], const uint32_t block[3], fg_program **out) {
  FG_REQUIRE(dev && source && func_name && out && grid && block, "fg_compile: null argument");
  FG_REQUIRE(num_args >= 0, "fg_compile: negative num_args");
  fg::Driver *drv = fg::driver();
  if (!drv->ok) return fg::set_error(FG_ERR_CUDA, "CUDA driver entry points unavailable");
  FG_CUDA_TRY(cudaSetDevice(dev->ordinal));
  nvrtcProgram prog;
  if (nvrtcCreateProgram(&prog, source, "fg_kernel.cu", 0, nullptr, nullptr) != NVRTC_SUCCESS)
    return fg::set_error(FG_ERR_COMPILE, "nvrtcCreateProgram failed");
  const char *opts[] = {"-arch=sm_100a", "--std=c++17", "-default-device", "-lineinfo"};
  nvrtcResult r = nvrtcCompileProgram(prog, 4, opts);
  if (r != NVRTC_SUCCESS) {
    size_t logsz = 0;
    nvrtcGetProgramLogSize(prog, &logsz);
    std::string log(logsz, '\0');
    if (logsz) nvrtcGetProgramLog(prog, &log[0]);
    nvrtcDestroyProgram(&prog);
    return fg::set_error(FG_ERR_COMPILE, "nvrtc compilation failed:\n%s", log.c_str());
  }
  size_t cubin_size = 0;
  nvrtcGetCUBINSize(prog, &cubin_size);
  std::vector<char> cubin(cubin_size);
  nvrtcGetCUBIN(prog, cubin.data());
  nvrtcDestroyProgram(&prog);
  CUmodule mod;
  CUresult cr = drv->moduleLoadData(&mod, cubin.data());
  if (cr != CUDA_SUCCESS) return fg::set_error(FG_ERR_CUDA, "cuModuleLoadData failed (%d)", (int)cr);
  CUfunction fn;
  cr = drv->moduleGetFunction(&fn, mod, func_name);
  if (cr != CUDA_SUCCESS) {
    drv->moduleUnload(mod);
    return fg::set_error(FG_ERR_COMPILE, "symbol '%s' not found (%d)", func_name, (int)cr);
  }
  fg_program *p = new fg_program;
  p->dev = dev;
  p->module = mod;
  p->func = fn;
  p->num_args = num_args;
  for (int i = 0; i < 3; i++) {
    p->grid[i] = grid[i] ? grid[i] : 1;
    p->block[i] = block[i] ? block[i] : 1;
  }
  *out = p;
  return FG_OK;
}

int fg_program_free(fg_program *prog) {
  if (!prog) return FG_OK;
  fg::Driver *drv = fg::driver();
  if (drv->ok) drv->moduleUnload(prog->module);
  delete prog;
  return FG_OK;
}

int fg_execute(fg_program *prog, const fg_kernel_arg *args, int nargs) {
  FG_REQUIRE(prog, "fg_execute: null program");
  FG_REQUIRE(nargs == prog->num_args, "expected %d kernel args, got %d", prog->num_args, nargs);
  FG_REQUIRE(nargs == 0 || args, "fg_execute: null args");
  std::vector<void *> ptrs(nargs);
  std::vector<void *> params(nargs);
  for (int i = 0; i < nargs; i++) {
    switch (args[i].kind) {
      case FG_ARG_BUFFER:
        FG_REQUIRE(args[i].v.buffer, "fg_execute: arg %d: null buffer", i);
        FG_REQUIRE(args[i].v.buffer->dev->ordinal == prog->dev->ordinal,
                   "fg_execute: arg %d: buffer belongs to another device", i);
        ptrs[i] = args[i].v.buffer->dptr;
        params[i] = &ptrs[i];
        break;
      case FG_ARG_I32: params[i] = (void *)&args[i].v.i32; break;
      case FG_ARG_F32: params[i] = (void *)&args[i].v.f32; break;
      case FG_ARG_BOOL: params[i] = (void *)&args[i].v.b; break;
      default: return fg::set_error(FG_ERR_INVALID, "fg_execute: arg %d: unknown kind", i);
    }
  }
  FG_CUDA_TRY(cudaSetDevice(prog->dev->ordinal));
  CUresult cr = fg::driver()->launchKernel(prog->func, prog->grid[0], prog->grid[1], prog->grid[2],
                                           prog->block[0], prog->block[1], prog->block[2], 0,
                                           (CUstream)prog->dev->stream, params.data(), nullptr);
  if (cr != CUDA_SUCCESS) return fg::set_error(FG_ERR_CUDA, "cuLaunchKernel failed (%d)", (int)cr);
  fg::count_launch();
  return FG_OK;
}

}  // extern "C"
