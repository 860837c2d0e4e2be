// Internal host-side helpers shared by the translation units of libferro_cuda.
#pragma once
#include <cuda_runtime.h>
#include <stdarg.h>
#include <stdint.h>
#include <stdio.h>
#include <string>

#include "../../include/ferro_cuda.h"

// Opaque handle of the C ABI (one per opened ordinal).
struct fg_device {
  int ordinal;
  cudaStream_t stream;
};

namespace fg {

int set_error(int code, const char *fmt, ...);
void clear_error();

// Per-device state, created lazily for the current device.
struct DevCtx {
  int ordinal = -1;
  unsigned int *d_err = nullptr;  // error word kernels set when a bounded wait expires
  void *workspace = nullptr;      // scratch for multi-pass kernels (grown on demand)
  size_t ws_bytes = 0;
  int num_sms = 0;
};
DevCtx *ctx_current();
// Returns a scratch pointer of at least `bytes` on the current device; the
// previous contents are not preserved.  Must not be called during capture
// with a size larger than the current workspace.
void *workspace(size_t bytes, int *status);
void count_launch(int n = 1);

}  // namespace fg

#define FG_CUDA_TRY(expr)                                                                   \
  do {                                                                                      \
    cudaError_t fg_e_ = (expr);                                                             \
    if (fg_e_ != cudaSuccess)                                                               \
      return fg::set_error(FG_ERR_CUDA, "%s failed: %s (%s:%d)", #expr,                     \
                           cudaGetErrorString(fg_e_), __FILE__, __LINE__);                 \
  } while (0)

#define FG_LAUNCH_TRY()                                                                     \
  do {                                                                                      \
    cudaError_t fg_e_ = cudaGetLastError();                                                 \
    if (fg_e_ != cudaSuccess)                                                               \
      return fg::set_error(FG_ERR_CUDA, "kernel launch failed: %s (%s:%d)",                 \
                           cudaGetErrorString(fg_e_), __FILE__, __LINE__);                 \
    fg::count_launch();                                                                     \
  } while (0)

#define FG_REQUIRE(cond, ...)                                                               \
  do {                                                                                      \
    if (!(cond)) return fg::set_error(FG_ERR_INVALID, __VA_ARGS__);                         \
  } while (0)
