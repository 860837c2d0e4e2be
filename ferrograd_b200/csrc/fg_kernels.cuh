// Launchers of the HBM-bound kernels (fg_kernels.cu), shared with the MLP plan.
#pragma once
#include <cuda_runtime.h>
#include <stddef.h>

#include "../../include/ferro_cuda.h"

// Rows of per-row scratch held in the library's static device array for
// fg_xent_fwd_bwd_noalloc (262144 floats = 1 MiB per GPU).
constexpr int kFgXentNoallocMaxRows = FG_XENT_NOALLOC_MAX_ROWS;

namespace fg {

constexpr int kMaxSgdSegments = 8;
struct SgdSegments {
  int count;
  float *p[kMaxSgdSegments];
  const float *g[kMaxSgdSegments];
  float *lo[kMaxSgdSegments];
  size_t n[kMaxSgdSegments];
};

int launch_ew_fma_relu_scale(const float *a, const float *b, const float *c, float *out, size_t n,
                             float scale, cudaStream_t st);
int launch_reduce_rows(int dtype, int op, const void *x, void *out, size_t rows, size_t cols,
                       cudaStream_t st);
// scratch == nullptr: use the per-device workspace.
int launch_reduce_cols(int dtype, int op, const void *x, void *out, size_t rows, size_t cols,
                       cudaStream_t st, void *scratch, size_t scratch_bytes);
size_t reduce_cols_scratch_bytes(size_t rows, size_t cols);
// row_scratch == nullptr: use the per-device workspace (rows floats).
// loss = loss_scale * mean over the rows; dx scaled by gscale.
int launch_xent(const float *x, const float *t, size_t rows, size_t cols, float *loss, float *dx,
                float gscale, cudaStream_t st, float *row_scratch, float loss_scale = 1.0f);
int launch_sgd_multi(const SgdSegments &segs, float lr, cudaStream_t st);
int launch_split_lo(const float *x, float *lo, size_t n, cudaStream_t st);
int launch_copy2(const float *src_a, float *dst_a, size_t na, const float *src_b, float *dst_b,
                 size_t nb, cudaStream_t st);

}  // namespace fg
