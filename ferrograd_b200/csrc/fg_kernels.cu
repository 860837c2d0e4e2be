// HBM-bound building blocks: fused elementwise chain, row / column
// reductions (f32 and bit-exact i32), fused cross-entropy forward+backward,
// SGD update and the TF32 residual split.
//
// All of these stream their operands once: 128-bit loads and stores where
// the layout allows, grids sized in multiples of the SM count, warp-shuffle
// reductions with a fixed (deterministic) order.
#include <cuda_runtime.h>
#include <stdint.h>

#include <cooperative_groups.h>
#include <mutex>

#include "fg_internal.h"
#include "fg_kernels.cuh"

namespace fg {

namespace cg = cooperative_groups;

// Reference op semantics (src/codegen/clang.rs:216-229): max is a ternary,
// every op rounds separately (no FMA contraction).
__device__ __forceinline__ float ref_max(float a, float b) { return (a > b) ? a : b; }
__device__ __forceinline__ int32_t ref_max_i(int32_t a, int32_t b) { return (a > b) ? a : b; }
__device__ __forceinline__ int32_t add_wrap(int32_t a, int32_t b) {
  return (int32_t)((uint32_t)a + (uint32_t)b);
}

static int grid_for(size_t work_items, int threads, int per_sm = 8) {
  DevCtx *c = ctx_current();
  int sms = (c && c->num_sms) ? c->num_sms : 148;
  size_t want = (work_items + threads - 1) / threads;
  size_t cap = (size_t)sms * per_sm;
  if (want > cap) want = cap;
  if (want < 1) want = 1;
  return (int)want;
}

// ---------------------------------------------------------------------------
// relu(a*b+c)*scale: t = a*b; t = t + c; r = (0 < t) ? t : 0; out = r*scale
// ---------------------------------------------------------------------------
__device__ __forceinline__ float ew_one(float a, float b, float c, float s) {
  float t = __fmul_rn(a, b);
  t = __fadd_rn(t, c);
  float r = (0.0f < t) ? t : 0.0f;
  return __fmul_rn(r, s);
}

__global__ void __launch_bounds__(256) k_ew_fma_relu_scale_v4(const float4 *__restrict__ a,
                                                              const float4 *__restrict__ b,
                                                              const float4 *__restrict__ c,
                                                              float4 *__restrict__ out,
                                                              size_t n4, float s) {
  size_t stride = (size_t)gridDim.x * blockDim.x;
  size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
  // Two independent 16-byte loads per operand in flight per iteration.
  for (; i + stride < n4; i += 2 * stride) {
    float4 a0 = __ldcs(a + i), b0 = __ldcs(b + i), c0 = __ldcs(c + i);
    float4 a1 = __ldcs(a + i + stride), b1 = __ldcs(b + i + stride), c1 = __ldcs(c + i + stride);
    float4 r0, r1;
    r0.x = ew_one(a0.x, b0.x, c0.x, s); r0.y = ew_one(a0.y, b0.y, c0.y, s);
    r0.z = ew_one(a0.z, b0.z, c0.z, s); r0.w = ew_one(a0.w, b0.w, c0.w, s);
    r1.x = ew_one(a1.x, b1.x, c1.x, s); r1.y = ew_one(a1.y, b1.y, c1.y, s);
    r1.z = ew_one(a1.z, b1.z, c1.z, s); r1.w = ew_one(a1.w, b1.w, c1.w, s);
    __stcs(out + i, r0);
    __stcs(out + i + stride, r1);
  }
  if (i < n4) {
    float4 a0 = __ldcs(a + i), b0 = __ldcs(b + i), c0 = __ldcs(c + i);
    float4 r0;
    r0.x = ew_one(a0.x, b0.x, c0.x, s); r0.y = ew_one(a0.y, b0.y, c0.y, s);
    r0.z = ew_one(a0.z, b0.z, c0.z, s); r0.w = ew_one(a0.w, b0.w, c0.w, s);
    __stcs(out + i, r0);
  }
}

__global__ void k_ew_fma_relu_scale_tail(const float *__restrict__ a, const float *__restrict__ b,
                                         const float *__restrict__ c, float *__restrict__ out,
                                         size_t begin, size_t n, float s) {
  size_t i = begin + (size_t)blockIdx.x * blockDim.x + threadIdx.x;
  for (; i < n; i += (size_t)gridDim.x * blockDim.x) out[i] = ew_one(a[i], b[i], c[i], s);
}

static bool aligned16(const void *p) { return ((uintptr_t)p & 15) == 0; }

int launch_ew_fma_relu_scale(const float *a, const float *b, const float *c, float *out, size_t n,
                             float scale, cudaStream_t st) {
  if (n == 0) return FG_OK;
  size_t n4 = 0;
  if (aligned16(a) && aligned16(b) && aligned16(c) && aligned16(out)) n4 = n / 4;
  if (n4) {
    k_ew_fma_relu_scale_v4<<<grid_for(n4 / 2 + 1, 256, 16), 256, 0, st>>>(
        (const float4 *)a, (const float4 *)b, (const float4 *)c, (float4 *)out, n4, scale);
    FG_LAUNCH_TRY();
  }
  if (n4 * 4 < n) {
    k_ew_fma_relu_scale_tail<<<grid_for(n - n4 * 4, 256), 256, 0, st>>>(a, b, c, out, n4 * 4, n,
                                                                         scale);
    FG_LAUNCH_TRY();
  }
  return FG_OK;
}

// ---------------------------------------------------------------------------
// Row reductions: one warp per row, 16-byte loads, shuffle tree.
// ---------------------------------------------------------------------------
template <typename T, int OP>
__device__ __forceinline__ T red_identity();
template <> __device__ __forceinline__ float red_identity<float, FG_REDUCE_SUM>() { return 0.0f; }
template <> __device__ __forceinline__ float red_identity<float, FG_REDUCE_MAX>() { return -INFINITY; }
template <> __device__ __forceinline__ int32_t red_identity<int32_t, FG_REDUCE_SUM>() { return 0; }
template <> __device__ __forceinline__ int32_t red_identity<int32_t, FG_REDUCE_MAX>() { return INT32_MIN; }

template <int OP>
__device__ __forceinline__ float red_op(float a, float b) {
  return OP == FG_REDUCE_SUM ? __fadd_rn(a, b) : ref_max(a, b);
}
template <int OP>
__device__ __forceinline__ int32_t red_op(int32_t a, int32_t b) {
  return OP == FG_REDUCE_SUM ? add_wrap(a, b) : ref_max_i(a, b);
}

template <typename T, int OP>
__device__ __forceinline__ T warp_reduce(T v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = red_op<OP>(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

template <typename T, int OP>
__device__ __forceinline__ T red4(const uint4 &u) {
  const T *f = reinterpret_cast<const T *>(&u);
  return red_op<OP>(red_op<OP>(f[0], f[1]), red_op<OP>(f[2], f[3]));
}

// One warp per row, 16-byte loads.  The row is walked in batches of kRowBatch
// loads per lane, and the next batch is in flight while the current one is
// folded, so each warp keeps its loads outstanding for the whole row instead
// of draining at every batch; the grid is a fixed multiple of the SM count
// and warps stride over the rows.
constexpr int kRowBatch = 8;

template <typename T, int OP>
__global__ void __launch_bounds__(128) k_reduce_rows_v4(const T *__restrict__ x, T *__restrict__ out,
                                                        size_t rows, size_t cols) {
  const int lane = threadIdx.x & 31;
  size_t row = (size_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const size_t wstride = (size_t)gridDim.x * (blockDim.x >> 5);
  const size_t nv = cols / 4;  // 16-byte vectors per row
  const T id = red_identity<T, OP>();
  const uint4 idv = [&] {
    uint4 v;
    T *f = reinterpret_cast<T *>(&v);
    f[0] = f[1] = f[2] = f[3] = id;
    return v;
  }();
  for (; row < rows; row += wstride) {
    const uint4 *pv = reinterpret_cast<const uint4 *>(x + row * cols);
    T acc0 = id, acc1 = id;
    uint4 cur[kRowBatch];
#pragma unroll
    for (int k = 0; k < kRowBatch; k++) {
      const size_t j = lane + 32 * (size_t)k;
      cur[k] = j < nv ? __ldcs(pv + j) : idv;
    }
    for (size_t base = 32 * kRowBatch; base < nv + 32 * kRowBatch; base += 32 * kRowBatch) {
      uint4 nxt[kRowBatch];
      const bool more = base < nv;
      if (more) {
#pragma unroll
        for (int k = 0; k < kRowBatch; k++) {
          const size_t j = base + lane + 32 * (size_t)k;
          nxt[k] = j < nv ? __ldcs(pv + j) : idv;
        }
      }
#pragma unroll
      for (int k = 0; k < kRowBatch; k++) {
        const T g = red4<T, OP>(cur[k]);
        if (k & 1)
          acc1 = red_op<OP>(acc1, g);
        else
          acc0 = red_op<OP>(acc0, g);
      }
      if (!more) break;
#pragma unroll
      for (int k = 0; k < kRowBatch; k++) cur[k] = nxt[k];
    }
    T acc = warp_reduce<T, OP>(red_op<OP>(acc0, acc1));
    if (lane == 0) out[row] = acc;
  }
}

// Rows whose length is not a multiple of 4 (or unaligned): scalar loads.
template <typename T, int OP>
__global__ void __launch_bounds__(128) k_reduce_rows_scalar(const T *__restrict__ x,
                                                            T *__restrict__ out, size_t rows,
                                                            size_t cols) {
  const int lane = threadIdx.x & 31;
  size_t row = (size_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const size_t wstride = (size_t)gridDim.x * (blockDim.x >> 5);
  for (; row < rows; row += wstride) {
    const T *p = x + row * cols;
    T acc = red_identity<T, OP>();
    for (size_t j = lane; j < cols; j += 32) acc = red_op<OP>(acc, p[j]);
    acc = warp_reduce<T, OP>(acc);
    if (lane == 0) out[row] = acc;
  }
}

template <typename T, int OP>
static int launch_rows_t(const void *x, void *out, size_t rows, size_t cols, cudaStream_t st) {
  const bool vec = (cols % 4 == 0) && aligned16(x);
  // 4 warps per block, 8 blocks per SM: every warp strides over rows.
  int grid = grid_for(rows * 32, 128, 8);
  if (vec)
    k_reduce_rows_v4<T, OP><<<grid, 128, 0, st>>>((const T *)x, (T *)out, rows, cols);
  else
    k_reduce_rows_scalar<T, OP><<<grid, 128, 0, st>>>((const T *)x, (T *)out, rows, cols);
  FG_LAUNCH_TRY();
  return FG_OK;
}

int launch_reduce_rows(int dtype, int op, const void *x, void *out, size_t rows, size_t cols,
                       cudaStream_t st) {
  if (rows == 0) return FG_OK;
  if (dtype == FG_F32)
    return op == FG_REDUCE_SUM ? launch_rows_t<float, FG_REDUCE_SUM>(x, out, rows, cols, st)
                               : launch_rows_t<float, FG_REDUCE_MAX>(x, out, rows, cols, st);
  return op == FG_REDUCE_SUM ? launch_rows_t<int32_t, FG_REDUCE_SUM>(x, out, rows, cols, st)
                             : launch_rows_t<int32_t, FG_REDUCE_MAX>(x, out, rows, cols, st);
}

// ---------------------------------------------------------------------------
// Column reductions (axis 0).  Pass 1: each block owns a 256-column strip and
// a chunk of rows, threads run down the columns (coalesced), partial results
// go to scratch [nchunks, cols].  Pass 2 folds the chunks in chunk order.
// ---------------------------------------------------------------------------
constexpr int kColTile = 256;

template <typename T, int OP>
__global__ void __launch_bounds__(256) k_reduce_cols_partial(const T *__restrict__ x,
                                                             T *__restrict__ part, size_t rows,
                                                             size_t cols, size_t rows_per_chunk) {
  size_t col = (size_t)blockIdx.x * kColTile + threadIdx.x;
  size_t r0 = (size_t)blockIdx.y * rows_per_chunk;
  size_t r1 = r0 + rows_per_chunk < rows ? r0 + rows_per_chunk : rows;
  if (col >= cols) return;
  T a0 = red_identity<T, OP>(), a1 = red_identity<T, OP>();
  T a2 = red_identity<T, OP>(), a3 = red_identity<T, OP>();
  size_t r = r0;
  for (; r + 4 <= r1; r += 4) {
    a0 = red_op<OP>(a0, __ldcs(x + r * cols + col));
    a1 = red_op<OP>(a1, __ldcs(x + (r + 1) * cols + col));
    a2 = red_op<OP>(a2, __ldcs(x + (r + 2) * cols + col));
    a3 = red_op<OP>(a3, __ldcs(x + (r + 3) * cols + col));
  }
  for (; r < r1; r++) a0 = red_op<OP>(a0, __ldcs(x + r * cols + col));
  part[blockIdx.y * cols + col] = red_op<OP>(red_op<OP>(a0, a1), red_op<OP>(a2, a3));
}

// 16-byte variant: a thread owns 4 adjacent columns, 8 rows in flight.
template <typename T, int OP>
__global__ void __launch_bounds__(64) k_reduce_cols_partial_v4(const T *__restrict__ x,
                                                               T *__restrict__ part, size_t rows,
                                                               size_t cols,
                                                               size_t rows_per_chunk) {
  const size_t col = ((size_t)blockIdx.x * 64 + threadIdx.x) * 4;
  const size_t r0 = (size_t)blockIdx.y * rows_per_chunk;
  const size_t r1 = r0 + rows_per_chunk < rows ? r0 + rows_per_chunk : rows;
  if (col >= cols) return;
  T a[4], b[4];
#pragma unroll
  for (int q = 0; q < 4; q++) a[q] = b[q] = red_identity<T, OP>();
  size_t r = r0;
  for (; r + 8 <= r1; r += 8) {
    uint4 u[8];
#pragma unroll
    for (int k = 0; k < 8; k++) u[k] = __ldcs(reinterpret_cast<const uint4 *>(x + (r + k) * cols + col));
#pragma unroll
    for (int k = 0; k < 8; k++) {
      const T *f = reinterpret_cast<const T *>(&u[k]);
#pragma unroll
      for (int q = 0; q < 4; q++) {
        if (k & 1)
          b[q] = red_op<OP>(b[q], f[q]);
        else
          a[q] = red_op<OP>(a[q], f[q]);
      }
    }
  }
  for (; r < r1; r++) {
    uint4 u = __ldcs(reinterpret_cast<const uint4 *>(x + r * cols + col));
    const T *f = reinterpret_cast<const T *>(&u);
#pragma unroll
    for (int q = 0; q < 4; q++) a[q] = red_op<OP>(a[q], f[q]);
  }
  uint4 o;
  T *oe = reinterpret_cast<T *>(&o);
#pragma unroll
  for (int q = 0; q < 4; q++) oe[q] = red_op<OP>(a[q], b[q]);
  *reinterpret_cast<uint4 *>(part + blockIdx.y * cols + col) = o;
}

template <typename T, int OP>
__global__ void __launch_bounds__(256) k_reduce_cols_final(const T *__restrict__ part,
                                                           T *__restrict__ out, size_t nchunks,
                                                           size_t cols) {
  size_t col = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (col >= cols) return;
  T acc = red_identity<T, OP>();
  for (size_t c = 0; c < nchunks; c++) acc = red_op<OP>(acc, part[c * cols + col]);
  out[col] = acc;
}

// Wide column reductions in one kernel: a CTA owns a strip of 128 columns
// (a warp row of 16-byte loads) and one of kColChunks row chunks; the
// chunks of a strip form a thread-block cluster and fold their partial sums
// through distributed shared memory, rank 0 adding them in chunk order
// (deterministic).  No scratch, no second launch.
constexpr int kColChunks = 8;
constexpr int kColWarps = 16;

template <typename T, int OP>
__global__ void __cluster_dims__(1, kColChunks, 1) __launch_bounds__(kColWarps * 32)
    k_reduce_cols_cluster(const T *__restrict__ x, T *__restrict__ out, size_t rows, size_t cols) {
  __shared__ uint4 wpart[kColWarps][32];
  __shared__ uint4 cpart[32];
  cg::cluster_group cl = cg::this_cluster();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const size_t col = (size_t)blockIdx.x * 128 + (size_t)lane * 4;
  const bool active = col < cols;
  const size_t chunk = (rows + kColChunks - 1) / kColChunks;
  const size_t r0 = (size_t)blockIdx.y * chunk;
  const size_t r1 = r0 + chunk < rows ? r0 + chunk : rows;
  const T id = red_identity<T, OP>();
  T a[4] = {id, id, id, id}, b[4] = {id, id, id, id};
  size_t r = r0 + warp;
  if (active) {
    for (; r + 7 * kColWarps < r1; r += 8 * kColWarps) {
      uint4 u[8];
#pragma unroll
      for (int k = 0; k < 8; k++)
        u[k] = __ldcs(reinterpret_cast<const uint4 *>(x + (r + k * kColWarps) * cols + col));
#pragma unroll
      for (int k = 0; k < 8; k++) {
        const T *f = reinterpret_cast<const T *>(&u[k]);
#pragma unroll
        for (int q = 0; q < 4; q++) {
          if (k & 1)
            b[q] = red_op<OP>(b[q], f[q]);
          else
            a[q] = red_op<OP>(a[q], f[q]);
        }
      }
    }
    for (; r < r1; r += kColWarps) {
      uint4 u = __ldcs(reinterpret_cast<const uint4 *>(x + r * cols + col));
      const T *f = reinterpret_cast<const T *>(&u);
#pragma unroll
      for (int q = 0; q < 4; q++) a[q] = red_op<OP>(a[q], f[q]);
    }
  }
  {
    uint4 v;
    T *f = reinterpret_cast<T *>(&v);
#pragma unroll
    for (int q = 0; q < 4; q++) f[q] = red_op<OP>(a[q], b[q]);
    wpart[warp][lane] = v;
  }
  __syncthreads();
  if (warp == 0) {
    uint4 v = wpart[0][lane];
    T *s = reinterpret_cast<T *>(&v);
    for (int w = 1; w < kColWarps; w++) {
      const T *f = reinterpret_cast<const T *>(&wpart[w][lane]);
#pragma unroll
      for (int q = 0; q < 4; q++) s[q] = red_op<OP>(s[q], f[q]);
    }
    cpart[lane] = v;
  }
  cl.sync();
  if (cl.block_rank() == 0 && warp == 0) {
    uint4 v = cpart[lane];
    T *s = reinterpret_cast<T *>(&v);
    for (unsigned q = 1; q < (unsigned)kColChunks; q++) {
      const uint4 *rp = cl.map_shared_rank(cpart, q);
      uint4 w = rp[lane];
      const T *f = reinterpret_cast<const T *>(&w);
#pragma unroll
      for (int e = 0; e < 4; e++) s[e] = red_op<OP>(s[e], f[e]);
    }
    if (active) *reinterpret_cast<uint4 *>(out + col) = v;
  }
  cl.sync();  // keep every CTA's shared memory alive until rank 0 has read it
}

template <typename T, int OP>
static int launch_cols_t(const void *x, void *out, size_t rows, size_t cols, cudaStream_t st,
                         void *scratch, size_t scratch_bytes) {
  if (rows == 0) {  // empty reduction: the identity in every column
    k_reduce_cols_final<T, OP><<<(unsigned)((cols + 255) / 256), 256, 0, st>>>(nullptr, (T *)out, 0,
                                                                              cols);
    FG_LAUNCH_TRY();
    return FG_OK;
  }
  size_t col_tiles = (cols + kColTile - 1) / kColTile;
  DevCtx *c = ctx_current();
  size_t sms = (c && c->num_sms) ? c->num_sms : 148;
  // Wide inputs: the single-kernel cluster reduction, once its strips x
  // chunks cover every SM and each chunk has rows to stream.
  const size_t strips = (cols + 127) / 128;
  if (cols % 4 == 0 && aligned16(x) && aligned16(out) && strips * kColChunks >= sms &&
      rows >= (size_t)kColChunks * kColWarps) {
    dim3 g((unsigned)strips, kColChunks);
    k_reduce_cols_cluster<T, OP><<<g, kColWarps * 32, 0, st>>>((const T *)x, (T *)out, rows, cols);
    FG_LAUNCH_TRY();
    return FG_OK;
  }
  // Enough chunks that col_tiles * nchunks fills every SM ~16 times, each
  // chunk at least 32 rows.
  size_t nchunks = (sms * 16 + col_tiles - 1) / col_tiles;
  size_t max_chunks = (rows + 31) / 32;
  if (nchunks > max_chunks) nchunks = max_chunks;
  if (nchunks < 1) nchunks = 1;
  size_t rpc = (rows + nchunks - 1) / nchunks;
  nchunks = (rows + rpc - 1) / rpc;
  size_t need = nchunks * cols * sizeof(T);
  if (!scratch) {
    int status = FG_OK;
    scratch = workspace(need, &status);
    if (!scratch) return status;
  } else if (scratch_bytes < need) {
    return set_error(FG_ERR_INVALID, "column reduce needs %zu scratch bytes, have %zu", need,
                     scratch_bytes);
  }
  dim3 g1((unsigned)col_tiles, (unsigned)nchunks);
  if (cols % 4 == 0 && aligned16(x) && aligned16(scratch))
    k_reduce_cols_partial_v4<T, OP><<<g1, 64, 0, st>>>((const T *)x, (T *)scratch, rows, cols, rpc);
  else
    k_reduce_cols_partial<T, OP><<<g1, kColTile, 0, st>>>((const T *)x, (T *)scratch, rows, cols,
                                                          rpc);
  FG_LAUNCH_TRY();
  k_reduce_cols_final<T, OP><<<(unsigned)((cols + 255) / 256), 256, 0, st>>>((const T *)scratch,
                                                                            (T *)out, nchunks, cols);
  FG_LAUNCH_TRY();
  return FG_OK;
}

size_t reduce_cols_scratch_bytes(size_t rows, size_t cols) {
  // Upper bound used by callers that provide their own scratch.
  size_t col_tiles = (cols + kColTile - 1) / kColTile;
  size_t nchunks = (148 * 16 + col_tiles - 1) / col_tiles + 1;
  size_t max_chunks = (rows + 31) / 32;
  if (nchunks > max_chunks) nchunks = max_chunks;
  if (nchunks < 1) nchunks = 1;
  return nchunks * cols * 4;
}

int launch_reduce_cols(int dtype, int op, const void *x, void *out, size_t rows, size_t cols,
                       cudaStream_t st, void *scratch, size_t scratch_bytes) {
  if (cols == 0) return FG_OK;
#define FG_COLS(T, OP) launch_cols_t<T, OP>(x, out, rows, cols, st, scratch, scratch_bytes)
  if (dtype == FG_F32)
    return op == FG_REDUCE_SUM ? FG_COLS(float, FG_REDUCE_SUM) : FG_COLS(float, FG_REDUCE_MAX);
  return op == FG_REDUCE_SUM ? FG_COLS(int32_t, FG_REDUCE_SUM) : FG_COLS(int32_t, FG_REDUCE_MAX);
#undef FG_COLS
}

// ---------------------------------------------------------------------------
// Cross-entropy forward + backward (src/tensor.rs:715-752 and the autograd
// graph of src/gradient.rs:97-205), one warp per row.  Per row:
//   m = max x; s = x - m; e = exp2(s*log2e); se = sum e; lse = log2(se)*ln2
//   nps = -sum t*(s - lse)                          (loss term of the row)
//   g_lp = t*(-1/B); g_se = (ln2*(sum g_lp)) * (1/(se*ln2))
//   g_s = g_lp + log2e*((e*ln2)*g_se)
//   dx = g_s + (mask/count) * (-sum g_s),  mask = (x < m) ? 0 : 1
// The row's loss terms go to scratch and are summed in row order by a
// second kernel (deterministic).
// ---------------------------------------------------------------------------
constexpr float kLog2e = 1.44269504088896340736f;
constexpr float kLn2 = 0.693147180559945309417f;

template <typename T>
__device__ __forceinline__ T warp_sum(T v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}
__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = ref_max(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

// NV float4 of logits per lane held in registers: cols <= 128 * NV,
// cols % 4 == 0.  Targets are not kept: their row sums (sum t, sum t*x) are
// folded in as they arrive, and the gradient pass re-reads them, which hits
// L1 (the row was read moments before with L1 caching).  That keeps the
// kernel at ~60 registers, 4 blocks (32 warps) per SM.
template <int NV>
__global__ void __launch_bounds__(256, 1) k_xent_rows_v4(const float *__restrict__ x,
                                                      const float *__restrict__ t,
                                                      float *__restrict__ dx,
                                                      float *__restrict__ warp_loss, size_t rows,
                                                      int cols, float inv_n, float gscale) {
  const int lane = threadIdx.x & 31;
  size_t row = (size_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const size_t wstride = (size_t)gridDim.x * (blockDim.x >> 5);
  const int nv = cols / 4;
  const size_t gwarp = row;
  float wloss = 0.f;  // this warp's rows' losses, summed in row order
  // Software pipeline: the next row's logits and targets are loaded while
  // the current row is reduced and its gradient written.
  float4 xn[NV], tn[NV];
  if (row < rows) {
    const float4 *xv = reinterpret_cast<const float4 *>(x + row * (size_t)cols);
    const float4 *tv = reinterpret_cast<const float4 *>(t + row * (size_t)cols);
#pragma unroll
    for (int i = 0; i < NV; i++) {
      int j = lane + 32 * i;
      if (j < nv) {
        xn[i] = __ldcs(xv + j);
        tn[i] = __ldcs(tv + j);
      }
    }
  }
  for (; row < rows; row += wstride) {
    float4 xr[NV], tr[NV];
#pragma unroll
    for (int i = 0; i < NV; i++) {
      xr[i] = xn[i];
      tr[i] = tn[i];
    }
    const size_t nrow = row + wstride;
    if (nrow < rows) {
      const float4 *xv = reinterpret_cast<const float4 *>(x + nrow * (size_t)cols);
      const float4 *tv = reinterpret_cast<const float4 *>(t + nrow * (size_t)cols);
#pragma unroll
      for (int i = 0; i < NV; i++) {
        int j = lane + 32 * i;
        if (j < nv) {
          xn[i] = __ldcs(xv + j);
          tn[i] = __ldcs(tv + j);
        }
      }
    }
    float m = -INFINITY, st_ = 0.f, stx = 0.f;
#pragma unroll
    for (int i = 0; i < NV; i++) {
      int j = lane + 32 * i;
      if (j < nv) {
        const float4 tt = tr[i];
        m = ref_max(m, ref_max(ref_max(xr[i].x, xr[i].y), ref_max(xr[i].z, xr[i].w)));
        st_ += (tt.x + tt.y) + (tt.z + tt.w);
        stx += __fmul_rn(tt.x, xr[i].x) + __fmul_rn(tt.y, xr[i].y) + __fmul_rn(tt.z, xr[i].z) +
               __fmul_rn(tt.w, xr[i].w);
      }
    }
    m = warp_max(m);
    float se = 0.f, cnt = 0.f;
    uint32_t maxbits = 0;  // bit (4i+q) set where x == row max (mask of the max path)
#pragma unroll
    for (int i = 0; i < NV; i++) {
      int j = lane + 32 * i;
      if (j < nv) {
        float *xe = reinterpret_cast<float *>(&xr[i]);
#pragma unroll
        for (int q = 0; q < 4; q++) {
          const float e = exp2f(__fmul_rn(__fsub_rn(xe[q], m), kLog2e));
          se += e;
          if (!(xe[q] < m)) {
            cnt += 1.0f;
            maxbits |= 1u << (4 * i + q);
          }
          xe[q] = e;  // the register now holds e
        }
      }
    }
    se = warp_sum(se);
    st_ = warp_sum(st_);
    stx = warp_sum(stx);
    cnt = warp_sum(cnt);
    const float lse = __fmul_rn(log2f(se), kLn2);
    // nps = -sum_c t*(s - lse), s = x - m: -(sum t*x - m*sum t) + lse*sum t
    const float nps = -((stx - m * st_) - lse * st_);
    const float g_lp_scale = -inv_n * gscale;
    const float g_lse = -(g_lp_scale * st_);  // -(sum_c t * (-1/B))
    const float g_se = __fmul_rn(__fmul_rn(kLn2, g_lse), 1.0f / __fmul_rn(se, kLn2));
    // g_s = t*g_lp_scale + log2e*((e*ln2)*g_se).  Its row sum feeds the
    // ReduceAxis(Max) gradient; it is exactly zero in real arithmetic
    // (g_se = -g_lp_scale*sum(t)/sum(e)), so any fp32 evaluation is rounding
    // residue.  It is taken from the row sums instead of a fourth pass.
    const float gsum = __fadd_rn(__fmul_rn(g_lp_scale, st_),
                                 __fmul_rn(__fmul_rn(__fmul_rn(kLog2e, kLn2), g_se), se));
    const float wmax = __fmul_rn(1.0f / cnt, -gsum);
    if (dx) {
      float4 *dv = reinterpret_cast<float4 *>(dx + row * (size_t)cols);
#pragma unroll
      for (int i = 0; i < NV; i++) {
        int j = lane + 32 * i;
        if (j < nv) {
          const float4 tt = tr[i];
          const float *te = reinterpret_cast<const float *>(&tt);
          const float *e = reinterpret_cast<const float *>(&xr[i]);
          float4 o;
          float *oe = reinterpret_cast<float *>(&o);
#pragma unroll
          for (int q = 0; q < 4; q++) {
            const float gs = __fadd_rn(__fmul_rn(te[q], g_lp_scale),
                                       __fmul_rn(kLog2e, __fmul_rn(__fmul_rn(e[q], kLn2), g_se)));
            const float mask = ((maxbits >> (4 * i + q)) & 1u) ? 1.0f : 0.0f;
            oe[q] = __fadd_rn(gs, __fmul_rn(mask, wmax));
          }
          __stcs(dv + j, o);
        }
      }
    }
    wloss += nps;
  }
  if (lane == 0 && gwarp < rows) warp_loss[gwarp] = wloss;
}

// Generic path (any cols): three sweeps over the row from global memory.
__global__ void __launch_bounds__(256) k_xent_rows_generic(const float *__restrict__ x,
                                                           const float *__restrict__ t,
                                                           float *__restrict__ dx,
                                                           float *__restrict__ warp_loss,
                                                           size_t rows, int cols, float inv_n,
                                                           float gscale) {
  const int lane = threadIdx.x & 31;
  size_t row = (size_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const size_t wstride = (size_t)gridDim.x * (blockDim.x >> 5);
  const size_t gwarp = row;
  float wloss = 0.f;
  for (; row < rows; row += wstride) {
    const float *xr = x + row * (size_t)cols;
    const float *tr = t + row * (size_t)cols;
    float m = -INFINITY;
    for (int c = lane; c < cols; c += 32) m = ref_max(m, xr[c]);
    m = warp_max(m);
    float se = 0.f, st_ = 0.f, sts = 0.f, cnt = 0.f;
    for (int c = lane; c < cols; c += 32) {
      float s = __fsub_rn(xr[c], m);
      se += exp2f(__fmul_rn(s, kLog2e));
      st_ += tr[c];
      sts += __fmul_rn(tr[c], s);
      cnt += (xr[c] < m) ? 0.0f : 1.0f;
    }
    se = warp_sum(se);
    st_ = warp_sum(st_);
    sts = warp_sum(sts);
    cnt = warp_sum(cnt);
    const float lse = __fmul_rn(log2f(se), kLn2);
    const float nps = -(sts - lse * st_);
    const float g_lp_scale = -inv_n * gscale;
    const float g_lse = -(g_lp_scale * st_);
    const float g_se = __fmul_rn(__fmul_rn(kLn2, g_lse), 1.0f / __fmul_rn(se, kLn2));
    float gsum = 0.f;
    for (int c = lane; c < cols; c += 32) {
      float e = exp2f(__fmul_rn(__fsub_rn(xr[c], m), kLog2e));
      gsum += __fadd_rn(__fmul_rn(tr[c], g_lp_scale),
                        __fmul_rn(kLog2e, __fmul_rn(__fmul_rn(e, kLn2), g_se)));
    }
    gsum = warp_sum(gsum);
    const float wmax = __fmul_rn(1.0f / cnt, -gsum);
    if (dx) {
      for (int c = lane; c < cols; c += 32) {
        float e = exp2f(__fmul_rn(__fsub_rn(xr[c], m), kLog2e));
        float gs = __fadd_rn(__fmul_rn(tr[c], g_lp_scale),
                             __fmul_rn(kLog2e, __fmul_rn(__fmul_rn(e, kLn2), g_se)));
        float mask = (xr[c] < m) ? 0.0f : 1.0f;
        dx[row * (size_t)cols + c] = __fadd_rn(gs, __fmul_rn(mask, wmax));
      }
    }
    wloss += nps;
  }
  if (lane == 0 && gwarp < rows) warp_loss[gwarp] = wloss;
}

// Sum of the row loss terms in a fixed order (one block, strided partials
// combined by a fixed tree), times 1/B.
// Sums the per-warp loss partials (count of them, in warp order).
__global__ void __launch_bounds__(1024) k_xent_loss_final(const float *__restrict__ warp_loss,
                                                          size_t count, float inv_n,
                                                          float *__restrict__ loss,
                                                          float loss_scale) {
  __shared__ float sh[32];
  float acc = 0.f;
  for (size_t r = threadIdx.x; r < count; r += blockDim.x) acc += warp_loss[r];
  acc = warp_sum(acc);
  if ((threadIdx.x & 31) == 0) sh[threadIdx.x >> 5] = acc;
  __syncthreads();
  if (threadIdx.x < 32) {
    float v = (threadIdx.x < (blockDim.x >> 5)) ? sh[threadIdx.x] : 0.f;
    v = warp_sum(v);
    if (threadIdx.x == 0) loss[0] = __fmul_rn(__fmul_rn(v, inv_n), loss_scale);
  }
}

// Number of per-warp partials a row kernel of `grid` 256-thread blocks writes.
static size_t xent_partials(int grid, size_t rows) {
  size_t w = (size_t)grid * 8;
  return w < rows ? w : rows;
}

int launch_xent(const float *x, const float *t, size_t rows, size_t cols, float *loss, float *dx,
                float gscale, cudaStream_t st, float *row_scratch, float loss_scale) {
  if (rows == 0 || cols == 0) return set_error(FG_ERR_INVALID, "cross_entropy: empty logits");
  if (cols > (size_t)INT32_MAX) return set_error(FG_ERR_UNSUPPORTED, "cross_entropy: cols too large");
  float *scratch = row_scratch;
  if (!scratch) {
    int status = FG_OK;
    scratch = (float *)workspace(rows * sizeof(float), &status);
    if (!scratch) return status;
  }
  const float inv_n = 1.0f / (float)rows;
  const int c = (int)cols;
  const bool vec = (cols % 4 == 0) && aligned16(x) && aligned16(t) && (!dx || aligned16(dx));
  // One resident wave: blocks per SM from the kernel's occupancy, so every
  // warp strides over (almost) the same number of rows.
  int per_sm = 4;
  {
    const void *kern = (vec && cols <= 128)    ? (const void *)k_xent_rows_v4<1>
                       : (vec && cols <= 256)  ? (const void *)k_xent_rows_v4<2>
                       : (vec && cols <= 512)  ? (const void *)k_xent_rows_v4<4>
                       : (vec && cols <= 1024) ? (const void *)k_xent_rows_v4<8>
                                               : (const void *)k_xent_rows_generic;
    int occ = 0;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, kern, 256, 0) == cudaSuccess && occ > 0)
      per_sm = occ;
  }
  int grid = grid_for(rows * 32, 256, per_sm);
  if (vec && cols <= 128)
    k_xent_rows_v4<1><<<grid, 256, 0, st>>>(x, t, dx, scratch, rows, c, inv_n, gscale);
  else if (vec && cols <= 256)
    k_xent_rows_v4<2><<<grid, 256, 0, st>>>(x, t, dx, scratch, rows, c, inv_n, gscale);
  else if (vec && cols <= 512)
    k_xent_rows_v4<4><<<grid, 256, 0, st>>>(x, t, dx, scratch, rows, c, inv_n, gscale);
  else if (vec && cols <= 1024)
    k_xent_rows_v4<8><<<grid, 256, 0, st>>>(x, t, dx, scratch, rows, c, inv_n, gscale);
  else
    k_xent_rows_generic<<<grid, 256, 0, st>>>(x, t, dx, scratch, rows, c, inv_n, gscale);
  FG_LAUNCH_TRY();
  k_xent_loss_final<<<1, 1024, 0, st>>>(scratch, xent_partials(grid, rows), inv_n, loss,
                                        loss_scale);
  FG_LAUNCH_TRY();
  return FG_OK;
}

// ---------------------------------------------------------------------------
// Dataset path: IDX pixels (u8) -> f32 / divisor on the device, and dense
// one-hot targets, so a dataset is uploaded once as bytes and stays resident.
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(256) k_u8_to_f32_div(const uint8_t *__restrict__ src,
                                                       float *__restrict__ dst, size_t n,
                                                       float divisor) {
  const size_t stride = (size_t)gridDim.x * blockDim.x;
  size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
  const size_t n16 = (((uintptr_t)src | (uintptr_t)dst) & 15) == 0 ? n / 16 : 0;
  for (size_t v = i; v < n16; v += stride) {
    const uint4 u = __ldcs(reinterpret_cast<const uint4 *>(src) + v);
    const uint8_t *b = reinterpret_cast<const uint8_t *>(&u);
    float4 *o = reinterpret_cast<float4 *>(dst + v * 16);
#pragma unroll
    for (int q = 0; q < 4; q++)
      __stcs(o + q, make_float4(__fdiv_rn((float)b[4 * q], divisor),
                                __fdiv_rn((float)b[4 * q + 1], divisor),
                                __fdiv_rn((float)b[4 * q + 2], divisor),
                                __fdiv_rn((float)b[4 * q + 3], divisor)));
  }
  for (size_t j = n16 * 16 + i; j < n; j += stride) dst[j] = __fdiv_rn((float)src[j], divisor);
}

__global__ void __launch_bounds__(256) k_one_hot_u8(const uint8_t *__restrict__ labels,
                                                    float *__restrict__ out, size_t n,
                                                    int classes) {
  const size_t total = n * (size_t)classes;
  const size_t stride = (size_t)gridDim.x * blockDim.x;
  for (size_t j = (size_t)blockIdx.x * blockDim.x + threadIdx.x; j < total; j += stride) {
    const size_t row = j / (size_t)classes;
    const int c = (int)(j - row * (size_t)classes);
    out[j] = (int)labels[row] == c ? 1.0f : 0.0f;
  }
}

// ---------------------------------------------------------------------------
// SGD (src/optim.rs:60-71): p = p + (-(g*lr)); optional TF32 residual of p.
// ---------------------------------------------------------------------------
__device__ __forceinline__ float sgd_one(float p, float g, float lr) {
  return __fadd_rn(p, -__fmul_rn(g, lr));
}
__device__ __forceinline__ float tf32_lo(float v) {
  float hi = __uint_as_float(__float_as_uint(v) & 0xffffe000u);
  return __fsub_rn(v, hi);
}

__global__ void __launch_bounds__(256) k_sgd_multi(SgdSegments segs, float lr) {
  for (int s = 0; s < segs.count; s++) {
    float *p = segs.p[s];
    const float *g = segs.g[s];
    float *lo = segs.lo[s];
    const size_t n = segs.n[s];
    const bool vec = ((((uintptr_t)p) | ((uintptr_t)g) | ((uintptr_t)lo)) & 15) == 0;
    size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
    const size_t stride = (size_t)gridDim.x * blockDim.x;
    size_t done = 0;
    if (vec) {
      const size_t n4 = n / 4;
      for (size_t j = i; j < n4; j += stride) {
        float4 pv = reinterpret_cast<float4 *>(p)[j];
        float4 gv = __ldcs(reinterpret_cast<const float4 *>(g) + j);
        pv.x = sgd_one(pv.x, gv.x, lr); pv.y = sgd_one(pv.y, gv.y, lr);
        pv.z = sgd_one(pv.z, gv.z, lr); pv.w = sgd_one(pv.w, gv.w, lr);
        reinterpret_cast<float4 *>(p)[j] = pv;
        if (lo) {
          float4 lv = make_float4(tf32_lo(pv.x), tf32_lo(pv.y), tf32_lo(pv.z), tf32_lo(pv.w));
          reinterpret_cast<float4 *>(lo)[j] = lv;
        }
      }
      done = n4 * 4;
    }
    for (size_t j = done + i; j < n; j += stride) {
      float v = sgd_one(p[j], g[j], lr);
      p[j] = v;
      if (lo) lo[j] = tf32_lo(v);
    }
  }
}

int launch_sgd_multi(const SgdSegments &segs, float lr, cudaStream_t st) {
  size_t maxn = 0;
  for (int s = 0; s < segs.count; s++) maxn = segs.n[s] > maxn ? segs.n[s] : maxn;
  if (!maxn) return FG_OK;
  k_sgd_multi<<<grid_for(maxn / 4 + 1, 256, 16), 256, 0, st>>>(segs, lr);
  FG_LAUNCH_TRY();
  return FG_OK;
}

__global__ void __launch_bounds__(256) k_split_lo(const float *__restrict__ x,
                                                  float *__restrict__ lo, size_t n) {
  const size_t stride = (size_t)gridDim.x * blockDim.x;
  size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
  const bool vec = ((((uintptr_t)x) | ((uintptr_t)lo)) & 15) == 0;
  size_t done = 0;
  if (vec) {
    const size_t n4 = n / 4;
    for (size_t j = i; j < n4; j += stride) {
      float4 v = __ldcs(reinterpret_cast<const float4 *>(x) + j);
      float4 o = make_float4(tf32_lo(v.x), tf32_lo(v.y), tf32_lo(v.z), tf32_lo(v.w));
      __stcs(reinterpret_cast<float4 *>(lo) + j, o);
    }
    done = n4 * 4;
  }
  for (size_t j = done + i; j < n; j += stride) lo[j] = tf32_lo(x[j]);
}

int launch_split_lo(const float *x, float *lo, size_t n, cudaStream_t st) {
  if (!n) return FG_OK;
  k_split_lo<<<grid_for(n / 4 + 1, 256, 16), 256, 0, st>>>(x, lo, n);
  FG_LAUNCH_TRY();
  return FG_OK;
}

// dst_a <- src_a (na floats) and dst_b <- src_b (nb floats) in one launch on
// the SMs; every pointer 16-byte aligned, na and nb multiples of 4.  A
// device-to-device cudaMemcpyAsync may be given to a copy engine that is
// busy with a long host upload, so the step's own staging copy is a kernel.
__global__ void __launch_bounds__(256) k_copy2(const float4 *__restrict__ src_a,
                                               float4 *__restrict__ dst_a, size_t na4,
                                               const float4 *__restrict__ src_b,
                                               float4 *__restrict__ dst_b, size_t nb4) {
  const size_t stride = (size_t)gridDim.x * blockDim.x;
  const size_t i0 = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
  for (size_t i = i0; i < na4; i += stride) __stcs(dst_a + i, __ldcs(src_a + i));
  for (size_t i = i0; i < nb4; i += stride) __stcs(dst_b + i, __ldcs(src_b + i));
}

int launch_copy2(const float *src_a, float *dst_a, size_t na, const float *src_b, float *dst_b,
                 size_t nb, cudaStream_t st) {
  if (na % 4 || nb % 4 || !aligned16(src_a) || !aligned16(dst_a) || (nb && (!aligned16(src_b) ||
      !aligned16(dst_b))))
    return set_error(FG_ERR_INVALID, "copy2: sizes must be multiples of 4 floats, 16-byte aligned");
  const size_t n4 = (na > nb ? na : nb) / 4;
  if (!n4) return FG_OK;
  k_copy2<<<grid_for(n4, 256, 16), 256, 0, st>>>(reinterpret_cast<const float4 *>(src_a),
                                                 reinterpret_cast<float4 *>(dst_a), na / 4,
                                                 reinterpret_cast<const float4 *>(src_b),
                                                 reinterpret_cast<float4 *>(dst_b), nb / 4);
  FG_LAUNCH_TRY();
  return FG_OK;
}

}  // namespace fg

extern "C" {

int fg_ew_fma_relu_scale(const float *d_a, const float *d_b, const float *d_c, float *d_out,
                         size_t n, float scale, void *stream) {
  FG_REQUIRE(n == 0 || (d_a && d_b && d_c && d_out), "fg_ew_fma_relu_scale: null pointer");
  return fg::launch_ew_fma_relu_scale(d_a, d_b, d_c, d_out, n, scale, (cudaStream_t)stream);
}

int fg_reduce_rows(int dtype, int op, const void *d_x, void *d_out, size_t rows, size_t cols,
                   void *stream) {
  FG_REQUIRE(dtype == FG_F32 || dtype == FG_I32, "fg_reduce_rows: dtype must be F32 or I32");
  FG_REQUIRE(op == FG_REDUCE_SUM || op == FG_REDUCE_MAX, "fg_reduce_rows: unknown op %d", op);
  FG_REQUIRE(rows == 0 || (d_out && (cols == 0 || d_x)), "fg_reduce_rows: null pointer");
  return fg::launch_reduce_rows(dtype, op, d_x, d_out, rows, cols, (cudaStream_t)stream);
}

int fg_reduce_cols(int dtype, int op, const void *d_x, void *d_out, size_t rows, size_t cols,
                   void *stream) {
  FG_REQUIRE(dtype == FG_F32 || dtype == FG_I32, "fg_reduce_cols: dtype must be F32 or I32");
  FG_REQUIRE(op == FG_REDUCE_SUM || op == FG_REDUCE_MAX, "fg_reduce_cols: unknown op %d", op);
  FG_REQUIRE(cols == 0 || (d_out && (rows == 0 || d_x)), "fg_reduce_cols: null pointer");
  return fg::launch_reduce_cols(dtype, op, d_x, d_out, rows, cols, (cudaStream_t)stream, nullptr, 0);
}

int fg_xent_fwd_bwd(const float *d_logits, const float *d_targets, size_t rows, size_t cols,
                    float *d_loss, float *d_dx, float grad_scale, void *stream) {
  FG_REQUIRE(d_logits && d_targets && d_loss, "fg_xent_fwd_bwd: null pointer");
  return fg::launch_xent(d_logits, d_targets, rows, cols, d_loss, d_dx, grad_scale,
                         (cudaStream_t)stream, nullptr, 1.0f);
}

}  // extern "C"

// ---------------------------------------------------------------------------
// Cross-entropy without any device allocation.
//
// Some callers cannot allocate device memory once they are running: a host
// that reserves its whole device-memory budget at start-up (a serving
// process, or a runtime with its own pool) and must not call cudaMalloc later,
// because cudaMalloc / cudaFree can synchronise the device, can fail under
// fragmentation in the middle of a job, and bypass the caller's accounting.
// fg_xent_fwd_bwd_noalloc gives them the cross-entropy kernel with its
// per-row scratch in this file-scope array instead of the library's growable
// workspace.  The array is part of the library's device image, so every GPU
// that loads the library holds it (kFgXentNoallocMaxRows floats, 1 MiB)
// until the process exits.
//
// In host code the array's name is only a host-side stand-in, not a device
// address: the launcher passes the address that cudaGetSymbolAddress returned
// for the current device.  All calls share the array and each call
// overwrites every row it uses before reading it (nothing needs to start at
// zero), so calls that overlap on the GPU -- two streams, or two threads --
// race on it and must be serialised by the caller.
// ---------------------------------------------------------------------------
static __device__ __align__(256) float g_xent_noalloc_scratch[kFgXentNoallocMaxRows];

namespace fg {
namespace {

struct NoallocDevice {
  float *scratch = nullptr;  // device address of g_xent_noalloc_scratch
  int sms = 0;
  bool ready = false;
};
std::mutex g_noalloc_mu;
NoallocDevice g_noalloc[64];

// Once per device, with that device current: resolve the array's device
// address and the SM count.  Neither call allocates by itself, but under
// lazy module loading the symbol lookup (like the first launch of any kernel
// of this library) loads the library's device code on this device, and that
// allocates the array and the code; callers warm up once per device before
// they reserve their memory budget.
int noalloc_setup(NoallocDevice **out) {
  int dev = 0;
  FG_CUDA_TRY(cudaGetDevice(&dev));
  if (dev < 0 || dev >= 64) return set_error(FG_ERR_UNSUPPORTED, "device ordinal %d", dev);
  std::lock_guard<std::mutex> lock(g_noalloc_mu);
  NoallocDevice &d = g_noalloc[dev];
  if (!d.ready) {
    void *p = nullptr;
    cudaError_t e = cudaGetSymbolAddress(&p, g_xent_noalloc_scratch);
    if (e != cudaSuccess || !p)
      return set_error(FG_ERR_CUDA, "cudaGetSymbolAddress(g_xent_noalloc_scratch) failed: %s",
                       cudaGetErrorString(e));
    FG_CUDA_TRY(cudaDeviceGetAttribute(&d.sms, cudaDevAttrMultiProcessorCount, dev));
    d.scratch = (float *)p;
    d.ready = true;
  }
  *out = &d;
  return FG_OK;
}

}  // namespace
}  // namespace fg

extern "C" {

int fg_xent_fwd_bwd_noalloc(const float *d_logits, const float *d_targets, size_t rows,
                            size_t cols, float *d_loss, float *d_dx, float grad_scale,
                            void *stream) {
  FG_REQUIRE(d_logits && d_targets && d_loss, "fg_xent_fwd_bwd_noalloc: null pointer");
  FG_REQUIRE(rows > 0 && cols > 0, "fg_xent_fwd_bwd_noalloc: empty logits");
  FG_REQUIRE(rows <= (size_t)kFgXentNoallocMaxRows,
             "fg_xent_fwd_bwd_noalloc: %zu rows exceed the static scratch limit of %d rows", rows,
             kFgXentNoallocMaxRows);
  FG_REQUIRE(cols <= (size_t)INT32_MAX, "fg_xent_fwd_bwd_noalloc: cols too large");
  fg::NoallocDevice *nd = nullptr;
  int rc = fg::noalloc_setup(&nd);
  if (rc) return rc;
  cudaStream_t st = (cudaStream_t)stream;
  const float inv_n = 1.0f / (float)rows;
  const int c = (int)cols;
  size_t want = (rows * 32 + 255) / 256;
  size_t cap = (size_t)nd->sms * 16;
  const int grid = (int)(want < cap ? (want ? want : 1) : cap);
  const bool vec = (cols % 4 == 0) && fg::aligned16(d_logits) && fg::aligned16(d_targets) &&
                   (!d_dx || fg::aligned16(d_dx));
  float *scratch = nd->scratch;
  if (vec && cols <= 128)
    fg::k_xent_rows_v4<1><<<grid, 256, 0, st>>>(d_logits, d_targets, d_dx, scratch, rows, c, inv_n, grad_scale);
  else if (vec && cols <= 256)
    fg::k_xent_rows_v4<2><<<grid, 256, 0, st>>>(d_logits, d_targets, d_dx, scratch, rows, c, inv_n, grad_scale);
  else if (vec && cols <= 512)
    fg::k_xent_rows_v4<4><<<grid, 256, 0, st>>>(d_logits, d_targets, d_dx, scratch, rows, c, inv_n, grad_scale);
  else if (vec && cols <= 1024)
    fg::k_xent_rows_v4<8><<<grid, 256, 0, st>>>(d_logits, d_targets, d_dx, scratch, rows, c, inv_n, grad_scale);
  else
    fg::k_xent_rows_generic<<<grid, 256, 0, st>>>(d_logits, d_targets, d_dx, scratch, rows, c, inv_n, grad_scale);
  FG_LAUNCH_TRY();
  fg::k_xent_loss_final<<<1, 1024, 0, st>>>(scratch, fg::xent_partials(grid, rows), inv_n,
                                            d_loss, 1.0f);
  FG_LAUNCH_TRY();
  return FG_OK;
}

int fg_u8_to_f32_div(const uint8_t *d_src, float *d_dst, size_t n, float divisor, void *stream) {
  FG_REQUIRE(n == 0 || (d_src && d_dst), "fg_u8_to_f32_div: null pointer");
  FG_REQUIRE(divisor != 0.0f, "fg_u8_to_f32_div: zero divisor");
  if (n == 0) return FG_OK;
  fg::k_u8_to_f32_div<<<fg::grid_for(n / 16 + 1, 256, 16), 256, 0, (cudaStream_t)stream>>>(
      d_src, d_dst, n, divisor);
  FG_LAUNCH_TRY();
  return FG_OK;
}

int fg_one_hot_u8(const uint8_t *d_labels, float *d_out, size_t n, int classes, void *stream) {
  FG_REQUIRE(classes > 0 && classes <= 256, "fg_one_hot_u8: classes must be in 1..256");
  FG_REQUIRE(n == 0 || (d_labels && d_out), "fg_one_hot_u8: null pointer");
  if (n == 0) return FG_OK;
  fg::k_one_hot_u8<<<fg::grid_for(n * (size_t)classes, 256, 16), 256, 0, (cudaStream_t)stream>>>(
      d_labels, d_out, n, classes);
  FG_LAUNCH_TRY();
  return FG_OK;
}

int fg_sgd(float *d_p, const float *d_g, size_t n, float lr, float *d_p_lo, void *stream) {
  FG_REQUIRE(n == 0 || (d_p && d_g), "fg_sgd: null pointer");
  fg::SgdSegments s{};
  s.count = 1;
  s.p[0] = d_p;
  s.g[0] = d_g;
  s.lo[0] = d_p_lo;
  s.n[0] = n;
  return fg::launch_sgd_multi(s, lr, (cudaStream_t)stream);
}

int fg_split_lo(const float *d_x, float *d_lo, size_t n, void *stream) {
  FG_REQUIRE(n == 0 || (d_x && d_lo), "fg_split_lo: null pointer");
  return fg::launch_split_lo(d_x, d_lo, n, (cudaStream_t)stream);
}

int fg_kernel_arch(int *binary_version, int *ptx_version) {
  FG_REQUIRE(binary_version, "fg_kernel_arch: null pointer");
  cudaFuncAttributes a;
  FG_CUDA_TRY(cudaFuncGetAttributes(&a, fg::k_split_lo));
  *binary_version = a.binaryVersion;
  if (ptx_version) *ptx_version = a.ptxVersion;
  return FG_OK;
}

}  // extern "C"
