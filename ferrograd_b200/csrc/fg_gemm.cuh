// 3xTF32 tcgen05 GEMM plans (fg_gemm.cu), shared with the MLP step.
#pragma once
#include <cuda.h>
#include <cuda_runtime.h>

namespace fg {
namespace gemm {

struct GemmParams {
  int M, N, K;
  float *C;
  float *C_lo;
  int ldc;
  const float *bias;
  const float *mask;
  int ldmask;
  int epilogue;
  int one_pass;
  int a3d, b3d;  // MN-major operand loaded as one 3-D box (MN % 32 == 0)
  unsigned int *err;
  // Stream-K tail (set per launch): tiles [0, dp_tiles) are computed whole,
  // tile t by CTA t % grid, in waves; the k-blocks of the remaining tiles,
  // sk_units of them in (tile, k) order, are split evenly over the grid.  A
  // CTA whose range ends inside a tile leaves its partial accumulator in
  // sk_ws[blockIdx.x] and sets sk_flags[blockIdx.x]; the CTA holding that
  // tile's last k-block adds the partials in CTA order and writes C.
  int dp_tiles;
  long long sk_units;
  float *sk_ws;             // [grid][BM * BN] partial accumulators
  unsigned int *sk_flags;   // [grid], zero between launches
  // Segmented accumulation: the tensor cores accumulate at most seg_kb
  // k-blocks into a fresh TMEM accumulator; the epilogue warps add the
  // segments' sums with round-to-nearest fp32 adds in a per-CTA running
  // partial (seg_ws[blockIdx.x], [BN][BM] floats, L2-resident).  The
  // tensor cores' own fp32 accumulation rounds its additions coarsely, so
  // its error grows with the length of one accumulation chain; cutting the
  // chain bounds it.  seg_kb == 0 or no seg_ws: one chain per output tile.
  int seg_kb;
  float *seg_ws;
};

// Everything a launch needs, built once per (shape, pointers) and replayed.
struct GemmPlan {
  CUtensorMap a, alo, b, blo;
  GemmParams p;
  int bn;
  int bk;  // 8, 16 or 32 fp32 elements per k-block (FG_GEMM_BK, default 16)
  bool a_mn, b_mn;
  int max_ctas;  // persistent grid cap (0: one CTA per SM); leaves SMs to a concurrent collective
  // Stream-K workspace (null: whole tiles only).  Launches that share one
  // workspace must be ordered (same stream).
  float *sk_ws;
  unsigned int *sk_flags;
  float *seg_ws;  // running partials of segmented accumulation (null: off)
};

// Bytes of stream-K + segment workspace a plan needs for grids of up to
// `ctas` CTAs.
size_t stream_k_ws_bytes(int ctas);
// Lays out a zeroed workspace of stream_k_ws_bytes(ctas) bytes for plans.
void stream_k_attach(GemmPlan *pl, void *ws, int ctas);
// Per-(device, stream) workspace for one-shot launches (fg_gemm_3xtf32).
void attach_stream_ws(GemmPlan *pl, cudaStream_t st);

int make_plan(int M, int N, int K, const float *a, const float *a_lo, int lda, const float *b,
              const float *b_lo, int ldb, float *c, float *c_lo, int ldc, int flags, int epilogue,
              const float *bias, const float *mask, int ldmask, GemmPlan *pl);
int run_plan(const GemmPlan &pl, cudaStream_t st);

}  // namespace gemm
}  // namespace fg
