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
};

// Everything a launch needs, built once per (shape, pointers) and replayed.
struct GemmPlan {
  CUtensorMap a, alo, b, blo;
  GemmParams p;
  int bn;
  bool a_mn, b_mn;
  int max_ctas;  // persistent grid cap (0: one CTA per SM); leaves SMs to a concurrent collective
};

int make_plan(int M, int N, int K, const float *a, const float *a_lo, int lda, const float *b,
              const float *b_lo, int ldb, float *c, float *c_lo, int ldc, int flags, int epilogue,
              const float *bias, const float *mask, int ldmask, GemmPlan *pl);
int run_plan(const GemmPlan &pl, cudaStream_t st);

}  // namespace gemm
}  // namespace fg
