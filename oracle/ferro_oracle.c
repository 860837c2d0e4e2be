/*
 * ferro_oracle.c -- TEST INFRASTRUCTURE ONLY.
 *
 * A plain-C restatement of the arithmetic that ferrograd's clang CPU backend
 * performs for the MLP training path (forward -> cross_entropy -> backward ->
 * Sgd::step).  It is the parity oracle for the CUDA kernels and the timed CPU
 * baseline.  Nothing in the product path links or calls it: only tests/,
 * __graft_entry__.smoke() and bench.py's cpu_baseline / reference legs do.
 *
 * The reference (Rust) cannot be built on this machine (no rustc, no clang),
 * so this is a port.  It is pinned against every known-answer test the
 * reference ships for this path (tests/test_oracle_golden.py).
 *
 * Rules restated here, each from the reference source:
 *  - One C statement per op, no FMA contraction: the reference renders every
 *    ALU op as its own statement (src/codegen/clang.rs:205-239) and clang's
 *    default -ffp-contract=on does not fuse across statements.  Build with
 *    -ffp-contract=off -fno-fast-math to keep that.
 *  - exp2 / log2 are the DOUBLE libm calls on float arguments, rounded back
 *    to float on assignment (src/codegen/clang.rs:218-219).
 *  - max renders as ((a>b)?a:b) (src/codegen/clang.rs:224).
 *  - Reduction order (src/optimize/unroll.rs:36,41-66 and
 *    src/devectorize.rs:206-225,274-347): when the innermost reduce range has
 *    size R > 4 and R % 4 == 0 it is split into outer R/4 x inner 4 and each
 *    step does acc = acc OP (((v0 OP v1) OP v2) OP v3); otherwise
 *    acc = acc OP v sequentially.  Identity 0 (add) or -inf (max).
 *  - The i32 max identity is (int)(-INFINITY) in the reference, which is
 *    undefined behaviour in C; it is defined here as INT32_MIN.
 */
#include <float.h>
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif

#define ORC_SUM 0
#define ORC_MAX 1
#define ORC_UNROLL 4 /* REDUCE_UNROLL_FACTOR, src/optimize/unroll.rs:36 */

/* std::f32::consts::LOG2_E / LN_2 as f32 (src/tensor.rs:697-707); the f64
 * LN_2 constant from src/gradient.rs:114,119 prints as a float literal with an
 * 'f' suffix (src/codegen/clang.rs:104-111), which rounds to the same float. */
static const float LOG2E_F = 1.44269504088896340736f;
static const float LN2_F = 0.693147180559945309417f;

/* The reference's OPT "unroll" pass (src/optimize/mod.rs:80-112): with it
 * off (OPT=0, or a pass list without "unroll") every reduction is
 * sequential. */
static int orc_unroll_on = 1;
void orc_set_unroll(int on) { orc_unroll_on = on != 0; }
static int orc_blocked(long n) { return orc_unroll_on && n > ORC_UNROLL && n % ORC_UNROLL == 0; }
static inline float orc_maxf(float a, float b) { return (a > b) ? a : b; }
static inline int32_t orc_maxi(int32_t a, int32_t b) { return (a > b) ? a : b; }
static inline int32_t orc_addi(int32_t a, int32_t b) {
  return (int32_t)((uint32_t)a + (uint32_t)b);
}

void orc_set_threads(int n) {
#ifdef _OPENMP
  omp_set_num_threads(n > 0 ? n : 1);
#else
  (void)n;
#endif
}

int orc_max_threads(void) {
#ifdef _OPENMP
  return omp_get_max_threads();
#else
  return 1;
#endif
}

/* ---------------------------------------------------------------------------
 * Parameter init: src/nn.rs:12-47.  Thread-local LCG seeded with 42 that keeps
 * running across layers in construction order; Box-Muller pairs pushed
 * cos then sin; std = sqrt(2 / fan_in).  All f32 arithmetic, glibc logf /
 * cosf / sinf (what Rust's f32::ln / cos / sin lower to on Linux).
 * ------------------------------------------------------------------------- */
static float orc_next_unit(uint64_t *state) {
  uint64_t next = (*state) * 6364136223846793005ULL + 1ULL; /* wrapping */
  *state = next;
  return (float)(next >> 33) / (float)(1ULL << 31);
}

void orc_kaiming_normal(float *out, long numel, long fan_in, uint64_t *state) {
  float stdv = sqrtf(2.0f / (float)fan_in);
  long n = 0;
  while (n < numel) {
    float u1 = orc_next_unit(state);
    if (!(u1 >= FLT_MIN)) u1 = FLT_MIN; /* u1.max(f32::MIN_POSITIVE) */
    float u2 = orc_next_unit(state);
    float lg = logf(u1);
    float m2 = -2.0f * lg;
    float radius = sqrtf(m2) * stdv;
    float two_pi = 2.0f * 3.14159265358979323846f;
    float theta = two_pi * u2;
    out[n++] = radius * cosf(theta);
    if (n < numel) out[n++] = radius * sinf(theta);
  }
}

/* ---------------------------------------------------------------------------
 * Reductions: Tensor::sum / Tensor::max (src/tensor.rs:665-693) lowered by
 * src/schedule/indexing.rs:184-217, src/optimize/unroll.rs:41-113 and
 * src/devectorize.rs:206-347.
 * ------------------------------------------------------------------------- */
void orc_reduce_last_f32(const float *x, long rows, long cols, int op, float *out) {
  const int blocked = orc_blocked(cols);
#pragma omp parallel for schedule(static)
  for (long r = 0; r < rows; r++) {
    const float *p = x + r * cols;
    float acc = (op == ORC_MAX) ? -INFINITY : 0.0f;
    if (blocked) {
      for (long c = 0; c < cols; c += 4) {
        float g;
        if (op == ORC_MAX) {
          g = orc_maxf(p[c], p[c + 1]);
          g = orc_maxf(g, p[c + 2]);
          g = orc_maxf(g, p[c + 3]);
          acc = orc_maxf(acc, g);
        } else {
          g = p[c] + p[c + 1];
          g = g + p[c + 2];
          g = g + p[c + 3];
          acc = acc + g;
        }
      }
    } else {
      for (long c = 0; c < cols; c++)
        acc = (op == ORC_MAX) ? orc_maxf(acc, p[c]) : acc + p[c];
    }
    out[r] = acc;
  }
}

void orc_reduce_last_i32(const int32_t *x, long rows, long cols, int op, int32_t *out) {
  const int blocked = orc_blocked(cols);
#pragma omp parallel for schedule(static)
  for (long r = 0; r < rows; r++) {
    const int32_t *p = x + r * cols;
    int32_t acc = (op == ORC_MAX) ? INT32_MIN : 0;
    if (blocked) {
      for (long c = 0; c < cols; c += 4) {
        if (op == ORC_MAX) {
          int32_t g = orc_maxi(orc_maxi(orc_maxi(p[c], p[c + 1]), p[c + 2]), p[c + 3]);
          acc = orc_maxi(acc, g);
        } else {
          int32_t g = orc_addi(orc_addi(orc_addi(p[c], p[c + 1]), p[c + 2]), p[c + 3]);
          acc = orc_addi(acc, g);
        }
      }
    } else {
      for (long c = 0; c < cols; c++)
        acc = (op == ORC_MAX) ? orc_maxi(acc, p[c]) : orc_addi(acc, p[c]);
    }
    out[r] = acc;
  }
}

/* Reduce over axis 0 of a row-major [rows, cols] matrix: the reduce range is
 * the row axis, so the blocking rule applies to `rows`. */
#define ORC_COLCHUNK 256
void orc_reduce_axis0_f32(const float *x, long rows, long cols, int op, float *out) {
  const int blocked = orc_blocked(rows);
  long nchunks = (cols + ORC_COLCHUNK - 1) / ORC_COLCHUNK;
#pragma omp parallel for schedule(static)
  for (long ch = 0; ch < nchunks; ch++) {
    long c0 = ch * ORC_COLCHUNK;
    long w = cols - c0 < ORC_COLCHUNK ? cols - c0 : ORC_COLCHUNK;
    float acc[ORC_COLCHUNK];
    for (long j = 0; j < w; j++) acc[j] = (op == ORC_MAX) ? -INFINITY : 0.0f;
    if (blocked) {
      for (long r = 0; r < rows; r += 4) {
        const float *p0 = x + r * cols + c0, *p1 = p0 + cols, *p2 = p1 + cols, *p3 = p2 + cols;
        if (op == ORC_MAX) {
          for (long j = 0; j < w; j++) {
            float g = orc_maxf(orc_maxf(orc_maxf(p0[j], p1[j]), p2[j]), p3[j]);
            acc[j] = orc_maxf(acc[j], g);
          }
        } else {
          for (long j = 0; j < w; j++) {
            float g = p0[j] + p1[j];
            g = g + p2[j];
            g = g + p3[j];
            acc[j] = acc[j] + g;
          }
        }
      }
    } else {
      for (long r = 0; r < rows; r++) {
        const float *p = x + r * cols + c0;
        for (long j = 0; j < w; j++)
          acc[j] = (op == ORC_MAX) ? orc_maxf(acc[j], p[j]) : acc[j] + p[j];
      }
    }
    for (long j = 0; j < w; j++) out[c0 + j] = acc[j];
  }
}

void orc_reduce_axis0_i32(const int32_t *x, long rows, long cols, int op, int32_t *out) {
  const int blocked = orc_blocked(rows);
#pragma omp parallel for schedule(static)
  for (long c = 0; c < cols; c++) {
    int32_t acc = (op == ORC_MAX) ? INT32_MIN : 0;
    long step = blocked ? 4 : 1;
    for (long r = 0; r < rows; r += step) {
      if (blocked) {
        const int32_t v0 = x[r * cols + c], v1 = x[(r + 1) * cols + c];
        const int32_t v2 = x[(r + 2) * cols + c], v3 = x[(r + 3) * cols + c];
        int32_t g = (op == ORC_MAX) ? orc_maxi(orc_maxi(orc_maxi(v0, v1), v2), v3)
                                    : orc_addi(orc_addi(orc_addi(v0, v1), v2), v3);
        acc = (op == ORC_MAX) ? orc_maxi(acc, g) : orc_addi(acc, g);
      } else {
        acc = (op == ORC_MAX) ? orc_maxi(acc, x[r * cols + c]) : orc_addi(acc, x[r * cols + c]);
      }
    }
    out[c] = acc;
  }
}

/* ---------------------------------------------------------------------------
 * Elementwise chain relu(a*b+c)*s: Tensor::mul / add / relu
 * (src/tensor.rs:471-491,519-531).  relu is where(0 < x, x, zeros) with a
 * real zero buffer, so the false branch is +0.0f.
 * ------------------------------------------------------------------------- */
void orc_ew_fma_relu_scale(const float *a, const float *b, const float *c, float *out, long n,
                           float scale) {
#pragma omp parallel for schedule(static)
  for (long i = 0; i < n; i++) {
    float t = a[i] * b[i];
    t = t + c[i];
    float r = (0.0f < t) ? t : 0.0f;
    out[i] = r * scale;
  }
}

void orc_relu(const float *x, float *out, long n) {
  for (long i = 0; i < n; i++) out[i] = (0.0f < x[i]) ? x[i] : 0.0f;
}

/* ---------------------------------------------------------------------------
 * Contractions.  Tensor::matmul (src/tensor.rs:762-778) is
 * sum_k(expand(A)[m,n,k] * expand(Bt)[m,n,k]) with Bt = rhs.permute.contiguous,
 * i.e. [N, K].  Its two backward contractions come from the Mul and Expand
 * gradient rules (src/gradient.rs:100-106,165-176):
 *   dA[m,k]  = sum_n Bt[n,k] * G[m,n]   (ReduceAxis over axis 1)
 *   dBt[n,k] = sum_m A[m,k]  * G[m,n]   (ReduceAxis over axis 0)
 * Each product is one rounded f32 multiply; the sum follows the blocking rule
 * on the reduced extent.
 * ------------------------------------------------------------------------- */
#define ORC_NCHUNK 64

/* C[m,n] = sum_k A[m,k]*B[n,k]  (+ bias[n] if bias != NULL, as (acc + b)). */
void orc_gemm_fwd(const float *A, const float *B, const float *bias, long M, long N, long K,
                  float *C) {
  float *Bt = (float *)malloc(sizeof(float) * (size_t)K * (size_t)N);
  for (long n = 0; n < N; n++)
    for (long k = 0; k < K; k++) Bt[k * N + n] = B[n * K + k];
  const int blocked = orc_blocked(K);
  long nchunks = (N + ORC_NCHUNK - 1) / ORC_NCHUNK;
#pragma omp parallel for collapse(2) schedule(static)
  for (long m = 0; m < M; m++) {
    for (long ch = 0; ch < nchunks; ch++) {
      long n0 = ch * ORC_NCHUNK;
      long w = N - n0 < ORC_NCHUNK ? N - n0 : ORC_NCHUNK;
      float acc[ORC_NCHUNK];
      const float *a = A + m * K;
      for (long j = 0; j < w; j++) acc[j] = 0.0f;
      if (blocked) {
        for (long k = 0; k < K; k += 4) {
          const float a0 = a[k], a1 = a[k + 1], a2 = a[k + 2], a3 = a[k + 3];
          const float *b0 = Bt + k * N + n0, *b1 = b0 + N, *b2 = b1 + N, *b3 = b2 + N;
          for (long j = 0; j < w; j++) {
            float p0 = a0 * b0[j];
            float p1 = a1 * b1[j];
            float p2 = a2 * b2[j];
            float p3 = a3 * b3[j];
            float g = p0 + p1;
            g = g + p2;
            g = g + p3;
            acc[j] = acc[j] + g;
          }
        }
      } else {
        for (long k = 0; k < K; k++) {
          const float ak = a[k];
          const float *bk = Bt + k * N + n0;
          for (long j = 0; j < w; j++) {
            float p = ak * bk[j];
            acc[j] = acc[j] + p;
          }
        }
      }
      float *c = C + m * N + n0;
      if (bias) {
        for (long j = 0; j < w; j++) c[j] = acc[j] + bias[n0 + j];
      } else {
        for (long j = 0; j < w; j++) c[j] = acc[j];
      }
    }
  }
  free(Bt);
}

/* dA[m,k] = sum_n Bt[n,k] * G[m,n]   (G: [M,N], Bt: [N,K]) */
void orc_gemm_dx(const float *G, const float *Bt, long M, long N, long K, float *dA) {
  const int blocked = orc_blocked(N);
  long kchunks = (K + ORC_NCHUNK - 1) / ORC_NCHUNK;
#pragma omp parallel for collapse(2) schedule(static)
  for (long m = 0; m < M; m++) {
    for (long ch = 0; ch < kchunks; ch++) {
      long k0 = ch * ORC_NCHUNK;
      long w = K - k0 < ORC_NCHUNK ? K - k0 : ORC_NCHUNK;
      float acc[ORC_NCHUNK];
      const float *g = G + m * N;
      for (long j = 0; j < w; j++) acc[j] = 0.0f;
      if (blocked) {
        for (long n = 0; n < N; n += 4) {
          const float g0 = g[n], g1 = g[n + 1], g2 = g[n + 2], g3 = g[n + 3];
          const float *w0 = Bt + n * K + k0, *w1 = w0 + K, *w2 = w1 + K, *w3 = w2 + K;
          for (long j = 0; j < w; j++) {
            float p0 = w0[j] * g0;
            float p1 = w1[j] * g1;
            float p2 = w2[j] * g2;
            float p3 = w3[j] * g3;
            float s = p0 + p1;
            s = s + p2;
            s = s + p3;
            acc[j] = acc[j] + s;
          }
        }
      } else {
        for (long n = 0; n < N; n++) {
          const float gn = g[n];
          const float *wn = Bt + n * K + k0;
          for (long j = 0; j < w; j++) {
            float p = wn[j] * gn;
            acc[j] = acc[j] + p;
          }
        }
      }
      for (long j = 0; j < w; j++) dA[m * K + k0 + j] = acc[j];
    }
  }
}

/* dBt[n,k] = sum_m A[m,k] * G[m,n]   (A: [M,K], G: [M,N]) */
void orc_gemm_dw(const float *A, const float *G, long M, long N, long K, float *dBt) {
  const int blocked = orc_blocked(M);
  long kchunks = (K + ORC_NCHUNK - 1) / ORC_NCHUNK;
#pragma omp parallel for collapse(2) schedule(static)
  for (long n = 0; n < N; n++) {
    for (long ch = 0; ch < kchunks; ch++) {
      long k0 = ch * ORC_NCHUNK;
      long w = K - k0 < ORC_NCHUNK ? K - k0 : ORC_NCHUNK;
      float acc[ORC_NCHUNK];
      for (long j = 0; j < w; j++) acc[j] = 0.0f;
      if (blocked) {
        for (long m = 0; m < M; m += 4) {
          const float g0 = G[m * N + n], g1 = G[(m + 1) * N + n];
          const float g2 = G[(m + 2) * N + n], g3 = G[(m + 3) * N + n];
          const float *a0 = A + m * K + k0, *a1 = a0 + K, *a2 = a1 + K, *a3 = a2 + K;
          for (long j = 0; j < w; j++) {
            float p0 = a0[j] * g0;
            float p1 = a1[j] * g1;
            float p2 = a2[j] * g2;
            float p3 = a3[j] * g3;
            float s = p0 + p1;
            s = s + p2;
            s = s + p3;
            acc[j] = acc[j] + s;
          }
        }
      } else {
        for (long m = 0; m < M; m++) {
          const float gm = G[m * N + n];
          const float *am = A + m * K + k0;
          for (long j = 0; j < w; j++) {
            float p = am[j] * gm;
            acc[j] = acc[j] + p;
          }
        }
      }
      for (long j = 0; j < w; j++) dBt[n * K + k0 + j] = acc[j];
    }
  }
}

/* ---------------------------------------------------------------------------
 * log_softmax / cross_entropy forward and the gradient graph autograd builds
 * for them.  Forward: src/tensor.rs:697-752.  Backward rules: Mul/Neg/Add
 * (src/gradient.rs:99-107), Exp2 (:113-116), Log2 (:117-124), Expand ->
 * ReduceAxis (:165-176), ReduceAxis Add -> Expand (:185), ReduceAxis Max tie
 * mask (:186-198).  Class axis is the last axis; B rows, C classes.
 * ------------------------------------------------------------------------- */
static float orc_row_reduce(const float *v, long n, int op) {
  float acc = (op == ORC_MAX) ? -INFINITY : 0.0f;
  if (orc_blocked(n)) {
    for (long c = 0; c < n; c += 4) {
      if (op == ORC_MAX) {
        float g = orc_maxf(orc_maxf(orc_maxf(v[c], v[c + 1]), v[c + 2]), v[c + 3]);
        acc = orc_maxf(acc, g);
      } else {
        float g = v[c] + v[c + 1];
        g = g + v[c + 2];
        g = g + v[c + 3];
        acc = acc + g;
      }
    }
  } else {
    for (long c = 0; c < n; c++) acc = (op == ORC_MAX) ? orc_maxf(acc, v[c]) : acc + v[c];
  }
  return acc;
}

/* log_softmax(x, axis=1): writes log-probabilities [B, C]. */
void orc_log_softmax(const float *x, long B, long C, float *out) {
#pragma omp parallel for schedule(static)
  for (long b = 0; b < B; b++) {
    const float *xr = x + b * C;
    float *o = out + b * C;
    float m = orc_row_reduce(xr, C, ORC_MAX);
    float nm = -m;
    for (long c = 0; c < C; c++) {
      float s = xr[c] + nm;
      float ea = s * LOG2E_F;
      o[c] = (float)exp2((double)ea); /* e, temporarily */
    }
    float se = orc_row_reduce(o, C, ORC_SUM);
    float l2 = (float)log2((double)se);
    float lse = l2 * LN2_F;
    float nlse = -lse;
    for (long c = 0; c < C; c++) {
      float s = xr[c] + nm;
      o[c] = s + nlse;
    }
  }
}

/* cross_entropy(x, t) forward + d(loss)/d(x).  `dx` may be NULL (forward only).
 * Returns the loss. */
float orc_xent_fwd_bwd(const float *x, const float *t, long B, long C, float *dx) {
  const float inv_n = 1.0f / (float)B; /* 1.0 / per_sample.numel() as f32 */
  float *nps = (float *)malloc(sizeof(float) * (size_t)B);
#pragma omp parallel
  {
    float *s = (float *)malloc(sizeof(float) * (size_t)C);
    float *e = (float *)malloc(sizeof(float) * (size_t)C);
    float *tmp = (float *)malloc(sizeof(float) * (size_t)C);
    float *gs = (float *)malloc(sizeof(float) * (size_t)C);
#pragma omp for schedule(static)
    for (long b = 0; b < B; b++) {
      const float *xr = x + b * C;
      const float *tr = t + b * C;
      /* forward */
      float m = orc_row_reduce(xr, C, ORC_MAX);
      float nm = -m;
      for (long c = 0; c < C; c++) {
        s[c] = xr[c] + nm;
        float ea = s[c] * LOG2E_F;
        e[c] = (float)exp2((double)ea);
      }
      float se = orc_row_reduce(e, C, ORC_SUM);
      float l2 = (float)log2((double)se);
      float lse = l2 * LN2_F;
      float nlse = -lse;
      for (long c = 0; c < C; c++) {
        float lp = s[c] + nlse;
        tmp[c] = tr[c] * lp;
      }
      float ps = orc_row_reduce(tmp, C, ORC_SUM);
      nps[b] = -ps;
      if (!dx) continue;
      /* backward: root grad 1.0; Mul(sum, scale) -> scale * 1.0 */
      float g_tot = inv_n * 1.0f;
      float g_ps = -g_tot;
      for (long c = 0; c < C; c++) tmp[c] = tr[c] * g_ps; /* g_lp */
      float g_nlse = orc_row_reduce(tmp, C, ORC_SUM);
      float g_lse = -g_nlse;
      float g_l2 = LN2_F * g_lse;
      float den = se * LN2_F;
      float rcp = 1.0f / den;
      float g_se = g_l2 * rcp;
      for (long c = 0; c < C; c++) {
        float eln = e[c] * LN2_F;
        float g_ea = eln * g_se;
        float g_exp = LOG2E_F * g_ea;
        gs[c] = tmp[c] + g_exp; /* g_s = g_lp + exp-path grad */
      }
      float g_nm = orc_row_reduce(gs, C, ORC_SUM);
      float g_m = -g_nm;
      for (long c = 0; c < C; c++) tmp[c] = (xr[c] < m) ? 0.0f : 1.0f; /* mask */
      float count = orc_row_reduce(tmp, C, ORC_SUM);
      float rc = 1.0f / count;
      float *dr = dx + b * C;
      for (long c = 0; c < C; c++) {
        float wgt = tmp[c] * rc;
        float gmax = wgt * g_m;
        dr[c] = gs[c] + gmax;
      }
    }
    free(s);
    free(e);
    free(tmp);
    free(gs);
  }
  /* sum over axes [0, 1] of [B, 1]: the last reduce range has size 1, so no
   * unroll and the B axis is accumulated sequentially. */
  float tot = 0.0f;
  for (long b = 0; b < B; b++) tot = tot + nps[b];
  free(nps);
  return tot * inv_n;
}

/* ---------------------------------------------------------------------------
 * Sgd::step: param.assign(param.detach().sub(grad.mul(lr)))
 * (src/optim.rs:60-71) -> p + (-(g * lr)).
 * ------------------------------------------------------------------------- */
void orc_sgd(float *p, const float *g, long n, float lr) {
#pragma omp parallel for schedule(static)
  for (long i = 0; i < n; i++) {
    float gl = g[i] * lr;
    float ng = -gl;
    p[i] = p[i] + ng;
  }
}

/* ---------------------------------------------------------------------------
 * One MLP training step as examples/mnist.rs:90-97 runs it: Linear layers
 * (src/nn.rs:97-104) with ReLU between them (src/tensor.rs:519-531),
 * cross_entropy, backward, Sgd::step.  dims[0..nl] are the layer widths,
 * W[l] is [dims[l+1], dims[l]], b[l] is [dims[l+1]].  Parameters are updated
 * in place; dW / db (optional, may be NULL) receive the gradients; logits_out
 * (optional) the pre-update logits.  Returns the loss.
 * ------------------------------------------------------------------------- */
float orc_mlp_step_acts(int nl, const long *dims, long B, float lr, float **W, float **bias,
                        const float *x, const float *t, float **dW, float **db, float *logits_out,
                        float **acts_out);

float orc_mlp_step(int nl, const long *dims, long B, float lr, float **W, float **bias,
                   const float *x, const float *t, float **dW, float **db, float *logits_out) {
  return orc_mlp_step_acts(nl, dims, B, lr, W, bias, x, t, dW, db, logits_out, NULL);
}

/* As orc_mlp_step; acts_out (optional) receives each hidden layer's post-ReLU
 * activations [B, dims[l+1]] for l < nl-1. */
float orc_mlp_step_acts(int nl, const long *dims, long B, float lr, float **W, float **bias,
                        const float *x, const float *t, float **dW, float **db, float *logits_out,
                        float **acts_out) {
  float **z = (float **)calloc((size_t)nl, sizeof(float *)); /* pre-activations */
  float **a = (float **)calloc((size_t)nl, sizeof(float *)); /* post-ReLU acts */
  for (int l = 0; l < nl; l++) {
    long in = dims[l], out = dims[l + 1];
    const float *inp = (l == 0) ? x : a[l - 1];
    z[l] = (float *)malloc(sizeof(float) * (size_t)(B * out));
    orc_gemm_fwd(inp, W[l], bias[l], B, out, in, z[l]);
    if (l < nl - 1) {
      a[l] = (float *)malloc(sizeof(float) * (size_t)(B * out));
      orc_relu(z[l], a[l], B * out);
      if (acts_out && acts_out[l]) memcpy(acts_out[l], a[l], sizeof(float) * (size_t)(B * out));
    }
  }
  long C = dims[nl];
  float *g = (float *)malloc(sizeof(float) * (size_t)(B * C));
  float loss = orc_xent_fwd_bwd(z[nl - 1], t, B, C, g);
  if (logits_out) memcpy(logits_out, z[nl - 1], sizeof(float) * (size_t)(B * C));

  float **gw = (float **)calloc((size_t)nl, sizeof(float *));
  float **gb = (float **)calloc((size_t)nl, sizeof(float *));
  for (int l = nl - 1; l >= 0; l--) {
    long in = dims[l], out = dims[l + 1];
    const float *inp = (l == 0) ? x : a[l - 1];
    gw[l] = (float *)malloc(sizeof(float) * (size_t)(out * in));
    gb[l] = (float *)malloc(sizeof(float) * (size_t)out);
    orc_gemm_dw(inp, g, B, out, in, gw[l]);
    orc_reduce_axis0_f32(g, B, out, ORC_SUM, gb[l]);
    if (l > 0) {
      float *dh = (float *)malloc(sizeof(float) * (size_t)(B * in));
      orc_gemm_dx(g, W[l], B, out, in, dh);
      const float *zp = z[l - 1];
      for (long i = 0; i < B * in; i++) dh[i] = (0.0f < zp[i]) ? dh[i] : 0.0f;
      free(g);
      g = dh;
    }
  }
  free(g);
  for (int l = 0; l < nl; l++) {
    long in = dims[l], out = dims[l + 1];
    if (dW && dW[l]) memcpy(dW[l], gw[l], sizeof(float) * (size_t)(out * in));
    if (db && db[l]) memcpy(db[l], gb[l], sizeof(float) * (size_t)out);
    orc_sgd(W[l], gw[l], out * in, lr);
    orc_sgd(bias[l], gb[l], out, lr);
    free(gw[l]);
    free(gb[l]);
    free(z[l]);
    if (a[l]) free(a[l]);
  }
  free(gw);
  free(gb);
  free(z);
  free(a);
  return loss;
}
