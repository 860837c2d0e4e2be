// The MLP training step -- examples/mnist.rs:90-97 (forward, cross_entropy,
// zero_grad, backward, Sgd::step, loss.to_vec) -- as a fixed schedule of this
// library's kernels.  It is the schedule ferrograd's scheduler produces for
// Linear (src/nn.rs:97-104) / relu (src/tensor.rs:519-531) / cross_entropy
// (src/tensor.rs:738-752) / Sgd (src/optim.rs:60-71) graphs, with every
// proto-kernel routed to a hand-written building block:
//
//   Linear forward / dX / dW   -> 3xTF32 tcgen05 GEMM (fused bias+relu,
//                                  relu-mask and TF32-residual epilogues)
//   Linear with <= 16 outputs  -> "skinny" SIMT kernels (one HBM pass)
//   bias gradient (axis-0 sum) -> deterministic column reduction
//   cross_entropy fwd+bwd      -> one fused pass
//   Sgd::step                  -> one multi-tensor pass (+ TF32 residual of W)
//
// Data parallel: each rank holds batch rows, and the gradients are combined
// across ranks while the remaining backward GEMMs run, either by NCCL
// all-reduces on a second stream (one bucket per layer, enqueue_step), or by
// the peer-sharded exchange (enqueue_step_peer, fg_peer.cu): copy-engine
// reduce-scatter of each gradient chunk to its owning rank, the owner's fused
// reduce + SGD, copy-engine all-gather of the updated parameters.
#include <cuda_runtime.h>
#include <stdlib.h>
#include <string.h>

#include <vector>

#include "fg_comm.h"
#include "fg_gemm.cuh"
#include "fg_internal.h"
#include "fg_kernels.cuh"
#include "fg_peer.cuh"

namespace fg {

// ---------------------------------------------------------------------------
// Skinny layers (out features NJ <= 16): logits = act @ W^T + b and the
// fused backward pass.
// ---------------------------------------------------------------------------
constexpr int kSkinnyMax = 16;

// Each warp computes 4 rows; W is staged in shared memory when it fits.
template <int NJ, bool WSMEM>
__global__ void __launch_bounds__(256) k_skinny_fwd(const float *__restrict__ act,
                                                    const float *__restrict__ W,
                                                    const float *__restrict__ bias,
                                                    float *__restrict__ out, int M, int K) {
  extern __shared__ float4 sW4[];
  const int K4 = K / 4;
  const float4 *W4 = WSMEM ? sW4 : reinterpret_cast<const float4 *>(W);
  if (WSMEM) {
    const float4 *g = reinterpret_cast<const float4 *>(W);
    for (int i = threadIdx.x; i < NJ * K4; i += blockDim.x) sW4[i] = g[i];
    __syncthreads();
  }
  const int lane = threadIdx.x & 31;
  const int wid = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const int nw = gridDim.x * (blockDim.x >> 5);
  for (int r0 = wid * 4; r0 < M; r0 += nw * 4) {
    float acc[4][NJ];
#pragma unroll
    for (int r = 0; r < 4; r++)
#pragma unroll
      for (int j = 0; j < NJ; j++) acc[r][j] = 0.f;
    for (int k4 = lane; k4 < K4; k4 += 32) {
      float4 a[4];
#pragma unroll
      for (int r = 0; r < 4; r++)
        a[r] = (r0 + r < M) ? __ldcs(reinterpret_cast<const float4 *>(act + (size_t)(r0 + r) * K) + k4)
                            : make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
      for (int j = 0; j < NJ; j++) {
        const float4 w = WSMEM ? W4[j * K4 + k4] : __ldg(W4 + j * K4 + k4);
#pragma unroll
        for (int r = 0; r < 4; r++)
          acc[r][j] += a[r].x * w.x + a[r].y * w.y + a[r].z * w.z + a[r].w * w.w;
      }
    }
#pragma unroll
    for (int r = 0; r < 4; r++)
#pragma unroll
      for (int j = 0; j < NJ; j++) {
        float v = acc[r][j];
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
        acc[r][j] = v;
      }
    if (lane < NJ) {
#pragma unroll
      for (int r = 0; r < 4; r++) {
        if (r0 + r < M) {
          float v = 0.f;
#pragma unroll
          for (int j = 0; j < NJ; j++)
            if (j == lane) v = acc[r][j];
          out[(size_t)(r0 + r) * NJ + lane] = __fadd_rn(v, bias[lane]);
        }
      }
    }
  }
}

// Backward of a skinny layer.  Thread owns a float4 column slice k4 of the
// layer input and a chunk of rows:
//   dW partial[chunk][j][k] += G[m,j] * act[m,k]
//   Gprev[m,k] = (act[m,k] > 0) ? sum_j G[m,j] * W[j,k] : 0   (+ TF32 residual)
template <int NJ, bool DX>
__global__ void __launch_bounds__(256) k_skinny_bwd(const float *__restrict__ G,
                                                    const float *__restrict__ act,
                                                    const float *__restrict__ W,
                                                    float *__restrict__ part,
                                                    float *__restrict__ gprev,
                                                    float *__restrict__ gprev_lo, int M, int K,
                                                    int rows_per_chunk) {
  __shared__ float sG[64 * kSkinnyMax];
  const int K4 = K / 4;
  const int k4 = blockIdx.x * blockDim.x + threadIdx.x;
  const int r_begin = blockIdx.y * rows_per_chunk;
  const int r_end = min(M, r_begin + rows_per_chunk);
  const bool active = k4 < K4;
  float4 w[NJ];
  float4 dw[NJ];
#pragma unroll
  for (int j = 0; j < NJ; j++) {
    w[j] = (DX && active) ? __ldg(reinterpret_cast<const float4 *>(W + (size_t)j * K) + k4)
                          : make_float4(0.f, 0.f, 0.f, 0.f);
    dw[j] = make_float4(0.f, 0.f, 0.f, 0.f);
  }
  for (int rb = r_begin; rb < r_end; rb += 64) {
    const int nr = min(64, r_end - rb);
    __syncthreads();
    for (int i = threadIdx.x; i < nr * NJ; i += blockDim.x) sG[i] = G[(size_t)rb * NJ + i];
    __syncthreads();
    if (!active) continue;
    for (int r = 0; r < nr; r++) {
      const size_t m = (size_t)(rb + r);
      const float4 a = __ldcs(reinterpret_cast<const float4 *>(act + m * K) + k4);
      float4 dx = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
      for (int j = 0; j < NJ; j++) {
        const float g = sG[r * NJ + j];
        dw[j].x += g * a.x; dw[j].y += g * a.y; dw[j].z += g * a.z; dw[j].w += g * a.w;
        if (DX) {
          dx.x += g * w[j].x; dx.y += g * w[j].y; dx.z += g * w[j].z; dx.w += g * w[j].w;
        }
      }
      if (DX) {
        dx.x = (a.x > 0.f) ? dx.x : 0.f;
        dx.y = (a.y > 0.f) ? dx.y : 0.f;
        dx.z = (a.z > 0.f) ? dx.z : 0.f;
        dx.w = (a.w > 0.f) ? dx.w : 0.f;
        reinterpret_cast<float4 *>(gprev + m * K)[k4] = dx;
        if (gprev_lo) {
          float4 lo;
          lo.x = __fsub_rn(dx.x, __uint_as_float(__float_as_uint(dx.x) & 0xffffe000u));
          lo.y = __fsub_rn(dx.y, __uint_as_float(__float_as_uint(dx.y) & 0xffffe000u));
          lo.z = __fsub_rn(dx.z, __uint_as_float(__float_as_uint(dx.z) & 0xffffe000u));
          lo.w = __fsub_rn(dx.w, __uint_as_float(__float_as_uint(dx.w) & 0xffffe000u));
          reinterpret_cast<float4 *>(gprev_lo + m * K)[k4] = lo;
        }
      }
    }
  }
  if (active) {
#pragma unroll
    for (int j = 0; j < NJ; j++)
      reinterpret_cast<float4 *>(part + ((size_t)blockIdx.y * NJ + j) * K)[k4] = dw[j];
  }
}

// dW[j,k] = sum over chunks (in chunk order) of the partials.
__global__ void __launch_bounds__(256) k_skinny_dw_final(const float *__restrict__ part,
                                                         float *__restrict__ dW, int nchunks,
                                                         size_t jk) {
  size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= jk) return;
  float acc = 0.f;
  for (int c = 0; c < nchunks; c++) acc += part[(size_t)c * jk + i];
  dW[i] = acc;
}

template <int NJ>
static int launch_skinny_fwd_t(const float *act, const float *W, const float *b, float *out, int M,
                               int K, cudaStream_t st, int sms) {
  const size_t wbytes = (size_t)NJ * K * 4;
  const bool smem = wbytes <= 200 * 1024;
  const int warps_needed = (M + 3) / 4;
  int grid = (warps_needed + 7) / 8;
  const int cap = sms * (smem ? 1 : 4);
  if (grid > cap) grid = cap;
  if (grid < 1) grid = 1;
  if (smem) {
    auto kern = k_skinny_fwd<NJ, true>;
    static int attr_bytes[64] = {};
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev >= 0 && dev < 64 && attr_bytes[dev] < (int)wbytes) {
      FG_CUDA_TRY(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024));
      attr_bytes[dev] = 200 * 1024;
    }
    kern<<<grid, 256, wbytes, st>>>(act, W, b, out, M, K);
  } else {
    k_skinny_fwd<NJ, false><<<grid, 256, 0, st>>>(act, W, b, out, M, K);
  }
  FG_LAUNCH_TRY();
  return FG_OK;
}

static int launch_skinny_fwd(int nj, const float *act, const float *W, const float *b, float *out,
                             int M, int K, cudaStream_t st, int sms) {
  switch (nj) {
#define FG_NJ(n) \
  case n: return launch_skinny_fwd_t<n>(act, W, b, out, M, K, st, sms);
    FG_NJ(1) FG_NJ(2) FG_NJ(3) FG_NJ(4) FG_NJ(5) FG_NJ(6) FG_NJ(7) FG_NJ(8)
    FG_NJ(9) FG_NJ(10) FG_NJ(11) FG_NJ(12) FG_NJ(13) FG_NJ(14) FG_NJ(15) FG_NJ(16)
#undef FG_NJ
    default: return set_error(FG_ERR_UNSUPPORTED, "skinny layer with %d outputs", nj);
  }
}

struct SkinnyBwdShape {
  int threads, colblocks, nchunks, rows_per_chunk;
};

static SkinnyBwdShape skinny_bwd_shape(int M, int K, int sms) {
  SkinnyBwdShape s;
  const int K4 = K / 4;
  s.threads = K4 >= 256 ? 256 : ((K4 + 31) / 32) * 32;
  s.colblocks = (K4 + s.threads - 1) / s.threads;
  int want = (2 * sms + s.colblocks - 1) / s.colblocks;
  int max_chunks = (M + 15) / 16;
  if (want > max_chunks) want = max_chunks;
  if (want < 1) want = 1;
  s.rows_per_chunk = (M + want - 1) / want;
  s.nchunks = (M + s.rows_per_chunk - 1) / s.rows_per_chunk;
  return s;
}

template <int NJ>
static int launch_skinny_bwd_t(const float *G, const float *act, const float *W, float *part,
                               float *dW, float *gprev, float *gprev_lo, int M, int K,
                               cudaStream_t st, int sms) {
  SkinnyBwdShape s = skinny_bwd_shape(M, K, sms);
  dim3 grid(s.colblocks, s.nchunks);
  if (gprev)
    k_skinny_bwd<NJ, true><<<grid, s.threads, 0, st>>>(G, act, W, part, gprev, gprev_lo, M, K,
                                                       s.rows_per_chunk);
  else
    k_skinny_bwd<NJ, false><<<grid, s.threads, 0, st>>>(G, act, W, part, nullptr, nullptr, M, K,
                                                        s.rows_per_chunk);
  FG_LAUNCH_TRY();
  size_t jk = (size_t)NJ * K;
  k_skinny_dw_final<<<(unsigned)((jk + 255) / 256), 256, 0, st>>>(part, dW, s.nchunks, jk);
  FG_LAUNCH_TRY();
  return FG_OK;
}

static int launch_skinny_bwd(int nj, const float *G, const float *act, const float *W,
                             float *part, float *dW, float *gprev, float *gprev_lo, int M, int K,
                             cudaStream_t st, int sms) {
  switch (nj) {
#define FG_NJ(n) \
  case n: return launch_skinny_bwd_t<n>(G, act, W, part, dW, gprev, gprev_lo, M, K, st, sms);
    FG_NJ(1) FG_NJ(2) FG_NJ(3) FG_NJ(4) FG_NJ(5) FG_NJ(6) FG_NJ(7) FG_NJ(8)
    FG_NJ(9) FG_NJ(10) FG_NJ(11) FG_NJ(12) FG_NJ(13) FG_NJ(14) FG_NJ(15) FG_NJ(16)
#undef FG_NJ
    default: return set_error(FG_ERR_UNSUPPORTED, "skinny layer with %d outputs", nj);
  }
}

}  // namespace fg

// ---------------------------------------------------------------------------
// The plan
// ---------------------------------------------------------------------------
namespace {

struct Layer {
  int in = 0, out = 0;
  bool tc = false;  // tensor-core layer (out % 16 == 0, out >= 32) vs skinny (out <= 16)
  float *W = nullptr, *b = nullptr, *W_lo = nullptr;
  float *dW = nullptr, *db = nullptr;  // inside the flat gradient buffer
  size_t bucket_off = 0, bucket_len = 0;  // this layer's all-reduce bucket (floats)
  fg::gemm::GemmPlan fwd, bwd_w, bwd_x;
  // dW as two launches over the halves of its output rows, so that with a
  // communicator the first half's all-reduce overlaps the second half's GEMM
  // (every tensor-core layer; FG_COMM_SPLIT_ALL=0: layer 0 only, whose
  // bucket is the last one of the backward pass)
  bool can_split_w = false;
  fg::gemm::GemmPlan bwd_w_half[2];
  // Peer-sharded mode: this layer's parameters of even / odd steps inside
  // the exchange region, the GEMM plans that read each of them, and dW as
  // row blocks, one per gradient chunk.
  float *Wp[2] = {nullptr, nullptr}, *bp[2] = {nullptr, nullptr}, *W_lo_p[2] = {nullptr, nullptr};
  fg::gemm::GemmPlan fwd_p[2], bwd_x_p[2];
  fg::gemm::GemmPlan bwd_w_part[fg::kMaxPeerParts];
};

size_t pad64(size_t n) { return (n + 63) / 64 * 64; }

// With a communicator every tensor-core layer's dW is computed in two row
// halves (the upper layers' SGD still waits for their dX GEMM), so each
// bucket's first half is averaged while its second half is computed
// (8 x B200: 647 steps/s against 627 with only layer 0 split).
// FG_COMM_SPLIT_ALL=0 splits layer 0 only.
bool split_all_layers() {
  static const bool v = [] {
    const char *e = getenv("FG_COMM_SPLIT_ALL");
    return !(e && *e && atoi(e) == 0);
  }();
  return v;
}

}  // namespace

struct fg_mlp {
  fg_device *dev = nullptr;
  cudaStream_t st = nullptr, comm_st = nullptr;
  // With a communicator, Sgd::step's updates run on their own stream after
  // their bucket's all-reduce, so the comm stream goes straight on to the
  // next bucket.
  cudaStream_t sgd_st = nullptr;
  std::vector<cudaEvent_t> ev_ar;  // [2 * layer + part]: a bucket's all-reduce done
  cudaEvent_t ev_sgd_done = nullptr;
  int nl = 0, B = 0;
  float lr = 0.f;
  std::vector<int> dims;
  std::vector<Layer> L;
  float *x = nullptr, *x_lo = nullptr, *t = nullptr;
  std::vector<float *> act, act_lo;  // act[l] = output of layer l (post-ReLU; logits for the last)
  std::vector<float *> G, G_lo;      // G[l] = d loss / d (pre-activation output of layer l)
  float *grad = nullptr;
  size_t grad_count = 0;
  float *loss = nullptr;  // inside the flat gradient buffer (averaged with the layer-0 bucket)
  float *scratch = nullptr;
  size_t scratch_bytes = 0;
  std::vector<void *> allocations;
  fg_comm *comm = nullptr;
  std::vector<cudaEvent_t> ev_bucket, ev_wread;
  std::vector<cudaEvent_t> ev_half;  // per layer: first half of dW complete
  cudaEvent_t ev_comm_done = nullptr;
  bool use_graph = false;
  cudaGraphExec_t graph = nullptr;
  bool timing = false;
  std::vector<cudaEvent_t> ev_t0, ev_t1;  // one pair per GEMM launch of a step
  std::vector<double> gemm_flops;
  int gemm_launches = 0;
  std::vector<cudaEvent_t> ev_c0, ev_c1;  // one pair per all-reduce of a step
  std::vector<double> comm_bytes;
  int comm_launches = 0;
  int launches_per_step = 0;
  int sms = 148;
  float *sk_ws = nullptr;  // stream-K workspace shared by every GEMM plan
  // Peer-sharded data parallelism (fg_mlp_peer_prepare / fg_mlp_peer_connect).
  bool peer = false;  // connected: fg_mlp_step runs enqueue_step_peer
  int peer_rank = 0, peer_n = 0;
  fg::PeerLayout pl;
  float *region = nullptr;  // this rank's exchange region (fg_peer.cuh)
  float *pg = nullptr, *pstage = nullptr, *pP[2] = {nullptr, nullptr}, *pLO[2] = {nullptr, nullptr};
  unsigned int *pflags = nullptr;
  char *peer_base[fg::kMaxPeers] = {};  // other ranks' regions, mapped (null for self)
  int par = 0;                          // parameter buffer the next step reads
  int reduce_blocks = 64;
  // all-gather the TF32 residual with the parameters (else each rank
  // recomputes it for the chunks that arrive)
  bool push_lo = true;
  cudaStream_t rs_st[fg::kMaxPeers] = {}, ag_st[fg::kMaxPeers] = {};
  cudaStream_t red_st = nullptr, sig_rs_st = nullptr, sig_ag_st = nullptr, arr_st = nullptr;
  cudaEvent_t ev_ready = nullptr, ev_red = nullptr, ev_join = nullptr;
  cudaEvent_t ev_rs[fg::kMaxPeers] = {}, ev_ag[fg::kMaxPeers] = {};
  cudaGraphExec_t pgraph[2] = {nullptr, nullptr};
  // Overlapped uploads (fg_mlp_step_host_next): two device staging slots for
  // a batch and its targets, filled from host memory on copy_st while a step
  // runs; staged_x/staged_t are the host pointers slot next_slot holds.
  float *stage_x[2] = {nullptr, nullptr}, *stage_t[2] = {nullptr, nullptr};
  cudaStream_t copy_st = nullptr;
  cudaEvent_t ev_staged[2] = {nullptr, nullptr}, ev_consumed[2] = {nullptr, nullptr};
  int next_slot = 0;
  const float *staged_x = nullptr, *staged_t = nullptr;
};

namespace {

int mlp_alloc(fg_mlp *m, float **p, size_t n) {
  void *q = nullptr;
  FG_CUDA_TRY(cudaMalloc(&q, n * sizeof(float) + 256));
  FG_CUDA_TRY(cudaMemset(q, 0, n * sizeof(float) + 256));
  m->allocations.push_back(q);
  *p = (float *)q;
  return FG_OK;
}

int build_plans(fg_mlp *m) {
  const int B = m->B;
  for (int l = 0; l < m->nl; l++) {
    Layer &ly = m->L[l];
    if (!ly.tc) continue;
    const float *in = (l == 0) ? m->x : m->act[l - 1];
    const float *in_lo = (l == 0) ? m->x_lo : m->act_lo[l - 1];
    const bool last = (l == m->nl - 1);
    int rc = fg::gemm::make_plan(B, ly.out, ly.in, in, in_lo, ly.in, ly.W, ly.W_lo, ly.in,
                                 m->act[l], last ? nullptr : m->act_lo[l], ly.out, 0,
                                 last ? FG_EPI_BIAS : FG_EPI_BIAS_RELU, ly.b, nullptr, 0, &ly.fwd);
    if (rc) return rc;
    // dW[n,k] = sum_m G[m,n] * in[m,k]: A = G stored [B, out] (MN-major),
    // B = in stored [B, in] (MN-major), reduction over the batch.
    rc = fg::gemm::make_plan(ly.out, ly.in, B, m->G[l], m->G_lo[l], ly.out, in, in_lo, ly.in, ly.dW,
                             nullptr, ly.in, FG_GEMM_A_MN_MAJOR | FG_GEMM_B_MN_MAJOR, FG_EPI_NONE,
                             nullptr, nullptr, 0, &ly.bwd_w);
    if (rc) return rc;
    if ((l == 0 || split_all_layers()) && ly.out % 64 == 0) {
      const int half = ly.out / 2;
      for (int h = 0; h < 2; h++) {
        rc = fg::gemm::make_plan(half, ly.in, B, m->G[l] + h * half, m->G_lo[l] + h * half, ly.out,
                                 in, in_lo, ly.in, ly.dW + (size_t)h * half * ly.in, nullptr, ly.in,
                                 FG_GEMM_A_MN_MAJOR | FG_GEMM_B_MN_MAJOR, FG_EPI_NONE, nullptr,
                                 nullptr, 0, &ly.bwd_w_half[h]);
        if (rc) return rc;
      }
      ly.can_split_w = true;
    }
    if (l > 0) {
      // Gprev[m,k] = (act[m,k] > 0) ? sum_n G[m,n] W[n,k] : 0:
      // A = G [B, out] K-major, B = W stored [out, in] = [K, N] (MN-major).
      rc = fg::gemm::make_plan(B, ly.in, ly.out, m->G[l], m->G_lo[l], ly.out, ly.W, ly.W_lo, ly.in,
                               m->G[l - 1], m->G_lo[l - 1], ly.in, FG_GEMM_B_MN_MAJOR,
                               FG_EPI_RELU_MASK, nullptr, m->act[l - 1], ly.in, &ly.bwd_x);
      if (rc) return rc;
    }
  }
  return FG_OK;
}

int record(cudaEvent_t ev, cudaStream_t st) {
  cudaStreamCaptureStatus cs = cudaStreamCaptureStatusNone;
  FG_CUDA_TRY(cudaStreamIsCapturing(st, &cs));
  if (cs == cudaStreamCaptureStatusActive)
    FG_CUDA_TRY(cudaEventRecordWithFlags(ev, st, cudaEventRecordExternal));
  else
    FG_CUDA_TRY(cudaEventRecord(ev, st));
  return FG_OK;
}

// Launch one GEMM plan, bracketed by timing events when timing is on.
int run_gemm(fg_mlp *m, const fg::gemm::GemmPlan &pl, cudaStream_t st) {
  const int i = m->gemm_launches++;
  const bool t = m->timing && i < (int)m->ev_t0.size();
  int rc;
  if (t && (rc = record(m->ev_t0[i], st))) return rc;
  if ((rc = fg::gemm::run_plan(pl, st))) return rc;
  if (t) {
    m->gemm_flops[i] = 2.0 * pl.p.M * (double)pl.p.N * pl.p.K;
    if ((rc = record(m->ev_t1[i], st))) return rc;
  }
  return FG_OK;
}

// Sgd::step for layer l's weight and bias on `st`.
int sgd_layer(fg_mlp *m, int l, cudaStream_t st) {
  Layer &ly = m->L[l];
  fg::SgdSegments segs{};
  segs.count = 2;
  segs.p[0] = ly.W;
  segs.g[0] = ly.dW;
  segs.lo[0] = ly.tc ? ly.W_lo : nullptr;
  segs.n[0] = (size_t)ly.out * ly.in;
  segs.p[1] = ly.b;
  segs.g[1] = ly.db;
  segs.lo[1] = nullptr;
  segs.n[1] = (size_t)ly.out;
  return fg::launch_sgd_multi(segs, m->lr, st);
}

// Average [off, off+len) of the gradient buffer across ranks on the comm
// stream once everything enqueued on st so far has run.
int bucket_allreduce(fg_mlp *m, cudaEvent_t ev, size_t off, size_t len) {
  FG_CUDA_TRY(cudaEventRecord(ev, m->st));
  FG_CUDA_TRY(cudaStreamWaitEvent(m->comm_st, ev, 0));
  const int i = m->comm_launches++;
  const bool t = m->timing && i < (int)m->ev_c0.size();
  int rc;
  if (t && (rc = record(m->ev_c0[i], m->comm_st))) return rc;
  if ((rc = fg::comm_allreduce_sum(m->comm, m->grad + off, len, m->comm_st))) return rc;
  if (t) {
    m->comm_bytes[i] = (double)len * sizeof(float);
    if ((rc = record(m->ev_c1[i], m->comm_st))) return rc;
  }
  return FG_OK;
}

// Make m->sgd_st wait for everything enqueued on m->comm_st so far (the
// all-reduce of the bucket it is about to apply).
int sgd_after_comm(fg_mlp *m, int ev_index) {
  FG_CUDA_TRY(cudaEventRecord(m->ev_ar[(size_t)ev_index], m->comm_st));
  FG_CUDA_TRY(cudaStreamWaitEvent(m->sgd_st, m->ev_ar[(size_t)ev_index], 0));
  return FG_OK;
}

// Enqueue one training step on m->st (and m->comm_st, m->sgd_st).
int enqueue_step(fg_mlp *m) {
  cudaStream_t st = m->st;
  const int B = m->B;
  int rc;
  m->gemm_launches = 0;
  m->comm_launches = 0;
  // forward
  if (m->L[0].tc && (rc = fg::launch_split_lo(m->x, m->x_lo, (size_t)B * m->dims[0], st))) return rc;
  for (int l = 0; l < m->nl; l++) {
    Layer &ly = m->L[l];
    const float *in = (l == 0) ? m->x : m->act[l - 1];
    if (ly.tc) {
      if ((rc = run_gemm(m, ly.fwd, st))) return rc;
    } else {
      if ((rc = fg::launch_skinny_fwd(ly.out, in, ly.W, ly.b, m->act[l], B, ly.in, st, m->sms)))
        return rc;
    }
  }
  // cross_entropy forward + backward
  const int C = m->dims[m->nl];
  // With N ranks the local loss and its gradient are pre-scaled by 1/N so
  // that a plain sum across ranks (NVLS-eligible) yields the global mean.
  const float rank_scale = 1.0f / (float)fg::comm_nranks(m->comm);
  if ((rc = fg::launch_xent(m->act[m->nl - 1], m->t, (size_t)B, (size_t)C, m->loss, m->G[m->nl - 1],
                            rank_scale, st, m->scratch, rank_scale)))
    return rc;
  if (m->L[m->nl - 1].tc &&
      (rc = fg::launch_split_lo(m->G[m->nl - 1], m->G_lo[m->nl - 1], (size_t)B * C, st)))
    return rc;
  // backward, last layer first.  With a communicator each layer's bucket
  // [dW | db] is averaged across ranks on the comm stream as soon as it is
  // complete -- before this layer's dX GEMM, which does not contribute to it
  // -- and the layer's SGD follows on the comm stream once the dX GEMM (the
  // last reader of W) has run, overlapping the layers below.
  for (int l = m->nl - 1; l >= 0; l--) {
    Layer &ly = m->L[l];
    const float *in = (l == 0) ? m->x : m->act[l - 1];
    const bool split = m->comm && ly.tc && ly.can_split_w;
    const size_t half_elems = (size_t)(ly.out / 2) * ly.in;
    if (split) {
      // first half of dW's rows: average and apply it while the second half
      // is computed (layer 0 has no dX GEMM, nothing reads W afterwards)
      if ((rc = run_gemm(m, ly.bwd_w_half[0], st))) return rc;
      if ((rc = bucket_allreduce(m, m->ev_half[l], ly.bucket_off, half_elems))) return rc;
      if (l == 0) {
        fg::SgdSegments segs{};
        segs.count = 1;
        segs.p[0] = ly.W;
        segs.g[0] = ly.dW;
        segs.lo[0] = ly.W_lo;
        segs.n[0] = half_elems;
        if ((rc = sgd_after_comm(m, 2 * l))) return rc;
        if ((rc = fg::launch_sgd_multi(segs, m->lr, m->sgd_st))) return rc;
      }
      if ((rc = run_gemm(m, ly.bwd_w_half[1], st))) return rc;
    } else if (ly.tc) {
      if ((rc = run_gemm(m, ly.bwd_w, st))) return rc;
    } else {
      if ((rc = fg::launch_skinny_bwd(ly.out, m->G[l], in, ly.W, m->scratch, ly.dW,
                                      l > 0 ? m->G[l - 1] : nullptr,
                                      (l > 0 && m->L[l - 1].tc) ? m->G_lo[l - 1] : nullptr, B,
                                      ly.in, st, m->sms)))
        return rc;
    }
    if ((rc = fg::launch_reduce_cols(FG_F32, FG_REDUCE_SUM, m->G[l], ly.db, (size_t)B,
                                     (size_t)ly.out, st, m->scratch, m->scratch_bytes)))
      return rc;
    const size_t done = split ? half_elems : 0;
    if (m->comm &&
        (rc = bucket_allreduce(m, m->ev_bucket[l], ly.bucket_off + done, ly.bucket_len - done)))
      return rc;
    if (ly.tc && l > 0 && (rc = run_gemm(m, ly.bwd_x, st))) return rc;
    if (m->comm) {
      if ((rc = sgd_after_comm(m, 2 * l + 1))) return rc;
      if (ly.tc && l > 0) {  // SGD must not overtake the dX GEMM reading W
        FG_CUDA_TRY(cudaEventRecord(m->ev_wread[l], st));
        FG_CUDA_TRY(cudaStreamWaitEvent(m->sgd_st, m->ev_wread[l], 0));
      }
      if (split && l == 0) {
        fg::SgdSegments segs{};
        segs.count = 2;
        segs.p[0] = ly.W + half_elems;
        segs.g[0] = ly.dW + half_elems;
        segs.lo[0] = ly.W_lo + half_elems;
        segs.n[0] = (size_t)ly.out * ly.in - half_elems;
        segs.p[1] = ly.b;
        segs.g[1] = ly.db;
        segs.lo[1] = nullptr;
        segs.n[1] = (size_t)ly.out;
        if ((rc = fg::launch_sgd_multi(segs, m->lr, m->sgd_st))) return rc;
      } else if ((rc = sgd_layer(m, l, m->sgd_st))) {
        return rc;
      }
    }
  }
  if (m->comm) {
    FG_CUDA_TRY(cudaEventRecord(m->ev_comm_done, m->comm_st));
    FG_CUDA_TRY(cudaStreamWaitEvent(st, m->ev_comm_done, 0));
    FG_CUDA_TRY(cudaEventRecord(m->ev_sgd_done, m->sgd_st));
    FG_CUDA_TRY(cudaStreamWaitEvent(st, m->ev_sgd_done, 0));
    return FG_OK;
  }
  // Sgd::step over every parameter (weights of tensor-core layers also get
  // their TF32 residual for the next step's GEMMs).
  fg::SgdSegments segs{};
  for (int l = 0; l < m->nl; l++) {
    Layer &ly = m->L[l];
    segs.p[segs.count] = ly.W;
    segs.g[segs.count] = ly.dW;
    segs.lo[segs.count] = ly.tc ? ly.W_lo : nullptr;
    segs.n[segs.count] = (size_t)ly.out * ly.in;
    segs.count++;
    segs.p[segs.count] = ly.b;
    segs.g[segs.count] = ly.db;
    segs.lo[segs.count] = nullptr;
    segs.n[segs.count] = (size_t)ly.out;
    segs.count++;
    if (segs.count + 2 > fg::kMaxSgdSegments || l == m->nl - 1) {
      if ((rc = fg::launch_sgd_multi(segs, m->lr, st))) return rc;
      segs.count = 0;
    }
  }
  return FG_OK;
}

// ---- peer-sharded data parallelism ----------------------------------------
// Byte address of float `idx` of area `area` (0 grad, 1 stage, 2/3 P0/P1,
// 4/5 LO0/LO1) in rank j's region (this rank's own or a peer's mapping).
float *region_f(fg_mlp *m, int j, int area, size_t idx) {
  char *base = (j == m->peer_rank) ? reinterpret_cast<char *>(m->region) : m->peer_base[j];
  return reinterpret_cast<float *>(base) + (size_t)area * m->pl.grad + idx;
}

// Flag word of chunk ci set by sender `from` in rank j's region
// (phase 0: reduce-scatter, 1: all-gather).
unsigned int *region_flag(fg_mlp *m, int j, int phase, int ci, int from) {
  char *base = (j == m->peer_rank) ? reinterpret_cast<char *>(m->region) : m->peer_base[j];
  unsigned int *f = reinterpret_cast<unsigned int *>(reinterpret_cast<float *>(base) + 6 * m->pl.grad);
  return f + ((size_t)phase * m->pl.chunks.size() + ci) * fg::kMaxPeers + from;
}

// Current-parameter pointers of every layer (what get/set_params and the
// host see) follow the parity of the next step.
void peer_point(fg_mlp *m) {
  for (auto &ly : m->L) {
    ly.W = ly.Wp[m->par];
    ly.b = ly.bp[m->par];
    ly.W_lo = ly.W_lo_p[m->par];
  }
}

// Exchange of gradient chunk ci of a step that reads parameter buffer par:
//   1. reduce-scatter: once the chunk is complete on the compute stream,
//      this rank's part of every other rank's shard is copied (copy engine,
//      one stream per peer) into that rank's staging slot for this rank,
//      then the peers' flags are raised;
//   2. on the owner, a one-block kernel waits for every peer's flag, then
//      one pass sums the contributions in rank order and writes the SGD
//      update of its shard into buffer par ^ 1 (and its TF32 residual);
//   3. all-gather: the updated shard is copied into every peer's buffer
//      par ^ 1 and the peers' all-gather flags are raised.
// Flags carry par + 1, so a waiter can never mistake the previous step's
// value for the current one (ranks are at most one step apart).
int peer_chunk(fg_mlp *m, int ci, int par) {
  const fg::PeerChunk &c = m->pl.chunks[ci];
  const int n = m->peer_n, r = m->peer_rank, nx = par ^ 1;
  const size_t S = c.len / n;
  const unsigned int val = (unsigned int)par + 1;
  int rc;
  FG_CUDA_TRY(cudaEventRecord(m->ev_ready, m->st));
  for (int p = 0; p < n; p++) {
    if (p == r) continue;
    FG_CUDA_TRY(cudaStreamWaitEvent(m->rs_st[p], m->ev_ready, 0));
    FG_CUDA_TRY(cudaMemcpyAsync(region_f(m, p, 1, c.off + (size_t)r * S), m->pg + c.off + (size_t)p * S,
                                S * sizeof(float), cudaMemcpyDefault, m->rs_st[p]));
    FG_CUDA_TRY(cudaEventRecord(m->ev_rs[p], m->rs_st[p]));
    FG_CUDA_TRY(cudaStreamWaitEvent(m->sig_rs_st, m->ev_rs[p], 0));
  }
  fg::PeerFlagPtrs f{};
  for (int p = 0; p < n; p++) f.p[p] = (p == r) ? nullptr : region_flag(m, p, 0, ci, r);
  if ((rc = fg::launch_peer_signal(f, val, m->sig_rs_st))) return rc;

  FG_CUDA_TRY(cudaStreamWaitEvent(m->red_st, m->ev_ready, 0));
  const size_t loss = m->pl.loss_off;
  const long long loss_idx = (loss >= c.off && loss < c.off + c.len) ? (long long)(loss - c.off) : -1;
  fg::DevCtx *ctx = fg::ctx_current();
  if ((rc = fg::launch_peer_reduce_sgd(m->pg + c.off, m->pstage + c.off, m->pP[par] + c.off,
                                       m->pP[nx] + c.off, m->pLO[nx] + c.off, S, r, n, m->lr,
                                       loss_idx, region_flag(m, r, 0, ci, 0), val,
                                       ctx ? ctx->d_err : nullptr, m->reduce_blocks, m->red_st)))
    return rc;
  FG_CUDA_TRY(cudaEventRecord(m->ev_red, m->red_st));
  for (int p = 0; p < n; p++) {
    if (p == r) continue;
    const size_t at = c.off + (size_t)r * S;
    FG_CUDA_TRY(cudaStreamWaitEvent(m->ag_st[p], m->ev_red, 0));
    FG_CUDA_TRY(cudaMemcpyAsync(region_f(m, p, 2 + nx, at), m->pP[nx] + at, S * sizeof(float),
                                cudaMemcpyDefault, m->ag_st[p]));
    if (m->push_lo)
      FG_CUDA_TRY(cudaMemcpyAsync(region_f(m, p, 4 + nx, at), m->pLO[nx] + at, S * sizeof(float),
                                  cudaMemcpyDefault, m->ag_st[p]));
    FG_CUDA_TRY(cudaEventRecord(m->ev_ag[p], m->ag_st[p]));
    FG_CUDA_TRY(cudaStreamWaitEvent(m->sig_ag_st, m->ev_ag[p], 0));
  }
  for (int p = 0; p < n; p++) f.p[p] = (p == r) ? nullptr : region_flag(m, p, 1, ci, r);
  if ((rc = fg::launch_peer_signal(f, val, m->sig_ag_st))) return rc;
  if (m->push_lo) return FG_OK;
  // 4. without residuals on the wire: once every peer's shard of this chunk
  //    has landed (and this rank's own reduce is done), recompute the
  //    chunk's TF32 residual here
  FG_CUDA_TRY(cudaStreamWaitEvent(m->arr_st, m->ev_red, 0));
  if ((rc = fg::launch_peer_wait(region_flag(m, r, 1, ci, 0), 1, n, r, val,
                                 ctx ? ctx->d_err : nullptr, m->arr_st)))
    return rc;
  return fg::launch_peer_lo(m->pP[nx] + c.off, m->pLO[nx] + c.off, c.len, m->reduce_blocks,
                            m->arr_st);
}

int join_into(fg_mlp *m, cudaStream_t from) {
  FG_CUDA_TRY(cudaEventRecord(m->ev_join, from));
  FG_CUDA_TRY(cudaStreamWaitEvent(m->st, m->ev_join, 0));
  return FG_OK;
}

// One training step in peer-sharded mode, reading parameter buffer par and
// leaving the updated parameters (and the global loss) in buffer par ^ 1 on
// every rank.  Same kernels as enqueue_step; the gradient exchange of each
// chunk starts as soon as the chunk is complete and overlaps the remaining
// backward GEMMs; the step ends when every peer's all-gather has landed.
int enqueue_step_peer(fg_mlp *m, int par) {
  cudaStream_t st = m->st;
  const int B = m->B;
  int rc;
  m->gemm_launches = 0;
  m->comm_launches = 0;
  if (m->L[0].tc && (rc = fg::launch_split_lo(m->x, m->x_lo, (size_t)B * m->dims[0], st))) return rc;
  for (int l = 0; l < m->nl; l++) {
    Layer &ly = m->L[l];
    const float *in = (l == 0) ? m->x : m->act[l - 1];
    if (ly.tc) {
      if ((rc = run_gemm(m, ly.fwd_p[par], st))) return rc;
    } else if ((rc = fg::launch_skinny_fwd(ly.out, in, ly.Wp[par], ly.bp[par], m->act[l], B, ly.in,
                                           st, m->sms))) {
      return rc;
    }
  }
  const int C = m->dims[m->nl];
  const float rank_scale = 1.0f / (float)m->peer_n;
  if ((rc = fg::launch_xent(m->act[m->nl - 1], m->t, (size_t)B, (size_t)C, m->loss, m->G[m->nl - 1],
                            rank_scale, st, m->scratch, rank_scale)))
    return rc;
  if (m->L[m->nl - 1].tc &&
      (rc = fg::launch_split_lo(m->G[m->nl - 1], m->G_lo[m->nl - 1], (size_t)B * C, st)))
    return rc;
  for (int l = m->nl - 1; l >= 0; l--) {
    Layer &ly = m->L[l];
    const float *in = (l == 0) ? m->x : m->act[l - 1];
    const int c0 = m->pl.first_chunk[l], nc = m->pl.n_chunks[l];
    if (!ly.tc) {
      if ((rc = fg::launch_skinny_bwd(ly.out, m->G[l], in, ly.Wp[par], m->scratch, ly.dW,
                                      l > 0 ? m->G[l - 1] : nullptr,
                                      (l > 0 && m->L[l - 1].tc) ? m->G_lo[l - 1] : nullptr, B,
                                      ly.in, st, m->sms)))
        return rc;
    } else if (nc > 1) {  // dW row block q is chunk q (the last also holds db)
      for (int q = 0; q < nc; q++) {
        if ((rc = run_gemm(m, ly.bwd_w_part[q], st))) return rc;
        if (q == nc - 1 &&
            (rc = fg::launch_reduce_cols(FG_F32, FG_REDUCE_SUM, m->G[l], ly.db, (size_t)B,
                                         (size_t)ly.out, st, m->scratch, m->scratch_bytes)))
          return rc;
        if ((rc = peer_chunk(m, c0 + q, par))) return rc;
      }
      if (l > 0 && (rc = run_gemm(m, ly.bwd_x_p[par], st))) return rc;
      continue;
    } else if ((rc = run_gemm(m, ly.bwd_w, st))) {
      return rc;
    }
    if ((rc = fg::launch_reduce_cols(FG_F32, FG_REDUCE_SUM, m->G[l], ly.db, (size_t)B, (size_t)ly.out,
                                     st, m->scratch, m->scratch_bytes)))
      return rc;
    for (int q = 0; q < nc; q++)
      if ((rc = peer_chunk(m, c0 + q, par))) return rc;
    if (ly.tc && l > 0 && (rc = run_gemm(m, ly.bwd_x_p[par], st))) return rc;
  }
  for (int p = 0; p < m->peer_n; p++) {
    if (p == m->peer_rank) continue;
    if ((rc = join_into(m, m->rs_st[p])) || (rc = join_into(m, m->ag_st[p]))) return rc;
  }
  // join every side stream this step used (a stream with no work in a
  // captured step must not be joined: it is not part of the capture)
  for (cudaStream_t s2 : {m->red_st, m->sig_rs_st, m->sig_ag_st})
    if ((rc = join_into(m, s2))) return rc;
  if (!m->push_lo && (rc = join_into(m, m->arr_st))) return rc;
  fg::DevCtx *ctx = fg::ctx_current();
  return fg::launch_peer_wait(region_flag(m, m->peer_rank, 1, 0, 0), (int)m->pl.chunks.size(),
                              m->peer_n, m->peer_rank, (unsigned int)par + 1,
                              ctx ? ctx->d_err : nullptr, st);
}

}  // namespace

extern "C" {

int fg_mlp_create(fg_device *dev, int n_layers, const int *dims, int batch, float lr,
                  fg_mlp **out) {
  FG_REQUIRE(dev && dims && out, "fg_mlp_create: null argument");
  FG_REQUIRE(n_layers >= 1 && n_layers <= 3, "fg_mlp_create: 1 to 3 layers supported (got %d)",
             n_layers);
  FG_REQUIRE(batch > 0, "fg_mlp_create: batch must be positive");
  FG_CUDA_TRY(cudaSetDevice(dev->ordinal));
  fg_mlp *m = new fg_mlp;
  m->dev = dev;
  m->st = dev->stream;
  m->nl = n_layers;
  m->B = batch;
  m->lr = lr;
  m->dims.assign(dims, dims + n_layers + 1);
  fg::DevCtx *ctx = fg::ctx_current();
  if (ctx && ctx->num_sms) m->sms = ctx->num_sms;
  auto fail = [&](int rc) {
    fg_mlp_destroy(m);
    return rc;
  };
  for (int l = 0; l <= n_layers; l++)
    if (dims[l] <= 0 || (dims[l] % 4 != 0 && l < n_layers))
      return fail(fg::set_error(FG_ERR_UNSUPPORTED,
                                "fg_mlp_create: layer input widths must be multiples of 4 (dims[%d]=%d)",
                                l, dims[l]));
  m->L.resize(n_layers);
  size_t off = 0;
  int rc;
  for (int l = 0; l < n_layers; l++) {
    Layer &ly = m->L[l];
    ly.in = dims[l];
    ly.out = dims[l + 1];
    if (ly.out <= fg::kSkinnyMax) {
      ly.tc = false;
      if (l != n_layers - 1)
        return fail(fg::set_error(FG_ERR_UNSUPPORTED,
                                  "fg_mlp_create: a layer with <= 16 outputs must be the last"));
    } else if (ly.out % 16 == 0) {
      ly.tc = true;
    } else {
      return fail(fg::set_error(FG_ERR_UNSUPPORTED,
                                "fg_mlp_create: layer %d width %d (need <= 16 or a multiple of 16)", l,
                                ly.out));
    }
    ly.bucket_off = off;
    off += pad64((size_t)ly.out * ly.in) + pad64(ly.out) + (l == 0 ? 64 : 0);
    ly.bucket_len = off - ly.bucket_off;
  }
  m->grad_count = off;
  if ((rc = mlp_alloc(m, &m->grad, m->grad_count))) return fail(rc);
  for (int l = 0; l < n_layers; l++) {
    Layer &ly = m->L[l];
    ly.dW = m->grad + ly.bucket_off;
    ly.db = ly.dW + pad64((size_t)ly.out * ly.in);
    if (l == 0) m->loss = ly.db + pad64(ly.out);
    if ((rc = mlp_alloc(m, &ly.W, (size_t)ly.out * ly.in))) return fail(rc);
    if ((rc = mlp_alloc(m, &ly.b, ly.out))) return fail(rc);
    if (ly.tc && (rc = mlp_alloc(m, &ly.W_lo, (size_t)ly.out * ly.in))) return fail(rc);
  }
  if ((rc = mlp_alloc(m, &m->x, (size_t)batch * dims[0]))) return fail(rc);
  if ((rc = mlp_alloc(m, &m->x_lo, (size_t)batch * dims[0]))) return fail(rc);
  if ((rc = mlp_alloc(m, &m->t, (size_t)batch * dims[n_layers]))) return fail(rc);
  m->act.assign(n_layers, nullptr);
  m->act_lo.assign(n_layers, nullptr);
  m->G.assign(n_layers, nullptr);
  m->G_lo.assign(n_layers, nullptr);
  for (int l = 0; l < n_layers; l++) {
    size_t n = (size_t)batch * dims[l + 1];
    if ((rc = mlp_alloc(m, &m->act[l], n))) return fail(rc);
    if ((rc = mlp_alloc(m, &m->G[l], n))) return fail(rc);
    if (m->L[l].tc) {
      if ((rc = mlp_alloc(m, &m->act_lo[l], n))) return fail(rc);
      if ((rc = mlp_alloc(m, &m->G_lo[l], n))) return fail(rc);
    }
  }
  // scratch: column-reduce partials, skinny dW partials, xent row terms
  size_t need = (size_t)batch * 4;
  for (int l = 0; l < n_layers; l++) {
    size_t r = fg::reduce_cols_scratch_bytes((size_t)batch, (size_t)dims[l + 1]);
    if (r > need) need = r;
    if (!m->L[l].tc) {
      fg::SkinnyBwdShape s = fg::skinny_bwd_shape(batch, dims[l], m->sms);
      size_t p = (size_t)s.nchunks * dims[l + 1] * dims[l] * 4;
      if (p > need) need = p;
    }
  }
  m->scratch_bytes = need;
  if ((rc = mlp_alloc(m, &m->scratch, need / 4 + 1))) return fail(rc);
  if ((rc = build_plans(m))) return fail(rc);
  // One stream-K workspace for every GEMM of the step: they all run in
  // order on the step's compute stream.
  {
    float *ws = nullptr;
    if ((rc = mlp_alloc(m, &ws, fg::gemm::stream_k_ws_bytes(m->sms) / 4 + 1))) return fail(rc);
    m->sk_ws = ws;
    for (int l = 0; l < m->nl; l++) {
      Layer &ly = m->L[l];
      if (!ly.tc) continue;
      for (fg::gemm::GemmPlan *pl : {&ly.fwd, &ly.bwd_w, &ly.bwd_x, &ly.bwd_w_half[0],
                                     &ly.bwd_w_half[1]})
        fg::gemm::stream_k_attach(pl, ws, m->sms);
    }
  }
  FG_CUDA_TRY(cudaDeviceSynchronize());
  *out = m;
  return FG_OK;
}

int fg_mlp_destroy(fg_mlp *m) {
  if (!m) return FG_OK;
  cudaSetDevice(m->dev->ordinal);
  cudaDeviceSynchronize();
  if (m->graph) cudaGraphExecDestroy(m->graph);
  for (auto e : m->ev_t0) cudaEventDestroy(e);
  for (auto e : m->ev_t1) cudaEventDestroy(e);
  for (auto e : m->ev_c0) cudaEventDestroy(e);
  for (auto e : m->ev_c1) cudaEventDestroy(e);
  for (auto e : m->ev_bucket) cudaEventDestroy(e);
  for (auto e : m->ev_wread) cudaEventDestroy(e);
  if (m->ev_comm_done) cudaEventDestroy(m->ev_comm_done);
  for (auto e : m->ev_half) cudaEventDestroy(e);
  if (m->comm_st) cudaStreamDestroy(m->comm_st);
  for (auto e : m->ev_ar) cudaEventDestroy(e);
  if (m->ev_sgd_done) cudaEventDestroy(m->ev_sgd_done);
  if (m->sgd_st) cudaStreamDestroy(m->sgd_st);
  for (auto g : m->pgraph)
    if (g) cudaGraphExecDestroy(g);
  for (int j = 0; j < fg::kMaxPeers; j++) {
    if (m->peer_base[j]) cudaIpcCloseMemHandle(m->peer_base[j]);
    if (m->rs_st[j]) cudaStreamDestroy(m->rs_st[j]);
    if (m->ag_st[j]) cudaStreamDestroy(m->ag_st[j]);
    if (m->ev_rs[j]) cudaEventDestroy(m->ev_rs[j]);
    if (m->ev_ag[j]) cudaEventDestroy(m->ev_ag[j]);
  }
  for (cudaStream_t s2 : {m->red_st, m->sig_rs_st, m->sig_ag_st, m->arr_st})
    if (s2) cudaStreamDestroy(s2);
  for (cudaEvent_t e : {m->ev_ready, m->ev_red, m->ev_join, m->ev_staged[0], m->ev_staged[1],
                        m->ev_consumed[0], m->ev_consumed[1]})
    if (e) cudaEventDestroy(e);
  if (m->copy_st) cudaStreamDestroy(m->copy_st);
  for (void *p : m->allocations) cudaFree(p);
  delete m;
  return FG_OK;
}

int fg_mlp_set_params(fg_mlp *m, int layer, const float *h_weight, const float *h_bias) {
  FG_REQUIRE(m && layer >= 0 && layer < m->nl, "fg_mlp_set_params: bad layer");
  Layer &ly = m->L[layer];
  FG_CUDA_TRY(cudaSetDevice(m->dev->ordinal));
  if (h_weight) {
    FG_CUDA_TRY(cudaMemcpyAsync(ly.W, h_weight, sizeof(float) * ly.out * ly.in,
                                cudaMemcpyHostToDevice, m->st));
    if (ly.tc) {
      int rc = fg::launch_split_lo(ly.W, ly.W_lo, (size_t)ly.out * ly.in, m->st);
      if (rc) return rc;
    }
  }
  if (h_bias)
    FG_CUDA_TRY(cudaMemcpyAsync(ly.b, h_bias, sizeof(float) * ly.out, cudaMemcpyHostToDevice, m->st));
  FG_CUDA_TRY(cudaStreamSynchronize(m->st));
  return FG_OK;
}

int fg_mlp_get_params(fg_mlp *m, int layer, float *h_weight, float *h_bias) {
  FG_REQUIRE(m && layer >= 0 && layer < m->nl, "fg_mlp_get_params: bad layer");
  Layer &ly = m->L[layer];
  FG_CUDA_TRY(cudaSetDevice(m->dev->ordinal));
  if (h_weight)
    FG_CUDA_TRY(cudaMemcpyAsync(h_weight, ly.W, sizeof(float) * ly.out * ly.in,
                                cudaMemcpyDeviceToHost, m->st));
  if (h_bias)
    FG_CUDA_TRY(cudaMemcpyAsync(h_bias, ly.b, sizeof(float) * ly.out, cudaMemcpyDeviceToHost, m->st));
  FG_CUDA_TRY(cudaStreamSynchronize(m->st));
  return fg_check_device_error();
}

int fg_mlp_get_grads(fg_mlp *m, int layer, float *h_dweight, float *h_dbias) {
  FG_REQUIRE(m && layer >= 0 && layer < m->nl, "fg_mlp_get_grads: bad layer");
  Layer &ly = m->L[layer];
  FG_CUDA_TRY(cudaSetDevice(m->dev->ordinal));
  if (m->peer) {
    // Each shard's reduced gradient lives in its owner's gradient area.
    FG_CUDA_TRY(cudaStreamSynchronize(m->st));
    const int c0 = m->pl.first_chunk[layer], nc = m->pl.n_chunks[layer];
    const size_t base = m->pl.chunks[c0].off;
    const fg::PeerChunk &last = m->pl.chunks[c0 + nc - 1];
    std::vector<float> bucket(last.off + last.len - base);
    for (int ci = c0; ci < c0 + nc; ci++) {
      const fg::PeerChunk &c = m->pl.chunks[ci];
      const size_t S = c.len / m->peer_n;
      for (int j = 0; j < m->peer_n; j++)
        FG_CUDA_TRY(cudaMemcpy(bucket.data() + (c.off - base) + (size_t)j * S,
                               region_f(m, j, 0, c.off + (size_t)j * S), S * sizeof(float),
                               cudaMemcpyDefault));
    }
    if (h_dweight)
      memcpy(h_dweight, bucket.data() + (m->pl.w_off[layer] - base), sizeof(float) * ly.out * ly.in);
    if (h_dbias) memcpy(h_dbias, bucket.data() + (m->pl.b_off[layer] - base), sizeof(float) * ly.out);
    return fg_check_device_error();
  }
  if (h_dweight)
    FG_CUDA_TRY(cudaMemcpyAsync(h_dweight, ly.dW, sizeof(float) * ly.out * ly.in,
                                cudaMemcpyDeviceToHost, m->st));
  if (h_dbias)
    FG_CUDA_TRY(cudaMemcpyAsync(h_dbias, ly.db, sizeof(float) * ly.out, cudaMemcpyDeviceToHost, m->st));
  FG_CUDA_TRY(cudaStreamSynchronize(m->st));
  return fg_check_device_error();
}

int fg_mlp_attach_comm(fg_mlp *m, fg_comm *comm) {
  FG_REQUIRE(m, "fg_mlp_attach_comm: null mlp");
  FG_REQUIRE(!m->region, "fg_mlp_attach_comm: this step uses the peer-sharded exchange");
  FG_CUDA_TRY(cudaSetDevice(m->dev->ordinal));
  if (m->graph) {
    cudaGraphExecDestroy(m->graph);
    m->graph = nullptr;
  }
  m->comm = comm;
  // The backward GEMMs that run while gradient all-reduces are in flight
  // leave SMs to the collective's kernels; a persistent grid over every SM
  // would keep them from starting until the GEMM ends.
  const int reserve = comm && fg::comm_nranks(comm) > 1 ? fg::comm_sm_reserve() : 0;
  for (int l = 0; l < m->nl; l++) {
    Layer &ly = m->L[l];
    const int cap = reserve ? m->sms - reserve : 0;
    if (l < m->nl - 1) ly.bwd_x.max_ctas = cap;
    ly.bwd_w.max_ctas = (l < m->nl - 1) ? cap : 0;
    ly.bwd_w_half[0].max_ctas = cap;
    ly.bwd_w_half[1].max_ctas = cap;
  }
  if (comm && !m->comm_st) {
    FG_CUDA_TRY(cudaStreamCreateWithFlags(&m->comm_st, cudaStreamNonBlocking));
    m->ev_bucket.resize(m->nl);
    for (auto &e : m->ev_bucket) FG_CUDA_TRY(cudaEventCreateWithFlags(&e, cudaEventDisableTiming));
    m->ev_wread.resize(m->nl);
    for (auto &e : m->ev_wread) FG_CUDA_TRY(cudaEventCreateWithFlags(&e, cudaEventDisableTiming));
    FG_CUDA_TRY(cudaEventCreateWithFlags(&m->ev_comm_done, cudaEventDisableTiming));
    m->ev_half.resize(m->nl);
    for (auto &e : m->ev_half) FG_CUDA_TRY(cudaEventCreateWithFlags(&e, cudaEventDisableTiming));
    FG_CUDA_TRY(cudaStreamCreateWithFlags(&m->sgd_st, cudaStreamNonBlocking));
    m->ev_ar.resize(2 * (size_t)m->nl);
    for (auto &e : m->ev_ar) FG_CUDA_TRY(cudaEventCreateWithFlags(&e, cudaEventDisableTiming));
    FG_CUDA_TRY(cudaEventCreateWithFlags(&m->ev_sgd_done, cudaEventDisableTiming));
  }
  return FG_OK;
}

int fg_mlp_input_slots(fg_mlp *m, float **d_x, float **d_targets) {
  FG_REQUIRE(m, "fg_mlp_input_slots: null mlp");
  if (d_x) *d_x = m->x;
  if (d_targets) *d_targets = m->t;
  return FG_OK;
}

int fg_mlp_use_graph(fg_mlp *m, int enable) {
  FG_REQUIRE(m, "fg_mlp_use_graph: null mlp");
  m->use_graph = enable != 0;
  if (!m->use_graph && m->graph) {
    cudaGraphExecDestroy(m->graph);
    m->graph = nullptr;
  }
  for (auto &g : m->pgraph)
    if (!m->use_graph && g) {
      cudaGraphExecDestroy(g);
      g = nullptr;
    }
  return FG_OK;
}

int fg_mlp_step(fg_mlp *m, float *d_loss_out) {
  FG_REQUIRE(m, "fg_mlp_step: null mlp");
  FG_CUDA_TRY(cudaSetDevice(m->dev->ordinal));
  int rc;
  if (m->region) {
    FG_REQUIRE(m->peer, "fg_mlp_step: fg_mlp_peer_connect has not been called");
    const int par = m->par;
    if (m->use_graph && m->pgraph[par]) {
      FG_CUDA_TRY(cudaGraphLaunch(m->pgraph[par], m->st));
    } else {
      // the first step of each parity runs eagerly (every rank takes part),
      // then its graph is captured for the later steps of that parity
      uint64_t before = fg_kernel_launches();
      if ((rc = enqueue_step_peer(m, par))) return rc;
      m->launches_per_step = (int)(fg_kernel_launches() - before);
      if (m->use_graph) {
        FG_CUDA_TRY(cudaStreamSynchronize(m->st));
        cudaGraph_t g;
        FG_CUDA_TRY(cudaStreamBeginCapture(m->st, cudaStreamCaptureModeThreadLocal));
        rc = enqueue_step_peer(m, par);
        cudaError_t ce = cudaStreamEndCapture(m->st, &g);
        if (rc) {
          if (ce == cudaSuccess) cudaGraphDestroy(g);
          return rc;
        }
        FG_CUDA_TRY(ce);
        cudaError_t ie = cudaGraphInstantiate(&m->pgraph[par], g, 0);
        cudaGraphDestroy(g);
        FG_CUDA_TRY(ie);
      }
    }
    m->par ^= 1;
    peer_point(m);
    if (d_loss_out)
      FG_CUDA_TRY(cudaMemcpyAsync(d_loss_out, m->pP[m->par] + m->pl.loss_off, sizeof(float),
                                  cudaMemcpyDeviceToDevice, m->st));
    return FG_OK;
  }
  if (m->use_graph) {
    if (!m->graph) {
      // First call: run eagerly once (counts launches, settles lazy init),
      // then capture the same sequence.
      uint64_t before = fg_kernel_launches();
      if ((rc = enqueue_step(m))) return rc;
      m->launches_per_step = (int)(fg_kernel_launches() - before);
      FG_CUDA_TRY(cudaStreamSynchronize(m->st));
      cudaGraph_t g;
      FG_CUDA_TRY(cudaStreamBeginCapture(m->st, cudaStreamCaptureModeThreadLocal));
      rc = enqueue_step(m);
      cudaError_t ce = cudaStreamEndCapture(m->st, &g);
      if (rc) {
        if (ce == cudaSuccess) cudaGraphDestroy(g);
        return rc;
      }
      FG_CUDA_TRY(ce);
      cudaError_t ie = cudaGraphInstantiate(&m->graph, g, 0);
      cudaGraphDestroy(g);
      FG_CUDA_TRY(ie);
    } else {
      FG_CUDA_TRY(cudaGraphLaunch(m->graph, m->st));
    }
  } else {
    uint64_t before = fg_kernel_launches();
    if ((rc = enqueue_step(m))) return rc;
    m->launches_per_step = (int)(fg_kernel_launches() - before);
  }
  if (d_loss_out)
    FG_CUDA_TRY(cudaMemcpyAsync(d_loss_out, m->loss, sizeof(float), cudaMemcpyDeviceToDevice, m->st));
  return FG_OK;
}

int fg_mlp_step_host(fg_mlp *m, const float *h_x, const float *h_targets, float *h_loss) {
  FG_REQUIRE(m && h_x && h_targets, "fg_mlp_step_host: null argument");
  FG_CUDA_TRY(cudaSetDevice(m->dev->ordinal));
  FG_CUDA_TRY(cudaMemcpyAsync(m->x, h_x, sizeof(float) * (size_t)m->B * m->dims[0],
                              cudaMemcpyHostToDevice, m->st));
  FG_CUDA_TRY(cudaMemcpyAsync(m->t, h_targets, sizeof(float) * (size_t)m->B * m->dims[m->nl],
                              cudaMemcpyHostToDevice, m->st));
  int rc = fg_mlp_step(m, nullptr);
  if (rc) return rc;
  if (h_loss) {
    // peer-sharded: the global loss travels with the parameters it produced
    const float *src = m->region ? m->pP[m->par] + m->pl.loss_off : m->loss;
    FG_CUDA_TRY(cudaMemcpyAsync(h_loss, src, sizeof(float), cudaMemcpyDeviceToHost, m->st));
    FG_CUDA_TRY(cudaStreamSynchronize(m->st));
    return fg_check_device_error();
  }
  return FG_OK;
}

int fg_mlp_step_host_next(fg_mlp *m, const float *h_x, const float *h_targets,
                          const float *h_x_next, const float *h_targets_next, float *h_loss) {
  FG_REQUIRE(m && h_x && h_targets, "fg_mlp_step_host_next: null argument");
  FG_REQUIRE(!h_x_next == !h_targets_next,
             "fg_mlp_step_host_next: give both next-batch pointers or neither");
  FG_CUDA_TRY(cudaSetDevice(m->dev->ordinal));
  const size_t xb = sizeof(float) * (size_t)m->B * m->dims[0];
  const size_t tb = sizeof(float) * (size_t)m->B * m->dims[m->nl];
  int rc;
  if (!m->copy_st) {
    for (int i = 0; i < 2; i++) {
      if ((rc = mlp_alloc(m, &m->stage_x[i], (size_t)m->B * m->dims[0]))) return rc;
      if ((rc = mlp_alloc(m, &m->stage_t[i], (size_t)m->B * m->dims[m->nl]))) return rc;
      FG_CUDA_TRY(cudaEventCreateWithFlags(&m->ev_staged[i], cudaEventDisableTiming));
      FG_CUDA_TRY(cudaEventCreateWithFlags(&m->ev_consumed[i], cudaEventDisableTiming));
    }
    FG_CUDA_TRY(cudaStreamCreateWithFlags(&m->copy_st, cudaStreamNonBlocking));
  }
  // This step's batch: staged by the previous call when it named these
  // buffers as its next batch, else uploaded now.
  const int cur = m->next_slot;
  if (m->staged_x != h_x || m->staged_t != h_targets) {
    FG_CUDA_TRY(cudaStreamWaitEvent(m->copy_st, m->ev_consumed[cur], 0));
    FG_CUDA_TRY(cudaMemcpyAsync(m->stage_x[cur], h_x, xb, cudaMemcpyHostToDevice, m->copy_st));
    FG_CUDA_TRY(cudaMemcpyAsync(m->stage_t[cur], h_targets, tb, cudaMemcpyHostToDevice, m->copy_st));
    FG_CUDA_TRY(cudaEventRecord(m->ev_staged[cur], m->copy_st));
  }
  m->staged_x = m->staged_t = nullptr;
  FG_CUDA_TRY(cudaStreamWaitEvent(m->st, m->ev_staged[cur], 0));
  if ((size_t)m->B * m->dims[0] % 4 == 0 && (size_t)m->B * m->dims[m->nl] % 4 == 0) {
    if ((rc = fg::launch_copy2(m->stage_x[cur], m->x, (size_t)m->B * m->dims[0], m->stage_t[cur],
                               m->t, (size_t)m->B * m->dims[m->nl], m->st)))
      return rc;
  } else {
    FG_CUDA_TRY(cudaMemcpyAsync(m->x, m->stage_x[cur], xb, cudaMemcpyDeviceToDevice, m->st));
    FG_CUDA_TRY(cudaMemcpyAsync(m->t, m->stage_t[cur], tb, cudaMemcpyDeviceToDevice, m->st));
  }
  FG_CUDA_TRY(cudaEventRecord(m->ev_consumed[cur], m->st));
  // The next batch goes into the other slot on the copy stream while this
  // step computes (once that slot's previous batch has been moved out).
  if (h_x_next) {
    const int nxt = cur ^ 1;
    FG_CUDA_TRY(cudaStreamWaitEvent(m->copy_st, m->ev_consumed[nxt], 0));
    FG_CUDA_TRY(cudaMemcpyAsync(m->stage_x[nxt], h_x_next, xb, cudaMemcpyHostToDevice, m->copy_st));
    FG_CUDA_TRY(cudaMemcpyAsync(m->stage_t[nxt], h_targets_next, tb, cudaMemcpyHostToDevice,
                                m->copy_st));
    FG_CUDA_TRY(cudaEventRecord(m->ev_staged[nxt], m->copy_st));
    m->next_slot = nxt;
    m->staged_x = h_x_next;
    m->staged_t = h_targets_next;
  }
  if ((rc = fg_mlp_step(m, nullptr))) return rc;
  if (h_loss) {
    const float *src = m->region ? m->pP[m->par] + m->pl.loss_off : m->loss;
    FG_CUDA_TRY(cudaMemcpyAsync(h_loss, src, sizeof(float), cudaMemcpyDeviceToHost, m->st));
    FG_CUDA_TRY(cudaStreamSynchronize(m->st));
    return fg_check_device_error();
  }
  return FG_OK;
}

int fg_mlp_get_activations(fg_mlp *m, int layer, float *h_out) {
  FG_REQUIRE(m && h_out && layer >= 0 && layer < m->nl, "fg_mlp_get_activations: bad argument");
  FG_CUDA_TRY(cudaSetDevice(m->dev->ordinal));
  FG_CUDA_TRY(cudaMemcpyAsync(h_out, m->act[layer], sizeof(float) * (size_t)m->B * m->dims[layer + 1],
                              cudaMemcpyDeviceToHost, m->st));
  FG_CUDA_TRY(cudaStreamSynchronize(m->st));
  return fg_check_device_error();
}

int fg_mlp_get_logits(fg_mlp *m, float *h_logits) {
  FG_REQUIRE(m && h_logits, "fg_mlp_get_logits: null argument");
  FG_CUDA_TRY(cudaSetDevice(m->dev->ordinal));
  FG_CUDA_TRY(cudaMemcpyAsync(h_logits, m->act[m->nl - 1],
                              sizeof(float) * (size_t)m->B * m->dims[m->nl], cudaMemcpyDeviceToHost,
                              m->st));
  FG_CUDA_TRY(cudaStreamSynchronize(m->st));
  return fg_check_device_error();
}

int fg_mlp_enable_gemm_timing(fg_mlp *m, int enable) {
  FG_REQUIRE(m, "fg_mlp_enable_gemm_timing: null mlp");
  FG_CUDA_TRY(cudaSetDevice(m->dev->ordinal));
  if (m->graph) {  // the captured sequence changes
    cudaGraphExecDestroy(m->graph);
    m->graph = nullptr;
  }
  for (auto &g : m->pgraph)
    if (g) {
      cudaGraphExecDestroy(g);
      g = nullptr;
    }
  m->timing = enable != 0;
  if (m->timing && m->ev_t0.empty()) {
    const int n = 3 * m->nl + fg::kMaxPeerParts;
    m->ev_t0.resize(n);
    m->ev_t1.resize(n);
    m->gemm_flops.assign(n, 0.0);
    for (int i = 0; i < n; i++) {
      FG_CUDA_TRY(cudaEventCreate(&m->ev_t0[i]));
      FG_CUDA_TRY(cudaEventCreate(&m->ev_t1[i]));
    }
    const int nc = m->nl + 1;
    m->ev_c0.resize(nc);
    m->ev_c1.resize(nc);
    m->comm_bytes.assign(nc, 0.0);
    for (int i = 0; i < nc; i++) {
      FG_CUDA_TRY(cudaEventCreate(&m->ev_c0[i]));
      FG_CUDA_TRY(cudaEventCreate(&m->ev_c1[i]));
    }
  }
  return FG_OK;
}

int fg_mlp_gemm_times(fg_mlp *m, float *ms, double *flops, int capacity, int *count) {
  FG_REQUIRE(m && count && (capacity == 0 || (ms && flops)), "fg_mlp_gemm_times: null argument");
  FG_REQUIRE(m->timing, "fg_mlp_gemm_times: timing is not enabled");
  FG_CUDA_TRY(cudaSetDevice(m->dev->ordinal));
  FG_CUDA_TRY(cudaStreamSynchronize(m->st));
  int n = m->gemm_launches < (int)m->ev_t0.size() ? m->gemm_launches : (int)m->ev_t0.size();
  if (n > capacity) n = capacity;
  for (int i = 0; i < n; i++) {
    FG_CUDA_TRY(cudaEventElapsedTime(&ms[i], m->ev_t0[i], m->ev_t1[i]));
    flops[i] = m->gemm_flops[i];
  }
  *count = n;
  return FG_OK;
}

int fg_mlp_comm_times(fg_mlp *m, float *ms, double *bytes, int capacity, int *count) {
  FG_REQUIRE(m && count && (capacity == 0 || (ms && bytes)), "fg_mlp_comm_times: null argument");
  FG_REQUIRE(m->timing, "fg_mlp_comm_times: timing is not enabled");
  FG_CUDA_TRY(cudaSetDevice(m->dev->ordinal));
  FG_CUDA_TRY(cudaStreamSynchronize(m->st));
  int n = m->comm_launches < (int)m->ev_c0.size() ? m->comm_launches : (int)m->ev_c0.size();
  if (n > capacity) n = capacity;
  for (int i = 0; i < n; i++) {
    FG_CUDA_TRY(cudaEventElapsedTime(&ms[i], m->ev_c0[i], m->ev_c1[i]));
    bytes[i] = m->comm_bytes[i];
  }
  *count = n;
  return FG_OK;
}

int fg_mlp_launch_count(fg_mlp *m, int *count) {
  FG_REQUIRE(m && count, "fg_mlp_launch_count: null argument");
  *count = m->launches_per_step;
  return FG_OK;
}

// ---- peer-sharded data parallelism ----------------------------------------
// Handle bytes: [0, 64) cudaIpcMemHandle_t of the region, then region bytes
// (u64), rank, nranks, parts (i32 each), layout digest (u32), magic.
static const char kPeerMagic[8] = {'F', 'G', 'P', 'E', 'E', 'R', '0', '1'};
struct PeerHandle {
  cudaIpcMemHandle_t ipc;
  unsigned long long bytes;
  int rank, nranks, parts;
  unsigned int digest;
  char magic[8];
};
static_assert(sizeof(PeerHandle) <= FG_PEER_HANDLE_BYTES, "peer handle size");

static int env_int(const char *name, int dflt, int lo, int hi) {
  const char *e = getenv(name);
  int v = (e && *e) ? atoi(e) : dflt;
  return v < lo ? lo : (v > hi ? hi : v);
}

int fg_mlp_peer_prepare(fg_mlp *m, int rank, int nranks, int chunks,
                        char handle_out[FG_PEER_HANDLE_BYTES]) {
  FG_REQUIRE(m && handle_out, "fg_mlp_peer_prepare: null argument");
  FG_REQUIRE(!m->comm, "fg_mlp_peer_prepare: an NCCL communicator is attached");
  FG_REQUIRE(!m->region, "fg_mlp_peer_prepare: already prepared");
  FG_REQUIRE(nranks >= 2 && nranks <= fg::kMaxPeers && rank >= 0 && rank < nranks,
             "fg_mlp_peer_prepare: rank %d of %d (2 to %d ranks)", rank, nranks, fg::kMaxPeers);
  FG_CUDA_TRY(cudaSetDevice(m->dev->ordinal));
  fg::PeerLayout L;
  int rc = fg::peer_layout(m->nl, m->dims.data(), nranks, chunks, &L);
  if (rc) return rc;
  FG_CUDA_TRY(cudaStreamSynchronize(m->st));
  float *region = nullptr;
  if ((rc = mlp_alloc(m, &region, L.region))) return rc;
  // the zero fill runs on the legacy default stream, which does not order
  // with the step's non-blocking stream: finish it before the copies below
  FG_CUDA_TRY(cudaDeviceSynchronize());
  m->region = region;
  m->pl = L;
  m->peer_rank = rank;
  m->peer_n = nranks;
  m->pg = region;
  m->pstage = region + L.grad;
  for (int q = 0; q < 2; q++) {
    m->pP[q] = region + (size_t)(2 + q) * L.grad;
    m->pLO[q] = region + (size_t)(4 + q) * L.grad;
  }
  m->pflags = reinterpret_cast<unsigned int *>(region + 6 * L.grad);
  // the current parameters (and residuals) become buffer 0
  for (int l = 0; l < m->nl; l++) {
    Layer &ly = m->L[l];
    const size_t nw = (size_t)ly.out * ly.in;
    for (int q = 0; q < 2; q++) {
      ly.Wp[q] = m->pP[q] + L.w_off[l];
      ly.bp[q] = m->pP[q] + L.b_off[l];
      ly.W_lo_p[q] = m->pLO[q] + L.w_off[l];
    }
    FG_CUDA_TRY(cudaMemcpyAsync(ly.Wp[0], ly.W, nw * sizeof(float), cudaMemcpyDeviceToDevice, m->st));
    FG_CUDA_TRY(cudaMemcpyAsync(ly.bp[0], ly.b, ly.out * sizeof(float), cudaMemcpyDeviceToDevice, m->st));
    if ((rc = fg::launch_split_lo(ly.Wp[0], ly.W_lo_p[0], nw, m->st))) return rc;
    ly.dW = m->pg + L.w_off[l];
    ly.db = m->pg + L.b_off[l];
  }
  m->loss = m->pg + L.loss_off;
  // GEMM plans for both parameter buffers, and layer 0's dW row blocks
  for (int q = 1; q >= 0; q--) {
    m->par = q;
    peer_point(m);
    if ((rc = build_plans(m))) return rc;
    for (auto &ly : m->L) {
      ly.fwd_p[q] = ly.fwd;
      ly.bwd_x_p[q] = ly.bwd_x;
    }
  }
  for (int l = 0; l < m->nl; l++) {
    Layer &ly = m->L[l];
    const int parts = L.n_chunks[l];
    if (!ly.tc || parts < 2) continue;
    const int rows = ly.out / parts;
    const float *in = (l == 0) ? m->x : m->act[l - 1];
    const float *in_lo = (l == 0) ? m->x_lo : m->act_lo[l - 1];
    for (int q = 0; q < parts; q++)
      if ((rc = fg::gemm::make_plan(rows, ly.in, m->B, m->G[l] + q * rows, m->G_lo[l] + q * rows,
                                    ly.out, in, in_lo, ly.in, ly.dW + (size_t)q * rows * ly.in,
                                    nullptr, ly.in, FG_GEMM_A_MN_MAJOR | FG_GEMM_B_MN_MAJOR,
                                    FG_EPI_NONE, nullptr, nullptr, 0, &ly.bwd_w_part[q])))
        return rc;
  }
  // SMs left free beside the backward GEMMs (FG_PEER_SM_RESERVE, default 0:
  // the exchange moves bytes with the copy engines; the owner's reduce
  // kernel shares SMs with the GEMM's CTAs)
  const int reserve = env_int("FG_PEER_SM_RESERVE", 0, 0, 64);
  const int cap = reserve ? m->sms - reserve : 0;
  for (auto &ly : m->L) {
    if (!ly.tc) continue;
    for (fg::gemm::GemmPlan *p2 : {&ly.fwd_p[0], &ly.fwd_p[1], &ly.bwd_w, &ly.bwd_x_p[0], &ly.bwd_x_p[1],
                                   &ly.fwd, &ly.bwd_x})
      fg::gemm::stream_k_attach(p2, m->sk_ws, m->sms);
    ly.bwd_w.max_ctas = cap;
    ly.bwd_x_p[0].max_ctas = ly.bwd_x_p[1].max_ctas = cap;
    const int l = (int)(&ly - m->L.data());
    for (int q = 0; q < L.n_chunks[l] && L.n_chunks[l] > 1; q++) {
      fg::gemm::stream_k_attach(&ly.bwd_w_part[q], m->sk_ws, m->sms);
      ly.bwd_w_part[q].max_ctas = cap;
    }
  }
  m->reduce_blocks = env_int("FG_PEER_REDUCE_BLOCKS", 64, 1, 1024);
  m->push_lo = env_int("FG_PEER_PUSH_LO", 1, 0, 1) != 0;
  m->par = 0;
  peer_point(m);
  // streams: copies to each peer (reduce-scatter and all-gather apart, so
  // one chunk's all-gather never holds up the next chunk's reduce-scatter);
  // the owner's reduce and the two signal streams at the highest priority
  int lo_prio = 0, hi_prio = 0;
  FG_CUDA_TRY(cudaDeviceGetStreamPriorityRange(&lo_prio, &hi_prio));
  for (int p = 0; p < nranks; p++) {
    if (p == rank) continue;
    FG_CUDA_TRY(cudaStreamCreateWithFlags(&m->rs_st[p], cudaStreamNonBlocking));
    FG_CUDA_TRY(cudaStreamCreateWithFlags(&m->ag_st[p], cudaStreamNonBlocking));
    FG_CUDA_TRY(cudaEventCreateWithFlags(&m->ev_rs[p], cudaEventDisableTiming));
    FG_CUDA_TRY(cudaEventCreateWithFlags(&m->ev_ag[p], cudaEventDisableTiming));
  }
  for (cudaStream_t *s2 : {&m->red_st, &m->sig_rs_st, &m->sig_ag_st, &m->arr_st})
    FG_CUDA_TRY(cudaStreamCreateWithPriority(s2, cudaStreamNonBlocking, hi_prio));
  for (cudaEvent_t *e : {&m->ev_ready, &m->ev_red, &m->ev_join})
    FG_CUDA_TRY(cudaEventCreateWithFlags(e, cudaEventDisableTiming));
  if (m->graph) {
    cudaGraphExecDestroy(m->graph);
    m->graph = nullptr;
  }
  PeerHandle h;
  memset(&h, 0, sizeof(h));
  FG_CUDA_TRY(cudaIpcGetMemHandle(&h.ipc, region));
  h.bytes = (unsigned long long)L.region * sizeof(float);
  h.rank = rank;
  h.nranks = nranks;
  h.parts = L.parts;
  h.digest = L.digest;
  memcpy(h.magic, kPeerMagic, sizeof(kPeerMagic));
  memset(handle_out, 0, FG_PEER_HANDLE_BYTES);
  memcpy(handle_out, &h, sizeof(h));
  FG_CUDA_TRY(cudaStreamSynchronize(m->st));
  return FG_OK;
}

int fg_mlp_peer_connect(fg_mlp *m, const char *handles) {
  FG_REQUIRE(m && handles, "fg_mlp_peer_connect: null argument");
  FG_REQUIRE(m->region, "fg_mlp_peer_connect: fg_mlp_peer_prepare has not been called");
  FG_REQUIRE(!m->peer, "fg_mlp_peer_connect: already connected");
  FG_CUDA_TRY(cudaSetDevice(m->dev->ordinal));
  // every handle must describe the same layout, in rank order
  for (int j = 0; j < m->peer_n; j++) {
    PeerHandle h;
    memcpy(&h, handles + (size_t)j * FG_PEER_HANDLE_BYTES, sizeof(h));
    FG_REQUIRE(memcmp(h.magic, kPeerMagic, sizeof(kPeerMagic)) == 0,
               "fg_mlp_peer_connect: handle %d is not a peer handle", j);
    FG_REQUIRE(h.rank == j && h.nranks == m->peer_n,
               "fg_mlp_peer_connect: handle %d is rank %d of %d (expected %d of %d)", j, h.rank,
               h.nranks, j, m->peer_n);
    FG_REQUIRE(h.digest == m->pl.digest && h.bytes == (unsigned long long)m->pl.region * sizeof(float),
               "fg_mlp_peer_connect: rank %d has a different exchange layout (dims, ranks or chunks differ)",
               j);
  }
  for (int j = 0; j < m->peer_n; j++) {
    if (j == m->peer_rank) continue;
    PeerHandle h;
    memcpy(&h, handles + (size_t)j * FG_PEER_HANDLE_BYTES, sizeof(h));
    void *p = nullptr;
    cudaError_t e = cudaIpcOpenMemHandle(&p, h.ipc, cudaIpcMemLazyEnablePeerAccess);
    if (e != cudaSuccess) {
      for (int k = 0; k < j; k++)
        if (m->peer_base[k]) {
          cudaIpcCloseMemHandle(m->peer_base[k]);
          m->peer_base[k] = nullptr;
        }
      return fg::set_error(FG_ERR_CUDA, "fg_mlp_peer_connect: mapping rank %d's region failed: %s", j,
                           cudaGetErrorString(e));
    }
    m->peer_base[j] = static_cast<char *>(p);
  }
  m->peer = true;
  return FG_OK;
}

int fg_mlp_peer_disconnect(fg_mlp *m) {
  FG_REQUIRE(m, "fg_mlp_peer_disconnect: null mlp");
  FG_CUDA_TRY(cudaSetDevice(m->dev->ordinal));
  FG_CUDA_TRY(cudaDeviceSynchronize());
  for (int j = 0; j < fg::kMaxPeers; j++)
    if (m->peer_base[j]) {
      FG_CUDA_TRY(cudaIpcCloseMemHandle(m->peer_base[j]));
      m->peer_base[j] = nullptr;
    }
  m->peer = false;
  return fg_check_device_error();
}

}  // extern "C"
