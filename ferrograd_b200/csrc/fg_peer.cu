// Peer-sharded gradient exchange of the data-parallel MLP step.
//
// The reference is single-device (src/device.rs:37-41); this is the one
// exchange data parallelism adds, built for ranks that share an NVLink
// domain.  The bytes move with the copy engines (cudaMemcpyAsync into a
// peer's memory mapped through CUDA IPC), so the collective takes no SMs
// from the tensor-core GEMMs it overlaps; the SMs only do the owner's fused
// reduce + SGD pass over its shard, an HBM-bound kernel over local memory.
// Ranks order the phases with 32-bit flag words written into each other's
// regions; every wait is bounded by the global timer and sets the device
// error word (role 4) when it expires instead of hanging.
#include <string.h>

#include "fg_internal.h"
#include "fg_peer.cuh"

namespace fg {

constexpr unsigned kErrPeer = 4u << 16;

namespace {

size_t pad_to(size_t n, size_t unit) { return (n + unit - 1) / unit * unit; }

uint32_t fnv(uint32_t h, uint64_t v) {
  for (int i = 0; i < 8; i++) {
    h ^= (uint32_t)(v & 0xff);
    h *= 16777619u;
    v >>= 8;
  }
  return h;
}

__device__ __forceinline__ unsigned long long global_ns() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

__device__ __forceinline__ unsigned int ld_acquire_sys(const unsigned int *p) {
  unsigned int v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

__device__ __forceinline__ void st_release_sys(unsigned int *p, unsigned int v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

// Bounded wait until flags[j] == val for all j < n, j != skip.
__device__ bool wait_flags(const unsigned int *flags, int n, int skip, unsigned int val,
                           unsigned int *err, unsigned int code, unsigned long long wait_ns) {
  const unsigned long long t0 = global_ns();
  for (int j = 0; j < n; j++) {
    if (j == skip) continue;
    while (ld_acquire_sys(flags + j) != val) {
      if (global_ns() - t0 > wait_ns) {
        if (err) atomicOr(err, kErrPeer | code);
        return false;
      }
      __nanosleep(256);
    }
  }
  return true;
}

__device__ __forceinline__ float sgd_step(float p, float g, float lr) {
  return __fadd_rn(p, -__fmul_rn(g, lr));  // src/optim.rs:60-71: p + (-(g * lr))
}
__device__ __forceinline__ float tf32_rest(float v) {
  return __fsub_rn(v, __uint_as_float(__float_as_uint(v) & 0xffffe000u));
}
__device__ __forceinline__ float4 add4(float4 a, float4 b) {
  return make_float4(__fadd_rn(a.x, b.x), __fadd_rn(a.y, b.y), __fadd_rn(a.z, b.z),
                     __fadd_rn(a.w, b.w));
}

__global__ void k_peer_signal(PeerFlagPtrs ptrs, unsigned int val) {
  const int j = threadIdx.x;
  if (j < kMaxPeers && ptrs.p[j]) {
    __threadfence_system();
    st_release_sys(ptrs.p[j], val);
  }
}

// Runs after a one-block k_peer_wait on its stream has seen every sender's
// flag, so its blocks never sit on SMs waiting.  If a wait of the exchange
// gave up (the error word carries kErrPeer), the staged contributions may be
// stale: nothing is written, so no update built from them reaches the next
// step's parameters before the host reads the error.
__global__ void __launch_bounds__(256)
    k_peer_reduce_sgd(float *__restrict__ grad, const float *__restrict__ stage,
                      const float *__restrict__ p_cur, float *__restrict__ p_next,
                      float *__restrict__ lo_next, size_t shard, int rank, int nranks, float lr,
                      long long loss_idx, const unsigned int *err) {
  if (err && (*reinterpret_cast<const volatile unsigned int *>(err) & kErrPeer)) return;
  const size_t base = (size_t)rank * shard;
  const size_t n4 = shard / 4;
  const size_t stride = (size_t)gridDim.x * blockDim.x;
  for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < n4; i += stride) {
    float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
    for (int j = 0; j < nranks; j++) {
      // peers' contributions arrive through the copy engines: read them
      // from L2, never from a stale L1 line
      const float4 v = (j == rank) ? reinterpret_cast<const float4 *>(grad + base)[i]
                                   : __ldcg(reinterpret_cast<const float4 *>(stage + (size_t)j * shard) + i);
      acc = (j == 0) ? v : add4(acc, v);
    }
    reinterpret_cast<float4 *>(grad + base)[i] = acc;
    const float4 pc = __ldcs(reinterpret_cast<const float4 *>(p_cur + base) + i);
    float4 pn = make_float4(sgd_step(pc.x, acc.x, lr), sgd_step(pc.y, acc.y, lr),
                            sgd_step(pc.z, acc.z, lr), sgd_step(pc.w, acc.w, lr));
    const long long e = (long long)(base + 4 * i);
    if (loss_idx >= e && loss_idx < e + 4) {
      const int k = (int)(loss_idx - e);
      if (k == 0) pn.x = acc.x;
      if (k == 1) pn.y = acc.y;
      if (k == 2) pn.z = acc.z;
      if (k == 3) pn.w = acc.w;
    }
    reinterpret_cast<float4 *>(p_next + base)[i] = pn;
    reinterpret_cast<float4 *>(lo_next + base)[i] =
        make_float4(tf32_rest(pn.x), tf32_rest(pn.y), tf32_rest(pn.z), tf32_rest(pn.w));
  }
}

// TF32 residual of parameters that arrived from peers.
__global__ void __launch_bounds__(256) k_peer_lo(const float *__restrict__ p, float *__restrict__ lo,
                                                 size_t n4) {
  const size_t stride = (size_t)gridDim.x * blockDim.x;
  for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < n4; i += stride) {
    const float4 v = __ldcg(reinterpret_cast<const float4 *>(p) + i);
    reinterpret_cast<float4 *>(lo)[i] =
        make_float4(tf32_rest(v.x), tf32_rest(v.y), tf32_rest(v.z), tf32_rest(v.w));
  }
}

__global__ void k_peer_wait(const unsigned int *flags, int n_chunks, int nranks, int rank,
                            unsigned int val, unsigned int *err, unsigned long long wait_ns) {
  if (threadIdx.x != 0) return;
  for (int c = 0; c < n_chunks; c++)
    if (!wait_flags(flags + (size_t)c * kMaxPeers, nranks, rank, val, err, 2, wait_ns)) return;
}

// The exchange's kernels run beside the persistent GEMM, whose CTAs need
// ~198 KB of shared memory: an SM can host blocks of both only if they
// share its shared-memory carve-out, so these kernels ask for the largest
// one (they use almost no shared memory themselves).
template <typename K>
int prefer_max_shared(K kern, int slot) {
  static bool done[4][64] = {};
  int dev = 0;
  FG_CUDA_TRY(cudaGetDevice(&dev));
  if (dev >= 0 && dev < 64 && !done[slot][dev]) {
    FG_CUDA_TRY(cudaFuncSetAttribute(kern, cudaFuncAttributePreferredSharedMemoryCarveout,
                                     (int)cudaSharedmemCarveoutMaxShared));
    done[slot][dev] = true;
  }
  return FG_OK;
}

}  // namespace

bool peer_parts_ok(int out, int in, int nranks, int parts) {
  if (parts < 2 || parts > kMaxPeerParts || out % parts) return false;
  const size_t rows = (size_t)(out / parts);
  return rows % 32 == 0 && (rows * (size_t)in) % (64 * (size_t)nranks) == 0;
}

int peer_layout(int n_layers, const int *dims, int nranks, int parts, PeerLayout *out) {
  if (!dims || !out || n_layers < 1) return set_error(FG_ERR_INVALID, "peer_layout: bad arguments");
  if (nranks < 2 || nranks > kMaxPeers)
    return set_error(FG_ERR_INVALID, "peer exchange: %d ranks (2 to %d supported)", nranks, kMaxPeers);
  if (parts < 1 || parts > kMaxPeerParts)
    return set_error(FG_ERR_INVALID, "peer exchange: %d chunks for layer 0 (1 to %d)", parts,
                     kMaxPeerParts);
  PeerLayout L;
  L.nranks = nranks;
  L.parts = parts;
  const size_t unit = 64 * (size_t)nranks;  // every shard 256-byte aligned
  L.w_off.resize(n_layers);
  L.b_off.resize(n_layers);
  L.first_chunk.resize(n_layers);
  L.n_chunks.resize(n_layers);
  std::vector<std::vector<PeerChunk>> per(n_layers);
  size_t off = 0;
  for (int l = 0; l < n_layers; l++) {
    const size_t o = (size_t)dims[l + 1], in = (size_t)dims[l];
    if (!o || !in) return set_error(FG_ERR_INVALID, "peer_layout: zero width");
    L.w_off[l] = off;
    L.b_off[l] = off + pad_to(o * in, 64);
    size_t raw = pad_to(o * in, 64) + pad_to(o, 64);
    if (l == 0) {
      L.loss_off = off + raw;
      raw += 64;
    }
    const size_t end = off + pad_to(raw, unit);
    // every tensor-core layer's dW in row blocks, so each block's exchange
    // starts while the next block is computed
    const int p = (o > 16 && peer_parts_ok((int)o, (int)in, nranks, parts)) ? parts : 1;
    size_t c0 = off;
    for (int q = 0; q < p; q++) {
      PeerChunk c;
      c.off = c0;
      c.len = (q == p - 1) ? end - c0 : (o / p) * in;
      c.layer = l;
      c.part = q;
      per[l].push_back(c);
      c0 += c.len;
    }
    off = end;
  }
  L.grad = off;
  for (int l = n_layers - 1; l >= 0; l--) {  // backward order
    L.first_chunk[l] = (int)L.chunks.size();
    L.n_chunks[l] = (int)per[l].size();
    for (auto &c : per[l]) L.chunks.push_back(c);
  }
  L.flag_words = pad_to(2 * L.chunks.size() * kMaxPeers, 64);
  L.region = 6 * L.grad + L.flag_words;
  uint32_t h = 2166136261u;
  h = fnv(h, (uint64_t)nranks);
  h = fnv(h, (uint64_t)L.parts);
  h = fnv(h, (uint64_t)n_layers);
  for (int l = 0; l <= n_layers; l++) h = fnv(h, (uint64_t)dims[l]);
  for (auto &c : L.chunks) {
    h = fnv(h, c.off);
    h = fnv(h, c.len);
  }
  h = fnv(h, L.region);
  L.digest = h;
  *out = std::move(L);
  return FG_OK;
}

int launch_peer_signal(const PeerFlagPtrs &ptrs, unsigned int val, cudaStream_t st) {
  int rc = prefer_max_shared(k_peer_signal, 0);
  if (rc) return rc;
  k_peer_signal<<<1, 32, 0, st>>>(ptrs, val);
  FG_LAUNCH_TRY();
  return FG_OK;
}

int launch_peer_reduce_sgd(float *grad, const float *stage, const float *p_cur, float *p_next,
                           float *lo_next, size_t shard, int rank, int nranks, float lr,
                           long long loss_idx, const unsigned int *flags, unsigned int val,
                           unsigned int *err, int blocks, cudaStream_t st,
                           unsigned long long wait_ns) {
  if (shard % 4) return set_error(FG_ERR_INVALID, "peer reduce: shard of %zu floats", shard);
  int rc = launch_peer_wait(flags, 1, nranks, rank, val, err, st, wait_ns);
  if (rc || (rc = prefer_max_shared(k_peer_reduce_sgd, 1))) return rc;
  const size_t n4 = shard / 4;
  size_t need = (n4 + 255) / 256;
  int grid = blocks > 0 ? blocks : 64;
  if ((size_t)grid > need) grid = (int)(need ? need : 1);
  k_peer_reduce_sgd<<<grid, 256, 0, st>>>(grad, stage, p_cur, p_next, lo_next, shard, rank, nranks,
                                          lr, loss_idx, err);
  FG_LAUNCH_TRY();
  return FG_OK;
}

int launch_peer_lo(const float *p, float *lo, size_t n, int blocks, cudaStream_t st) {
  if (n % 4) return set_error(FG_ERR_INVALID, "peer residual: %zu floats", n);
  int rc = prefer_max_shared(k_peer_lo, 3);
  if (rc) return rc;
  const size_t need = (n / 4 + 255) / 256;
  int grid = blocks > 0 ? blocks : 64;
  if ((size_t)grid > need) grid = (int)(need ? need : 1);
  k_peer_lo<<<grid, 256, 0, st>>>(p, lo, n / 4);
  FG_LAUNCH_TRY();
  return FG_OK;
}

int launch_peer_wait(const unsigned int *flags, int n_chunks, int nranks, int rank,
                     unsigned int val, unsigned int *err, cudaStream_t st,
                     unsigned long long wait_ns) {
  int rc = prefer_max_shared(k_peer_wait, 2);
  if (rc) return rc;
  k_peer_wait<<<1, 32, 0, st>>>(flags, n_chunks, nranks, rank, val, err, wait_ns);
  FG_LAUNCH_TRY();
  return FG_OK;
}

}  // namespace fg

extern "C" int fg_peer_layout(int n_layers, const int *dims, int nranks, int chunks,
                              size_t *region_floats, size_t *chunk_off, size_t *chunk_len,
                              int capacity, int *n_chunks) {
  fg::PeerLayout L;
  int rc = fg::peer_layout(n_layers, dims, nranks, chunks, &L);
  if (rc) return rc;
  if (region_floats) *region_floats = L.region;
  const int n = (int)L.chunks.size();
  for (int i = 0; i < n && i < capacity; i++) {
    if (chunk_off) chunk_off[i] = L.chunks[i].off;
    if (chunk_len) chunk_len[i] = L.chunks[i].len;
  }
  if (n_chunks) *n_chunks = n;
  return FG_OK;
}

extern "C" int fg_peer_layout_offsets(int n_layers, const int *dims, int nranks, int chunks,
                                      size_t *w_off, size_t *b_off, size_t *loss_off) {
  fg::PeerLayout L;
  int rc = fg::peer_layout(n_layers, dims, nranks, chunks, &L);
  if (rc) return rc;
  for (int l = 0; l < n_layers; l++) {
    if (w_off) w_off[l] = L.w_off[l];
    if (b_off) b_off[l] = L.b_off[l];
  }
  if (loss_off) *loss_off = L.loss_off;
  return FG_OK;
}

extern "C" int fg_peer_reduce_sgd_local(float *d_grad, const float *d_stage, const float *d_p_cur,
                                        float *d_p_next, float *d_lo_next, size_t shard, int rank,
                                        int nranks, float lr, long long loss_idx,
                                        const unsigned int *d_flags, unsigned int val, int wait_ms,
                                        void *stream) {
  FG_REQUIRE(d_grad && d_stage && d_p_cur && d_p_next && d_lo_next && d_flags,
             "fg_peer_reduce_sgd_local: null pointer");
  FG_REQUIRE(nranks >= 2 && nranks <= fg::kMaxPeers && rank >= 0 && rank < nranks,
             "fg_peer_reduce_sgd_local: rank %d of %d", rank, nranks);
  FG_REQUIRE(wait_ms > 0 && wait_ms <= 60000, "fg_peer_reduce_sgd_local: wait of %d ms", wait_ms);
  FG_REQUIRE(loss_idx < (long long)(shard * (size_t)nranks),
             "fg_peer_reduce_sgd_local: loss index outside the chunk");
  fg::DevCtx *ctx = fg::ctx_current();
  if (!ctx) return fg::set_error(FG_ERR_CUDA, "fg_peer_reduce_sgd_local: no CUDA device context");
  cudaStream_t st = (cudaStream_t)stream;
  int rc = fg::launch_peer_reduce_sgd(d_grad, d_stage, d_p_cur, d_p_next, d_lo_next, shard, rank,
                                      nranks, lr, loss_idx, d_flags, val, ctx->d_err, 64, st,
                                      (unsigned long long)wait_ms * 1000000ull);
  if (rc) return rc;
  FG_CUDA_TRY(cudaStreamSynchronize(st));
  return fg_check_device_error();
}
