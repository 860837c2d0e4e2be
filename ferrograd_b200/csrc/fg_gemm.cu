// 3xTF32 GEMM on the sm_100a tensor cores (tcgen05 + TMEM), operands staged
// by TMA.  This is the kernel the schedule routes the reduce-of-broadcast-mul
// pattern to: Tensor::matmul (src/tensor.rs:762-778) and its two backward
// contractions (src/gradient.rs:100-106,165-176).
//
//   C[m,n] = sum_k A(m,k) B(n,k)  ~=  A*B + A*B_lo + A_lo*B
//
// The tensor cores read an fp32 operand as TF32 by dropping its low 13
// mantissa bits, so the raw matrix serves as the high part; *_lo holds the
// exact residual x - trunc_tf32(x).  The residual-times-residual term is
// dropped (relative size 2^-22).  Accumulation is fp32 in TMEM.
//
// Persistent CTA (one per SM, 6 warps) looping over 128 x BN output tiles:
//   warp 0     TMA producer (one elected lane), STAGES-deep smem ring
//   warp 1     TMEM allocator + MMA issuer (one elected lane); two TMEM
//              accumulators so tile i+1 accumulates while tile i drains
//   warps 2-5  epilogue: tcgen05.ld TMEM -> registers -> fused op -> global
// Operands are K-major ([rows, K], K contiguous) or MN-major ([K, rows]);
// both are loaded with 128-byte swizzle and described to tcgen05 directly,
// so no transposed copies are made.  Every TMA load fills only this CTA's own
// shared memory from this GPU's memory.
#include <cuda.h>
#include <cudaTypedefs.h>
#include <cuda_runtime.h>

#include <mutex>
#include <utility>
#include <vector>

#include "fg_gemm.cuh"
#include "fg_internal.h"
#include "fg_ptx.cuh"

namespace fg {
namespace gemm {

using namespace fg::ptx;

constexpr int BM = 128;
constexpr int UMMA_K = 8;   // K of one kind::tf32 MMA
constexpr int kThreads = 192;

// BK: fp32 elements per k-block.  32 is one 128-byte swizzle row per K-major
// operand row; 16 (64-byte swizzle) and 8 (32-byte swizzle) shrink a stage,
// so the same shared memory holds 2x / 4x the stages and more operand bytes
// are in flight while the tensor cores consume one stage (FG_GEMM_BK
// selects).
template <int BN, int BK>
struct Cfg {
  static constexpr int A_BYTES = BM * BK * 4;
  static constexpr int B_BYTES = BN * BK * 4;
  static constexpr int STAGE_BYTES = 2 * (A_BYTES + B_BYTES);
  static constexpr int STAGES = (BN <= 128 ? 3 : 2) * (32 / BK);
  static constexpr int TMEM_COLS = 2 * BN;  // two accumulators
  static constexpr int BAR_BYTES = 256;
  static constexpr int SMEM_BYTES = STAGES * STAGE_BYTES + BAR_BYTES + 1024;
  static_assert(SMEM_BYTES <= 227 * 1024, "shared memory budget");
};

__device__ __forceinline__ float tf32_residual(float v) {
  return __fsub_rn(v, __uint_as_float(__float_as_uint(v) & 0xffffe000u));
}

// Error codes written to the device error word (high 16 bits = role).
constexpr unsigned kErrProducer = 1u << 16;
constexpr unsigned kErrMma = 2u << 16;
constexpr unsigned kErrEpilogue = 3u << 16;

// Tile index -> (m block, n block).  Tiles are walked in groups of kGroupM
// row blocks, row block fastest, so the ~148 tiles in flight at any time
// share a few B panels and a few A panels (L2 reuse of both operands).
constexpr int kGroupM = 16;
__device__ __forceinline__ void tile_coords(int tile, int num_m, int num_n, int &mb, int &nb) {
  const int per_group = kGroupM * num_n;
  const int group = tile / per_group;
  const int first_m = group * kGroupM;
  const int gm = min(kGroupM, num_m - first_m);
  const int r = tile - group * per_group;
  mb = first_m + r % gm;
  nb = r / gm;
}

__device__ __forceinline__ void mbar_arrive(uint64_t *bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

// A CTA's work: its whole tiles (data-parallel waves), then its contiguous
// share of the stream-K units (k-blocks of the tail tiles in (tile, k)
// order), walked from its end to its start.  All three warp roles walk the
// same sequence of segments.
//
// Walking backwards makes every dependency short: the segment a CTA takes
// first is the head of a tile whose last k-block lies in a later CTA's
// range, and it leaves a partial; the segment it takes last is the tail of
// the tile its range starts in, and it finishes that tile, adding the
// partials that earlier CTAs produced at the start of their own walks.
struct Seg {
  int tile, k0, k1;
};

__device__ __forceinline__ long long sk_begin(const GemmParams &p, int c) {
  return p.sk_units * (long long)c / (long long)gridDim.x;
}

struct SegIter {
  int next_dp, dp_tiles, nk;
  long long lo, hi;  // SK units still to walk: [lo, hi), taken from hi down
  __device__ SegIter(const GemmParams &p, int nk_)
      : next_dp(blockIdx.x), dp_tiles(p.dp_tiles), nk(nk_), lo(sk_begin(p, blockIdx.x)),
        hi(sk_begin(p, blockIdx.x + 1)) {}
  __device__ bool next(Seg &s) {
    if (next_dp < dp_tiles) {
      s.tile = next_dp;
      s.k0 = 0;
      s.k1 = nk;
      next_dp += gridDim.x;
      return true;
    }
    if (hi <= lo) return false;
    const long long t = (hi - 1) / nk;
    const long long t0 = t * nk;
    const long long b = lo > t0 ? lo : t0;
    s.tile = dp_tiles + (int)t;
    s.k0 = (int)(b - t0);
    s.k1 = (int)(hi - t0);
    hi = b;
    return true;
  }
};

__device__ __forceinline__ void epi_bar() { asm volatile("bar.sync 1, 128;" ::: "memory"); }

// Bounded wait (~1 s of SM clocks) for a stream-K partial's flag.
__device__ __forceinline__ bool wait_flag(const unsigned int *flag, unsigned int *err) {
  const long long t0 = clock64();
  for (;;) {
    unsigned int v;
    asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(flag) : "memory");
    if (v) return true;
    if (clock64() - t0 > 2000000000LL) {
      if (err) atomicOr(err, kErrEpilogue | 3u);
      return false;
    }
    __nanosleep(64);
  }
}

// Persistent: one CTA per SM loops over output tiles.  The accumulator lives
// in one of two TMEM buffers (2 x BN columns): while the epilogue warps drain
// tile i from one buffer, the MMA warp already accumulates tile i+1 in the
// other.
template <int BN, bool A_MN, bool B_MN, int BK>
__global__ void __launch_bounds__(kThreads, 1)
    k_gemm3x(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmAlo,
             const __grid_constant__ CUtensorMap tmB, const __grid_constant__ CUtensorMap tmBlo,
             const GemmParams p) {
  using C = Cfg<BN, BK>;
  extern __shared__ uint8_t smem_raw[];
  // 128-byte swizzle atoms need 1024-byte aligned tiles.
  const uint32_t raw_addr = smem_u32(smem_raw);
  uint8_t *smem = smem_raw + ((1024u - (raw_addr & 1023u)) & 1023u);
  uint64_t *full = reinterpret_cast<uint64_t *>(smem + C::STAGES * C::STAGE_BYTES);
  uint64_t *empty = full + C::STAGES;
  uint64_t *tmem_full = empty + C::STAGES;  // [2]: accumulator ready for the epilogue
  uint64_t *tmem_empty = tmem_full + 2;     // [2]: epilogue drained the accumulator
  uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(tmem_empty + 2);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int num_m = (p.M + BM - 1) / BM;
  const int num_n = (p.N + BN - 1) / BN;
  const int nk = (p.K + BK - 1) / BK;
  const bool three = !p.one_pass;
  // k-blocks per accumulation chain (segmented accumulation, GemmParams)
  const int seglen = (p.seg_kb > 0 && p.seg_ws) ? p.seg_kb : nk;

  if (warp == 0 && lane == 0) {
    for (int s = 0; s < C::STAGES; s++) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int a = 0; a < 2; a++) {
      mbar_init(&tmem_full[a], 1);
      mbar_init(&tmem_empty[a], 128);  // every epilogue thread arrives
    }
    fence_mbar_init();
    prefetch_tmap(&tmA);
    prefetch_tmap(&tmB);
    if (three) {
      prefetch_tmap(&tmAlo);
      prefetch_tmap(&tmBlo);
    }
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, C::TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp == 0) {
    if (lane == 0) {
      // ---------------- TMA producer ----------------
      const uint32_t stage_tx = three ? (uint32_t)C::STAGE_BYTES
                                      : (uint32_t)(C::A_BYTES + C::B_BYTES);
      int it = 0;  // k-blocks issued so far, across segments
      bool ok = true;
      SegIter segs(p, nk);
      Seg sg;
      while (ok && segs.next(sg)) {
        int mb, nb;
        tile_coords(sg.tile, num_m, num_n, mb, nb);
        const int m0 = mb * BM, n0 = nb * BN;
        for (int kb = sg.k0; kb < sg.k1; kb++, it++) {
          const int s = it % C::STAGES;
          if (it >= C::STAGES) {
            ok = mbar_wait(&empty[s], ((it / C::STAGES) - 1) & 1, p.err, kErrProducer | 1);
            if (!ok) break;
          }
          uint8_t *sa = smem + s * C::STAGE_BYTES;
          uint8_t *salo = sa + C::A_BYTES;
          uint8_t *sb = salo + C::A_BYTES;
          uint8_t *sblo = sb + C::B_BYTES;
          const int k0 = kb * BK;
          mbar_arrive_expect_tx(&full[s], stage_tx);
          if (A_MN && p.a3d) {
            tma_load_3d(sa, &tmA, &full[s], 0, k0, m0 / 32);
            if (three) tma_load_3d(salo, &tmAlo, &full[s], 0, k0, m0 / 32);
          } else if (A_MN) {
#pragma unroll
            for (int j = 0; j < BM / 32; j++) {
              tma_load_2d(sa + j * (BK * 128), &tmA, &full[s], m0 + 32 * j, k0);
              if (three) tma_load_2d(salo + j * (BK * 128), &tmAlo, &full[s], m0 + 32 * j, k0);
            }
          } else {
            tma_load_2d(sa, &tmA, &full[s], k0, m0);
            if (three) tma_load_2d(salo, &tmAlo, &full[s], k0, m0);
          }
          if (B_MN && p.b3d) {
            tma_load_3d(sb, &tmB, &full[s], 0, k0, n0 / 32);
            if (three) tma_load_3d(sblo, &tmBlo, &full[s], 0, k0, n0 / 32);
          } else if (B_MN) {
#pragma unroll
            for (int j = 0; j < BN / 32; j++) {
              tma_load_2d(sb + j * (BK * 128), &tmB, &full[s], n0 + 32 * j, k0);
              if (three) tma_load_2d(sblo + j * (BK * 128), &tmBlo, &full[s], n0 + 32 * j, k0);
            }
          } else {
            tma_load_2d(sb, &tmB, &full[s], k0, n0);
            if (three) tma_load_2d(sblo, &tmBlo, &full[s], k0, n0);
          }
        }
      }
      if (!ok) {
        // Let loads already in flight land before the CTA exits.
        for (int i = it - C::STAGES < 0 ? 0 : it - C::STAGES; i < it; i++)
          mbar_wait(&full[i % C::STAGES], (i / C::STAGES) & 1, nullptr, 0);
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      // ---------------- MMA issuer ----------------
      constexpr uint32_t idesc = idesc_tf32(BM, BN, A_MN, B_MN);
      // K-major (BK*4-byte rows, 128B or 64B swizzle, 8-row atoms): the
      // next 8-element K slice is +32 bytes inside the swizzle row; SBO = 8
      // rows.  MN-major (128B swizzle with 32-byte atomicity, 4-row atoms):
      // a K row is 128 bytes (32 elements of M or N), the next 8 K rows are
      // +1024 bytes, SBO = 4 rows = 512 bytes, LBO = BK*128 bytes between the
      // 32-element MN chunks that TMA wrote as separate boxes.
      constexpr uint32_t kmaj_lay = BK == 32 ? kLayoutSw128 : BK == 16 ? kLayoutSw64 : kLayoutSw32;
      constexpr uint32_t a_kstep = A_MN ? 1024 : 32;
      constexpr uint32_t b_kstep = B_MN ? 1024 : 32;
      constexpr uint32_t a_lbo = A_MN ? BK * 128 : 16, a_sbo = A_MN ? 512 : 8 * BK * 4;
      constexpr uint32_t b_lbo = B_MN ? BK * 128 : 16, b_sbo = B_MN ? 512 : 8 * BK * 4;
      constexpr uint32_t a_lay = A_MN ? kLayoutSw128Base32 : kmaj_lay;
      constexpr uint32_t b_lay = B_MN ? kLayoutSw128Base32 : kmaj_lay;
      bool ok = true;
      int it = 0, local = 0;
      SegIter segs(p, nk);
      Seg sg;
      // one accumulation chain per sub-segment of at most seglen k-blocks
      for (; ok && segs.next(sg);)
        for (int s0 = sg.k0; ok && s0 < sg.k1; s0 += seglen, local++) {
        const int s1 = min(s0 + seglen, sg.k1);
        const int acc_buf = local & 1;
        if (local >= 2) {
          ok = mbar_wait(&tmem_empty[acc_buf], ((local >> 1) - 1) & 1, p.err, kErrMma | 2);
          if (!ok) break;
        }
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + (uint32_t)(acc_buf * BN);
        for (int kb = s0; kb < s1; kb++, it++) {
          const int s = it % C::STAGES;
          ok = mbar_wait(&full[s], (it / C::STAGES) & 1, p.err, kErrMma | 1);
          if (!ok) break;
          tc_fence_after();
          const uint32_t sa = smem_u32(smem + s * C::STAGE_BYTES);
          const uint32_t salo = sa + C::A_BYTES;
          const uint32_t sb = salo + C::A_BYTES;
          const uint32_t sblo = sb + C::B_BYTES;
#pragma unroll
          for (int kk = 0; kk < BK / UMMA_K; kk++) {
            const uint64_t da = smem_desc(sa + kk * a_kstep, a_lbo, a_sbo, a_lay);
            const uint64_t db = smem_desc(sb + kk * b_kstep, b_lbo, b_sbo, b_lay);
            const uint32_t acc = (kb > s0 || kk > 0) ? 1u : 0u;
            if (three) {
              const uint64_t dalo = smem_desc(salo + kk * a_kstep, a_lbo, a_sbo, a_lay);
              const uint64_t dblo = smem_desc(sblo + kk * b_kstep, b_lbo, b_sbo, b_lay);
              // small terms first, then the main product
              mma_tf32(d_tmem, dalo, db, idesc, acc);
              mma_tf32(d_tmem, da, dblo, idesc, 1u);
              mma_tf32(d_tmem, da, db, idesc, 1u);
            } else {
              mma_tf32(d_tmem, da, db, idesc, acc);
            }
          }
          mma_commit(&empty[s]);  // frees the stage once these MMAs have read it
        }
        if (ok) mma_commit(&tmem_full[acc_buf]);
      }
    }
  } else {
    // ---------------- epilogue (warps 2..5) ----------------
    const int q = warp & 3;  // TMEM lane quarter this warp may access
    const bool vec = ((p.ldc & 3) == 0) && ((((uintptr_t)p.C) & 15) == 0) &&
                     (!p.C_lo || (((uintptr_t)p.C_lo) & 15) == 0) &&
                     (!p.mask || (((p.ldmask & 3) == 0) && (((uintptr_t)p.mask) & 15) == 0));
    int local = 0;
    const int trow = 32 * q + lane;  // this thread's row within the tile
    // After a timed-out wait the warp stops touching TMEM and memory but
    // still takes every named barrier, so the other epilogue warps never
    // wait on a barrier this warp skipped.
    bool dead = false;
    SegIter segs(p, nk);
    Seg sg;
    // this CTA's running partial of segmented accumulation: [BN][BM]
    // floats, column-major so a warp's 32 rows of one column are one line
    float *run = p.seg_ws ? p.seg_ws + (size_t)blockIdx.x * (BM * BN) + trow : nullptr;
    while (segs.next(sg)) {
      int mb, nb;
      tile_coords(sg.tile, num_m, num_n, mb, nb);
      const int m0 = mb * BM, n0 = nb * BN;
      const int row = m0 + 32 * q + lane;
      const int nsub = (sg.k1 - sg.k0 + seglen - 1) / seglen;
      // Stream-K roles: a segment without the tile's last k-block leaves a
      // partial (it is the first segment its CTA walks); one with the last
      // k-block but not the first finishes the tile, adding the partials of
      // the CTAs below it that cover the tile's earlier k-blocks (the last
      // segment its CTA walks, so they are ready).
      const bool partial_out = sg.k1 < nk;
      const bool finisher = sg.k1 == nk && sg.k0 > 0;
      int c_lo = 0;  // contributors c_lo .. blockIdx.x-1, added from the top down
      for (int sub = 0; sub < nsub; sub++, local++) {
      const int acc_buf = local & 1;
      const bool last = sub == nsub - 1;
      if (last && finisher) {
        const long long tile_start = (long long)(sg.tile - p.dp_tiles) * nk;
        c_lo = blockIdx.x - 1;
        while (c_lo > 0 && sk_begin(p, c_lo) > tile_start) c_lo--;
        if (threadIdx.x == 64 && !dead)
          for (int c = (int)blockIdx.x - 1; c >= c_lo; c--)
            if (!wait_flag(p.sk_flags + c, p.err)) break;
        epi_bar();
        __threadfence();  // the partial loads below stay after the acquire
      }
      if (!dead && !mbar_wait(&tmem_full[acc_buf], (local >> 1) & 1, p.err, kErrEpilogue | 1))
        dead = true;
      tc_fence_after();
      float *my_ws = partial_out ? p.sk_ws + (size_t)blockIdx.x * (BM * BN) + (size_t)trow * BN
                                 : nullptr;
#pragma unroll 1
      for (int c0 = 0; c0 < BN && !dead; c0 += 32) {
        uint32_t r[32];
        __syncwarp();
        tmem_ld_32x32b_x32(tmem_base + ((uint32_t)(32 * q) << 16) + (uint32_t)(acc_buf * BN + c0),
                           r);
        tmem_ld_wait();
        float v[32];
#pragma unroll
        for (int j = 0; j < 32; j++) v[j] = __uint_as_float(r[j]);
        // Fold this chain's sum into the running partial (round to
        // nearest).  All 32 loads are issued before the first add: the
        // cache-hinted loads and stores keep their program order, so a
        // load-add-store per column would pay one L2 round trip per column.
        if (sub > 0) {
          float w[32];
#pragma unroll
          for (int j = 0; j < 32; j++) w[j] = __ldcg(run + (size_t)(c0 + j) * BM);
#pragma unroll
          for (int j = 0; j < 32; j++) v[j] = __fadd_rn(w[j], v[j]);
        }
        if (!last) {
#pragma unroll
          for (int j = 0; j < 32; j++) __stcg(run + (size_t)(c0 + j) * BM, v[j]);
          continue;
        }
        if (partial_out) {
#pragma unroll
          for (int j = 0; j < 32; j += 4)
            __stcg(reinterpret_cast<float4 *>(my_ws + c0 + j),
                   make_float4(v[j], v[j + 1], v[j + 2], v[j + 3]));
          continue;
        }
        if (row >= p.M || n0 + c0 >= p.N) continue;
        const int col0 = n0 + c0;
        if (finisher) {
          for (int c = (int)blockIdx.x - 1; c >= c_lo; c--) {
            const float *w = p.sk_ws + (size_t)c * (BM * BN) + (size_t)trow * BN + c0;
#pragma unroll
            for (int j = 0; j < 32; j += 4) {
              const float4 u = __ldcg(reinterpret_cast<const float4 *>(w + j));
              v[j] = __fadd_rn(v[j], u.x);
              v[j + 1] = __fadd_rn(v[j + 1], u.y);
              v[j + 2] = __fadd_rn(v[j + 2], u.z);
              v[j + 3] = __fadd_rn(v[j + 3], u.w);
            }
          }
        }
        if (p.epilogue == FG_EPI_BIAS || p.epilogue == FG_EPI_BIAS_RELU) {
#pragma unroll
          for (int j = 0; j < 32; j++) {
            const float b = (col0 + j < p.N) ? __ldg(p.bias + col0 + j) : 0.f;
            float z = __fadd_rn(v[j], b);
            if (p.epilogue == FG_EPI_BIAS_RELU) z = (0.0f < z) ? z : 0.0f;
            v[j] = z;
          }
        } else if (p.epilogue == FG_EPI_RELU_MASK) {
          const float *mrow = p.mask + (size_t)row * p.ldmask + col0;
#pragma unroll
          for (int j = 0; j < 32; j++) {
            const float mk = (col0 + j < p.N) ? __ldg(mrow + j) : 0.f;
            v[j] = (mk > 0.0f) ? v[j] : 0.0f;
          }
        }
        float *crow = p.C + (size_t)row * p.ldc + col0;
        float *lrow = p.C_lo ? p.C_lo + (size_t)row * p.ldc + col0 : nullptr;
        if (vec && col0 + 32 <= p.N) {
#pragma unroll
          for (int j = 0; j < 32; j += 4) {
            *reinterpret_cast<float4 *>(crow + j) = make_float4(v[j], v[j + 1], v[j + 2], v[j + 3]);
            if (lrow)
              *reinterpret_cast<float4 *>(lrow + j) =
                  make_float4(tf32_residual(v[j]), tf32_residual(v[j + 1]),
                              tf32_residual(v[j + 2]), tf32_residual(v[j + 3]));
          }
        } else {
#pragma unroll
          for (int j = 0; j < 32; j++) {
            if (col0 + j < p.N) {
              crow[j] = v[j];
              if (lrow) lrow[j] = tf32_residual(v[j]);
            }
          }
        }
      }
      // every TMEM load of this buffer has completed (tcgen05.wait::ld above)
      tc_fence_before();
      if (!dead) mbar_arrive(&tmem_empty[acc_buf]);
      }
      if (partial_out) {
        // publish: every thread's stores, then one release of the flag
        __threadfence();
        epi_bar();
        if (threadIdx.x == 64) {
          __threadfence();
          asm volatile("st.release.gpu.global.u32 [%0], %1;" ::"l"(p.sk_flags + blockIdx.x),
                       "r"(1u)
                       : "memory");
        }
      } else if (finisher) {
        epi_bar();  // all partials read
        if (threadIdx.x == 64)
          for (int c = (int)blockIdx.x - 1; c >= c_lo; c--) p.sk_flags[c] = 0u;
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, C::TMEM_COLS);
  }
}

// ---------------------------------------------------------------------------
// Host side
// ---------------------------------------------------------------------------
static PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    cudaDriverEntryPointQueryResult q;
    void *ptr = nullptr;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = (PFN_cuTensorMapEncodeTiled_v12000)ptr;
  });
  return fn;
}

// Tensor map over a row-major fp32 matrix of `outer` rows x `inner` columns
// with row pitch `ld` elements; box = 32 columns x box_rows rows.  K-major
// tiles use the 128-byte swizzle; MN-major tiles the 128-byte swizzle with
// 32-byte atoms (the layout tcgen05 reads MN-major tf32 operands in).
static int make_map(CUtensorMap *map, const float *ptr, int inner, int outer, int ld,
                    int box_rows, bool mn_major, int bk) {
  auto fn = encode_fn();
  if (!fn) return set_error(FG_ERR_CUDA, "cuTensorMapEncodeTiled unavailable");
  cuuint64_t dims[2] = {(cuuint64_t)inner, (cuuint64_t)outer};
  cuuint64_t strides[1] = {(cuuint64_t)ld * 4};
  // K-major: bk columns of K per row; MN-major: 32 columns of M or N
  cuuint32_t box[2] = {(cuuint32_t)(mn_major ? 32 : bk), (cuuint32_t)box_rows};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, (void *)ptr, dims, strides, box, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE,
                  mn_major  ? CU_TENSOR_MAP_SWIZZLE_128B_ATOM_32B
                  : bk == 32 ? CU_TENSOR_MAP_SWIZZLE_128B
                  : bk == 16 ? CU_TENSOR_MAP_SWIZZLE_64B
                             : CU_TENSOR_MAP_SWIZZLE_32B,
                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS)
    return set_error(FG_ERR_CUDA,
                     "cuTensorMapEncodeTiled failed (%d): inner=%d outer=%d ld=%d box_rows=%d",
                     (int)r, inner, outer, ld, box_rows);
  return FG_OK;
}

// MN-major operand [K, mn] (pitch ld) viewed as 3-D {32, K, mn/32} with the
// 32-element chunks 128 bytes apart, so one box {32, 32, rows/32} lands in
// shared memory as rows/32 chunks of 32 K-rows x 128 bytes -- the same layout
// the per-chunk 2-D loads produce.  Only valid when mn % 32 == 0 (the last
// chunk then ends exactly at the end of the row).
static int make_map_mn3d(CUtensorMap *map, const float *ptr, int mn, int K, int ld, int box_rows,
                         int bk) {
  auto fn = encode_fn();
  if (!fn) return set_error(FG_ERR_CUDA, "cuTensorMapEncodeTiled unavailable");
  cuuint64_t dims[3] = {32, (cuuint64_t)K, (cuuint64_t)(mn / 32)};
  cuuint64_t strides[2] = {(cuuint64_t)ld * 4, 128};
  cuuint32_t box[3] = {32, (cuuint32_t)bk, (cuuint32_t)(box_rows / 32)};
  cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 3, (void *)ptr, dims, strides, box, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B_ATOM_32B,
                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? FG_OK : FG_ERR_UNSUPPORTED;
}

// Splits a launch into whole-tile waves and a stream-K tail; returns the
// grid.  Whole waves keep the grouped tile order (operand panels shared in
// L2); only the last, partial wave's tiles are cut into k-ranges, so every
// CTA ends at the same k-block count instead of a fraction of the SMs
// running one more tile.  Used only when whole waves would waste >= 5% (a
// 1024-tile grid on 148 SMs wastes 1%: measured slower with the split).  A
// tail share under 1/4 tile per CTA borrows the previous whole wave; the
// grid shrinks so that every CTA gets >= max(nk/8, 24) k-blocks, and below
// one CTA per tail tile the split is not used.
static int plan_stream_k(GemmParams &p, int ntiles, int nk, int cap, float *ws,
                         unsigned int *flags, int min_kb) {
  p.dp_tiles = ntiles;
  p.sk_units = 0;
  p.sk_ws = ws;
  p.sk_flags = flags;
  int grid = ntiles < cap ? ntiles : cap;
  static const int mode = [] {
    const char *e = getenv("FG_GEMM_STREAM_K");
    return e && *e ? atoi(e) : 1;
  }();
  if (mode == 0 || !ws || !flags || nk < 8 || ntiles % cap == 0) return grid;
  // Only when whole-tile waves would leave enough of the last wave idle.
  static const double min_gain = [] {
    const char *e = getenv("FG_GEMM_STREAM_K_MIN_GAIN");
    return e && *e ? atof(e) : 0.05;
  }();
  const double waves = (double)ntiles / cap;
  const double whole = (double)((ntiles + cap - 1) / cap);
  if (whole / waves - 1.0 < min_gain) return grid;
  long long full = ntiles / cap;
  long long units = (long long)(ntiles - full * cap) * nk;
  if (full >= 1 && units < (long long)cap * (nk / 4)) {
    full -= 1;
    units += (long long)cap * nk;
  }
  // Each partial costs about one epilogue pass (~2-3 k-blocks of MMA time),
  // so a CTA's share must be long enough to amortise it.
  const long long min_share = nk / 8 > min_kb ? nk / 8 : min_kb;
  long long g = units / min_share;
  if (g > cap) g = cap;
  if (full > 0 && g < cap) return grid;  // waves need the whole grid
  if (g <= ntiles - full * cap) return grid;  // no better than whole tiles
  p.dp_tiles = (int)(full * cap);
  p.sk_units = units;
  return (int)g;
}

// Workspace layout: [ctas][BM * 256] stream-K partials, [ctas][BM * 256]
// segment running partials, then [ctas] stream-K flags.
size_t stream_k_ws_bytes(int ctas) {
  return 2 * (size_t)ctas * BM * 256 * sizeof(float) + (size_t)ctas * sizeof(unsigned int) + 256;
}

void stream_k_attach(GemmPlan *pl, void *ws, int ctas) {
  const size_t part = (size_t)ctas * BM * 256 * sizeof(float);
  pl->sk_ws = static_cast<float *>(ws);
  pl->seg_ws = ws ? reinterpret_cast<float *>(static_cast<char *>(ws) + part) : nullptr;
  pl->sk_flags =
      ws ? reinterpret_cast<unsigned int *>(static_cast<char *>(ws) + 2 * part) : nullptr;
}

// k-blocks per tensor-core accumulation chain (FG_GEMM_SEG_KB, default 32,
// i.e. 1024 products of each output; 0 = one chain per tile), applied to
// GEMMs whose K is at least FG_GEMM_SEG_MIN_K (default 0: every GEMM).
static int seg_kb_setting() {
  static const int v = [] {
    const char *e = getenv("FG_GEMM_SEG_KB");
    const int x = e && *e ? atoi(e) : 32;
    return x < 0 ? 0 : x;
  }();
  return v;
}
static int seg_min_k_setting() {
  static const int v = [] {
    const char *e = getenv("FG_GEMM_SEG_MIN_K");
    const int x = e && *e ? atoi(e) : 0;
    return x < 0 ? 0 : x;
  }();
  return v;
}

template <int BN, bool A_MN, bool B_MN, int BK>
static int launch_t(const GemmPlan &pl, cudaStream_t st) {
  using C = Cfg<BN, BK>;
  auto kern = k_gemm3x<BN, A_MN, B_MN, BK>;
  static bool attr_done[64] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev >= 0 && dev < 64 && !attr_done[dev]) {
    FG_CUDA_TRY(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                     C::SMEM_BYTES));
    attr_done[dev] = true;
  }
  const int ntiles = ((pl.p.N + BN - 1) / BN) * ((pl.p.M + BM - 1) / BM);
  const int nk = (pl.p.K + BK - 1) / BK;
  DevCtx *ctx = ctx_current();
  const int sms = (ctx && ctx->num_sms) ? ctx->num_sms : 148;
  int cap = sms;  // persistent: one CTA per SM
  if (pl.max_ctas > 0 && pl.max_ctas < cap) cap = pl.max_ctas;
  GemmParams p = pl.p;
  // stream-K shares and segment lengths are set in 32-deep k-block units
  const int grid = plan_stream_k(p, ntiles, nk, cap, pl.sk_ws, pl.sk_flags, 24 * 32 / BK);
  p.seg_ws = pl.seg_ws;
  p.seg_kb = p.K >= seg_min_k_setting() ? seg_kb_setting() * 32 / BK : 0;
  kern<<<grid, kThreads, C::SMEM_BYTES, st>>>(pl.a, pl.alo, pl.b, pl.blo, p);
  FG_LAUNCH_TRY();
  return FG_OK;
}

int make_plan(int M, int N, int K, const float *a, const float *a_lo, int lda, const float *b,
              const float *b_lo, int ldb, float *c, float *c_lo, int ldc, int flags, int epilogue,
              const float *bias, const float *mask, int ldmask, GemmPlan *pl) {
  FG_REQUIRE(M > 0 && N > 0 && K > 0, "gemm: M, N, K must be positive (got %d, %d, %d)", M, N, K);
  FG_REQUIRE(a && b && c, "gemm: null operand");
  const bool a_mn = flags & FG_GEMM_A_MN_MAJOR, b_mn = flags & FG_GEMM_B_MN_MAJOR;
  const bool one = flags & FG_GEMM_1XTF32;
  FG_REQUIRE(one || (a_lo && b_lo), "gemm: 3xTF32 needs the A and B residuals");
  FG_REQUIRE(lda % 4 == 0 && ldb % 4 == 0, "gemm: lda/ldb must be multiples of 4 elements");
  FG_REQUIRE(lda >= (a_mn ? M : K) && ldb >= (b_mn ? N : K) && ldc >= N, "gemm: pitch too small");
  auto al = [](const void *q) { return q == nullptr || (((uintptr_t)q) & 15) == 0; };
  FG_REQUIRE(al(a) && al(a_lo) && al(b) && al(b_lo), "gemm: operands must be 16-byte aligned");
  FG_REQUIRE(epilogue >= FG_EPI_NONE && epilogue <= FG_EPI_RELU_MASK, "gemm: bad epilogue %d",
             epilogue);
  FG_REQUIRE(epilogue != FG_EPI_BIAS && epilogue != FG_EPI_BIAS_RELU ? true : bias != nullptr,
             "gemm: epilogue needs a bias");
  FG_REQUIRE(epilogue != FG_EPI_RELU_MASK || (mask && ldmask >= N), "gemm: epilogue needs a mask");
  // 128 x 256 tiles need ~25% less shared-memory operand traffic per flop
  // than 128 x 128 (the tensor cores re-read A for every 8-deep K slice);
  // narrow outputs keep the 128-wide tile.
  const int bn = (N >= 256) ? 256 : 128;
  static const int bk = [] {
    const char *e = getenv("FG_GEMM_BK");
    const int v = e && *e ? atoi(e) : 16;
    return v == 8 || v == 32 ? v : 16;
  }();
  int rc;
  // A: [M,K] K-major (box 32 x BM rows) or [K,M] MN-major (box 32 x 32)
  if (a_mn) {
    if ((rc = make_map(&pl->a, a, M, K, lda, bk, true, bk))) return rc;
    if ((rc = make_map(&pl->alo, one ? a : a_lo, M, K, lda, bk, true, bk))) return rc;
  } else {
    if ((rc = make_map(&pl->a, a, K, M, lda, BM, false, bk))) return rc;
    if ((rc = make_map(&pl->alo, one ? a : a_lo, K, M, lda, BM, false, bk))) return rc;
  }
  if (b_mn) {
    if ((rc = make_map(&pl->b, b, N, K, ldb, bk, true, bk))) return rc;
    if ((rc = make_map(&pl->blo, one ? b : b_lo, N, K, ldb, bk, true, bk))) return rc;
  } else {
    if ((rc = make_map(&pl->b, b, K, N, ldb, bn, false, bk))) return rc;
    if ((rc = make_map(&pl->blo, one ? b : b_lo, K, N, ldb, bn, false, bk))) return rc;
  }
  pl->bk = bk;
  // single 3-D boxes for MN-major operands whose extent is a multiple of 32
  pl->p.a3d = 0;
  pl->p.b3d = 0;
  if (a_mn && M % 32 == 0) {
    CUtensorMap t0, t1;
    if (make_map_mn3d(&t0, a, M, K, lda, BM, bk) == FG_OK &&
        make_map_mn3d(&t1, one ? a : a_lo, M, K, lda, BM, bk) == FG_OK) {
      pl->a = t0;
      pl->alo = t1;
      pl->p.a3d = 1;
    }
  }
  if (b_mn && N % 32 == 0) {
    CUtensorMap t0, t1;
    if (make_map_mn3d(&t0, b, N, K, ldb, bn, bk) == FG_OK &&
        make_map_mn3d(&t1, one ? b : b_lo, N, K, ldb, bn, bk) == FG_OK) {
      pl->b = t0;
      pl->blo = t1;
      pl->p.b3d = 1;
    }
  }
  fg::clear_error();
  DevCtx *ctx = ctx_current();
  if (!ctx) return set_error(FG_ERR_CUDA, "no CUDA device context");
  GemmParams &p = pl->p;
  p.M = M;
  p.N = N;
  p.K = K;
  p.C = c;
  p.C_lo = c_lo;
  p.ldc = ldc;
  p.bias = bias;
  p.mask = mask;
  p.ldmask = ldmask;
  p.epilogue = epilogue;
  p.one_pass = one ? 1 : 0;
  p.err = ctx->d_err;
  pl->bn = bn;
  pl->a_mn = a_mn;
  pl->b_mn = b_mn;
  pl->max_ctas = 0;
  pl->sk_ws = nullptr;
  pl->sk_flags = nullptr;
  pl->seg_ws = nullptr;
  p.seg_ws = nullptr;
  p.seg_kb = 0;
  return FG_OK;
}

// One stream-K workspace per (device, stream) for the one-shot entry point:
// launches on one stream are ordered, so they can share it; launches on
// different streams get their own.  Allocated (zeroed) on first use outside
// stream capture; a capturing stream without one runs whole tiles only.
void attach_stream_ws(GemmPlan *pl, cudaStream_t st) {
  static std::mutex mu;
  static std::vector<std::pair<std::pair<int, cudaStream_t>, void *>> pool;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return;
  DevCtx *ctx = ctx_current();
  const int sms = (ctx && ctx->num_sms) ? ctx->num_sms : 148;
  std::lock_guard<std::mutex> lock(mu);
  for (auto &e : pool)
    if (e.first.first == dev && e.first.second == st) {
      stream_k_attach(pl, e.second, sms);
      return;
    }
  cudaStreamCaptureStatus cs = cudaStreamCaptureStatusNone;
  if (cudaStreamIsCapturing(st, &cs) != cudaSuccess || cs != cudaStreamCaptureStatusNone) {
    cudaGetLastError();
    return;
  }
  void *ws = nullptr;
  const size_t bytes = stream_k_ws_bytes(sms);
  // zero-filled on the GEMM's own stream, so the fill is ordered before the
  // first launch that reads the stream-K flags
  if (cudaMalloc(&ws, bytes) != cudaSuccess || cudaMemsetAsync(ws, 0, bytes, st) != cudaSuccess) {
    cudaGetLastError();
    if (ws) cudaFree(ws);
    return;
  }
  pool.push_back({{dev, st}, ws});
  stream_k_attach(pl, ws, sms);
}

template <int BK>
static int run_plan_bk(const GemmPlan &pl, cudaStream_t st) {
  if (pl.bn == 128) {
    if (!pl.a_mn && !pl.b_mn) return launch_t<128, false, false, BK>(pl, st);
    if (!pl.a_mn && pl.b_mn) return launch_t<128, false, true, BK>(pl, st);
    if (pl.a_mn && !pl.b_mn) return launch_t<128, true, false, BK>(pl, st);
    return launch_t<128, true, true, BK>(pl, st);
  }
  if (pl.bn == 256) {
    if (!pl.a_mn && !pl.b_mn) return launch_t<256, false, false, BK>(pl, st);
    if (!pl.a_mn && pl.b_mn) return launch_t<256, false, true, BK>(pl, st);
    if (pl.a_mn && !pl.b_mn) return launch_t<256, true, false, BK>(pl, st);
    return launch_t<256, true, true, BK>(pl, st);
  }
  return set_error(FG_ERR_UNSUPPORTED, "gemm: tile width %d not built", pl.bn);
}

int run_plan(const GemmPlan &pl, cudaStream_t st) {
  if (pl.bk == 8) return run_plan_bk<8>(pl, st);
  return pl.bk == 16 ? run_plan_bk<16>(pl, st) : run_plan_bk<32>(pl, st);
}

}  // namespace gemm
}  // namespace fg

extern "C" int fg_gemm_3xtf32(int M, int N, int K, const float *d_a, const float *d_a_lo, int lda,
                              const float *d_b, const float *d_b_lo, int ldb, float *d_c,
                              float *d_c_lo, int ldc, int flags, int epilogue, const float *d_bias,
                              const float *d_mask, int ldmask, void *stream) {
  fg::gemm::GemmPlan pl;
  int rc = fg::gemm::make_plan(M, N, K, d_a, d_a_lo, lda, d_b, d_b_lo, ldb, d_c, d_c_lo, ldc, flags,
                               epilogue, d_bias, d_mask, ldmask, &pl);
  if (rc) return rc;
  fg::gemm::attach_stream_ws(&pl, (cudaStream_t)stream);
  return fg::gemm::run_plan(pl, (cudaStream_t)stream);
}
