
#include <barrier>
#include <cmath>
#include <cstring>
#include <memory>
#include <thread>
#include <vector>
struct fg_dim3 { unsigned x, y, z; };
static thread_local fg_dim3 blockIdx, threadIdx;
#define __global__
#define __launch_bounds__(x)
#define __restrict__ __restrict
#define __shared__ static
struct float4 { float x, y, z, w; };
struct int4 { int x, y, z, w; };
struct uchar4 { unsigned char x, y, z, w; };
static inline float4 make_float4(float a, float b, float c, float d) { return {a, b, c, d}; }
static inline int4 make_int4(int a, int b, int c, int d) { return {a, b, c, d}; }
static inline uchar4 make_uchar4(unsigned char a, unsigned char b, unsigned char c,
                                 unsigned char d) { return {a, b, c, d}; }
// Cooperative kernels (warp shuffles, __syncthreads) run with one host
// thread per CUDA thread of a block: a barrier per warp and one per block.
static std::unique_ptr<std::barrier<>> fg_block_bar;
static std::vector<std::unique_ptr<std::barrier<>>> fg_warp_bar;
static double fg_xch[1024];
static inline void __syncthreads() { fg_block_bar->arrive_and_wait(); }
template <class T>
static inline T __shfl_xor_sync(unsigned, T v, int off) {
  const unsigned t = threadIdx.x;
  std::barrier<> &b = *fg_warp_bar[t >> 5];
  std::memcpy(&fg_xch[t], &v, sizeof(T));
  b.arrive_and_wait();
  T r;
  std::memcpy(&r, &fg_xch[t ^ (unsigned)off], sizeof(T));
  b.arrive_and_wait();
  return r;
}
static inline float __fadd_rn(float a, float b) { return a + b; }
static inline float __fmul_rn(float a, float b) { return a * b; }
static inline float __frcp_rn(float a) { return 1.0f / a; }
static inline float __fsqrt_rn(float a) { return std::sqrt(a); }
static inline float __int_as_float(int i) { float f; std::memcpy(&f, &i, 4); return f; }
static inline float __uint_as_float(unsigned i) { float f; std::memcpy(&f, &i, 4); return f; }
static inline unsigned __float_as_uint(float f) { unsigned i; std::memcpy(&i, &f, 4); return i; }
static inline float __fsub_rn(float a, float b) { return a - b; }
using std::exp2;
using std::log2;
// rendered by the ferrograd_b200 front end
#ifndef INFINITY
#define INFINITY __int_as_float(0x7f800000)
#endif
#ifndef NAN
#define NAN __int_as_float(0x7fffffff)
#endif
extern "C" __global__ void __launch_bounds__(1024) fg_kernel(float* __restrict__ p0, const float* __restrict__ p1, const float* __restrict__ p2) {
  __shared__ float fg_sm_f[1024];
  const int fg_lane = threadIdx.x & 31, fg_warp = threadIdx.x >> 5;
  const bool fg_in = (long long)blockIdx.x * 32LL + fg_lane < 128LL;
  const long long e0 = fg_in ? (long long)blockIdx.x * 32LL + fg_lane : 128LL - 1LL;
  float res0 = 0.0f;
  long long st0 = -1;
   {
    const long long i0 = e0;
    const long long i1 = i0;
    const float v2 = p0[i1];
    float acc3 = 0.0f;
    float acc4 = 0.0f;
    float acc5 = 0.0f;
    float acc6 = 0.0f;
    float acc7 = 0.0f;
    float acc8 = 0.0f;
    float acc9 = 0.0f;
    float acc10 = 0.0f;
    float acc11 = 0.0f;
    for (long long r12 = fg_warp; r12 < 256LL; r12 += 256LL) {
      const long long i13 = r12 * 128LL + i1;
      const long long i14 = i13;
      const float v15 = p1[i14];
      const float v16 = __fadd_rn(acc4, v15);
      acc4 = v16;
      const long long i17 = r12 + 32LL;
      if (i17 < 256LL) {
        const long long i18 = i17 * 128LL + i1;
        const long long i19 = i18;
        const float v20 = p1[i19];
        const float v21 = __fadd_rn(acc5, v20);
        acc5 = v21;
      }
      const long long i22 = r12 + 64LL;
      if (i22 < 256LL) {
        const long long i23 = i22 * 128LL + i1;
        const long long i24 = i23;
        const float v25 = p1[i24];
        const float v26 = __fadd_rn(acc6, v25);
        acc6 = v26;
      }
      const long long i27 = r12 + 96LL;
      if (i27 < 256LL) {
        const long long i28 = i27 * 128LL + i1;
        const long long i29 = i28;
        const float v30 = p1[i29];
        const float v31 = __fadd_rn(acc7, v30);
        acc7 = v31;
      }
      const long long i32 = r12 + 128LL;
      if (i32 < 256LL) {
        const long long i33 = i32 * 128LL + i1;
        const long long i34 = i33;
        const float v35 = p1[i34];
        const float v36 = __fadd_rn(acc8, v35);
        acc8 = v36;
      }
      const long long i37 = r12 + 160LL;
      if (i37 < 256LL) {
        const long long i38 = i37 * 128LL + i1;
        const long long i39 = i38;
        const float v40 = p1[i39];
        const float v41 = __fadd_rn(acc9, v40);
        acc9 = v41;
      }
      const long long i42 = r12 + 192LL;
      if (i42 < 256LL) {
        const long long i43 = i42 * 128LL + i1;
        const long long i44 = i43;
        const float v45 = p1[i44];
        const float v46 = __fadd_rn(acc10, v45);
        acc10 = v46;
      }
      const long long i47 = r12 + 224LL;
      if (i47 < 256LL) {
        const long long i48 = i47 * 128LL + i1;
        const long long i49 = i48;
        const float v50 = p1[i49];
        const float v51 = __fadd_rn(acc11, v50);
        acc11 = v51;
      }
    }
    const float v52 = __fadd_rn(acc4, acc8);
    acc4 = v52;
    const float v53 = __fadd_rn(acc5, acc9);
    acc5 = v53;
    const float v54 = __fadd_rn(acc6, acc10);
    acc6 = v54;
    const float v55 = __fadd_rn(acc7, acc11);
    acc7 = v55;
    const float v56 = __fadd_rn(acc4, acc6);
    acc4 = v56;
    const float v57 = __fadd_rn(acc5, acc7);
    acc5 = v57;
    const float v58 = __fadd_rn(acc4, acc5);
    acc4 = v58;
    acc3 = acc4;
    fg_sm_f[threadIdx.x] = acc3;
    __syncthreads();
    if (fg_warp == 0) {
      const float v59 = __fadd_rn(acc3, fg_sm_f[32 + fg_lane]);
      acc3 = v59;
      const float v60 = __fadd_rn(acc3, fg_sm_f[64 + fg_lane]);
      acc3 = v60;
      const float v61 = __fadd_rn(acc3, fg_sm_f[96 + fg_lane]);
      acc3 = v61;
      const float v62 = __fadd_rn(acc3, fg_sm_f[128 + fg_lane]);
      acc3 = v62;
      const float v63 = __fadd_rn(acc3, fg_sm_f[160 + fg_lane]);
      acc3 = v63;
      const float v64 = __fadd_rn(acc3, fg_sm_f[192 + fg_lane]);
      acc3 = v64;
      const float v65 = __fadd_rn(acc3, fg_sm_f[224 + fg_lane]);
      acc3 = v65;
      const float v66 = __fadd_rn(acc3, fg_sm_f[256 + fg_lane]);
      acc3 = v66;
      const float v67 = __fadd_rn(acc3, fg_sm_f[288 + fg_lane]);
      acc3 = v67;
      const float v68 = __fadd_rn(acc3, fg_sm_f[320 + fg_lane]);
      acc3 = v68;
      const float v69 = __fadd_rn(acc3, fg_sm_f[352 + fg_lane]);
      acc3 = v69;
      const float v70 = __fadd_rn(acc3, fg_sm_f[384 + fg_lane]);
      acc3 = v70;
      const float v71 = __fadd_rn(acc3, fg_sm_f[416 + fg_lane]);
      acc3 = v71;
      const float v72 = __fadd_rn(acc3, fg_sm_f[448 + fg_lane]);
      acc3 = v72;
      const float v73 = __fadd_rn(acc3, fg_sm_f[480 + fg_lane]);
      acc3 = v73;
      const float v74 = __fadd_rn(acc3, fg_sm_f[512 + fg_lane]);
      acc3 = v74;
      const float v75 = __fadd_rn(acc3, fg_sm_f[544 + fg_lane]);
      acc3 = v75;
      const float v76 = __fadd_rn(acc3, fg_sm_f[576 + fg_lane]);
      acc3 = v76;
      const float v77 = __fadd_rn(acc3, fg_sm_f[608 + fg_lane]);
      acc3 = v77;
      const float v78 = __fadd_rn(acc3, fg_sm_f[640 + fg_lane]);
      acc3 = v78;
      const float v79 = __fadd_rn(acc3, fg_sm_f[672 + fg_lane]);
      acc3 = v79;
      const float v80 = __fadd_rn(acc3, fg_sm_f[704 + fg_lane]);
      acc3 = v80;
      const float v81 = __fadd_rn(acc3, fg_sm_f[736 + fg_lane]);
      acc3 = v81;
      const float v82 = __fadd_rn(acc3, fg_sm_f[768 + fg_lane]);
      acc3 = v82;
      const float v83 = __fadd_rn(acc3, fg_sm_f[800 + fg_lane]);
      acc3 = v83;
      const float v84 = __fadd_rn(acc3, fg_sm_f[832 + fg_lane]);
      acc3 = v84;
      const float v85 = __fadd_rn(acc3, fg_sm_f[864 + fg_lane]);
      acc3 = v85;
      const float v86 = __fadd_rn(acc3, fg_sm_f[896 + fg_lane]);
      acc3 = v86;
      const float v87 = __fadd_rn(acc3, fg_sm_f[928 + fg_lane]);
      acc3 = v87;
      const float v88 = __fadd_rn(acc3, fg_sm_f[960 + fg_lane]);
      acc3 = v88;
      const float v89 = __fadd_rn(acc3, fg_sm_f[992 + fg_lane]);
      acc3 = v89;
      fg_sm_f[fg_lane] = acc3;
    }
    __syncthreads();
    acc3 = fg_sm_f[fg_lane];
    __syncthreads();
    const float v90 = p2[0];
    const float v91 = __fmul_rn(acc3, v90);
    const float v92 = (-v91);
    const float v93 = __fadd_rn(v2, v92);
    res0 = v93;
    st0 = i1;
  }
  if (fg_warp == 0 && fg_in && st0 >= 0) p0[st0] = res0;
}

extern "C" void fg_host_launch(void **a, unsigned grid, unsigned block) {
  fg_block_bar.reset(new std::barrier<>(block));
  fg_warp_bar.clear();
  for (unsigned w = 0; w < (block + 31) / 32; w++)
    fg_warp_bar.emplace_back(new std::barrier<>(block - 32 * w < 32 ? block - 32 * w : 32));
  std::vector<std::thread> team;
  for (unsigned t = 0; t < block; t++) team.emplace_back([=] {
    threadIdx.x = t;
    for (unsigned b = 0; b < grid; b++) {
      blockIdx.x = b;
      fg_kernel(*(float*  *)a[0], *( const float*  *)a[1], *( const float*  *)a[2]);
      fg_block_bar->arrive_and_wait();
    }
  });
  for (auto &th : team) th.join();
}
