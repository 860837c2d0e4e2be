
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
extern "C" __global__ void __launch_bounds__(1024) fg_kernel(float* __restrict__ p0, const float* __restrict__ p1, const float* __restrict__ p2, const float* __restrict__ p3, const float* __restrict__ p4) {
  __shared__ float fg_sm_f[1024];
  const int fg_lane = threadIdx.x & 31, fg_warp = threadIdx.x >> 5;
  const bool fg_in = (long long)blockIdx.x * 32LL + fg_lane < 1280LL;
  const long long e0 = fg_in ? (long long)blockIdx.x * 32LL + fg_lane : 1280LL - 1LL;
  float res0 = 0.0f;
  long long st0 = -1;
   {
    const long long i0 = e0;
    const long long i1 = (i0 / 128LL);
    const long long i2 = (i0 % 128LL);
    const long long i3 = i1 * 128LL + i2;
    const long long i4 = i3;
    const float v5 = p0[i4];
    float acc6 = 0.0f;
    float acc7 = 0.0f;
    float acc8 = 0.0f;
    float acc9 = 0.0f;
    float acc10 = 0.0f;
    float acc11 = 0.0f;
    float acc12 = 0.0f;
    float acc13 = 0.0f;
    float acc14 = 0.0f;
    for (long long r15 = fg_warp; r15 < 256LL; r15 += 256LL) {
      const long long i16 = r15 * 128LL + i2;
      const long long i17 = i16;
      const float v18 = p2[i17];
      const bool v19 = (0.0f < v18);
      const float v20 = (v19 ? v18 : 0.0f);
      const long long i21 = r15 * 10LL + i1;
      const long long i22 = i21;
      const float v23 = p3[i22];
      const float v24 = __fmul_rn(v20, v23);
      const float v25 = __fadd_rn(acc7, v24);
      acc7 = v25;
      const long long i26 = r15 + 32LL;
      if (i26 < 256LL) {
        const long long i27 = i26 * 128LL + i2;
        const long long i28 = i27;
        const float v29 = p2[i28];
        const bool v30 = (0.0f < v29);
        const float v31 = (v30 ? v29 : 0.0f);
        const long long i32 = i26 * 10LL + i1;
        const long long i33 = i32;
        const float v34 = p3[i33];
        const float v35 = __fmul_rn(v31, v34);
        const float v36 = __fadd_rn(acc8, v35);
        acc8 = v36;
      }
      const long long i37 = r15 + 64LL;
      if (i37 < 256LL) {
        const long long i38 = i37 * 128LL + i2;
        const long long i39 = i38;
        const float v40 = p2[i39];
        const bool v41 = (0.0f < v40);
        const float v42 = (v41 ? v40 : 0.0f);
        const long long i43 = i37 * 10LL + i1;
        const long long i44 = i43;
        const float v45 = p3[i44];
        const float v46 = __fmul_rn(v42, v45);
        const float v47 = __fadd_rn(acc9, v46);
        acc9 = v47;
      }
      const long long i48 = r15 + 96LL;
      if (i48 < 256LL) {
        const long long i49 = i48 * 128LL + i2;
        const long long i50 = i49;
        const float v51 = p2[i50];
        const bool v52 = (0.0f < v51);
        const float v53 = (v52 ? v51 : 0.0f);
        const long long i54 = i48 * 10LL + i1;
        const long long i55 = i54;
        const float v56 = p3[i55];
        const float v57 = __fmul_rn(v53, v56);
        const float v58 = __fadd_rn(acc10, v57);
        acc10 = v58;
      }
      const long long i59 = r15 + 128LL;
      if (i59 < 256LL) {
        const long long i60 = i59 * 128LL + i2;
        const long long i61 = i60;
        const float v62 = p2[i61];
        const bool v63 = (0.0f < v62);
        const float v64 = (v63 ? v62 : 0.0f);
        const long long i65 = i59 * 10LL + i1;
        const long long i66 = i65;
        const float v67 = p3[i66];
        const float v68 = __fmul_rn(v64, v67);
        const float v69 = __fadd_rn(acc11, v68);
        acc11 = v69;
      }
      const long long i70 = r15 + 160LL;
      if (i70 < 256LL) {
        const long long i71 = i70 * 128LL + i2;
        const long long i72 = i71;
        const float v73 = p2[i72];
        const bool v74 = (0.0f < v73);
        const float v75 = (v74 ? v73 : 0.0f);
        const long long i76 = i70 * 10LL + i1;
        const long long i77 = i76;
        const float v78 = p3[i77];
        const float v79 = __fmul_rn(v75, v78);
        const float v80 = __fadd_rn(acc12, v79);
        acc12 = v80;
      }
      const long long i81 = r15 + 192LL;
      if (i81 < 256LL) {
        const long long i82 = i81 * 128LL + i2;
        const long long i83 = i82;
        const float v84 = p2[i83];
        const bool v85 = (0.0f < v84);
        const float v86 = (v85 ? v84 : 0.0f);
        const long long i87 = i81 * 10LL + i1;
        const long long i88 = i87;
        const float v89 = p3[i88];
        const float v90 = __fmul_rn(v86, v89);
        const float v91 = __fadd_rn(acc13, v90);
        acc13 = v91;
      }
      const long long i92 = r15 + 224LL;
      if (i92 < 256LL) {
        const long long i93 = i92 * 128LL + i2;
        const long long i94 = i93;
        const float v95 = p2[i94];
        const bool v96 = (0.0f < v95);
        const float v97 = (v96 ? v95 : 0.0f);
        const long long i98 = i92 * 10LL + i1;
        const long long i99 = i98;
        const float v100 = p3[i99];
        const float v101 = __fmul_rn(v97, v100);
        const float v102 = __fadd_rn(acc14, v101);
        acc14 = v102;
      }
    }
    const float v103 = __fadd_rn(acc7, acc11);
    acc7 = v103;
    const float v104 = __fadd_rn(acc8, acc12);
    acc8 = v104;
    const float v105 = __fadd_rn(acc9, acc13);
    acc9 = v105;
    const float v106 = __fadd_rn(acc10, acc14);
    acc10 = v106;
    const float v107 = __fadd_rn(acc7, acc9);
    acc7 = v107;
    const float v108 = __fadd_rn(acc8, acc10);
    acc8 = v108;
    const float v109 = __fadd_rn(acc7, acc8);
    acc7 = v109;
    acc6 = acc7;
    fg_sm_f[threadIdx.x] = acc6;
    __syncthreads();
    if (fg_warp == 0) {
      const float v110 = __fadd_rn(acc6, fg_sm_f[32 + fg_lane]);
      acc6 = v110;
      const float v111 = __fadd_rn(acc6, fg_sm_f[64 + fg_lane]);
      acc6 = v111;
      const float v112 = __fadd_rn(acc6, fg_sm_f[96 + fg_lane]);
      acc6 = v112;
      const float v113 = __fadd_rn(acc6, fg_sm_f[128 + fg_lane]);
      acc6 = v113;
      const float v114 = __fadd_rn(acc6, fg_sm_f[160 + fg_lane]);
      acc6 = v114;
      const float v115 = __fadd_rn(acc6, fg_sm_f[192 + fg_lane]);
      acc6 = v115;
      const float v116 = __fadd_rn(acc6, fg_sm_f[224 + fg_lane]);
      acc6 = v116;
      const float v117 = __fadd_rn(acc6, fg_sm_f[256 + fg_lane]);
      acc6 = v117;
      const float v118 = __fadd_rn(acc6, fg_sm_f[288 + fg_lane]);
      acc6 = v118;
      const float v119 = __fadd_rn(acc6, fg_sm_f[320 + fg_lane]);
      acc6 = v119;
      const float v120 = __fadd_rn(acc6, fg_sm_f[352 + fg_lane]);
      acc6 = v120;
      const float v121 = __fadd_rn(acc6, fg_sm_f[384 + fg_lane]);
      acc6 = v121;
      const float v122 = __fadd_rn(acc6, fg_sm_f[416 + fg_lane]);
      acc6 = v122;
      const float v123 = __fadd_rn(acc6, fg_sm_f[448 + fg_lane]);
      acc6 = v123;
      const float v124 = __fadd_rn(acc6, fg_sm_f[480 + fg_lane]);
      acc6 = v124;
      const float v125 = __fadd_rn(acc6, fg_sm_f[512 + fg_lane]);
      acc6 = v125;
      const float v126 = __fadd_rn(acc6, fg_sm_f[544 + fg_lane]);
      acc6 = v126;
      const float v127 = __fadd_rn(acc6, fg_sm_f[576 + fg_lane]);
      acc6 = v127;
      const float v128 = __fadd_rn(acc6, fg_sm_f[608 + fg_lane]);
      acc6 = v128;
      const float v129 = __fadd_rn(acc6, fg_sm_f[640 + fg_lane]);
      acc6 = v129;
      const float v130 = __fadd_rn(acc6, fg_sm_f[672 + fg_lane]);
      acc6 = v130;
      const float v131 = __fadd_rn(acc6, fg_sm_f[704 + fg_lane]);
      acc6 = v131;
      const float v132 = __fadd_rn(acc6, fg_sm_f[736 + fg_lane]);
      acc6 = v132;
      const float v133 = __fadd_rn(acc6, fg_sm_f[768 + fg_lane]);
      acc6 = v133;
      const float v134 = __fadd_rn(acc6, fg_sm_f[800 + fg_lane]);
      acc6 = v134;
      const float v135 = __fadd_rn(acc6, fg_sm_f[832 + fg_lane]);
      acc6 = v135;
      const float v136 = __fadd_rn(acc6, fg_sm_f[864 + fg_lane]);
      acc6 = v136;
      const float v137 = __fadd_rn(acc6, fg_sm_f[896 + fg_lane]);
      acc6 = v137;
      const float v138 = __fadd_rn(acc6, fg_sm_f[928 + fg_lane]);
      acc6 = v138;
      const float v139 = __fadd_rn(acc6, fg_sm_f[960 + fg_lane]);
      acc6 = v139;
      const float v140 = __fadd_rn(acc6, fg_sm_f[992 + fg_lane]);
      acc6 = v140;
      fg_sm_f[fg_lane] = acc6;
    }
    __syncthreads();
    acc6 = fg_sm_f[fg_lane];
    __syncthreads();
    const float v141 = p4[0];
    const float v142 = __fmul_rn(acc6, v141);
    const float v143 = (-v142);
    const float v144 = __fadd_rn(v5, v143);
    res0 = v144;
    st0 = i4;
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
      fg_kernel(*(float*  *)a[0], *( const float*  *)a[1], *( const float*  *)a[2], *( const float*  *)a[3], *( const float*  *)a[4]);
      fg_block_bar->arrive_and_wait();
    }
  });
  for (auto &th : team) th.join();
}
