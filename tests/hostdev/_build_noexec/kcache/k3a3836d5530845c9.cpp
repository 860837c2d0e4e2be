
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
extern "C" __global__ void __launch_bounds__(256) fg_kernel(float* __restrict__ p0, const float* __restrict__ p1, const float* __restrict__ p2, const float* __restrict__ p3, const float* __restrict__ p4) {
  const int fg_lane = threadIdx.x & 31;
  const long long e0 = (long long)blockIdx.x * 8LL + (threadIdx.x >> 5);
  float res0 = 0.0f;
  long long st0 = -1;
  if (e0 < 2560LL) {
    const long long i0 = e0;
    const long long i1 = (i0 / 10LL);
    const long long i2 = (i0 % 10LL);
    float acc3 = 0.0f;
    float acc4 = 0.0f;
    float acc5 = 0.0f;
    float acc6 = 0.0f;
    float acc7 = 0.0f;
    float acc8 = 0.0f;
    float acc9 = 0.0f;
    float acc10 = 0.0f;
    float acc11 = 0.0f;
    for (long long r12 = fg_lane * 4LL; r12 < 128LL; r12 += 512LL) {
      const long long i13 = r12 + 1LL;
      const long long i14 = r12 + 2LL;
      const long long i15 = r12 + 3LL;
      const long long i16 = i2 * 128LL + r12;
      const long long i17 = i16;
      const float4 q18 = *reinterpret_cast<const float4 *>(p3 + i17);
      const long long i19 = i1 * 128LL + r12;
      const long long i20 = i19;
      const float v21 = p2[i20];
      const bool v22 = (0.0f < v21);
      const float v23 = (v22 ? v21 : 0.0f);
      const float v24 = __fmul_rn(v23, q18.x);
      const float v25 = __fadd_rn(acc4, v24);
      acc4 = v25;
      const long long i26 = i1 * 128LL + i13;
      const long long i27 = i26;
      const float v28 = p2[i27];
      const bool v29 = (0.0f < v28);
      const float v30 = (v29 ? v28 : 0.0f);
      const float v31 = __fmul_rn(v30, q18.y);
      const float v32 = __fadd_rn(acc4, v31);
      acc4 = v32;
      const long long i33 = i1 * 128LL + i14;
      const long long i34 = i33;
      const float v35 = p2[i34];
      const bool v36 = (0.0f < v35);
      const float v37 = (v36 ? v35 : 0.0f);
      const float v38 = __fmul_rn(v37, q18.z);
      const float v39 = __fadd_rn(acc4, v38);
      acc4 = v39;
      const long long i40 = i1 * 128LL + i15;
      const long long i41 = i40;
      const float v42 = p2[i41];
      const bool v43 = (0.0f < v42);
      const float v44 = (v43 ? v42 : 0.0f);
      const float v45 = __fmul_rn(v44, q18.w);
      const float v46 = __fadd_rn(acc4, v45);
      acc4 = v46;
      const long long i47 = r12 + 128LL;
      if (i47 < 128LL) {
        const long long i48 = i47 + 1LL;
        const long long i49 = i47 + 2LL;
        const long long i50 = i47 + 3LL;
        const long long i51 = i2 * 128LL + i47;
        const long long i52 = i51;
        const float4 q53 = *reinterpret_cast<const float4 *>(p3 + i52);
        const long long i54 = i1 * 128LL + i47;
        const long long i55 = i54;
        const float v56 = p2[i55];
        const bool v57 = (0.0f < v56);
        const float v58 = (v57 ? v56 : 0.0f);
        const float v59 = __fmul_rn(v58, q53.x);
        const float v60 = __fadd_rn(acc5, v59);
        acc5 = v60;
        const long long i61 = i1 * 128LL + i48;
        const long long i62 = i61;
        const float v63 = p2[i62];
        const bool v64 = (0.0f < v63);
        const float v65 = (v64 ? v63 : 0.0f);
        const float v66 = __fmul_rn(v65, q53.y);
        const float v67 = __fadd_rn(acc5, v66);
        acc5 = v67;
        const long long i68 = i1 * 128LL + i49;
        const long long i69 = i68;
        const float v70 = p2[i69];
        const bool v71 = (0.0f < v70);
        const float v72 = (v71 ? v70 : 0.0f);
        const float v73 = __fmul_rn(v72, q53.z);
        const float v74 = __fadd_rn(acc5, v73);
        acc5 = v74;
        const long long i75 = i1 * 128LL + i50;
        const long long i76 = i75;
        const float v77 = p2[i76];
        const bool v78 = (0.0f < v77);
        const float v79 = (v78 ? v77 : 0.0f);
        const float v80 = __fmul_rn(v79, q53.w);
        const float v81 = __fadd_rn(acc5, v80);
        acc5 = v81;
      }
      const long long i82 = r12 + 256LL;
      if (i82 < 128LL) {
        const long long i83 = i82 + 1LL;
        const long long i84 = i82 + 2LL;
        const long long i85 = i82 + 3LL;
        const long long i86 = i2 * 128LL + i82;
        const long long i87 = i86;
        const float4 q88 = *reinterpret_cast<const float4 *>(p3 + i87);
        const long long i89 = i1 * 128LL + i82;
        const long long i90 = i89;
        const float v91 = p2[i90];
        const bool v92 = (0.0f < v91);
        const float v93 = (v92 ? v91 : 0.0f);
        const float v94 = __fmul_rn(v93, q88.x);
        const float v95 = __fadd_rn(acc6, v94);
        acc6 = v95;
        const long long i96 = i1 * 128LL + i83;
        const long long i97 = i96;
        const float v98 = p2[i97];
        const bool v99 = (0.0f < v98);
        const float v100 = (v99 ? v98 : 0.0f);
        const float v101 = __fmul_rn(v100, q88.y);
        const float v102 = __fadd_rn(acc6, v101);
        acc6 = v102;
        const long long i103 = i1 * 128LL + i84;
        const long long i104 = i103;
        const float v105 = p2[i104];
        const bool v106 = (0.0f < v105);
        const float v107 = (v106 ? v105 : 0.0f);
        const float v108 = __fmul_rn(v107, q88.z);
        const float v109 = __fadd_rn(acc6, v108);
        acc6 = v109;
        const long long i110 = i1 * 128LL + i85;
        const long long i111 = i110;
        const float v112 = p2[i111];
        const bool v113 = (0.0f < v112);
        const float v114 = (v113 ? v112 : 0.0f);
        const float v115 = __fmul_rn(v114, q88.w);
        const float v116 = __fadd_rn(acc6, v115);
        acc6 = v116;
      }
      const long long i117 = r12 + 384LL;
      if (i117 < 128LL) {
        const long long i118 = i117 + 1LL;
        const long long i119 = i117 + 2LL;
        const long long i120 = i117 + 3LL;
        const long long i121 = i2 * 128LL + i117;
        const long long i122 = i121;
        const float4 q123 = *reinterpret_cast<const float4 *>(p3 + i122);
        const long long i124 = i1 * 128LL + i117;
        const long long i125 = i124;
        const float v126 = p2[i125];
        const bool v127 = (0.0f < v126);
        const float v128 = (v127 ? v126 : 0.0f);
        const float v129 = __fmul_rn(v128, q123.x);
        const float v130 = __fadd_rn(acc7, v129);
        acc7 = v130;
        const long long i131 = i1 * 128LL + i118;
        const long long i132 = i131;
        const float v133 = p2[i132];
        const bool v134 = (0.0f < v133);
        const float v135 = (v134 ? v133 : 0.0f);
        const float v136 = __fmul_rn(v135, q123.y);
        const float v137 = __fadd_rn(acc7, v136);
        acc7 = v137;
        const long long i138 = i1 * 128LL + i119;
        const long long i139 = i138;
        const float v140 = p2[i139];
        const bool v141 = (0.0f < v140);
        const float v142 = (v141 ? v140 : 0.0f);
        const float v143 = __fmul_rn(v142, q123.z);
        const float v144 = __fadd_rn(acc7, v143);
        acc7 = v144;
        const long long i145 = i1 * 128LL + i120;
        const long long i146 = i145;
        const float v147 = p2[i146];
        const bool v148 = (0.0f < v147);
        const float v149 = (v148 ? v147 : 0.0f);
        const float v150 = __fmul_rn(v149, q123.w);
        const float v151 = __fadd_rn(acc7, v150);
        acc7 = v151;
      }
    }
    const float v152 = __fadd_rn(acc4, acc6);
    acc4 = v152;
    const float v153 = __fadd_rn(acc5, acc7);
    acc5 = v153;
    const float v154 = __fadd_rn(acc4, acc5);
    acc4 = v154;
    acc3 = acc4;
     {
      const float t155 = __shfl_xor_sync(0xffffffffu, acc3, 16);
      const float v156 = __fadd_rn(acc3, t155);
      acc3 = v156;
    }
     {
      const float t157 = __shfl_xor_sync(0xffffffffu, acc3, 8);
      const float v158 = __fadd_rn(acc3, t157);
      acc3 = v158;
    }
     {
      const float t159 = __shfl_xor_sync(0xffffffffu, acc3, 4);
      const float v160 = __fadd_rn(acc3, t159);
      acc3 = v160;
    }
     {
      const float t161 = __shfl_xor_sync(0xffffffffu, acc3, 2);
      const float v162 = __fadd_rn(acc3, t161);
      acc3 = v162;
    }
     {
      const float t163 = __shfl_xor_sync(0xffffffffu, acc3, 1);
      const float v164 = __fadd_rn(acc3, t163);
      acc3 = v164;
    }
    const float v165 = p4[i2];
    const float v166 = __fadd_rn(acc3, v165);
    res0 = v166;
    st0 = i0;
  }
  if (fg_lane == 0 && st0 >= 0) p0[st0] = res0;
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
