// fg_init.cpp -- host-side parameter initialisation (src/nn.rs:12-47).
// Kept free of CUDA so every build of the C ABI shares one definition.
#include <cmath>
#include <cstdint>
#include <cstdio>

#include "../../include/ferro_cuda.h"

namespace fg {
int set_error(int code, const char *fmt, ...);  // defined by each build of the C ABI
}

extern "C" {

int fg_kaiming_normal(float *h_out, size_t numel, size_t fan_in, uint64_t *state) {
  if (!state || (numel != 0 && !h_out))
    return fg::set_error(FG_ERR_INVALID, "fg_kaiming_normal: null argument");
  if (fan_in == 0) return fg::set_error(FG_ERR_INVALID, "fg_kaiming_normal: fan_in must be positive");
  const float stdv = sqrtf(2.0f / (float)fan_in);
  auto next_unit = [state]() {
    const uint64_t next = *state * 6364136223846793005ULL + 1ULL;
    *state = next;
    return (float)(next >> 33) / (float)(1ULL << 31);
  };
  size_t n = 0;
  while (n < numel) {
    float u1 = next_unit();
    if (!(u1 >= 1.17549435e-38f)) u1 = 1.17549435e-38f;  // max(u1, f32::MIN_POSITIVE)
    const float u2 = next_unit();
    const float radius = sqrtf(-2.0f * logf(u1)) * stdv;
    const float theta = (2.0f * 3.14159265358979323846f) * u2;
    h_out[n++] = radius * cosf(theta);
    if (n < numel) h_out[n++] = radius * sinf(theta);
  }
  return FG_OK;
}

}  // extern "C"
