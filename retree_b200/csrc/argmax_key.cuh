// Order-preserving argmax key of a logit, shared by the lm_head projection's
// argmax epilogue (linear.cu) and its host-built test.
//
// Larger value -> larger key; -0.0 and +0.0 share a key; every NaN maps above
// +inf (torch.argmax returns the first NaN's index); the low 32 bits hold
// 0xFFFFFFFF - row, so on equal values the smaller row has the larger key.
// The argmax of a row is then the row encoded in the maximum key.
#pragma once

#include <stdint.h>

#ifdef __CUDACC__
#define RT_AK_HD __host__ __device__ __forceinline__
#else
#define RT_AK_HD inline
#endif

namespace rt {

RT_AK_HD unsigned long long argmax_key(float x, uint32_t row) {
  union {
    float f;
    uint32_t u;
  } v;
  v.f = x;
  uint32_t b = v.u;
  uint32_t k;
  if (x != x) {
    k = 0xFFFFFFFFu;
  } else {
    if (b == 0x80000000u) b = 0u;
    k = (b & 0x80000000u) ? ~b : (b | 0x80000000u);
  }
  return (static_cast<unsigned long long>(k) << 32) | (0xFFFFFFFFu - row);
}

RT_AK_HD int64_t argmax_row(unsigned long long key) {
  return key == 0ull ? -1 : static_cast<int64_t>(0xFFFFFFFFu - static_cast<uint32_t>(key));
}

}  // namespace rt
