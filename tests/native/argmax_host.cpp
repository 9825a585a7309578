// Host build of the argmax key (retree_b200/csrc/argmax_key.cuh) for the CPU tests.
#include "../../retree_b200/csrc/argmax_key.cuh"

extern "C" int64_t host_argmax(const float* x, int n) {
  unsigned long long best = 0ull;
  for (int i = 0; i < n; ++i) {
    const unsigned long long k = rt::argmax_key(x[i], static_cast<uint32_t>(i));
    if (k > best) best = k;
  }
  return rt::argmax_row(best);
}
