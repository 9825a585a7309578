// Exact tree walk + commit bookkeeping, and the dense-mask -> bitmask bridge.
#include "common.cuh"
#include "host_util.h"

namespace rt {

// One warp: at each step the 32 lanes scan the node list for a child of the
// current node carrying the target's token.
__global__ void tree_walk_kernel(const int32_t* __restrict__ parents, const int64_t* __restrict__ tokens,
                                 int count, const int32_t* count_dev, const int64_t* __restrict__ posterior,
                                 int64_t* __restrict__ accepted, int32_t* accepted_len, int64_t* next_token,
                                 const int64_t* __restrict__ verify_ids, int64_t* output_ids, int64_t output_len,
                                 int64_t* start_dev, int* status) {
  const int lane = threadIdx.x;
  const int cnt = count_dev != nullptr ? *count_dev : count;
  int cur = 0, len = 1;
  int64_t nxt = posterior[0];
  if (lane == 0) accepted[0] = 0;
  for (int step = 0; step <= cnt; ++step) {
    int found = -1;
    for (int base = 1; base <= cnt; base += 32) {
      const int i = base + lane;
      const bool hit = i <= cnt && parents[i] == cur && tokens[i - 1] == nxt;
      const unsigned b = __ballot_sync(0xFFFFFFFFu, hit);
      if (b) found = base + 31 - __clz(b);  // keep the highest-numbered match
    }
    if (found < 0) break;
    cur = found;
    if (lane == 0) accepted[len] = cur;
    ++len;
    nxt = posterior[cur];
  }
  if (lane == 0) {
    *accepted_len = len;
    *next_token = nxt;
  }
  if (output_ids != nullptr) {
    const int64_t start = *start_dev;
    if (start < 0 || start + len >= output_len) {
      if (lane == 0) set_status(status, RT_DEV_OVERFLOW);
      return;
    }
    __syncwarp();
    for (int i = lane; i < len; i += 32) output_ids[start + i] = verify_ids[accepted[i]];
    if (lane == 0) {
      output_ids[start + len] = nxt;
      start_dev[1] = start;
      start_dev[0] = start + len;
    }
  }
}

template <typename T>
__device__ __forceinline__ bool is_zero(T v);
template <>
__device__ __forceinline__ bool is_zero<float>(float v) { return v == 0.0f; }
template <>
__device__ __forceinline__ bool is_zero<__nv_bfloat16>(__nv_bfloat16 v) { return __bfloat162float(v) == 0.0f; }
template <>
__device__ __forceinline__ bool is_zero<__half>(__half v) { return __half2float(v) == 0.0f; }

template <typename T>
__global__ void mask_from_dense_kernel(const T* dense, int64_t ld, int64_t col0, int n, uint32_t* mask,
                                       int mask_words) {
  const int row = blockIdx.x;
  for (int w = threadIdx.x; w < mask_words; w += blockDim.x) {
    uint32_t bits = 0;
    for (int b = 0; b < 32; ++b) {
      const int j = w * 32 + b;
      if (j < n && is_zero<T>(dense[row * ld + col0 + j])) bits |= 1u << b;
    }
    mask[static_cast<int64_t>(row) * mask_words + w] = bits;
  }
}

}  // namespace rt

using namespace rt;

extern "C" int rt_tree_walk(const int32_t* parents, const int64_t* node_tokens, int count, const int32_t* count_dev,
                            const int64_t* posterior, int64_t* accepted, int32_t* accepted_len,
                            int64_t* next_token, const int64_t* verify_ids, int64_t* output_ids,
                            int64_t output_len, int64_t* start_dev, int* status, rt_stream_t stream) {
  if (count < 0 || !parents || !posterior || !accepted || !accepted_len || !next_token)
    return RT_ERR_INVALID_ARGUMENT;
  if (count > 0 && node_tokens == nullptr && count_dev == nullptr) return RT_ERR_INVALID_ARGUMENT;
  if (output_ids != nullptr && (verify_ids == nullptr || start_dev == nullptr)) return RT_ERR_INVALID_ARGUMENT;
  tree_walk_kernel<<<1, 32, 0, reinterpret_cast<cudaStream_t>(stream)>>>(
      parents, node_tokens, count, count_dev, posterior, accepted, accepted_len, next_token, verify_ids, output_ids,
      output_len, start_dev, status);
  return check_launch();
}

extern "C" int rt_mask_from_dense(const void* dense, int dtype, int64_t ld, int64_t col0, int n, uint32_t* mask,
                                  int mask_words, rt_stream_t stream) {
  if (n < 0 || !dense || !mask || mask_words < (n + 31) / 32 || col0 < 0 || ld < col0 + n)
    return RT_ERR_INVALID_ARGUMENT;
  if (n == 0) return RT_OK;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  const int threads = 32;
  switch (dtype) {
    case 0:
      mask_from_dense_kernel<float><<<n, threads, 0, s>>>(static_cast<const float*>(dense), ld, col0, n, mask,
                                                          mask_words);
      break;
    case 1:
      mask_from_dense_kernel<__nv_bfloat16><<<n, threads, 0, s>>>(static_cast<const __nv_bfloat16*>(dense), ld,
                                                                  col0, n, mask, mask_words);
      break;
    case 2:
      mask_from_dense_kernel<__half><<<n, threads, 0, s>>>(static_cast<const __half*>(dense), ld, col0, n, mask,
                                                           mask_words);
      break;
    default:
      return RT_ERR_INVALID_ARGUMENT;
  }
  return check_launch();
}
