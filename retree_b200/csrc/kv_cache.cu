// KV-cache maintenance kernels: in-place append and commit-time compaction.
//
// Both are pure data movement (HBM-bound, and at tree sizes launch-bound):
// rows are moved in the widest vector unit the alignment allows (16 B for
// bf16 rows of 128 elements), one CTA per (slab, head) for compaction so the
// gather-then-scatter happens through shared memory with no scratch in HBM.
#include "common.cuh"
#include "host_util.h"

namespace rt {

template <typename Unit>
__global__ void __launch_bounds__(256) kv_compact_kernel(void* const* slabs, char* base, int64_t slab_stride,
                                                         int n_heads, int64_t head_stride, int64_t row_stride,
                                                         int row_bytes, int64_t past_len_host,
                                                         const int64_t* past_len_dev, int64_t cur_len,
                                                         const int64_t* __restrict__ keep, int n_keep,
                                                         const int32_t* n_keep_dev, int* status) {
  extern __shared__ __align__(16) unsigned char stage[];
  __shared__ int bad;
  const int slab = blockIdx.x / n_heads;
  const int head = blockIdx.x % n_heads;
  int nk = n_keep;
  if (n_keep_dev != nullptr) nk = min(max(*n_keep_dev, 0), n_keep);
  const int64_t past_len = past_len_dev != nullptr ? *past_len_dev : past_len_host;
  // Same no-op rule as the reference: nothing kept, or everything kept.
  if (nk == 0 || nk == cur_len) return;
  if (threadIdx.x == 0) bad = 0;
  __syncthreads();
  for (int i = threadIdx.x; i < nk; i += blockDim.x) {
    const int64_t k = keep[i];
    if (k < 0 || k >= cur_len) bad = 1;
  }
  __syncthreads();
  if (bad || past_len < 0) {
    if (threadIdx.x == 0) set_status(status, RT_DEV_BAD_INDEX);
    return;
  }
  char* col = (slabs != nullptr ? static_cast<char*>(slabs[slab]) : base + slab * slab_stride) + head * head_stride;
  const int units = row_bytes / static_cast<int>(sizeof(Unit));
  const int total = nk * units;
  Unit* st = reinterpret_cast<Unit*>(stage);
  for (int u = threadIdx.x; u < total; u += blockDim.x) {
    const int i = u / units, c = u - i * units;
    const Unit* src = reinterpret_cast<const Unit*>(col + (past_len + keep[i]) * row_stride) + c;
    st[u] = *src;
  }
  __syncthreads();
  for (int u = threadIdx.x; u < total; u += blockDim.x) {
    const int i = u / units, c = u - i * units;
    Unit* dst = reinterpret_cast<Unit*>(col + (past_len + i) * row_stride) + c;
    *dst = st[u];
  }
}

template <typename Unit>
__global__ void __launch_bounds__(256) kv_append_kernel(char* k_cache, char* v_cache, int64_t c_head_stride,
                                                        int64_t c_row_stride, const char* k_new,
                                                        const char* v_new, int64_t n_head_stride,
                                                        int64_t n_row_stride, int n_heads, int n_new,
                                                        int row_bytes, int64_t capacity, int64_t offset,
                                                        const int64_t* offset_dev, int* status) {
  const int64_t off = offset_dev != nullptr ? *offset_dev : offset;
  char* dst_base = blockIdx.y == 0 ? k_cache : v_cache;
  const char* src_base = blockIdx.y == 0 ? k_new : v_new;
  const int units = row_bytes / static_cast<int>(sizeof(Unit));
  const int64_t total = static_cast<int64_t>(n_heads) * n_new * units;
  for (int64_t u = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; u < total;
       u += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int c = static_cast<int>(u % units);
    const int64_t hr = u / units;
    const int r = static_cast<int>(hr % n_new);
    const int h = static_cast<int>(hr / n_new);
    const int64_t row = off + r;
    if (row < 0 || row >= capacity) {
      if (c == 0) set_status(status, RT_DEV_OVERFLOW);
      continue;
    }
    const Unit* src = reinterpret_cast<const Unit*>(src_base + h * n_head_stride + r * n_row_stride) + c;
    Unit* dst = reinterpret_cast<Unit*>(dst_base + h * c_head_stride + row * c_row_stride) + c;
    *dst = *src;
  }
}

}  // namespace rt

using namespace rt;

extern "C" int rt_kv_compact(void* const* slabs, void* base, int n_slabs, int64_t slab_stride, int n_heads,
                             int64_t head_stride, int64_t row_stride, int row_bytes, int64_t past_len,
                             const int64_t* past_len_dev, int64_t cur_len, const int64_t* keep, int n_keep,
                             const int32_t* n_keep_dev, int* status, rt_stream_t stream) {
  if (n_slabs < 0 || n_heads < 0 || row_bytes <= 0 || past_len < 0 || cur_len < 0 || n_keep < 0)
    return RT_ERR_INVALID_ARGUMENT;
  if (n_keep > cur_len) return RT_ERR_INVALID_ARGUMENT;  // ddtree.py:55
  if (n_slabs == 0 || n_heads == 0 || n_keep == 0 || cur_len == 0) return RT_OK;
  if (n_keep_dev == nullptr && n_keep == cur_len) return RT_OK;  // ddtree.py:57-59
  if (keep == nullptr || (slabs == nullptr && base == nullptr)) return RT_ERR_INVALID_ARGUMENT;
  const size_t smem = static_cast<size_t>(n_keep) * row_bytes;
  if (smem > 200 * 1024) return RT_ERR_UNSUPPORTED;
  const uint64_t align_bits = reinterpret_cast<uint64_t>(base) | static_cast<uint64_t>(slab_stride) |
                              static_cast<uint64_t>(head_stride) | static_cast<uint64_t>(row_stride) |
                              static_cast<uint64_t>(row_bytes);
  const dim3 grid(n_slabs * n_heads);
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  // Slab pointers from a device array are assumed 16-byte aligned only if the
  // strides and row size are (checked above); torch allocations always are.
  if ((align_bits & 15) == 0) {
    set_smem_limit(kv_compact_kernel<uint4>, smem);
    kv_compact_kernel<uint4><<<grid, 256, smem, s>>>(slabs, static_cast<char*>(base), slab_stride, n_heads,
                                                     head_stride, row_stride, row_bytes, past_len, past_len_dev, cur_len, keep,
                                                     n_keep, n_keep_dev, status);
  } else if ((align_bits & 3) == 0) {
    set_smem_limit(kv_compact_kernel<uint32_t>, smem);
    kv_compact_kernel<uint32_t><<<grid, 256, smem, s>>>(slabs, static_cast<char*>(base), slab_stride, n_heads,
                                                        head_stride, row_stride, row_bytes, past_len, past_len_dev, cur_len,
                                                        keep, n_keep, n_keep_dev, status);
  } else if ((align_bits & 1) == 0) {
    set_smem_limit(kv_compact_kernel<uint16_t>, smem);
    kv_compact_kernel<uint16_t><<<grid, 256, smem, s>>>(slabs, static_cast<char*>(base), slab_stride, n_heads,
                                                        head_stride, row_stride, row_bytes, past_len, past_len_dev, cur_len,
                                                        keep, n_keep, n_keep_dev, status);
  } else {
    return RT_ERR_UNSUPPORTED;
  }
  return check_launch();
}

extern "C" int rt_kv_append(void* k_cache, void* v_cache, int64_t cache_head_stride, int64_t cache_row_stride,
                            const void* k_new, const void* v_new, int64_t new_head_stride, int64_t new_row_stride,
                            int n_heads, int n_new, int row_bytes, int64_t capacity, int64_t offset,
                            const int64_t* offset_dev, int* status, rt_stream_t stream) {
  if (n_heads < 0 || n_new < 0 || row_bytes <= 0 || capacity < 0) return RT_ERR_INVALID_ARGUMENT;
  if (n_heads == 0 || n_new == 0) return RT_OK;
  if (!k_cache || !v_cache || !k_new || !v_new) return RT_ERR_INVALID_ARGUMENT;
  if (offset_dev == nullptr && (offset < 0 || offset + n_new > capacity)) return RT_ERR_INVALID_ARGUMENT;
  const uint64_t align_bits =
      reinterpret_cast<uint64_t>(k_cache) | reinterpret_cast<uint64_t>(v_cache) |
      reinterpret_cast<uint64_t>(k_new) | reinterpret_cast<uint64_t>(v_new) |
      static_cast<uint64_t>(cache_head_stride) | static_cast<uint64_t>(cache_row_stride) |
      static_cast<uint64_t>(new_head_stride) | static_cast<uint64_t>(new_row_stride) |
      static_cast<uint64_t>(row_bytes);
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  const int64_t units16 = static_cast<int64_t>(n_heads) * n_new * (row_bytes / 2);
  const int blocks = static_cast<int>(std::min<int64_t>((units16 + 255) / 256, 1184));
  const dim3 grid(std::max(blocks, 1), 2);
#define RT_APPEND(U)                                                                                        \
  kv_append_kernel<U><<<grid, 256, 0, s>>>(static_cast<char*>(k_cache), static_cast<char*>(v_cache),      \
                                           cache_head_stride, cache_row_stride,                            \
                                           static_cast<const char*>(k_new), static_cast<const char*>(v_new), \
                                           new_head_stride, new_row_stride, n_heads, n_new, row_bytes,      \
                                           capacity, offset, offset_dev, status)
  if ((align_bits & 15) == 0) {
    RT_APPEND(uint4);
  } else if ((align_bits & 3) == 0) {
    RT_APPEND(uint32_t);
  } else if ((align_bits & 1) == 0) {
    RT_APPEND(uint16_t);
  } else {
    return RT_ERR_UNSUPPORTED;
  }
#undef RT_APPEND
  return check_launch();
}
