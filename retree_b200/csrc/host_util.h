// Host-side helpers shared by the entry points.
#pragma once

#include <cuda_runtime.h>

#include <algorithm>

#include "../../include/retree_b200.h"
#include <cstdint>

namespace rt {

// Last CUDA error seen on this host thread (returned by rt_last_cuda_error).
extern thread_local int g_last_cuda_error;

inline int check_launch() {
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) {
    g_last_cuda_error = static_cast<int>(e);
    return RT_ERR_CUDA;
  }
  return RT_OK;
}

inline int record_cuda(cudaError_t e) {
  if (e != cudaSuccess) {
    g_last_cuda_error = static_cast<int>(e);
    return RT_ERR_CUDA;
  }
  return RT_OK;
}

// Raise a kernel's dynamic shared-memory limit when a launch needs more than
// the 48 KiB default (idempotent; cheap after the first call).
template <typename Kernel>
inline void set_smem_limit(Kernel k, size_t bytes) {
  if (bytes > 48 * 1024) cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(bytes));
}

inline size_t align_up(size_t x, size_t a) { return (x + a - 1) / a * a; }

}  // namespace rt
