// Host-side helpers shared by the entry points.
#pragma once

#include <cuda_runtime.h>

#include <algorithm>
#include <utility>

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

// Whether launches of the verify-forward kernels carry the programmatic
// stream-serialisation attribute (RETREE_B200_PDL=0 turns it off).
bool pdl_enabled();

// cudaLaunchKernelEx with programmatic dependent launch (when enabled) and an
// optional (1, cluster_y, 1) thread-block cluster.  Every kernel launched
// through here calls pdl_wait() before it reads or writes data that earlier
// kernels of the stream produce or consume.
template <typename... KArgs, typename... Args>
inline cudaError_t launch_ex(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t stream,
                             int cluster_y, Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attrs[2];
  unsigned n = 0;
  if (pdl_enabled()) {
    attrs[n].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attrs[n].val.programmaticStreamSerializationAllowed = 1;
    ++n;
  }
  if (cluster_y > 1) {
    attrs[n].id = cudaLaunchAttributeClusterDimension;
    attrs[n].val.clusterDim.x = 1;
    attrs[n].val.clusterDim.y = static_cast<unsigned>(cluster_y);
    attrs[n].val.clusterDim.z = 1;
    ++n;
  }
  cfg.attrs = attrs;
  cfg.numAttrs = n;
  return cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
}

// The same with a (cx, cy, cz) thread-block cluster (no cluster when all are 1).
template <typename... KArgs, typename... Args>
inline cudaError_t launch_ex_cluster(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem,
                                     cudaStream_t stream, dim3 cluster, Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attrs[2];
  unsigned n = 0;
  if (pdl_enabled()) {
    attrs[n].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attrs[n].val.programmaticStreamSerializationAllowed = 1;
    ++n;
  }
  if (cluster.x * cluster.y * cluster.z > 1) {
    attrs[n].id = cudaLaunchAttributeClusterDimension;
    attrs[n].val.clusterDim.x = cluster.x;
    attrs[n].val.clusterDim.y = cluster.y;
    attrs[n].val.clusterDim.z = cluster.z;
    ++n;
  }
  cfg.attrs = attrs;
  cfg.numAttrs = n;
  return cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
}

}  // namespace rt
