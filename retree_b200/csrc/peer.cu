// Attention-output exchange of a KV-head split over NVLink peer memory.
//
// Under the split (one request, G ranks, rank r owning kv heads
// [r*Hkv/G, (r+1)*Hkv/G)), o_proj needs every rank's attention output in head
// order -- the all-gather that headsplit.gather_heads does with NCCL.  Here the
// ranks map each other's exchange buffers (CUDA IPC, plain peer mappings, no
// multicast object) and:
//   rt_peer_signal   after rank r's attention has written its rows into its
//                    own buffer, one warp stores the layer's epoch into slot r
//                    of every rank's flag array (release, system scope);
//   rt_peer_gather   each CTA takes one source rank and a range of rows, waits
//                    (bounded) until its local flag slot for that rank reaches
//                    the epoch, and copies the rows over NVLink into the
//                    destination's column block of that rank.
// The epoch of a layer is read from a device counter (+ a constant per layer)
// so a captured CUDA graph replays with fresh epochs: rt_peer_epoch_step
// advances the counter once per forward.  Flags only grow, so a slot that
// already holds a later epoch also satisfies the wait.
#include <cstring>

#include "common.cuh"
#include "host_util.h"

namespace rt {
namespace {

constexpr int kMaxPeers = 8;
constexpr int kGatherThreads = 256;
constexpr uint32_t kPeerWaitLimit = 1u << 22;  // polls (system-scope load + ~100 ns sleep): 0.5 s or more

struct PeerPtrs {
  char* p[kMaxPeers];
};

__device__ __forceinline__ int64_t ld_acquire_sys(const int64_t* p) {
  int64_t v;
  asm volatile("ld.acquire.sys.global.s64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}

__device__ __forceinline__ void st_release_sys(int64_t* p, int64_t v) {
  asm volatile("st.release.sys.global.s64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}

__global__ void __launch_bounds__(32) peer_signal_kernel(PeerPtrs flags, int world, int rank,
                                                         const int64_t* epoch_dev, int64_t epoch_add) {
  const int p = threadIdx.x;
  if (p >= world) return;
  // the attention rows were written by earlier kernels of this stream; make
  // them visible to the peers before the flag that announces them
  __threadfence_system();
  st_release_sys(reinterpret_cast<int64_t*>(flags.p[p]) + rank, *epoch_dev + epoch_add);
}

__global__ void __launch_bounds__(kGatherThreads) peer_gather_kernel(PeerPtrs bufs, int world, int rows,
                                                                     int64_t row_bytes, int64_t src_ld,
                                                                     char* out, int64_t out_ld,
                                                                     const int64_t* flags_local,
                                                                     const int64_t* epoch_dev, int64_t epoch_add,
                                                                     int rows_per_cta, int* status) {
  __shared__ int ok;
  const int src = blockIdx.y;
  const int r0 = blockIdx.x * rows_per_cta;
  const int r1 = min(rows, r0 + rows_per_cta);
  const int64_t epoch = *epoch_dev + epoch_add;
  if (threadIdx.x == 0) {
    int good = 0;
    for (uint32_t i = 0; i < kPeerWaitLimit; ++i) {
      if (ld_acquire_sys(flags_local + src) >= epoch) {
        good = 1;
        break;
      }
      __nanosleep(100);
    }
    if (!good) set_status(status, RT_DEV_WAIT_TIMEOUT);
    ok = good;
  }
  __syncthreads();
  if (!ok) return;
  // every thread orders its own reads after the announcement
  (void)ld_acquire_sys(flags_local + src);
  const char* base = bufs.p[src];
  const int64_t vec = row_bytes / 16;
  const int64_t total = static_cast<int64_t>(r1 - r0) * vec;
  for (int64_t i = threadIdx.x; i < total; i += kGatherThreads) {
    const int64_t r = r0 + i / vec, c = i % vec;
    const uint4 v = __ldcv(reinterpret_cast<const uint4*>(base + r * src_ld) + c);
    reinterpret_cast<uint4*>(out + r * out_ld + src * row_bytes)[c] = v;
  }
}

__global__ void peer_epoch_step_kernel(int64_t* epoch_dev, int64_t add) { *epoch_dev += add; }

bool peers_ok(const void* const* ptrs, int world) {
  if (ptrs == nullptr || world < 1 || world > kMaxPeers) return false;
  for (int i = 0; i < world; ++i)
    if (ptrs[i] == nullptr || (reinterpret_cast<uintptr_t>(ptrs[i]) & 15)) return false;
  return true;
}

}  // namespace
}  // namespace rt

using namespace rt;

extern "C" int rt_ipc_alloc(size_t bytes, void** ptr, void* handle) {
  if (bytes == 0 || ptr == nullptr || handle == nullptr) return RT_ERR_INVALID_ARGUMENT;
  *ptr = nullptr;
  void* p = nullptr;
  int rc = record_cuda(cudaMalloc(&p, bytes));
  if (rc != RT_OK) return rc;
  rc = record_cuda(cudaMemset(p, 0, bytes));
  // zero before any peer can store into it
  if (rc == RT_OK) rc = record_cuda(cudaDeviceSynchronize());
  if (rc == RT_OK) rc = record_cuda(cudaIpcGetMemHandle(static_cast<cudaIpcMemHandle_t*>(handle), p));
  if (rc != RT_OK) {
    cudaFree(p);
    return rc;
  }
  *ptr = p;
  return RT_OK;
}

extern "C" int rt_ipc_free(void* ptr) { return ptr == nullptr ? RT_OK : record_cuda(cudaFree(ptr)); }

extern "C" int rt_ipc_open(const void* handle, void** ptr) {
  if (handle == nullptr || ptr == nullptr) return RT_ERR_INVALID_ARGUMENT;
  cudaIpcMemHandle_t h;
  memcpy(&h, handle, sizeof(h));
  return record_cuda(cudaIpcOpenMemHandle(ptr, h, cudaIpcMemLazyEnablePeerAccess));
}

extern "C" int rt_ipc_close(void* ptr) { return ptr == nullptr ? RT_OK : record_cuda(cudaIpcCloseMemHandle(ptr)); }

extern "C" int rt_peer_epoch_step(int64_t* epoch_dev, int64_t add, rt_stream_t stream) {
  if (epoch_dev == nullptr) return RT_ERR_INVALID_ARGUMENT;
  peer_epoch_step_kernel<<<1, 1, 0, reinterpret_cast<cudaStream_t>(stream)>>>(epoch_dev, add);
  return check_launch();
}

extern "C" int rt_peer_signal(void* const* peer_flags, int world, int rank, const int64_t* epoch_dev,
                              int64_t epoch_add, rt_stream_t stream) {
  if (!peers_ok(peer_flags, world) || rank < 0 || rank >= world || epoch_dev == nullptr)
    return RT_ERR_INVALID_ARGUMENT;
  PeerPtrs f{};
  for (int i = 0; i < world; ++i) f.p[i] = static_cast<char*>(peer_flags[i]);
  peer_signal_kernel<<<1, 32, 0, reinterpret_cast<cudaStream_t>(stream)>>>(f, world, rank, epoch_dev, epoch_add);
  return check_launch();
}

extern "C" int rt_peer_gather(void* const* peer_bufs, int world, int rows, int64_t row_bytes, int64_t src_ld,
                              void* out, int64_t out_ld, const int64_t* flags_local, const int64_t* epoch_dev,
                              int64_t epoch_add, int* status, rt_stream_t stream) {
  if (!peers_ok(peer_bufs, world) || rows < 0 || row_bytes <= 0 || row_bytes % 16 || src_ld < row_bytes ||
      src_ld % 16 || out == nullptr || (reinterpret_cast<uintptr_t>(out) & 15) || out_ld < world * row_bytes ||
      out_ld % 16 || flags_local == nullptr || epoch_dev == nullptr)
    return RT_ERR_INVALID_ARGUMENT;
  if (rows == 0) return RT_OK;
  PeerPtrs b{};
  for (int i = 0; i < world; ++i) b.p[i] = static_cast<char*>(peer_bufs[i]);
  // about 16 KB of rows per CTA
  const int rows_per_cta = static_cast<int>(std::max<int64_t>(1, 16384 / row_bytes));
  const dim3 grid((rows + rows_per_cta - 1) / rows_per_cta, world);
  peer_gather_kernel<<<grid, kGatherThreads, 0, reinterpret_cast<cudaStream_t>(stream)>>>(
      b, world, rows, row_bytes, src_ld, static_cast<char*>(out), out_ld, flags_local, epoch_dev, epoch_add,
      rows_per_cta, status);
  return check_launch();
}
