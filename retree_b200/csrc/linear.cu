// Projections of the verify forward on tcgen05: Y[m, N] = X[m, K] . W[N, K]^T
// for a few hundred tree nodes m against a weight matrix W that streams from
// HBM once per round (transformers' nn.Linear in Qwen3Attention / Qwen3MLP,
// modeling_qwen3.py:236-247 and :70-83, and the lm_head).
//
// At tree sizes the product is weight-bandwidth bound, so the kernel is built
// around the weight stream:
//   * swap AB: the MMA's M = 128 side is 128 weight rows (output features),
//     its N side the m tokens (padded to 16; two MMAs when m > 256), K in
//     64-element (128-byte, SW128) blocks.  Accumulators live in TMEM.
//   * warp 0 issues TMA loads of the W tile and the X rows into a ring of
//     stages (one 64-column K block a stage, or four where K is split over a
//     cluster: fewer, longer transfers per weight row), warp 1 issues
//     tcgen05.mma (one thread) and owns TMEM, warps 2-5 run the epilogue.
//     Small m fits two CTAs per SM.
//   * split-K fills the machine when N / 128 is small: the CTAs of one tile
//     form a thread-block cluster along the split dimension; each parks its
//     fp32 partial tile in shared memory and every CTA sums, for the tokens it
//     owns, the partials of all ranks over DSMEM in rank order (deterministic,
//     no global scratch, no second launch) and runs the epilogue on them.
//   * programmatic dependent launch: the W stages of the ring are requested
//     before the kernel waits for the previous kernel in the stream (the
//     weights are not written by the round), so the weight stream starts
//     while the producer of X is still finishing.
//   * fused epilogues on the finished tile, staged in shared memory as the bf16
//     values the library GEMM would have produced:
//       RT_EPI_STORE     Y rows to `out`;
//       RT_EPI_SILU_MUL  W = [gate; up]: a tile takes 64 gate rows and the 64
//                        matching up rows, and writes silu(gate) * up
//                        (Qwen3MLP.forward, :81-83);
//       RT_EPI_QKV_ROPE  W = [Wq; Wk; Wv]: a tile is one head; query/key heads
//                        get the per-head RMSNorm and rotary embedding, keys
//                        and values go straight into the KV cache
//                        (Qwen3Attention.forward :262-271, cache_utils.py:102-121).
// Every wait is bounded (common.cuh); a CTA that gives up records
// RT_DEV_WAIT_TIMEOUT, drains what it issued, frees TMEM and exits.
#include <cuda.h>

#include <map>
#include <mutex>

#include "argmax_key.cuh"
#include "common.cuh"
#include "host_util.h"
#include "layer_math.cuh"
#include "tmap.h"

namespace rt {
namespace {

constexpr int kLinThreads = 192;
constexpr int kBK = 64;
constexpr uint32_t kWTileBytes = 128 * kBK * 2;  // 16 KB
constexpr int kMaxStages = 8;
constexpr int kMaxTokens = 512;

struct LinearParams {
  int m, n_out, k;
  int chunks, chunk_rows;  // token chunks of chunk_rows (multiple of 16, <= 256)
  int kblocks, splits, per, tiles;  // kblocks: ring stages over K (bps 64-column blocks each)
  int epi, stages, bps;
  uint32_t stage_bytes, tmem_cols;
  __nv_bfloat16* out;
  int64_t ld_out;
  rt_qkv_epilogue qkv;
  int* status;
  // gathered X (rt_linear_gather): K block kb lives on rank kb / g_blocks,
  // announced by g_flags[rank] reaching *g_epoch + g_epoch_add
  int g_blocks;
  const int64_t* g_flags;
  const int64_t* g_epoch;
  int64_t g_epoch_add;
  // rt_linear_argmax: per token the max of argmax_key over the output row (zeroed before the launch)
  unsigned long long* am_keys;
};

// kMode: kPlain, kGatherX (X gathered from the ranks of a split, rt_linear_gather)
// or kArgmax (store + per-token argmax keys, rt_linear_argmax).
constexpr int kPlain = 0, kGatherX = 1, kArgmax = 2;

// X sources of rt_linear_gather: one tensor map per rank's column block
// (peer memory for the other ranks; plain, non-multicast TMA loads).  The
// other modes carry one unused map, not eight (1 KB less of kernel
// parameters per launch).
constexpr int kMaxGather = 8;
template <int kMode>
struct XSources {
  CUtensorMap map[kMode == kGatherX ? kMaxGather : 1];
};

constexpr uint32_t kPeerWaitLimit = 1u << 22;  // polls (system-scope load + ~64 ns sleep): 0.5 s or more

// Bounded wait for a peer's announcement; on success the async proxy (TMA)
// is ordered after the acquire.
__device__ __forceinline__ bool wait_peer_flag(const int64_t* flag, int64_t epoch, volatile int* abort,
                                               int* status) {
  for (uint32_t i = 0; i < kPeerWaitLimit; ++i) {
    int64_t v;
    asm volatile("ld.acquire.sys.global.s64 %0, [%1];" : "=l"(v) : "l"(flag) : "memory");
    if (v >= epoch) {
      asm volatile("fence.proxy.async.global;" ::: "memory");
      return true;
    }
    if ((i & 255u) == 255u && *abort) return false;
    __nanosleep(64);
  }
  *abort = 1;
  set_status(status, RT_DEV_WAIT_TIMEOUT);
  return false;
}

struct LinBars {
  uint64_t full[kMaxStages], empty[kMaxStages], acc;
  uint32_t tmem_base;
  int abort_flag;
};

constexpr uint32_t kPartBytes = 32 * 128 * 4;  // one 32-token fp32 partial slice (split-K exchange)

template <int kMode>
__global__ void __launch_bounds__(kLinThreads, 2) linear_kernel(const __grid_constant__ CUtensorMap tmap_w,
                                                             const __grid_constant__ CUtensorMap tmap_x,
                                                             const __grid_constant__ XSources<kMode> xs,
                                                             const LinearParams p) {
  extern __shared__ unsigned char smem_raw[];
  unsigned char* smem =
      reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  LinBars& bar = *reinterpret_cast<LinBars*>(smem + p.stages * p.stage_bytes);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  constexpr bool kGather = kMode == kGatherX;
  const int tile = blockIdx.x, split = blockIdx.y;
  const int kb0 = split * p.per;
  const int nk = max(0, min(p.kblocks, kb0 + p.per) - kb0);
  const bool dual = p.epi == RT_EPI_SILU_MUL;

  if (threadIdx.x == 0) {
    for (int s = 0; s < p.stages; ++s) {
      mbar_init(&bar.full[s], 1);
      mbar_init(&bar.empty[s], 1);
    }
    mbar_init(&bar.acc, 1);
    bar.abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 1) {
    tmem_alloc(&bar.tmem_base, p.tmem_cols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = bar.tmem_base;
  volatile int* abort_flag = &bar.abort_flag;

  pdl_launch_dependents();
  if (warp == 0) {
    // ------------------------------ TMA producer ------------------------------
    if (lane == 0) {
      prefetch_tmap(&tmap_w);
      prefetch_tmap(&tmap_x);
      auto load_w = [&](int it) {
        const int s = it % p.stages;
        unsigned char* st = smem + s * p.stage_bytes;
        mbar_arrive_expect_tx(&bar.full[s], p.stage_bytes);
        for (int b = 0; b < p.bps; ++b) {
          const int kx = ((kb0 + it) * p.bps + b) * kBK;
          unsigned char* wb = st + b * kWTileBytes;
          if (dual) {
            tma_load_2d(wb, &tmap_w, &bar.full[s], kx, tile * 64);
            tma_load_2d(wb + kWTileBytes / 2, &tmap_w, &bar.full[s], kx, p.n_out / 2 + tile * 64);
          } else {
            tma_load_2d(wb, &tmap_w, &bar.full[s], kx, tile * 128);
          }
        }
      };
      uint32_t ready = 0;  // gathered X: ranks whose rows this CTA has seen announced
      int64_t epoch = 0;
      auto load_x = [&](int it) -> bool {
        const int s = it % p.stages;
        unsigned char* xst = smem + s * p.stage_bytes + p.bps * kWTileBytes;
        for (int b = 0; b < p.bps; ++b) {
          const int kx = ((kb0 + it) * p.bps + b) * kBK;
          if constexpr (kGather) {
            const int src = (kx / kBK) / p.g_blocks;
            if (!(ready & (1u << src))) {
              if (!wait_peer_flag(p.g_flags + src, epoch, abort_flag, p.status)) {
                // the stage was armed for these X bytes: count them so its barrier completes
                mbar_complete_tx(&bar.full[s], static_cast<uint32_t>((p.bps - b) * p.chunks * p.chunk_rows * 128));
                return false;
              }
              ready |= 1u << src;
            }
            const int lx = kx - src * p.g_blocks * kBK;
            for (int c = 0; c < p.chunks; ++c)
              tma_load_2d(xst + (b * p.chunks + c) * p.chunk_rows * 128, &xs.map[src], &bar.full[s], lx,
                          c * p.chunk_rows);
          } else {
            for (int c = 0; c < p.chunks; ++c)
              tma_load_2d(xst + (b * p.chunks + c) * p.chunk_rows * 128, &tmap_x, &bar.full[s], kx,
                          c * p.chunk_rows);
          }
        }
        return true;
      };
      // the first pass over the ring needs no free slot: weights first, then X
      // once the kernel that writes it has finished
      const int pre = min(nk, p.stages);
      for (int it = 0; it < pre; ++it) load_w(it);
      pdl_wait();
      if constexpr (kGather) epoch = *p.g_epoch + p.g_epoch_add;
      int issued = pre;
      int x_stages = 0;  // first-pass stages whose X loads went out
      for (int it = 0; it < pre; ++it) {
        if (!load_x(it)) break;
        x_stages = it + 1;
      }
      if constexpr (kGather) {
        // gave up inside stage x_stages (load_x settled its bytes): the first-pass
        // stages after it were armed for X that never comes
        for (int it = x_stages + 1; it < pre; ++it)
          mbar_complete_tx(&bar.full[it % p.stages], static_cast<uint32_t>(p.bps * p.chunks * p.chunk_rows * 128));
      }
      for (int it = pre; it < nk && !(kGather && *abort_flag); ++it) {
        const int s = it % p.stages;
        if (!mbar_wait(&bar.empty[s], ((it / p.stages) & 1) ^ 1, abort_flag, p.status, RT_DEV_WAIT_TIMEOUT)) break;
        load_w(it);
        issued = it + 1;
        if (!load_x(it)) break;
      }
      if (*abort_flag) {
        // let the copies still in flight land before the block's memory goes away
        for (int it = max(0, issued - p.stages); it < issued; ++it)
          mbar_wait_drain(&bar.full[it % p.stages], (it / p.stages) & 1);
      }
    } else {
      pdl_wait();
    }
  } else if (warp == 1) {
    // ------------------------------ MMA issuer --------------------------------
    pdl_wait();
    if (lane == 0) {
      const uint32_t idesc = idesc_bf16_f32(128, p.chunk_rows, false, false);
      for (int it = 0; it < nk; ++it) {
        const int s = it % p.stages;
        if (!mbar_wait(&bar.full[s], (it / p.stages) & 1, abort_flag, p.status, RT_DEV_WAIT_TIMEOUT)) break;
        tc_fence_after();
        const uint32_t st = smem_u32(smem + s * p.stage_bytes);
        for (int b = 0; b < p.bps; ++b) {
          const uint32_t sw = st + b * kWTileBytes;
          for (int c = 0; c < p.chunks; ++c) {
            const uint32_t sx = st + p.bps * kWTileBytes + (b * p.chunks + c) * p.chunk_rows * 128;
#pragma unroll
            for (int kk = 0; kk < kBK / 16; ++kk) {
              umma_f16(tmem + c * 256, smem_desc_sw128(sw + kk * 32, 16, 1024),
                       smem_desc_sw128(sx + kk * 32, 16, 1024), idesc, (it > 0 || b > 0 || kk > 0) ? 1u : 0u);
            }
          }
        }
        umma_commit(&bar.empty[s]);
      }
      // arrives once every MMA issued above has completed (also on the abort path)
      umma_commit(&bar.acc);
      // the TMEM is freed after the final block barrier: on the abort path the
      // epilogue does not wait for the accumulator, so this lane does
      if (*abort_flag) mbar_wait_drain(&bar.acc, 0);
    }
  } else {
    pdl_wait();
  }
  __syncwarp();  // the producer / MMA lanes rejoin their warps before the aligned barriers below

  // ------------------------------ epilogue ------------------------------------
  // Warps 2-5 read the accumulator (warp w may read TMEM lanes 32*(w%4)..+31);
  // every warp of every CTA takes part in the cluster barriers.
  const bool epi_warp = warp >= 2;
  const int et = threadIdx.x - 64;  // 0..127 on the epilogue warps
  const int quad = warp & 3;
  const int r = quad * 32 + lane;   // tile row = output feature
  const int S = p.splits;
  const int rank = split;           // cluster (1, S, 1): rank = blockIdx.y
  bool ok = true;
  if (epi_warp) {
    ok = mbar_wait(&bar.acc, 0, abort_flag, p.status, RT_DEV_WAIT_TIMEOUT);
    ok = __all_sync(0xFFFFFFFFu, ok) && nk > 0;
    tc_fence_after();
  }
  // the ring is free once the accumulator is final: [0, 16 KB) exchange slice,
  // then the bf16 result tile [m][128]
  float* part = reinterpret_cast<float*>(smem);
  __nv_bfloat16* stile = reinterpret_cast<__nv_bfloat16*>(smem + kPartBytes);
  const uint32_t lane_base = static_cast<uint32_t>(quad * 32) << 16;
  if (S == 1) {
    if (epi_warp) {
      for (int c = 0; c < p.chunks; ++c) {
        for (int c0 = 0; c0 < p.chunk_rows; c0 += 32) {
          uint32_t v[32];
          tmem_ld32(tmem + lane_base + c * 256 + c0, v);
          tmem_wait_ld();
          if (ok) {
#pragma unroll
            for (int j = 0; j < 32; ++j) {
              const int t = c * p.chunk_rows + c0 + j;
              if (c0 + j < p.chunk_rows && t < p.m) stile[t * 128 + r] = __float2bfloat16_rn(__uint_as_float(v[j]));
            }
          }
        }
      }
    }
  } else {
    // split-K (one token chunk): 32 tokens at a time, every rank parks its
    // partial slice, then sums the slices of all ranks for the tokens it owns
    // (t % S == rank), rank 0 first
    const int rounds = (p.m + 31) / 32;
    for (int rnd = 0; rnd < rounds; ++rnd) {
      if (epi_warp) {
        uint32_t v[32];
        tmem_ld32(tmem + lane_base + rnd * 32, v);
        tmem_wait_ld();
#pragma unroll
        for (int j = 0; j < 32; ++j) part[j * 128 + r] = ok ? __uint_as_float(v[j]) : 0.f;
      }
      cluster_sync_all();
      if (epi_warp) {
        // owned tokens of this 32-token pass: j = j0, j0 + S, ... (t % S == rank); all
        // remote loads of a token are issued before any is summed
        const int j0 = ((rank - rnd * 32) % S + S) % S;
        for (int j = j0; j < 32; j += S) {
          const int t = rnd * 32 + j;
          if (t >= p.m) break;
          const uint32_t a = smem_u32(part + j * 128 + r);
          float v[8];
#pragma unroll
          for (int q = 0; q < 8; ++q) v[q] = q < S ? ld_cluster_f32(cluster_map(a, q)) : 0.f;
          float acc = 0.f;
#pragma unroll
          for (int q = 0; q < 8; ++q)
            if (q < S) acc = __fadd_rn(acc, v[q]);
          stile[t * 128 + r] = __float2bfloat16_rn(acc);
        }
      }
      cluster_sync_all();
    }
  }
  tc_fence_before();
  __syncthreads();
  if (epi_warp && ok) {
    // tokens this CTA finishes: all of them, or t % S == rank under split-K
    const int own = (p.m - rank + S - 1) / S;
    if (p.epi == RT_EPI_STORE) {
      for (int i = et; i < own * 16; i += 128) {
        const int t = (i >> 4) * S + rank, c = i & 15;
        const uint4 v = reinterpret_cast<const uint4*>(stile)[t * 16 + c];
        *reinterpret_cast<uint4*>(p.out + t * p.ld_out + tile * 128 + c * 8) = v;
      }
      if constexpr (kMode == kArgmax) {
        // one warp per token: the best of the tile's 128 bf16 values (4 a lane), then one
        // 64-bit atomicMax per (tile, token); equal values resolve to the smaller row
        for (int i = et >> 5; i < own; i += 4) {
          const int t = i * S + rank;
          float x[4];
          unpack4(reinterpret_cast<const uint2*>(stile)[t * 32 + lane], x);
          unsigned long long best = 0ull;
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const unsigned long long key = argmax_key(x[e], static_cast<uint32_t>(tile * 128 + lane * 4 + e));
            best = key > best ? key : best;
          }
#pragma unroll
          for (int off = 16; off > 0; off >>= 1) {
            const unsigned long long o = __shfl_xor_sync(0xFFFFFFFFu, best, off);
            best = o > best ? o : best;
          }
          if (lane == 0) atomicMax(p.am_keys + t, best);
        }
      }
    } else if (p.epi == RT_EPI_SILU_MUL) {
      for (int i = et; i < own * 8; i += 128) {
        const int t = (i >> 3) * S + rank, c = i & 7;
        float g[8], u[8], y[8];
        unpack8(reinterpret_cast<const Vec8*>(stile)[t * 16 + c], g);
        unpack8(reinterpret_cast<const Vec8*>(stile)[t * 16 + 8 + c], u);
#pragma unroll
        for (int e = 0; e < 8; ++e) y[e] = silu_mul_bf16(g[e], u[e]);
        *reinterpret_cast<Vec8*>(p.out + t * p.ld_out + tile * 64 + c * 8) = pack8(y);
      }
    } else {
      const rt_qkv_epilogue& e = p.qkv;
      const int h = tile;  // a 128-row tile is one head of [q | k | v]
      const bool is_q = h < e.num_q_heads, is_v = h >= e.num_q_heads + e.num_kv_heads;
      const int64_t off = (e.offset_dev != nullptr ? *e.offset_dev : 0) + e.offset;
      for (int i = et >> 5; i < own; i += 4) {
        const int t = i * S + rank;
        uint2 res = reinterpret_cast<const uint2*>(stile)[t * 32 + lane];
        if (!is_v) {
          float x[4];
          unpack4(res, x);
          int64_t pos = e.positions[t];
          if (pos < 0 || pos >= e.table_len) {
            if (lane == 0) set_status(p.status, RT_DEV_BAD_INDEX);
            pos = 0;
          }
          res = qk_norm_rope4(x, static_cast<const __nv_bfloat16*>(is_q ? e.q_norm_weight : e.k_norm_weight), e.eps,
                              static_cast<const __nv_bfloat16*>(e.cos_table) + pos * 128,
                              static_cast<const __nv_bfloat16*>(e.sin_table) + pos * 128, lane);
        }
        if (is_q) {
          reinterpret_cast<uint2*>(static_cast<__nv_bfloat16*>(e.q_out) +
                                   (static_cast<int64_t>(t) * e.num_q_heads + h) * 128)[lane] = res;
        } else {
          const int64_t row = off + t;
          if (off < 0 || row >= e.capacity) {
            if (lane == 0) set_status(p.status, RT_DEV_OVERFLOW);
          } else {
            const int g = is_v ? h - e.num_q_heads - e.num_kv_heads : h - e.num_q_heads;
            char* dst =
                static_cast<char*>(is_v ? e.v_cache : e.k_cache) + g * e.cache_head_stride + row * e.cache_row_stride;
            reinterpret_cast<uint2*>(dst)[lane] = res;
          }
        }
      }
    }
  }
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, p.tmem_cols);
  }
}

struct Plan {
  int chunks, chunk_rows, kblocks, tiles, splits, per, stages, bps;
  uint32_t stage_bytes, tmem_cols;
  size_t smem;
};

int sm_count() {
  static int n = [] {
    int dev = 0, v = 148;
    if (cudaGetDevice(&dev) == cudaSuccess) cudaDeviceGetAttribute(&v, cudaDevAttrMultiProcessorCount, dev);
    return v > 0 ? v : 148;
  }();
  return n;
}

// 64-column K blocks per ring stage.  Where the 128-row tiles do not cover
// the SMs (K split over a cluster, one CTA per SM) a stage takes kSplitBps
// blocks: fewer, longer transfers per weight row and fewer ring round trips
// (measured at 17 rows: down_proj 18.1 -> 14.5 us with two blocks, 13.8 with
// four; the ring depth itself, 8 or 12 one-block stages, made no difference).
// Where the tiles cover the SMs a stage takes one block, so two CTAs share an
// SM with a ring each.
constexpr int kSplitBps = 4;
int linear_bps(int tiles, int chunks) { return (chunks == 1 && tiles < sm_count()) ? kSplitBps : 1; }

// CTAs (clusters of `cluster`) of linear_kernel that fit on the GPU at once
// with `smem` bytes each (cached per shape of the launch).
int max_active_clusters(int cluster, size_t smem, int tiles) {
  static std::mutex mu;
  static std::map<std::pair<int, size_t>, int> cache;
  std::lock_guard<std::mutex> lock(mu);
  const auto key = std::make_pair(cluster, smem);
  auto it = cache.find(key);
  if (it != cache.end()) return it->second;
  set_smem_limit(linear_kernel<kPlain>, smem);
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(tiles, cluster);
  cfg.blockDim = dim3(kLinThreads);
  cfg.dynamicSmemBytes = smem;
  cudaLaunchAttribute attr;
  attr.id = cudaLaunchAttributeClusterDimension;
  attr.val.clusterDim.x = 1;
  attr.val.clusterDim.y = static_cast<unsigned>(cluster);
  attr.val.clusterDim.z = 1;
  cfg.attrs = &attr;
  cfg.numAttrs = 1;
  int n = 0;
  if (cudaOccupancyMaxActiveClusters(&n, linear_kernel<kPlain>, &cfg) != cudaSuccess) {
    cudaGetLastError();
    n = 0;
  }
  cache[key] = n;
  return n;
}

// Shape checks, and (when `choose`) the launch plan: the largest split of K
// (cluster of <= 8 CTAs per 128-row tile) whose clusters all fit on the GPU at
// once -- a second wave would double the time of a weight-streaming launch --
// with the deeper one-CTA-per-SM ring preferred over two CTAs per SM.
int make_plan(int m, int n_out, int k, int epi, Plan* pl, bool choose) {
  if (m <= 0 || m > kMaxTokens || k < 8 || k % 8 || n_out <= 0 || n_out % 128) return RT_ERR_INVALID_ARGUMENT;
  if (epi < RT_EPI_STORE || epi > RT_EPI_QKV_ROPE) return RT_ERR_INVALID_ARGUMENT;
  const int m_pad = (m + 15) / 16 * 16;
  pl->chunks = m_pad > 256 ? 2 : 1;
  pl->chunk_rows = pl->chunks == 1 ? m_pad : ((m_pad / 2 + 15) / 16 * 16);
  const uint32_t fixed = sizeof(LinBars) + 1024;
  const uint32_t block_bytes = kWTileBytes + static_cast<uint32_t>(pl->chunks * pl->chunk_rows * 128);
  // K blocks per stage: as many as the preference allows with >= 2 stages in 200 KB
  pl->bps = linear_bps(n_out / 128, pl->chunks);
  while (pl->bps > 1 && 2 * pl->bps * block_bytes > 200u * 1024u) pl->bps >>= 1;
  pl->kblocks = (k + kBK * pl->bps - 1) / (kBK * pl->bps);
  pl->tiles = n_out / 128;
  pl->stage_bytes = pl->bps * block_bytes;
  if (2 * pl->stage_bytes + fixed > 227u * 1024u) return RT_ERR_UNSUPPORTED;
  const int stages1 = std::max(2, std::min(kMaxStages, static_cast<int>((200u * 1024u) / pl->stage_bytes)));
  const int stages2 = std::min(kMaxStages, static_cast<int>((113u * 1024u - fixed) / pl->stage_bytes));
  const size_t need = kPartBytes + static_cast<size_t>(m) * 256;  // exchange slice + result tile
  if (static_cast<size_t>(stages1) * pl->stage_bytes < need) return RT_ERR_UNSUPPORTED;
  uint32_t cols = 32;
  while (cols < (pl->chunks == 1 ? static_cast<uint32_t>(m_pad) : 512u)) cols <<= 1;
  pl->tmem_cols = cols;
  auto set = [&](int splits, int stages) {
    pl->per = (pl->kblocks + splits - 1) / splits;
    pl->splits = (pl->kblocks + pl->per - 1) / pl->per;
    pl->stages = stages;
    pl->smem = static_cast<size_t>(stages) * pl->stage_bytes + fixed;
  };
  const bool two_ok = stages2 >= 3 && static_cast<size_t>(stages2) * pl->stage_bytes >= need;
  set(1, two_ok ? stages2 : stages1);
  if (!choose) return RT_OK;
  const int sms = sm_count();
  if (pl->chunks != 1 || pl->tiles >= sms) return RT_OK;
  for (int s = std::min(8, pl->kblocks / 2); s >= 2; --s) {
    const int per = (pl->kblocks + s - 1) / s;
    const int splits = (pl->kblocks + per - 1) / per;
    if (splits != s) continue;
    if (pl->tiles <= max_active_clusters(s, static_cast<size_t>(stages1) * pl->stage_bytes + fixed, pl->tiles)) {
      set(s, stages1);
      return RT_OK;
    }
    if (two_ok &&
        pl->tiles <= max_active_clusters(s, static_cast<size_t>(stages2) * pl->stage_bytes + fixed, pl->tiles)) {
      set(s, stages2);
      return RT_OK;
    }
  }
  return RT_OK;
}

bool al16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; }

}  // namespace
}  // namespace rt

using namespace rt;

extern "C" int rt_linear_check(int m, int n_out, int k, int epilogue) {
  Plan pl;
  return make_plan(m, n_out, k, epilogue, &pl, false);
}

extern "C" int rt_linear_plan(int m, int n_out, int k, int epilogue, int* splits, int* stages, int* smem_bytes) {
  Plan pl;
  const int rc = make_plan(m, n_out, k, epilogue, &pl, true);
  if (rc != RT_OK) return rc;
  if (splits) *splits = pl.splits;
  if (stages) *stages = pl.stages;
  if (smem_bytes) *smem_bytes = static_cast<int>(pl.smem);
  return RT_OK;
}

extern "C" int rt_linear(const void* x, int64_t ld_x, int m, int k, const void* w, int n_out, int epilogue,
                         void* out, int64_t ld_out, const rt_qkv_epilogue* qkv, int* status, rt_stream_t stream) {
  Plan pl;
  int rc = make_plan(m, n_out, k, epilogue, &pl, true);
  if (rc != RT_OK) return rc;
  if (!x || !w || !al16(x) || !al16(w) || ld_x < k || (ld_x * 2) % 16) return RT_ERR_INVALID_ARGUMENT;
  if (epilogue == RT_EPI_QKV_ROPE) {
    if (!qkv || qkv->num_q_heads <= 0 || qkv->num_kv_heads <= 0 ||
        n_out != (qkv->num_q_heads + 2 * qkv->num_kv_heads) * 128 || !qkv->cos_table || !qkv->sin_table ||
        qkv->table_len <= 0 || !qkv->positions || !qkv->q_out || !qkv->k_cache || !qkv->v_cache ||
        qkv->capacity <= 0 || (qkv->q_norm_weight == nullptr) != (qkv->k_norm_weight == nullptr) ||
        qkv->cache_head_stride % 8 || qkv->cache_row_stride % 8 ||
        reinterpret_cast<uintptr_t>(qkv->k_cache) % 8 || reinterpret_cast<uintptr_t>(qkv->v_cache) % 8 ||
        reinterpret_cast<uintptr_t>(qkv->q_out) % 8)
      return RT_ERR_INVALID_ARGUMENT;
  } else {
    const int width = epilogue == RT_EPI_SILU_MUL ? n_out / 2 : n_out;
    if (!out || !al16(out) || ld_out < width || (ld_out * 2) % 16) return RT_ERR_INVALID_ARGUMENT;
  }
  CUtensorMap tw, tx;
  rc = make_bf16_2d_tmap(&tw, w, n_out, k, k, epilogue == RT_EPI_SILU_MUL ? 64 : 128);
  if (rc != RT_OK) return rc;
  rc = make_bf16_2d_tmap(&tx, x, m, k, ld_x, static_cast<uint32_t>(pl.chunk_rows));
  if (rc != RT_OK) return rc;
  LinearParams p{};
  p.m = m;
  p.n_out = n_out;
  p.k = k;
  p.chunks = pl.chunks;
  p.chunk_rows = pl.chunk_rows;
  p.kblocks = pl.kblocks;
  p.splits = pl.splits;
  p.per = pl.per;
  p.tiles = pl.tiles;
  p.epi = epilogue;
  p.stages = pl.stages;
  p.stage_bytes = pl.stage_bytes;
  p.bps = pl.bps;
  p.tmem_cols = pl.tmem_cols;
  p.out = static_cast<__nv_bfloat16*>(out);
  p.ld_out = ld_out;
  if (qkv) p.qkv = *qkv;
  p.status = status;
  set_smem_limit(linear_kernel<kPlain>, pl.smem);
  static const XSources<kPlain> no_sources{};
  return record_cuda(launch_ex(linear_kernel<kPlain>, dim3(pl.tiles, pl.splits), dim3(kLinThreads), pl.smem,
                               static_cast<cudaStream_t>(stream), pl.splits, tw, tx, no_sources, p));
}

extern "C" int rt_linear_gather(const void* const* x_ranks, int world, int cols_per_rank, int64_t ld_x, int m,
                                const void* w, int n_out, int k, void* out, int64_t ld_out,
                                const int64_t* flags_local, const int64_t* epoch_dev, int64_t epoch_add, int* status,
                                rt_stream_t stream) {
  if (x_ranks == nullptr || world < 1 || world > kMaxGather || cols_per_rank <= 0 || cols_per_rank % kBK ||
      k != world * cols_per_rank || ld_x < cols_per_rank || (ld_x * 2) % 16 || flags_local == nullptr ||
      epoch_dev == nullptr)
    return RT_ERR_INVALID_ARGUMENT;
  Plan pl;
  int rc = make_plan(m, n_out, k, RT_EPI_STORE, &pl, true);
  if (rc != RT_OK) return rc;
  if (!w || !al16(w) || !out || !al16(out) || ld_out < n_out || (ld_out * 2) % 16) return RT_ERR_INVALID_ARGUMENT;
  for (int r = 0; r < world; ++r)
    if (x_ranks[r] == nullptr || !al16(x_ranks[r])) return RT_ERR_INVALID_ARGUMENT;
  CUtensorMap tw;
  rc = make_bf16_2d_tmap(&tw, w, n_out, k, k, 128);
  if (rc != RT_OK) return rc;
  XSources<kGatherX> xs{};
  for (int r = 0; r < world; ++r) {
    rc = make_bf16_2d_tmap(&xs.map[r], x_ranks[r], m, cols_per_rank, ld_x, static_cast<uint32_t>(pl.chunk_rows));
    if (rc != RT_OK) return rc;
  }
  LinearParams p{};
  p.m = m;
  p.n_out = n_out;
  p.k = k;
  p.chunks = pl.chunks;
  p.chunk_rows = pl.chunk_rows;
  p.kblocks = pl.kblocks;
  p.splits = pl.splits;
  p.per = pl.per;
  p.tiles = pl.tiles;
  p.epi = RT_EPI_STORE;
  p.stages = pl.stages;
  p.stage_bytes = pl.stage_bytes;
  p.bps = pl.bps;
  p.tmem_cols = pl.tmem_cols;
  p.out = static_cast<__nv_bfloat16*>(out);
  p.ld_out = ld_out;
  p.status = status;
  p.g_blocks = cols_per_rank / kBK;
  p.g_flags = flags_local;
  p.g_epoch = epoch_dev;
  p.g_epoch_add = epoch_add;
  set_smem_limit(linear_kernel<kGatherX>, pl.smem);
  return record_cuda(launch_ex(linear_kernel<kGatherX>, dim3(pl.tiles, pl.splits), dim3(kLinThreads), pl.smem,
                               static_cast<cudaStream_t>(stream), pl.splits, tw, xs.map[0], xs, p));
}

namespace rt {
namespace {
__global__ void argmax_index_kernel(const unsigned long long* keys, int n, int64_t* index) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i < n) index[i] = argmax_row(keys[i]);
}
}  // namespace
}  // namespace rt

extern "C" int rt_linear_argmax(const void* x, int64_t ld_x, int m, int k, const void* w, int n_out, void* out,
                                int64_t ld_out, void* keys, int64_t* index, int* status, rt_stream_t stream) {
  Plan pl;
  int rc = make_plan(m, n_out, k, RT_EPI_STORE, &pl, true);
  if (rc != RT_OK) return rc;
  if (!x || !w || !al16(x) || !al16(w) || ld_x < k || (ld_x * 2) % 16) return RT_ERR_INVALID_ARGUMENT;
  if (!out || !al16(out) || ld_out < n_out || (ld_out * 2) % 16) return RT_ERR_INVALID_ARGUMENT;
  if (!keys || (reinterpret_cast<uintptr_t>(keys) & 7) || !index) return RT_ERR_INVALID_ARGUMENT;
  CUtensorMap tw, tx;
  rc = make_bf16_2d_tmap(&tw, w, n_out, k, k, 128);
  if (rc != RT_OK) return rc;
  rc = make_bf16_2d_tmap(&tx, x, m, k, ld_x, static_cast<uint32_t>(pl.chunk_rows));
  if (rc != RT_OK) return rc;
  LinearParams p{};
  p.m = m;
  p.n_out = n_out;
  p.k = k;
  p.chunks = pl.chunks;
  p.chunk_rows = pl.chunk_rows;
  p.kblocks = pl.kblocks;
  p.splits = pl.splits;
  p.per = pl.per;
  p.tiles = pl.tiles;
  p.epi = RT_EPI_STORE;
  p.stages = pl.stages;
  p.stage_bytes = pl.stage_bytes;
  p.bps = pl.bps;
  p.tmem_cols = pl.tmem_cols;
  p.out = static_cast<__nv_bfloat16*>(out);
  p.ld_out = ld_out;
  p.status = status;
  p.am_keys = static_cast<unsigned long long*>(keys);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  rc = record_cuda(cudaMemsetAsync(keys, 0, static_cast<size_t>(m) * 8, s));
  if (rc != RT_OK) return rc;
  set_smem_limit(linear_kernel<kArgmax>, pl.smem);
  static const XSources<kArgmax> no_sources{};
  rc = record_cuda(launch_ex(linear_kernel<kArgmax>, dim3(pl.tiles, pl.splits), dim3(kLinThreads), pl.smem, s,
                             pl.splits, tw, tx, no_sources, p));
  if (rc != RT_OK) return rc;
  argmax_index_kernel<<<(m + 127) / 128, 128, 0, s>>>(static_cast<const unsigned long long*>(keys), m, index);
  return check_launch();
}
