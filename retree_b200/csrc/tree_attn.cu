// Tree-verify attention for B200 (sm_100a): bf16 GQA, head_dim 128, packed
// ancestor bitmask over the tree block, every prefix key visible.
//
// tcgen05 path (n * group >= 64 query rows per kv head)
// ---------------------------------------------------------------------------
// Grid (split, kv_head, m_tile).  A CTA owns 128 query rows of one kv head --
// row r of the tile is (node (t*128+r)/group, q head kv_head*group + (..)%group),
// so the GQA group shares every K/V tile without repeat_kv -- and a contiguous
// range of 128-key blocks.  Ten warps:
//   warp 8  TMA producer: Q, then K (lane 0) and V (lane 1) blocks -- two
//           64-column SW128 boxes each -- into 2-stage rings, no multicast;
//   warp 9  MMA issuer (one lane): S_j = Q K_j^T into a double-buffered TMEM
//           tile, then O += P_{j-1} V_{j-1} with P read from TMEM; owns the
//           TMEM allocation (S0 | S1 | O | P0 P1, 512 columns);
//   warps 0-7 softmax, two threads per query row (TMEM lane; 64 key columns
//           each, row max and sum exchanged through shared memory): scale and
//           mask S_j, online softmax in the exp2 domain (scale-and-shift and
//           row sums as paired fp32 operations) with a lazy (>8 in log2)
//           rescale of O done in TMEM, P_j as bf16 pairs into TMEM, and the
//           tile's result.
// When the key range is split, the splits of one (kv head, tile) either form
// a thread-block cluster and merge their partial O rows over distributed
// shared memory at the end of the kernel, or write fp32 partials + (m, l) to
// a workspace that attn_combine_kernel merges (two warps per output row up to
// kFastSplits splits, all loads of a row in flight at once; one warp beyond).
// Every mbarrier wait is bounded (common.cuh): on time-out the CTA records
// RT_DEV_WAIT_TIMEOUT, drains what it issued, frees TMEM and exits.
//
// warp-level path (fewer rows): one warp per query row set, shuffle-reduced
// dot products and online softmax; same partial format.

#include <cuda.h>
#include <cuda_fp16.h>

#include <mutex>

#include "common.cuh"
#include "host_util.h"
#include "tmap.h"

namespace rt {

constexpr int kHD = 128;
constexpr int kBM = 128;
constexpr int kBN = 128;
constexpr int kSoftmaxThreads = 256;  // warps 0-7: two threads per tile row
constexpr int kProducerWarp = 8;
constexpr int kMmaWarp = 9;
constexpr int kAttnThreads = 320;
constexpr uint32_t kTile = 128 * 128 * 2;  // one 128x128 bf16 tile
constexpr uint32_t kHalf = kTile / 2;      // one 128-row x 64-column SW128 box
constexpr uint32_t kOffQ = 0;
constexpr uint32_t kOffK = kTile;           // 2 stages
constexpr uint32_t kOffV = 3 * kTile;       // 2 stages
constexpr uint32_t kOffBar = 5 * kTile;     // (P lives in TMEM)
constexpr uint32_t kAttnSmem = kOffBar + 1536 + 1024;  // + barriers/exchange + alignment slack
// In-kernel split merge: once a CTA's last PV product is final, the Q / K / V
// ring is idle and holds the CTA's unnormalised fp32 O tile (rows of 512 B,
// 16-byte chunks XOR-swizzled by row) and its rows' (m, l).
constexpr uint32_t kOffStage = 0;
constexpr uint32_t kOffMl = 2 * kTile;
constexpr uint32_t kOffWeights = 3 * kTile;  // [owned rows][kMaxMerge] fp32 merge weights
constexpr int kMaxMerge = 16;  // cluster size limit (16 needs the non-portable cluster attribute)
constexpr uint32_t kTmemCols = 512;                   // S0 | S1 | O | P0 P1
// P_b (bf16, two keys per 32-bit column, row r in lane r) at TMEM columns
// kPCol + 64*b: the A operand of the PV product, read by the tensor core
// straight from TMEM.
constexpr uint32_t kPCol = 3 * 128;
constexpr float kRescaleThreshold = 8.0f;             // log2 units

struct AttnParams {
  const char* q;
  int64_t q_tok_stride, q_head_stride;
  char* out;
  int64_t out_tok_stride, out_head_stride;
  const uint32_t* mask;
  int mask_words;
  int n;
  int64_t prefix_len;
  const int64_t* prefix_len_dev;
  int group, num_kv_heads, tiles, num_splits;
  int merge;       // 1: the splits of a (kv head, tile) form one cluster and are merged in the kernel
  float scale_log2;
  float* ws_o;     // [split][kv_head][tiles*128][128]
  float2* ws_ml;   // [split][kv_head][tiles*128]  (m in log2 units, l)
  int* status;
  // warp-level path only
  const char* k;
  const char* v;
  int64_t kv_head_stride, kv_row_stride;
};

struct Barriers {
  uint64_t full_q, full_k[2], full_v[2], empty_k[2], empty_v[2], s_full[2], s_free[2], p_full[2], o_done[2], fin;
  uint32_t tmem_base;
  int abort_flag;
  float xchg[2][kBM];  // per-row partial max / sum of the two column halves
};

__device__ __forceinline__ int64_t key_count(const AttnParams& p) {
  const int64_t L = p.prefix_len_dev != nullptr ? *p.prefix_len_dev : p.prefix_len;
  return L + p.n;
}

// Block range [b0, b1) of this split: the blocks spread evenly (range sizes
// differ by at most one, so no split runs two blocks while another idles).
__device__ __forceinline__ void split_range(int64_t total_keys, int split, int splits, int64_t blk, int64_t& b0,
                                            int64_t& b1) {
  const int64_t nblk = (total_keys + blk - 1) / blk;
  b0 = nblk * split / splits;
  b1 = nblk * (split + 1) / splits;
}

__device__ __forceinline__ void write_neutral_partial(const AttnParams& p, int split, int kvh, int row0, int rows) {
  const int64_t rows_ws = static_cast<int64_t>(p.tiles) * kBM;
  for (int r = threadIdx.x; r < rows; r += blockDim.x) {
    p.ws_ml[(static_cast<int64_t>(split) * p.num_kv_heads + kvh) * rows_ws + row0 + r] = make_float2(-INFINITY, 0.f);
  }
}

// Raw S -> running max with four independent accumulators.
__device__ __forceinline__ float max128(const uint32_t (&s)[4][32]) {
  float a[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};
#pragma unroll
  for (int c4 = 0; c4 < 4; ++c4)
#pragma unroll
    for (int c = 0; c < 32; ++c) a[c & 3] = fmaxf(a[c & 3], __uint_as_float(s[c4][c]));
  return fmaxf(fmaxf(a[0], a[1]), fmaxf(a[2], a[3]));
}

// Visibility of the 32 keys [k0, k0+32) for one node: prefix keys (< L) are
// visible, tree key t = key - L uses bit t of the node's mask row, keys at or
// past L + n are hidden.
__device__ __forceinline__ uint32_t visible_word(int64_t k0, int64_t L, int n, const uint32_t* mrow, int words) {
  const int64_t pre = L - k0;  // prefix columns at the start of the window
  if (pre >= 32) return 0xFFFFFFFFu;
  uint32_t bits = pre > 0 ? ((1u << pre) - 1u) : 0u;
  const int64_t t0 = k0 - L;  // tree index of column 0 (negative: starts in the prefix)
  uint32_t tb;
  if (t0 >= 0) {
    const int w = static_cast<int>(t0 >> 5), sh = static_cast<int>(t0 & 31);
    const uint32_t lo = w < words ? mrow[w] : 0u;
    const uint32_t hi = (sh != 0 && w + 1 < words) ? mrow[w + 1] : 0u;
    tb = sh ? ((lo >> sh) | (hi << (32 - sh))) : lo;
  } else {
    tb = mrow[0] << static_cast<int>(-t0);
  }
  // tree columns past the last node are hidden
  const int64_t lim = static_cast<int64_t>(n) - t0;  // columns c < lim have t < n
  if (lim < 32) tb &= lim <= 0 ? 0u : ((1u << lim) - 1u);
  return bits | tb;
}

__device__ __forceinline__ float2 ld_cluster_f32x2(uint32_t addr) {
  float2 v;
  asm volatile("ld.shared::cluster.v2.f32 {%0, %1}, [%2];" : "=f"(v.x), "=f"(v.y) : "r"(addr) : "memory");
  return v;
}
__device__ __forceinline__ float4 ld_cluster_f32x4(uint32_t addr) {
  float4 v;
  asm volatile("ld.shared::cluster.v4.f32 {%0, %1, %2, %3}, [%4];"
               : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w)
               : "r"(addr)
               : "memory");
  return v;
}

// Byte offset of 16-byte chunk `c` (0..31) of row `r` in the merge's O stage.
__device__ __forceinline__ uint32_t stage_off(int r, int c) {
  return kOffStage + static_cast<uint32_t>(r) * 512u + static_cast<uint32_t>((c ^ (r & 31)) << 4);
}

// The split merge inside the cluster (every thread of every CTA calls it; the
// cluster is the S = num_splits CTAs of one (kv head, tile), rank = split).
// Each CTA has staged its unnormalised O rows and (m, l) in its own shared
// memory.  Rank c merges the tile rows r = c, c + S, ...: the rank weights of
// a row are 2^(m_s - M) / L (L = sum_s 2^(m_s - M) l_s, in rank order), and the
// chunks are summed in rank order (a rank of weight 0 -- no key of the row, or
// a row it did not stage -- is skipped, never multiplied) into the bf16
// output.  When every thread has at most one (row, 4-dim chunk) item, each
// item's thread loads every rank's (m, l) and chunk at once and forms the
// weights itself: one distributed-shared-memory round trip.  Otherwise one
// thread per row forms the weights into a shared table first and the item
// threads then load only the chunks.  The last barrier keeps every CTA's
// shared memory until all ranks have read it.
__device__ __forceinline__ float4 merge_chunk(const float4 (&o)[kMaxMerge], int S, const float* wrow) {
  float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
  for (int u = 0; u < kMaxMerge; ++u) {
    const float wu = wrow[u];
    if (u < S && wu != 0.f) {
      acc.x = fmaf(wu, o[u].x, acc.x);
      acc.y = fmaf(wu, o[u].y, acc.y);
      acc.z = fmaf(wu, o[u].z, acc.z);
      acc.w = fmaf(wu, o[u].w, acc.w);
    }
  }
  return acc;
}

// The rank weights of one row from every rank's (m, l).
__device__ __forceinline__ void merge_weights(const float2 (&ml)[kMaxMerge], float (&w)[kMaxMerge]) {
  float M = -INFINITY;
#pragma unroll
  for (int u = 0; u < kMaxMerge; ++u) M = fmaxf(M, ml[u].x);
  float lsum = 0.f;
#pragma unroll
  for (int u = 0; u < kMaxMerge; ++u) {
    w[u] = (M == -INFINITY || ml[u].x == -INFINITY) ? 0.f : ex2(ml[u].x - M);
    lsum = fmaf(w[u], ml[u].y, lsum);
  }
  const float inv = lsum > 0.f ? 1.f / lsum : 0.f;
#pragma unroll
  for (int u = 0; u < kMaxMerge; ++u) w[u] = w[u] * inv;
}

__device__ __forceinline__ void merge_splits(const AttnParams& p, unsigned char* smem, int rank, int kvh, int row0,
                                             int rows_total) {
  __syncwarp();
  cluster_sync_all();
  const int tid = threadIdx.x;
  const int S = p.num_splits, G = p.group;
  const int rows_here = min(kBM, rows_total - row0);
  const int owned = rows_here > rank ? (rows_here - rank + S - 1) / S : 0;
  const uint32_t base = smem_u32(smem);
  float* wtab = reinterpret_cast<float*>(smem + kOffWeights);
  auto store = [&](int rr, int c, const float4& acc) {
    const int R = row0 + rr;
    const int node = R / G, h = kvh * G + (R - node * G);
    uint2 pk;
    pk.x = pack_bf16x2(acc.x, acc.y);
    pk.y = pack_bf16x2(acc.z, acc.w);
    *reinterpret_cast<uint2*>(p.out + node * p.out_tok_stride + h * p.out_head_stride + c * 8) = pk;
  };
  if (owned * 32 <= kAttnThreads) {  // the same in every thread of the CTA
    const int it = tid;
    if (it < owned * 32) {
      const int i = it >> 5, c = it & 31;
      const int rr = rank + S * i;
      const uint32_t off = base + stage_off(rr, c);
      float2 ml[kMaxMerge];
      float4 o[kMaxMerge];
#pragma unroll
      for (int u = 0; u < kMaxMerge; ++u) {
        ml[u] = make_float2(-INFINITY, 0.f);
        o[u] = make_float4(0.f, 0.f, 0.f, 0.f);
        if (u < S) {
          ml[u] = ld_cluster_f32x2(cluster_map(base + kOffMl + rr * 8, u));
          o[u] = ld_cluster_f32x4(cluster_map(off, u));
        }
      }
      float w[kMaxMerge];
      merge_weights(ml, w);
      store(rr, c, merge_chunk(o, S, w));
    }
  } else {
    for (int i = tid; i < owned; i += kAttnThreads) {
      const int rr = rank + S * i;
      float2 ml[kMaxMerge];
#pragma unroll
      for (int u = 0; u < kMaxMerge; ++u)
        ml[u] = u < S ? ld_cluster_f32x2(cluster_map(base + kOffMl + rr * 8, u)) : make_float2(-INFINITY, 0.f);
      float w[kMaxMerge];
      merge_weights(ml, w);
#pragma unroll
      for (int u = 0; u < kMaxMerge; ++u) wtab[i * kMaxMerge + u] = w[u];
    }
    __syncthreads();
    for (int it = tid; it < owned * 32; it += kAttnThreads) {
      const int i = it >> 5, c = it & 31;
      const int rr = rank + S * i;
      const uint32_t off = base + stage_off(rr, c);
      float4 o[kMaxMerge];
#pragma unroll
      for (int u = 0; u < kMaxMerge; ++u) {
        o[u] = make_float4(0.f, 0.f, 0.f, 0.f);
        if (u < S && wtab[i * kMaxMerge + u] != 0.f) o[u] = ld_cluster_f32x4(cluster_map(off, u));
      }
      store(rr, c, merge_chunk(o, S, wtab + i * kMaxMerge));
    }
  }
  __syncwarp();
  cluster_sync_all();
}


__global__ void __launch_bounds__(kAttnThreads, 1)
    tree_attn_tc_kernel(const __grid_constant__ CUtensorMap tmap_k, const __grid_constant__ CUtensorMap tmap_v,
                        const __grid_constant__ CUtensorMap tmap_q, const AttnParams p, const int q_tma) {
  extern __shared__ unsigned char smem_raw[];
  // 1024-byte alignment for the SW128 atoms
  unsigned char* smem =
      reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  Barriers& bar = *reinterpret_cast<Barriers*>(smem + kOffBar);
  // Programmatic dependent launch: the prefix rows of the KV cache are not
  // written while the round's forward runs (only rows from prefix_len on, by
  // this layer's projection), so the producer requests the leading pure-prefix
  // K/V blocks before waiting for the previous kernel; Q, the tree block, the
  // mask and every write come after the wait.  Dependents are released only
  // once this CTA holds its TMEM columns (below): a dependent CTA on the same
  // SM that allocated first and then waited for this grid would otherwise
  // leave this CTA's allocation waiting for columns that never free.
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int split = blockIdx.x, kvh = blockIdx.y, mt = blockIdx.z;
  const int G = p.group;
  const int rows_total = p.n * G;
  const int row0 = mt * kBM;

  const int64_t total_keys = key_count(p);
  const int64_t L = total_keys - p.n;
  int64_t b0, b1;
  split_range(total_keys, split, p.num_splits, kBN, b0, b1);
  const int nb = static_cast<int>(b1 - b0);
  if (nb <= 0) {
    pdl_wait();
    if (p.merge > 1) {
      // no keys here: neutral (m, l) for every row, then this rank's share of the merge
      float2* ml = reinterpret_cast<float2*>(smem + kOffMl);
      for (int r = tid; r < kBM; r += kAttnThreads) ml[r] = make_float2(-INFINITY, 0.f);
      __syncthreads();
      merge_splits(p, smem, split, kvh, row0, rows_total);
      return;
    }
    if (p.num_splits > 1) write_neutral_partial(p, split, kvh, row0, min(kBM, rows_total - row0));
    return;
  }
  // leading blocks of this split that hold prefix keys only (at most the ring depth)
  int pre = 0;
  while (pre < min(2, nb) && (b0 + pre + 1) * kBN <= L) ++pre;

  // The producer lane sets up the barriers and sends the pure-prefix K/V loads
  // out at once, while the MMA warp allocates TMEM (nothing before the block
  // barrier below waits for another warp).
  auto load_kv = [&](uint64_t* full, const CUtensorMap* map, unsigned char* dst, int key0) {
    mbar_arrive_expect_tx(full, kTile);
    tma_load_3d(dst, map, full, 0, key0, kvh);
    tma_load_3d(dst + kHalf, map, full, 64, key0, kvh);
  };
  if (warp == kProducerWarp && lane == 0) {
    prefetch_tmap(&tmap_k);
    prefetch_tmap(&tmap_v);
    if (q_tma) prefetch_tmap(&tmap_q);
    mbar_init(&bar.full_q, 1);
    for (int i = 0; i < 2; ++i) {
      mbar_init(&bar.full_k[i], 1);
      mbar_init(&bar.full_v[i], 1);
      mbar_init(&bar.empty_k[i], 1);
      mbar_init(&bar.empty_v[i], 1);
      mbar_init(&bar.s_full[i], 1);
      mbar_init(&bar.s_free[i], kSoftmaxThreads);
      mbar_init(&bar.p_full[i], kSoftmaxThreads);
      mbar_init(&bar.o_done[i], 1);
    }
    mbar_init(&bar.fin, 1);
    bar.abort_flag = 0;
    fence_mbar_init();
    fence_proxy_async_smem();
    for (int j = 0; j < pre; ++j) {
      const int key0 = static_cast<int>((b0 + j) * kBN);
      load_kv(&bar.full_k[j], &tmap_k, smem + kOffK + j * kTile, key0);
      load_kv(&bar.full_v[j], &tmap_v, smem + kOffV + j * kTile, key0);
    }
  }
  if (warp == kMmaWarp) {
    tmem_alloc(&bar.tmem_base, kTmemCols);
    tmem_relinquish();
  }
  if (!q_tma) {
    pdl_wait();
    // Q tile -> SW128 K-major smem by plain loads (group sizes that do not tile 128 rows)
    constexpr int kPer = (kBM * 16 + kAttnThreads - 1) / kAttnThreads;
    uint4 v[kPer];
#pragma unroll
    for (int i = 0; i < kPer; ++i) {
      const int c = tid + i * kAttnThreads;
      const int r = c >> 4, ch = c & 15, R = row0 + r;
      v[i] = make_uint4(0, 0, 0, 0);
      if (c < kBM * 16 && R < rows_total) {
        const int node = R / G, h = kvh * G + (R - node * G);
        v[i] = *reinterpret_cast<const uint4*>(p.q + node * p.q_tok_stride + h * p.q_head_stride + ch * 16);
      }
    }
#pragma unroll
    for (int i = 0; i < kPer; ++i) {
      const int c = tid + i * kAttnThreads;
      if (c < kBM * 16) {
        const int r = c >> 4, ch = c & 15;
        const uint32_t off = kOffQ + (ch >> 3) * kHalf + r * 128 + (((ch & 7) ^ (r & 7)) << 4);
        *reinterpret_cast<uint4*>(smem + off) = v[i];
      }
    }
    fence_proxy_async_smem();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  pdl_launch_dependents();
  const uint32_t tmem = bar.tmem_base;
  volatile int* abort_flag = &bar.abort_flag;

  if (warp == kProducerWarp) {
    // ---------------- TMA producer: lane 0 Q and K, lane 1 V ----------------
    // (the first `pre` K and V blocks went out in the prologue)
    if (lane == 0) {
      auto issue_q = [&] {
        pdl_wait();
        if (q_tma) {
          mbar_arrive_expect_tx(&bar.full_q, kTile);
          const int tok0 = mt * (kBM / G);
          tma_load_3d(smem + kOffQ, &tmap_q, &bar.full_q, 0, kvh * G, tok0);
          tma_load_3d(smem + kOffQ + kHalf, &tmap_q, &bar.full_q, 64, kvh * G, tok0);
        } else {
          mbar_arrive(&bar.full_q);
        }
      };
      int issued = pre;
      bool q_issued = false;
      for (int j = pre; j < nb; ++j) {
        if (j == pre) {
          issue_q();
          q_issued = true;
        }
        const int st = j & 1;
        // stage st is free once S(j-2) has consumed it
        if (!mbar_wait(&bar.empty_k[st], ((j >> 1) & 1) ^ 1, abort_flag, p.status, RT_DEV_WAIT_TIMEOUT)) break;
        load_kv(&bar.full_k[st], &tmap_k, smem + kOffK + st * kTile, static_cast<int>((b0 + j) * kBN));
        issued = j + 1;
      }
      if (!q_issued) issue_q();
      if (*abort_flag) {
        mbar_wait_drain(&bar.full_q, 0);
        for (int j = max(0, issued - 2); j < issued; ++j) mbar_wait_drain(&bar.full_k[j & 1], (j >> 1) & 1);
      }
    } else if (lane == 1) {
      int issued = pre;
      for (int j = pre; j < nb; ++j) {
        if (j == pre) pdl_wait();
        const int st = j & 1;
        // stage st is free once PV(j-2) has consumed it
        if (!mbar_wait(&bar.empty_v[st], ((j >> 1) & 1) ^ 1, abort_flag, p.status, RT_DEV_WAIT_TIMEOUT)) break;
        load_kv(&bar.full_v[st], &tmap_v, smem + kOffV + st * kTile, static_cast<int>((b0 + j) * kBN));
        issued = j + 1;
      }
      if (*abort_flag)
        for (int j = max(0, issued - 2); j < issued; ++j) mbar_wait_drain(&bar.full_v[j & 1], (j >> 1) & 1);
      pdl_wait();
    } else {
      pdl_wait();
    }
  } else if (warp == kMmaWarp) {
    pdl_wait();
    // ---------------- MMA issuer ----------------
    if (lane == 0) {
      constexpr uint32_t idesc_qk = idesc_bf16_f32(kBM, kBN, false, false);
      constexpr uint32_t idesc_pv = idesc_bf16_f32(kBM, kHD, false, true);
      const uint32_t sq = smem_u32(smem + kOffQ);
      bool ok = mbar_wait(&bar.full_q, 0, abort_flag, p.status, RT_DEV_WAIT_TIMEOUT);
      for (int j = 0; j <= nb && ok; ++j) {
        if (j < nb) {
          const int st = j & 1, b = j & 1;
          const uint32_t ph = (j >> 1) & 1;
          ok = mbar_wait(&bar.full_k[st], ph, abort_flag, p.status, RT_DEV_WAIT_TIMEOUT) &&
               mbar_wait(&bar.s_free[b], ph ^ 1, abort_flag, p.status, RT_DEV_WAIT_TIMEOUT);
          if (!ok) break;
          tc_fence_after();
          const uint32_t sk = smem_u32(smem + kOffK + st * kTile);
#pragma unroll
          for (int kk = 0; kk < kHD / 16; ++kk) {
            const uint32_t koff = (kk >> 2) * kHalf + (kk & 3) * 32;
            umma_f16(tmem + b * kBN, smem_desc_sw128(sq + koff, 16, 1024), smem_desc_sw128(sk + koff, 16, 1024),
                     idesc_qk, kk > 0);
          }
          umma_commit(&bar.s_full[b]);
          umma_commit(&bar.empty_k[st]);
        }
        if (j >= 1) {
          const int jp = j - 1, pb = jp & 1;
          const uint32_t pph = (jp >> 1) & 1;
          ok = mbar_wait(&bar.p_full[pb], pph, abort_flag, p.status, RT_DEV_WAIT_TIMEOUT) &&
               mbar_wait(&bar.full_v[pb], pph, abort_flag, p.status, RT_DEV_WAIT_TIMEOUT);
          if (!ok) break;
          tc_fence_after();
          const uint32_t sv = smem_u32(smem + kOffV + pb * kTile);
#pragma unroll
          for (int kk = 0; kk < kBN / 16; ++kk) {
            // P from TMEM: 16 keys = 8 packed columns.  V is MN-major: 16 keys =
            // two 8-row SW128 atoms (1024 B apart); the second 64-column half
            // of head_dim sits one box (LBO) away.
            umma_f16_ts(tmem + 2 * kBN, tmem + kPCol + pb * 64 + kk * 8,
                        smem_desc_sw128(sv + kk * 2048, kHalf, 1024), idesc_pv, (jp > 0 || kk > 0) ? 1u : 0u);
          }
          umma_commit(&bar.o_done[pb]);
          umma_commit(&bar.empty_v[pb]);
        }
      }
      // all issued MMAs complete before TMEM is released
      umma_commit(&bar.fin);
      mbar_wait_drain(&bar.fin, 0);  // also on the abort path: no MMA may outlive the TMEM
    }
  } else {
    // ---------------- softmax / epilogue (warps 0-7) ----------------
    pdl_wait();
    // Warp w reads TMEM lanes 32*(w%4)..+31 (its sub-partition) and owns key /
    // head-dim columns [64*half, 64*half + 64) with half = w / 4, so every tile
    // row is handled by two threads that exchange their partial max and sum.
    const int half = warp >> 2;
    const int r = tid & (kBM - 1);  // TMEM lane == tile row
    const int R = row0 + r;
    const bool valid = R < rows_total;
    const bool warp_live = row0 + (warp & 3) * 32 < rows_total;  // some row of this warp is a real query
    const int node = valid ? R / G : 0;
    const uint32_t lane_base = static_cast<uint32_t>((warp & 3) * 32) << 16;
    const uint32_t col0 = half * 64;  // this thread's S / O columns
    const uint32_t* mrow = p.mask + static_cast<int64_t>(node) * p.mask_words;
    const float sl2 = p.scale_log2;
    float m = -INFINITY, l = 0.f;  // m in scaled log2 units; l = this half's partial sum
    bool ok = true;
    uint32_t sreg[2][32];
    // Every softmax thread passes both named barriers of every block, whatever
    // happens to its waits: after a time-out `ok` turns false (warp-uniformly)
    // and the thread only keeps the barrier count, so no thread is left waiting.
    for (int j = 0; j < nb; ++j) {
      const int b = j & 1;
      const uint32_t ph = (j >> 1) & 1;
      if (ok) ok = mbar_wait(&bar.s_full[b], ph, abort_flag, p.status, RT_DEV_WAIT_TIMEOUT);
      ok = __all_sync(0xFFFFFFFFu, ok);
      const bool work = ok && warp_live;
      float mloc = -INFINITY;
      if (work) {
        tc_fence_after();
#pragma unroll
        for (int c2 = 0; c2 < 2; ++c2) tmem_ld32(tmem + lane_base + b * kBN + col0 + c2 * 32, sreg[c2]);
        tmem_wait_ld();
        tc_fence_before();
      }
      mbar_arrive(&bar.s_free[b]);
      if (work) {
        const int64_t key0 = (b0 + j) * kBN + col0;
        if (!valid || key0 + 64 > L) {
          // columns reach the tree keys (or the end): hide per a 32-bit visibility word
#pragma unroll
          for (int c2 = 0; c2 < 2; ++c2) {
            const uint32_t vm = valid ? visible_word(key0 + c2 * 32, L, p.n, mrow, p.mask_words) : 0u;
            if (vm != 0xFFFFFFFFu) {
#pragma unroll
              for (int c = 0; c < 32; ++c)
                if (!((vm >> c) & 1u)) sreg[c2][c] = __float_as_uint(-INFINITY);
            }
          }
        }
        float a[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};
#pragma unroll
        for (int c2 = 0; c2 < 2; ++c2)
#pragma unroll
          for (int c = 0; c < 32; ++c) a[c & 3] = fmaxf(a[c & 3], __uint_as_float(sreg[c2][c]));
        mloc = fmaxf(fmaxf(a[0], a[1]), fmaxf(a[2], a[3]));
      }
      // row max over both halves (named barrier among the 256 softmax threads)
      bar.xchg[half][r] = mloc;
      asm volatile("bar.sync 1, %0;" ::"n"(kSoftmaxThreads) : "memory");
      const float mrow_max = fmaxf(bar.xchg[0][r], bar.xchg[1][r]);
      asm volatile("bar.sync 1, %0;" ::"n"(kSoftmaxThreads) : "memory");
      if (!work) {
        mbar_arrive(&bar.p_full[b]);
        continue;
      }
      const float m_new = fmaxf(m, mrow_max * sl2);
      const bool need = m_new > m + kRescaleThreshold;  // identical in both halves; false while -inf
      if (__any_sync(0xFFFFFFFFu, need) && j > 0) {
        // O must hold blocks <= j-1 before it is rescaled
        ok = mbar_wait(&bar.o_done[(j - 1) & 1], ((j - 1) >> 1) & 1, abort_flag, p.status, RT_DEV_WAIT_TIMEOUT);
        ok = __all_sync(0xFFFFFFFFu, ok);
        if (ok) {
          tc_fence_after();
          const float f = need ? ex2(m - m_new) : 1.f;  // ex2(-inf) = 0 when m was -inf
          uint32_t o[32];
#pragma unroll
          for (int c2 = 0; c2 < 2; ++c2) {
            tmem_ld32(tmem + lane_base + 2 * kBN + col0 + c2 * 32, o);
            tmem_wait_ld();
#pragma unroll
            for (int c = 0; c < 32; ++c) o[c] = __float_as_uint(__uint_as_float(o[c]) * f);
            tmem_st32(tmem + lane_base + 2 * kBN + col0 + c2 * 32, o);
          }
          tmem_wait_st();
          l *= f;
        }
      }
      if (need) m = m_new;
      const float mu = (m == -INFINITY) ? 0.f : m;
      if (ok && j >= 2) {
        // P buffer b was last read by PV(j-2)
        ok = mbar_wait(&bar.o_done[b], ((j - 2) >> 1) & 1, abort_flag, p.status, RT_DEV_WAIT_TIMEOUT);
      }
      if (!ok) {
        mbar_arrive(&bar.p_full[b]);
        continue;
      }
      // P = exp2(s*scale - m), summed in fp32, stored as bf16 pairs into this
      // half's 32 columns of the TMEM P buffer (keys 2i, 2i+1 in column i); the
      // scale-and-shift and the running sums go two keys per instruction
      const float2 sc2 = make_float2(sl2, sl2), sh2 = make_float2(-mu, -mu);
      float2 acc[2] = {make_float2(0.f, 0.f), make_float2(0.f, 0.f)};
#pragma unroll
      for (int c2 = 0; c2 < 2; ++c2) {
        uint32_t pk[16];
#pragma unroll
        for (int i = 0; i < 16; ++i) {
          const float2 x = ffma2(make_float2(__uint_as_float(sreg[c2][2 * i]), __uint_as_float(sreg[c2][2 * i + 1])),
                                 sc2, sh2);
          const float p0 = ex2(x.x), p1 = ex2(x.y);
          acc[i & 1] = fadd2(acc[i & 1], make_float2(p0, p1));
          pk[i] = pack_bf16x2(p0, p1);
        }
        tmem_st16(tmem + lane_base + kPCol + b * 64 + half * 32 + c2 * 16, pk);
      }
      l += (acc[0].x + acc[1].x) + (acc[0].y + acc[1].y);
      tmem_wait_st();
      tc_fence_before();
      mbar_arrive(&bar.p_full[b]);
    }
    // full row sum = both halves
    if (ok) ok = mbar_wait(&bar.o_done[(nb - 1) & 1], ((nb - 1) >> 1) & 1, abort_flag, p.status, RT_DEV_WAIT_TIMEOUT);
    ok = __all_sync(0xFFFFFFFFu, ok);
    bar.xchg[half][r] = l;
    asm volatile("bar.sync 1, %0;" ::"n"(kSoftmaxThreads) : "memory");
    const float lrow = bar.xchg[0][r] + bar.xchg[1][r];
    if (p.merge > 1) {
      // park the unnormalised O rows and (m, l) for the in-cluster merge (the
      // ring is idle: every load was consumed and the last PV product is final)
      if (ok && warp_live) {
        tc_fence_after();
#pragma unroll
        for (int c2 = 0; c2 < 2; ++c2) {
          uint32_t o[32];
          tmem_ld32(tmem + lane_base + 2 * kBN + col0 + c2 * 32, o);
          tmem_wait_ld();
#pragma unroll
          for (int q = 0; q < 8; ++q)
            *reinterpret_cast<uint4*>(smem + stage_off(r, (col0 + c2 * 32) / 4 + q)) =
                make_uint4(o[q * 4], o[q * 4 + 1], o[q * 4 + 2], o[q * 4 + 3]);
        }
      }
      if (half == 0)
        reinterpret_cast<float2*>(smem + kOffMl)[r] =
            (ok && warp_live) ? make_float2(m, lrow) : make_float2(-INFINITY, 0.f);
    } else if (ok && warp_live) {
      tc_fence_after();
      const int64_t rows_ws = static_cast<int64_t>(p.tiles) * kBM;
      const int h = valid ? kvh * G + (R - node * G) : 0;
#pragma unroll
      for (int c2 = 0; c2 < 2; ++c2) {
        uint32_t o[32];
        tmem_ld32(tmem + lane_base + 2 * kBN + col0 + c2 * 32, o);
        tmem_wait_ld();
        if (!valid) continue;
        const int d0 = col0 + c2 * 32;  // head-dim offset of these 32 values
        if (p.num_splits == 1) {
          const float inv = 1.f / lrow;
          char* dst = p.out + node * p.out_tok_stride + h * p.out_head_stride + d0 * 2;
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            uint4 pk;
            pk.x = pack_bf16x2(__uint_as_float(o[q * 8 + 0]) * inv, __uint_as_float(o[q * 8 + 1]) * inv);
            pk.y = pack_bf16x2(__uint_as_float(o[q * 8 + 2]) * inv, __uint_as_float(o[q * 8 + 3]) * inv);
            pk.z = pack_bf16x2(__uint_as_float(o[q * 8 + 4]) * inv, __uint_as_float(o[q * 8 + 5]) * inv);
            pk.w = pack_bf16x2(__uint_as_float(o[q * 8 + 6]) * inv, __uint_as_float(o[q * 8 + 7]) * inv);
            *reinterpret_cast<uint4*>(dst + q * 16) = pk;
          }
        } else {
          float* dst = p.ws_o + ((static_cast<int64_t>(split) * p.num_kv_heads + kvh) * rows_ws + R) * kHD + d0;
#pragma unroll
          for (int q = 0; q < 8; ++q)
            *reinterpret_cast<float4*>(dst + q * 4) =
                make_float4(__uint_as_float(o[q * 4]), __uint_as_float(o[q * 4 + 1]), __uint_as_float(o[q * 4 + 2]),
                            __uint_as_float(o[q * 4 + 3]));
        }
      }
      if (valid && half == 0 && p.num_splits > 1)
        p.ws_ml[(static_cast<int64_t>(split) * p.num_kv_heads + kvh) * rows_ws + R] = make_float2(m, lrow);
    }
    tc_fence_before();
  }
  __syncthreads();
  if (p.merge > 1) merge_splits(p, smem, split, kvh, row0, rows_total);
  if (warp == kMmaWarp) {
    __syncwarp();
    tc_fence_after();
    tmem_dealloc(tmem, kTmemCols);
  }
}

// ---------------------------------------------------------------------------
// Warp-level path: CTA = (split, kv head), 4 warps, K/V blocks of 64 keys in
// shared memory; warp w handles query rows w, w+4, ...  Each lane owns 4 of the
// 128 dims; dot products are shuffle-reduced.
// ---------------------------------------------------------------------------
constexpr int kSimtKeys = 64;

__global__ void __launch_bounds__(128) tree_attn_simt_kernel(const AttnParams p) {
  pdl_launch_dependents();
  pdl_wait();
  __shared__ __align__(16) __nv_bfloat16 ks[kSimtKeys][kHD];
  __shared__ __align__(16) __nv_bfloat16 vs[kSimtKeys][kHD];
  const int split = blockIdx.x, kvh = blockIdx.y;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int G = p.group, rows = p.n * G;
  const int64_t total_keys = key_count(p);
  const int64_t L = total_keys - p.n;
  int64_t b0, b1;
  split_range(total_keys, split, p.num_splits, kSimtKeys, b0, b1);
  constexpr int kMaxRowsPerWarp = 16;
  float qv[kMaxRowsPerWarp][4];
  float acc[kMaxRowsPerWarp][4];
  float m[kMaxRowsPerWarp], l[kMaxRowsPerWarp];
#pragma unroll
  for (int i = 0; i < kMaxRowsPerWarp; ++i) {
    m[i] = -INFINITY;
    l[i] = 0.f;
    const int R = warp + 4 * i;
#pragma unroll
    for (int d = 0; d < 4; ++d) {
      acc[i][d] = 0.f;
      qv[i][d] = 0.f;
    }
    if (R < rows) {
      const int node = R / G, h = kvh * G + (R - node * G);
      const __nv_bfloat16* qp =
          reinterpret_cast<const __nv_bfloat16*>(p.q + node * p.q_tok_stride + h * p.q_head_stride) + lane * 4;
#pragma unroll
      for (int d = 0; d < 4; ++d) qv[i][d] = __bfloat162float(qp[d]) * p.scale_log2;
    }
  }
  for (int64_t blk = b0; blk < b1; ++blk) {
    const int64_t key0 = blk * kSimtKeys;
    __syncthreads();
    for (int c = threadIdx.x; c < kSimtKeys * 16; c += 128) {
      const int kr = c >> 4, ch = c & 15;
      const int64_t key = key0 + kr;
      uint4 kv4 = make_uint4(0, 0, 0, 0), vv4 = make_uint4(0, 0, 0, 0);
      if (key < total_keys) {
        kv4 = *reinterpret_cast<const uint4*>(p.k + kvh * p.kv_head_stride + key * p.kv_row_stride + ch * 16);
        vv4 = *reinterpret_cast<const uint4*>(p.v + kvh * p.kv_head_stride + key * p.kv_row_stride + ch * 16);
      }
      *reinterpret_cast<uint4*>(&ks[kr][ch * 8]) = kv4;
      *reinterpret_cast<uint4*>(&vs[kr][ch * 8]) = vv4;
    }
    __syncthreads();
#pragma unroll
    for (int i = 0; i < kMaxRowsPerWarp; ++i) {
      const int R = warp + 4 * i;
      if (R >= rows) break;
      const int node = R / G;
      // scores of keys `lane` and `lane + 32`
      float s2[2];
#pragma unroll
      for (int half = 0; half < 2; ++half) {
        float mine = -INFINITY;
        for (int kk = 0; kk < 32; ++kk) {
          const int kr = half * 32 + kk;
          const __nv_bfloat16* kp = &ks[kr][lane * 4];
          float d = qv[i][0] * __bfloat162float(kp[0]) + qv[i][1] * __bfloat162float(kp[1]) +
                    qv[i][2] * __bfloat162float(kp[2]) + qv[i][3] * __bfloat162float(kp[3]);
#pragma unroll
          for (int o = 16; o > 0; o >>= 1) d += __shfl_xor_sync(0xFFFFFFFFu, d, o);
          if (kk == lane) mine = d;
        }
        const int64_t key = key0 + half * 32 + lane;
        bool vis = key < L;
        if (!vis && key < total_keys) {
          const int64_t t = key - L;
          vis = (p.mask[static_cast<int64_t>(node) * p.mask_words + (t >> 5)] >> (t & 31)) & 1u;
        }
        s2[half] = vis ? mine : -INFINITY;
      }
      float bm = fmaxf(s2[0], s2[1]);
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) bm = fmaxf(bm, __shfl_xor_sync(0xFFFFFFFFu, bm, o));
      const float m_new = fmaxf(m[i], bm);
      const float mu = m_new == -INFINITY ? 0.f : m_new;
      const float f = ex2(m[i] - mu);
      const float e0 = ex2(s2[0] - mu), e1 = ex2(s2[1] - mu);
      float es = e0 + e1;
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) es += __shfl_xor_sync(0xFFFFFFFFu, es, o);
      l[i] = l[i] * f + es;
      m[i] = m_new;
#pragma unroll
      for (int d = 0; d < 4; ++d) acc[i][d] *= f;
      for (int kk = 0; kk < kSimtKeys; ++kk) {
        const float pk = __shfl_sync(0xFFFFFFFFu, kk < 32 ? e0 : e1, kk & 31);
        const __nv_bfloat16* vp = &vs[kk][lane * 4];
#pragma unroll
        for (int d = 0; d < 4; ++d) acc[i][d] += pk * __bfloat162float(vp[d]);
      }
    }
  }
  const int64_t rows_ws = static_cast<int64_t>(p.tiles) * kBM;
#pragma unroll
  for (int i = 0; i < kMaxRowsPerWarp; ++i) {
    const int R = warp + 4 * i;
    if (R >= rows) break;
    const int node = R / G, h = kvh * G + (R - node * G);
    if (p.num_splits == 1) {
      const float inv = 1.f / l[i];
      uint2 pk;
      pk.x = pack_bf16x2(acc[i][0] * inv, acc[i][1] * inv);
      pk.y = pack_bf16x2(acc[i][2] * inv, acc[i][3] * inv);
      *reinterpret_cast<uint2*>(p.out + node * p.out_tok_stride + h * p.out_head_stride + lane * 8) = pk;
    } else {
      const int64_t idx = (static_cast<int64_t>(split) * p.num_kv_heads + kvh) * rows_ws + R;
      *reinterpret_cast<float4*>(p.ws_o + idx * kHD + lane * 4) =
          make_float4(acc[i][0], acc[i][1], acc[i][2], acc[i][3]);
      if (lane == 0) p.ws_ml[idx] = make_float2(m[i], l[i]);
    }
  }
}

// ---------------------------------------------------------------------------
// Split merge: one warp per (kv head, tile row); lane owns 4 dims.
// ---------------------------------------------------------------------------
constexpr int kFastSplits = 24;  // up to this many splits: every load of a row issued at once

__global__ void __launch_bounds__(128) attn_combine_kernel(const AttnParams p) {
  pdl_launch_dependents();
  pdl_wait();
  const int lane = threadIdx.x & 31;
  const int rows = p.n * p.group;
  const int64_t rows_ws = static_cast<int64_t>(p.tiles) * kBM;
  const int S = p.num_splits;
  const float2 none = make_float2(-INFINITY, 0.f);
  if (S <= kFastSplits) {
    // Two warps per (kv head, row), one per 64-dim half, lane owns 2 dims.
    // Every load of the row is independent of the others, so all of them --
    // the splits' partial rows and (max, sum) pairs -- go out at once: one
    // L2 round trip instead of one for the maxima and one per batch of rows.
    // A split whose weight is zero (max -inf) is skipped, never multiplied;
    // the per-element sum runs over the splits in order, as below.
    const int gw = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    if (gw >= 2 * p.num_kv_heads * rows) return;
    const int half = gw & 1, pair = gw >> 1;
    const int kvh = pair / rows, R = pair - kvh * rows;
    auto slot = [&](int s) { return (static_cast<int64_t>(s) * p.num_kv_heads + kvh) * rows_ws + R; };
    const int d0 = half * 64 + lane * 2;
    float2 o[kFastSplits];
#pragma unroll
    for (int u = 0; u < kFastSplits; ++u)
      o[u] = u < S ? *reinterpret_cast<const float2*>(p.ws_o + slot(u) * kHD + d0) : make_float2(0.f, 0.f);
    const float2 ml = lane < S ? p.ws_ml[slot(lane)] : none;
    float M = ml.x;
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) M = fmaxf(M, __shfl_xor_sync(0xFFFFFFFFu, M, off));
    float2 acc = make_float2(0.f, 0.f);
    float lsum = 0.f;
    if (M > -INFINITY) {
      const float w = ml.x == -INFINITY ? 0.f : ex2(ml.x - M);
      lsum = w * ml.y;
#pragma unroll
      for (int u = 0; u < kFastSplits; ++u) {
        const float wu = __shfl_sync(0xFFFFFFFFu, w, u);
        if (u < S && wu != 0.f) {
          acc.x = fmaf(wu, o[u].x, acc.x);
          acc.y = fmaf(wu, o[u].y, acc.y);
        }
      }
#pragma unroll
      for (int off = 16; off > 0; off >>= 1) lsum += __shfl_xor_sync(0xFFFFFFFFu, lsum, off);
    }
    const float inv = lsum > 0.f ? 1.f / lsum : 0.f;
    const int node = R / p.group, h = kvh * p.group + (R - node * p.group);
    *reinterpret_cast<uint32_t*>(p.out + node * p.out_tok_stride + h * p.out_head_stride + d0 * 2) =
        pack_bf16x2(acc.x * inv, acc.y * inv);
    return;
  }
  const int gw = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  if (gw >= p.num_kv_heads * rows) return;
  const int kvh = gw / rows, R = gw - kvh * rows;
  auto slot = [&](int s) { return (static_cast<int64_t>(s) * p.num_kv_heads + kvh) * rows_ws + R; };
  // lane s holds split s's (max, sum); one load per lane instead of a serial walk
  const float2 first = lane < S ? p.ws_ml[slot(lane)] : none;
  float M = first.x;
  for (int base = 32; base < S; base += 32) M = fmaxf(M, base + lane < S ? p.ws_ml[slot(base + lane)].x : -INFINITY);
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) M = fmaxf(M, __shfl_xor_sync(0xFFFFFFFFu, M, o));
  float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
  float lsum = 0.f;
  if (M > -INFINITY) {
    for (int base = 0; base < S; base += 32) {
      const float2 ml = base == 0 ? first : (base + lane < S ? p.ws_ml[slot(base + lane)] : none);
      const float w = ml.x == -INFINITY ? 0.f : ex2(ml.x - M);
      lsum += w * ml.y;
      const int cnt = min(32, S - base);
      for (int j = 0; j < cnt; j += 8) {
        float4 o[8];
        float ww[8];
#pragma unroll
        for (int u = 0; u < 8; ++u) {
          ww[u] = __shfl_sync(0xFFFFFFFFu, w, (j + u) & 31);
          o[u] = make_float4(0.f, 0.f, 0.f, 0.f);
          if (j + u < cnt && ww[u] != 0.f)
            o[u] = *reinterpret_cast<const float4*>(p.ws_o + slot(base + j + u) * kHD + lane * 4);
        }
#pragma unroll
        for (int u = 0; u < 8; ++u) {
          acc.x = fmaf(ww[u], o[u].x, acc.x);
          acc.y = fmaf(ww[u], o[u].y, acc.y);
          acc.z = fmaf(ww[u], o[u].z, acc.z);
          acc.w = fmaf(ww[u], o[u].w, acc.w);
        }
      }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) lsum += __shfl_xor_sync(0xFFFFFFFFu, lsum, o);
  }
  const float inv = lsum > 0.f ? 1.f / lsum : 0.f;
  const int node = R / p.group, h = kvh * p.group + (R - node * p.group);
  uint2 pk;
  pk.x = pack_bf16x2(acc.x * inv, acc.y * inv);
  pk.y = pack_bf16x2(acc.z * inv, acc.w * inv);
  *reinterpret_cast<uint2*>(p.out + node * p.out_tok_stride + h * p.out_head_stride + lane * 8) = pk;
}

// ---------------------------------------------------------------------------
// Host side
// ---------------------------------------------------------------------------
static int make_kv_tmap(CUtensorMap* m, const void* base, int64_t head_stride, int64_t row_stride, int64_t capacity,
                        int heads) {
  EncodeTiledFn fn = encode_fn();
  if (fn == nullptr) return RT_ERR_CUDA;
  const cuuint64_t dims[3] = {static_cast<cuuint64_t>(kHD), static_cast<cuuint64_t>(capacity),
                              static_cast<cuuint64_t>(heads)};
  const cuuint64_t strides[2] = {static_cast<cuuint64_t>(row_stride), static_cast<cuuint64_t>(head_stride)};
  const cuuint32_t box[3] = {64, static_cast<cuuint32_t>(kBN), 1};
  const cuuint32_t estr[3] = {1, 1, 1};
  const CUresult r = fn(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void*>(base), dims, strides, box, estr,
                        CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                        CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? RT_OK : RT_ERR_INVALID_ARGUMENT;
}

// Q viewed as [n tokens][Hq heads][128] (any token / head strides): one box is
// 128/G tokens x G heads x 64 dims, i.e. the 128 tile rows in (node, head) order.
static int make_q_tmap(CUtensorMap* m, const void* q, int64_t tok_stride, int64_t head_stride, int n, int hq,
                       int G) {
  EncodeTiledFn fn = encode_fn();
  if (fn == nullptr) return RT_ERR_CUDA;
  const cuuint64_t dims[3] = {static_cast<cuuint64_t>(kHD), static_cast<cuuint64_t>(hq), static_cast<cuuint64_t>(n)};
  const cuuint64_t strides[2] = {static_cast<cuuint64_t>(head_stride), static_cast<cuuint64_t>(tok_stride)};
  const cuuint32_t box[3] = {64, static_cast<cuuint32_t>(G), static_cast<cuuint32_t>(kBM / G)};
  const cuuint32_t estr[3] = {1, 1, 1};
  const CUresult r = fn(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void*>(q), dims, strides, box, estr,
                        CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                        CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? RT_OK : RT_ERR_INVALID_ARGUMENT;
}

static int tiles_for(int n, int G) { return (n * G + kBM - 1) / kBM; }

static int default_splits(int n, int G, int hkv, int64_t prefix_len, bool tc) {
  const int64_t keys = prefix_len + n;
  const int blk = tc ? kBN : kSimtKeys;
  const int64_t nblk = (keys + blk - 1) / blk;
  const int tiles = tc ? tiles_for(n, G) : 1;
  const int64_t ctas = static_cast<int64_t>(hkv) * tiles;
  // one wave: at most one CTA per SM (the tcgen05 kernel holds a whole SM)
  const int64_t target = std::min<int64_t>(256, std::max<int64_t>(1, 148 / ctas));
  const int64_t per = std::max<int64_t>(1, (nblk + target - 1) / target);    // blocks per split
  return static_cast<int>(std::max<int64_t>(1, (nblk + per - 1) / per));
}

static bool use_tc(int n, int G, int path) { return path == 1 || (path == 0 && n * G >= 64); }

// Clusters of `c` tcgen05-path CTAs (cluster (c, 1, 1)) that fit on the GPU at
// once (0 when the query fails, e.g. without a device); cached per size.
static int clusters_fit(int c) {
  static std::mutex mu;
  static int cache[kMaxMerge + 1] = {};
  static bool done[kMaxMerge + 1] = {};
  std::lock_guard<std::mutex> lock(mu);
  if (c < 2 || c > kMaxMerge) return 0;
  if (done[c]) return cache[c];
  int n = 0;
  if (cudaFuncSetAttribute(tree_attn_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                           static_cast<int>(kAttnSmem)) == cudaSuccess &&
      (c <= 8 || cudaFuncSetAttribute(tree_attn_tc_kernel, cudaFuncAttributeNonPortableClusterSizeAllowed, 1) ==
                     cudaSuccess)) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(c, 1, 1);
    cfg.blockDim = dim3(kAttnThreads);
    cfg.dynamicSmemBytes = kAttnSmem;
    cudaLaunchAttribute attr;
    attr.id = cudaLaunchAttributeClusterDimension;
    attr.val.clusterDim.x = static_cast<unsigned>(c);
    attr.val.clusterDim.y = 1;
    attr.val.clusterDim.z = 1;
    cfg.attrs = &attr;
    cfg.numAttrs = 1;
    if (cudaOccupancyMaxActiveClusters(&n, tree_attn_tc_kernel, &cfg) != cudaSuccess) n = 0;
  }
  cudaGetLastError();
  cache[c] = n;
  done[c] = true;
  return n;
}

// How a launch runs: the path, the key splits, and whether the splits of a
// (kv head, tile) are merged inside the kernel by a cluster of `splits` CTAs
// (tcgen05 path, 2..16 splits, every cluster resident at once) or by the
// combine kernel through the caller's workspace.
struct AttnPlan {
  bool tc;
  int splits;
  bool merge;
};

static AttnPlan plan_attn(int n, int G, int hkv, int64_t prefix_len, int num_splits, int path) {
  AttnPlan pl{use_tc(n, G, path), num_splits, false};
  if (!pl.tc) {
    if (pl.splits <= 0) pl.splits = default_splits(n, G, hkv, prefix_len, false);
    return pl;
  }
  const int pairs = hkv * tiles_for(n, G);
  const int64_t nblk = (prefix_len + n + kBN - 1) / kBN;
  if (num_splits > 0) {
    // a requested split count is merged in the kernel when its clusters fit
    pl.merge = num_splits >= 2 && num_splits <= kMaxMerge && pairs <= clusters_fit(num_splits);
    return pl;
  }
  pl.splits = default_splits(n, G, hkv, prefix_len, true);  // one wave of CTAs
  if (pl.splits < 2) return pl;
  // the largest cluster (<= the one-wave split count) whose clusters all fit at once
  const int want = static_cast<int>(std::min<int64_t>(std::min<int64_t>(kMaxMerge, nblk), pl.splits));
  int c = want;
  while (c >= 2 && pairs > clusters_fit(c)) --c;
  if (c < 2) return pl;
  // Merged in the kernel when the cluster takes every split of the wave, or
  // leaves each CTA at most three key blocks (a latency-bound launch, where the
  // combine launch costs more than the CTAs it would add; measured on B200:
  // 17 blocks merge faster in a 10-CTA cluster than in 17 workspace splits,
  // 33 blocks run equally, 257 blocks twice as fast in workspace splits).
  // (The largest such cluster, not the fewest splits with the same most blocks
  // a CTA takes: a CUDA-graph round plans once for the cache capacity while the
  // live prefix grows, and fewer splits would leave CTAs more blocks of it.)
  if (c == pl.splits || nblk <= 3 * c) {
    pl.splits = c;
    pl.merge = true;
  }
  return pl;
}

}  // namespace rt

using namespace rt;

extern "C" int rt_tree_attn_default_splits(int n, int num_q_heads, int num_kv_heads, int64_t prefix_len) {
  if (n <= 0 || num_kv_heads <= 0 || num_q_heads <= 0 || num_q_heads % num_kv_heads) return 1;
  const int G = num_q_heads / num_kv_heads;
  return plan_attn(n, G, num_kv_heads, prefix_len, 0, 0).splits;
}

extern "C" int rt_tree_attn_plan(int n, int num_q_heads, int num_kv_heads, int64_t prefix_len, int num_splits,
                                 int path, int* splits_out, int* merged_out, int* tcgen05_out) {
  if (n <= 0 || num_kv_heads <= 0 || num_q_heads <= 0 || num_q_heads % num_kv_heads || path < 0 || path > 2)
    return RT_ERR_INVALID_ARGUMENT;
  const AttnPlan pl = plan_attn(n, num_q_heads / num_kv_heads, num_kv_heads, prefix_len, num_splits, path);
  if (splits_out) *splits_out = pl.splits;
  if (merged_out) *merged_out = pl.merge ? 1 : 0;
  if (tcgen05_out) *tcgen05_out = pl.tc ? 1 : 0;
  return RT_OK;
}

// Bytes of workspace a launch of this shape may need, whatever path it takes
// (a launch whose splits merge in the kernel uses none of it).
extern "C" size_t rt_tree_attn_workspace_size(int n, int num_q_heads, int num_kv_heads, int head_dim,
                                              int64_t prefix_len, int num_splits) {
  if (n <= 0 || num_kv_heads <= 0 || num_q_heads <= 0 || num_q_heads % num_kv_heads || head_dim != kHD) return 0;
  const int G = num_q_heads / num_kv_heads;
  if (num_splits <= 0) num_splits = plan_attn(n, G, num_kv_heads, prefix_len, 0, 0).splits;
  if (num_splits <= 1) return 0;
  const size_t rows_ws = static_cast<size_t>(tiles_for(n, G)) * kBM;
  const size_t slots = static_cast<size_t>(num_splits) * num_kv_heads * rows_ws;
  return align_up(slots * kHD * 4, 256) + align_up(slots * 8, 256);
}

extern "C" int rt_tree_attn(const void* q, int64_t q_tok_stride, int64_t q_head_stride, const void* k, const void* v,
                            int64_t kv_head_stride, int64_t kv_row_stride, int64_t kv_capacity, void* out,
                            int64_t out_tok_stride, int64_t out_head_stride, const uint32_t* mask, int mask_words,
                            int n, int64_t prefix_len, const int64_t* prefix_len_dev, int num_q_heads,
                            int num_kv_heads, int head_dim, float scale, int num_splits, int path, void* workspace,
                            size_t workspace_bytes, int* status, rt_stream_t stream) {
  if (!q || !k || !v || !out || !mask) return RT_ERR_INVALID_ARGUMENT;
  if (n <= 0 || num_kv_heads <= 0 || num_q_heads <= 0 || num_q_heads % num_kv_heads || prefix_len < 0)
    return RT_ERR_INVALID_ARGUMENT;
  if (head_dim != kHD) return RT_ERR_UNSUPPORTED;
  if (mask_words < (n + 31) / 32) return RT_ERR_INVALID_ARGUMENT;
  if (prefix_len_dev == nullptr && prefix_len + n > kv_capacity) return RT_ERR_INVALID_ARGUMENT;
  const uint64_t align_bits = reinterpret_cast<uint64_t>(q) | reinterpret_cast<uint64_t>(k) |
                              reinterpret_cast<uint64_t>(v) | reinterpret_cast<uint64_t>(out) |
                              static_cast<uint64_t>(q_tok_stride) | static_cast<uint64_t>(q_head_stride) |
                              static_cast<uint64_t>(kv_head_stride) | static_cast<uint64_t>(kv_row_stride) |
                              static_cast<uint64_t>(out_tok_stride) | static_cast<uint64_t>(out_head_stride);
  if (align_bits & 15) return RT_ERR_INVALID_ARGUMENT;
  if (path < 0 || path > 2) return RT_ERR_INVALID_ARGUMENT;
  const int G = num_q_heads / num_kv_heads;
  const AttnPlan plan = plan_attn(n, G, num_kv_heads, prefix_len, num_splits, path);
  const bool tc = plan.tc;
  if (!tc && n * G > 64) return RT_ERR_UNSUPPORTED;  // warp-level path holds <= 64 rows
  if (kv_capacity > INT32_MAX) return RT_ERR_UNSUPPORTED;
  num_splits = plan.splits;
  AttnParams p{};
  p.q = static_cast<const char*>(q);
  p.q_tok_stride = q_tok_stride;
  p.q_head_stride = q_head_stride;
  p.out = static_cast<char*>(out);
  p.out_tok_stride = out_tok_stride;
  p.out_head_stride = out_head_stride;
  p.mask = mask;
  p.mask_words = mask_words;
  p.n = n;
  p.prefix_len = prefix_len;
  p.prefix_len_dev = prefix_len_dev;
  p.group = G;
  p.num_kv_heads = num_kv_heads;
  p.tiles = tiles_for(n, G);
  p.num_splits = num_splits;
  p.merge = plan.merge ? num_splits : 1;
  p.scale_log2 = scale * 1.4426950408889634f;
  p.status = status;
  p.k = static_cast<const char*>(k);
  p.v = static_cast<const char*>(v);
  p.kv_head_stride = kv_head_stride;
  p.kv_row_stride = kv_row_stride;
  if (num_splits > 1 && !plan.merge) {
    const size_t need = rt_tree_attn_workspace_size(n, num_q_heads, num_kv_heads, head_dim, prefix_len, num_splits);
    if (workspace == nullptr || workspace_bytes < need) return RT_ERR_WORKSPACE;
    const size_t rows_ws = static_cast<size_t>(p.tiles) * kBM;
    const size_t slots = static_cast<size_t>(num_splits) * num_kv_heads * rows_ws;
    p.ws_o = static_cast<float*>(workspace);
    p.ws_ml = reinterpret_cast<float2*>(static_cast<char*>(workspace) + align_up(slots * kHD * 4, 256));
  }
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  if (tc) {
    CUtensorMap tk, tv;
    int rc = make_kv_tmap(&tk, k, kv_head_stride, kv_row_stride, kv_capacity, num_kv_heads);
    if (rc != RT_OK) return rc;
    rc = make_kv_tmap(&tv, v, kv_head_stride, kv_row_stride, kv_capacity, num_kv_heads);
    if (rc != RT_OK) return rc;
    CUtensorMap tq = tk;
    int q_tma = (kBM % G == 0 && q_tok_stride > 0 && q_head_stride > 0) ? 1 : 0;
    if (q_tma && make_q_tmap(&tq, q, q_tok_stride, q_head_stride, n, num_q_heads, G) != RT_OK) {
      tq = tk;
      q_tma = 0;
    }
    set_smem_limit(tree_attn_tc_kernel, kAttnSmem);
    const dim3 grid(num_splits, num_kv_heads, p.tiles);
    rc = record_cuda(launch_ex_cluster(tree_attn_tc_kernel, grid, dim3(kAttnThreads), kAttnSmem, s,
                                       dim3(plan.merge ? num_splits : 1, 1, 1), tk, tv, tq, p, q_tma));
    if (rc != RT_OK) return rc;
    if (plan.merge) return RT_OK;
  } else {
    const dim3 grid(num_splits, num_kv_heads);
    int rc = record_cuda(launch_ex(tree_attn_simt_kernel, grid, dim3(128), 0, s, 1, p));
    if (rc != RT_OK) return rc;
  }
  if (num_splits == 1) return RT_OK;
  // two warps per output row on the combine's fast path (up to kFastSplits splits), one otherwise
  const int warps = num_kv_heads * n * G * (num_splits <= kFastSplits ? 2 : 1);
  return record_cuda(launch_ex(attn_combine_kernel, dim3((warps + 3) / 4), dim3(128), 0, s, 1, p));
}

// ---------------------------------------------------------------------------
// Allocation-free variant: the split partials live in a fixed device array.
//
// Some callers cannot allocate device memory when they call this kernel:
// code that runs while a CUDA stream is being captured into a graph (a
// cudaMalloc there is not allowed), serving runtimes that hand every byte of
// device memory to their own pool up front, and plain C hosts that bind only
// this ABI and have no allocator to carve a workspace from.  For them the
// scratch is a file-scope __device__ array of kNoAllocScratchBytes that every
// GPU loading this library holds until the process exits.
//
// Its device address is looked up once per device (cudaGetSymbolAddress with
// that device current) on the first call on that device, so that first call
// must not be made while a stream is being captured.  The address is kept for
// the life of the process; a device reset (cudaDeviceReset, or a destroyed
// primary context) leaves it stale.  All calls share the one
// array: calls whose launches overlap on the GPU (different streams, or
// different host threads) race on it.  Nothing in it has to start at zero --
// every split writes all of its partial rows (or its neutral -inf/0 row)
// before the merge reads them -- and it keeps the last call's contents.
// ---------------------------------------------------------------------------
namespace rt {
constexpr size_t kNoAllocScratchBytes = size_t(16) << 20;  // 16 MiB
static __device__ __align__(256) unsigned char g_attn_scratch[kNoAllocScratchBytes];

constexpr int kMaxDevices = 64;
static void* g_scratch_ptr[kMaxDevices] = {};
static std::mutex g_scratch_mutex;

static int scratch_for_current_device(void** out) {
  int dev = -1;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return record_cuda(e);
  if (dev < 0 || dev >= kMaxDevices) return RT_ERR_UNSUPPORTED;
  std::lock_guard<std::mutex> lock(g_scratch_mutex);
  if (g_scratch_ptr[dev] == nullptr) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_attn_scratch);  // host code must not use the symbol itself
    if (e != cudaSuccess) return record_cuda(e);
    g_scratch_ptr[dev] = p;
  }
  *out = g_scratch_ptr[dev];
  return RT_OK;
}
}  // namespace rt

extern "C" size_t rt_tree_attn_noalloc_max_bytes(void) { return rt::kNoAllocScratchBytes; }

extern "C" int rt_tree_attn_noalloc(const void* q, int64_t q_tok_stride, int64_t q_head_stride, const void* k,
                                    const void* v, int64_t kv_head_stride, int64_t kv_row_stride,
                                    int64_t kv_capacity, void* out, int64_t out_tok_stride, int64_t out_head_stride,
                                    const uint32_t* mask, int mask_words, int n, int64_t prefix_len,
                                    const int64_t* prefix_len_dev, int num_q_heads, int num_kv_heads, int head_dim,
                                    float scale, int num_splits, int path, int* status, rt_stream_t stream) {
  if (n <= 0 || num_kv_heads <= 0 || num_q_heads <= 0 || num_q_heads % num_kv_heads || head_dim <= 0)
    return RT_ERR_INVALID_ARGUMENT;
  const int G = num_q_heads / num_kv_heads;
  const rt::AttnPlan plan = rt::plan_attn(n, G, num_kv_heads, prefix_len, num_splits, path);
  num_splits = plan.splits;
  const size_t need =
      plan.merge ? 0 : rt_tree_attn_workspace_size(n, num_q_heads, num_kv_heads, head_dim, prefix_len, num_splits);
  if (need > rt::kNoAllocScratchBytes) return RT_ERR_WORKSPACE;  // beyond the fixed scratch: use rt_tree_attn
  void* ws = nullptr;
  if (need > 0) {
    const int rc = rt::scratch_for_current_device(&ws);
    if (rc != RT_OK) return rc;
  }
  return rt_tree_attn(q, q_tok_stride, q_head_stride, k, v, kv_head_stride, kv_row_stride, kv_capacity, out,
                      out_tok_stride, out_head_stride, mask, mask_words, n, prefix_len, prefix_len_dev, num_q_heads,
                      num_kv_heads, head_dim, scale, num_splits, path, ws, need, status, stream);
}
