// Draft-logit top-k and log-normaliser on the device.
//
// Two launches, both HBM/L2-light:
//   1. topk_chunk: each CTA owns a contiguous chunk of one row.  It widens the
//      logits to fp32, turns them into order-preserving uint32 keys in shared
//      memory, accumulates a binary64 (max, sum exp) partial for logsumexp,
//      and radix-selects the chunk's top min(k, chunk) keys (four 8-bit digit
//      passes with shared-memory histograms).  Survivors are written in index
//      order.
//   2. topk_merge: one CTA per row radix-selects the global top k from the
//      concatenated survivors (still in index order, so ties keep resolving to
//      the smallest index), bitonic-sorts them by (value desc, index asc),
//      merges the logsumexp partials and writes logp = fp32(top - log_z).
#include <cuda_fp16.h>

#include <type_traits>

#include "common.cuh"
#include "host_util.h"

namespace rt {

constexpr int kTopkThreads = 256;
constexpr int kMaxCandidates = 24576;  // merge stage shared-memory budget (8 B each)

// Order-preserving key: larger float -> larger key; -0.0 == +0.0; every NaN
// maps above +inf (torch.topk ranks NaN first).
__device__ __forceinline__ uint32_t order_key(float x) {
  uint32_t b = __float_as_uint(x);
  if (x != x) return 0xFFFFFFFFu;
  if (b == 0x80000000u) b = 0u;
  return (b & 0x80000000u) ? ~b : (b | 0x80000000u);
}
__device__ __forceinline__ float key_value(uint32_t k) {
  if (k == 0xFFFFFFFFu) return __uint_as_float(0x7FC00000u);
  const uint32_t b = (k & 0x80000000u) ? (k & 0x7FFFFFFFu) : ~k;
  return __uint_as_float(b);
}

// 8-bit digit passes that decide a key widened from T (its significant leading bits).
template <typename T>
__host__ __device__ constexpr int key_passes() {
  return sizeof(T) == 4 ? 4 : (std::is_same<T, __half>::value ? 3 : 2);
}

template <typename T>
__device__ __forceinline__ float load_logit(const T* p);
template <>
__device__ __forceinline__ float load_logit<float>(const float* p) { return *p; }
template <>
__device__ __forceinline__ float load_logit<__nv_bfloat16>(const __nv_bfloat16* p) { return __bfloat162float(*p); }
template <>
__device__ __forceinline__ float load_logit<__half>(const __half* p) { return __half2float(*p); }

// Block-wide exclusive scan of one int per thread (kTopkThreads threads).
__device__ __forceinline__ int block_exclusive_scan(int v, int* warp_tot, int* total) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  int x = v;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int y = __shfl_up_sync(0xFFFFFFFFu, x, o);
    if (lane >= o) x += y;
  }
  if (lane == 31) warp_tot[warp] = x;
  __syncthreads();
  if (warp == 0) {
    int t = lane < kTopkThreads / 32 ? warp_tot[lane] : 0;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int y = __shfl_up_sync(0xFFFFFFFFu, t, o);
      if (lane >= o) t += y;
    }
    if (lane < kTopkThreads / 32) warp_tot[lane] = t;  // inclusive
    if (lane == kTopkThreads / 32 - 1) *total = t;
  }
  __syncthreads();
  const int before = warp == 0 ? 0 : warp_tot[warp - 1];
  const int r = before + x - v;
  __syncthreads();
  return r;
}

struct SelectShared {
  uint32_t hist[256];
  int warp_tot[kTopkThreads / 32];
  int total;
  uint32_t prefix;
  int need;
};

// Select the `k` largest of keys[0..len) (ties -> smaller position first) and
// write them, in position order, to out_key/out_idx (idx = idx_base + position,
// or idx_in[position] when idx_in is non-null).  `passes` 8-bit digits decide
// (4 for fp32 logits; keys widened from bf16 / fp16 carry only their top 16 /
// 24 bits, the rest being all zeros for positive and all ones for negative
// values, so 2 / 3 digit passes find the k-th key).
__device__ void block_select(const uint32_t* keys, const int* idx_in, int idx_base, int len, int k,
                             uint32_t* out_key, int* out_idx, SelectShared& sh, int passes) {
  const int tid = threadIdx.x;
  if (tid == 0) {
    sh.prefix = 0;
    sh.need = k;
  }
  uint32_t himask = 0;
  const int last_shift = 32 - 8 * passes;
  for (int shift = 24; shift >= last_shift; shift -= 8) {
    sh.hist[tid] = 0;  // kTopkThreads == 256 bins
    __syncthreads();
    const uint32_t prefix = sh.prefix;
    // Warp-aggregated counting: logits share their leading key bytes (sign and
    // exponent), so most live keys of a pass land in a handful of bins; one
    // atomic per distinct bin per warp instead of one per key.
    for (int base = 0; base < len; base += kTopkThreads) {  // same trip count on every lane
      const int i = base + tid;
      uint32_t bin = 256u;  // no bin
      if (i < len) {
        const uint32_t key = keys[i];
        if (((key ^ prefix) & himask) == 0) bin = (key >> shift) & 255u;
      }
      const uint32_t peers = __match_any_sync(0xFFFFFFFFu, bin);
      if (bin < 256u && (tid & 31) == __ffs(peers) - 1) atomicAdd(&sh.hist[bin], static_cast<uint32_t>(__popc(peers)));
    }
    __syncthreads();
    if (tid < 32) {
      // lane l owns bins 255-8l .. 248-8l (highest first)
      uint32_t c[8];
      uint32_t s = 0;
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        c[j] = sh.hist[255 - (tid * 8 + j)];
        s += c[j];
      }
      uint32_t incl = s;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const uint32_t y = __shfl_up_sync(0xFFFFFFFFu, incl, o);
        if (tid >= o) incl += y;
      }
      uint32_t p = incl - s;
      const uint32_t need = static_cast<uint32_t>(sh.need);
      if (p < need && need <= incl) {
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          if (p + c[j] >= need) {
            sh.prefix = prefix | (static_cast<uint32_t>(255 - (tid * 8 + j)) << shift);
            sh.need = static_cast<int>(need - p);
            break;
          }
          p += c[j];
        }
      }
    }
    himask |= 0xFFu << shift;
    __syncthreads();
  }
  // the k-th key: the selected digits, and below them the fill of its sign
  const uint32_t low = last_shift > 0 ? (1u << last_shift) - 1u : 0u;
  const uint32_t T = sh.prefix | ((sh.prefix & 0x80000000u) ? 0u : low);
  const int eq_take = sh.need;
  // Stable compaction over contiguous per-thread ranges (position order).
  const int per = (len + kTopkThreads - 1) / kTopkThreads;
  const int lo = min(len, tid * per), hi = min(len, lo + per);
  int gt = 0, eq = 0;
  for (int i = lo; i < hi; ++i) {
    const uint32_t key = keys[i];
    gt += key > T;
    eq += key == T;
  }
  const int gt_before = block_exclusive_scan(gt, sh.warp_tot, &sh.total);
  const int eq_before = block_exclusive_scan(eq, sh.warp_tot, &sh.total);
  int slot = gt_before + min(eq_before, eq_take);
  int eq_rank = eq_before;
  for (int i = lo; i < hi; ++i) {
    const uint32_t key = keys[i];
    bool take = key > T;
    if (key == T) {
      take = eq_rank < eq_take;
      ++eq_rank;
    }
    if (take) {
      out_key[slot] = key;
      out_idx[slot] = idx_in != nullptr ? idx_in[i] : idx_base + i;
      ++slot;
    }
  }
  __syncthreads();
}

template <typename T>
__global__ void __launch_bounds__(kTopkThreads) topk_chunk_kernel(const T* __restrict__ logits, int64_t ld,
                                                                  int vocab, int k, int chunk_len, int n_chunks,
                                                                  uint32_t* __restrict__ cand_key,
                                                                  int* __restrict__ cand_idx,
                                                                  double2* __restrict__ lse_part) {
  extern __shared__ __align__(16) unsigned char smem_raw[];
  uint32_t* keys = reinterpret_cast<uint32_t*>(smem_raw);
  __shared__ SelectShared sh;
  __shared__ float red_f[kTopkThreads / 32];
  __shared__ double red_d[kTopkThreads / 32];
  __shared__ int red_nan;
  const int chunk = blockIdx.x, row = blockIdx.y, tid = threadIdx.x;
  const int c0 = chunk * chunk_len;
  const int len = min(chunk_len, vocab - c0);
  const T* src = logits + row * ld + c0;
  if (tid == 0) red_nan = 0;
  __syncthreads();
  float m = -INFINITY;
  bool nan = false;
  for (int i = tid; i < len; i += kTopkThreads) {
    const float x = load_logit<T>(src + i);
    keys[i] = order_key(x);
    nan |= (x != x);
    m = fmaxf(m, x);
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xFFFFFFFFu, m, o));
  if ((tid & 31) == 0) red_f[tid >> 5] = m;
  if (nan) red_nan = 1;
  __syncthreads();
  m = red_f[0];
#pragma unroll
  for (int w = 1; w < kTopkThreads / 32; ++w) m = fmaxf(m, red_f[w]);
  // sum of exp(x - m): each term in fp32 (expf, within 2 ulp; x - m is exact
  // whenever x is within a factor of two of m, which covers every term that
  // carries weight), summed in binary64, so the rounded log_z stays within an
  // ulp of the all-binary64 one
  double s = 0.0;
  if (m > -INFINITY && m < INFINITY) {
    float f[4] = {0.f, 0.f, 0.f, 0.f};
    double d = 0.0;
    int c = 0;
    for (int i = tid; i < len; i += kTopkThreads, ++c) {
      f[c & 3] = expf(key_value(keys[i]) - m);
      if ((c & 3) == 3) {
        d += static_cast<double>(f[0]) + static_cast<double>(f[1]) + static_cast<double>(f[2]) +
             static_cast<double>(f[3]);
        f[0] = f[1] = f[2] = f[3] = 0.f;
      }
    }
    s = d + (static_cast<double>(f[0]) + static_cast<double>(f[1]) + static_cast<double>(f[2]) +
             static_cast<double>(f[3]));
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xFFFFFFFFu, s, o);
  if ((tid & 31) == 0) red_d[tid >> 5] = s;
  __syncthreads();
  if (tid == 0) {
    double t = 0.0;
    for (int w = 0; w < kTopkThreads / 32; ++w) t += red_d[w];
    lse_part[row * n_chunks + chunk] = make_double2(red_nan ? static_cast<double>(NAN) : static_cast<double>(m), t);
  }
  const int kk = min(k, len);
  const int64_t base = (static_cast<int64_t>(row) * n_chunks + chunk) * k;
  block_select(keys, nullptr, c0, len, kk, cand_key + base, cand_idx + base, sh, key_passes<T>());
}

__global__ void __launch_bounds__(kTopkThreads) topk_merge_kernel(int vocab, int k, int chunk_len, int n_chunks,
                                                                  int passes,
                                                                  const uint32_t* __restrict__ cand_key,
                                                                  const int* __restrict__ cand_idx,
                                                                  const double2* __restrict__ lse_part,
                                                                  float* __restrict__ top_logp,
                                                                  int64_t* __restrict__ top_ids,
                                                                  float* __restrict__ log_z_out, int sort_len) {
  extern __shared__ __align__(16) unsigned char smem_raw[];
  __shared__ SelectShared sh;
  __shared__ float log_z_sh;
  const int row = blockIdx.x, tid = threadIdx.x;
  // layout: keys[total] | idx[total] | sorted u64[sort_len]
  int total = 0;
  for (int c = 0; c < n_chunks; ++c) total += min(k, min(chunk_len, vocab - c * chunk_len));
  uint32_t* keys = reinterpret_cast<uint32_t*>(smem_raw);
  int* idx = reinterpret_cast<int*>(keys + total);
  unsigned long long* srt = reinterpret_cast<unsigned long long*>(
      smem_raw + ((static_cast<size_t>(total) * 8 + 15) & ~static_cast<size_t>(15)));
  // every chunk but the last contributed exactly k survivors, in chunk order
  for (int j = tid; j < total; j += kTopkThreads) {
    const int c = j / k, i = j - c * k;
    const int64_t base = (static_cast<int64_t>(row) * n_chunks + c) * k;
    keys[j] = cand_key[base + i];
    idx[j] = cand_idx[base + i];
  }
  if (tid < 32) {
    // logsumexp of the chunk partials (binary64), one warp
    double M = -INFINITY;
    bool nan = false;
    for (int c = tid; c < n_chunks; c += 32) {
      const double mc = lse_part[row * n_chunks + c].x;
      if (mc != mc) nan = true;
      else M = fmax(M, mc);
    }
    nan = __any_sync(0xFFFFFFFFu, nan);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) M = fmax(M, __shfl_xor_sync(0xFFFFFFFFu, M, o));
    double S = 0.0;
    if (!nan && M > -INFINITY && M < INFINITY) {
      for (int c = tid; c < n_chunks; c += 32) {
        const double2 pc = lse_part[row * n_chunks + c];
        if (pc.x > -INFINITY) S += pc.y * exp(pc.x - M);
      }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) S += __shfl_xor_sync(0xFFFFFFFFu, S, o);
    if (tid == 0) {
      const double lz = nan ? static_cast<double>(NAN) : ((M == INFINITY || M == -INFINITY) ? M : M + log(S));
      log_z_sh = static_cast<float>(lz);
    }
  }
  __syncthreads();
  // select the row's top k (in index order), staging them in the sort buffer
  uint32_t* sel_key = reinterpret_cast<uint32_t*>(srt);  // reuse: packed below
  int* sel_idx = reinterpret_cast<int*>(sel_key + sort_len);
  block_select(keys, idx, 0, total, k, sel_key, sel_idx, sh, passes);
  // pack (key desc, index asc) into 64-bit keys, pad to the power-of-two length
  // (sort_len <= 1024: at most 4 per thread; threads past a short length idle)
  unsigned long long packed[4];
  const int per = sort_len / kTopkThreads > 0 ? sort_len / kTopkThreads : 1;
  for (int j = 0; j < per; ++j) {
    const int i = tid * per + j;
    packed[j] = (i < k && i < sort_len)
                    ? ((static_cast<unsigned long long>(sel_key[i]) << 32) |
                       static_cast<unsigned long long>(0xFFFFFFFFu - static_cast<uint32_t>(sel_idx[i])))
                    : 0ull;
  }
  __syncthreads();
  for (int j = 0; j < per; ++j) {
    const int i = tid * per + j;
    if (i < sort_len) srt[i] = packed[j];
  }
  __syncthreads();
  // bitonic sort, descending
  for (int size = 2; size <= sort_len; size <<= 1) {
    for (int stride = size >> 1; stride > 0; stride >>= 1) {
      for (int i = tid; i < sort_len; i += kTopkThreads) {
        const int j = i ^ stride;
        if (j > i) {
          const bool desc = (i & size) == 0;
          const unsigned long long a = srt[i], b = srt[j];
          if (desc ? (a < b) : (a > b)) {
            srt[i] = b;
            srt[j] = a;
          }
        }
      }
      __syncthreads();
    }
  }
  const float lz = log_z_sh;
  for (int i = tid; i < k; i += kTopkThreads) {
    const unsigned long long p = srt[i];
    const float v = key_value(static_cast<uint32_t>(p >> 32));
    const uint32_t id = 0xFFFFFFFFu - static_cast<uint32_t>(p & 0xFFFFFFFFull);
    top_logp[static_cast<int64_t>(row) * k + i] = __fsub_rn(v, lz);
    top_ids[static_cast<int64_t>(row) * k + i] = static_cast<int64_t>(id);
  }
  if (tid == 0 && log_z_out != nullptr) log_z_out[row] = lz;
}

struct TopkPlan {
  int chunk_len, n_chunks, total, sort_len;
  size_t ws_key, ws_idx, ws_lse, ws_total, smem1, smem2;
};

static TopkPlan topk_plan(int rows, int vocab, int k) {
  TopkPlan p{};
  const int max_chunks = std::max(1, kMaxCandidates / k);
  int cl = std::max(4096, (vocab + max_chunks - 1) / max_chunks);
  cl = std::max(cl, k);
  cl = (cl + 255) / 256 * 256;
  p.chunk_len = cl;
  p.n_chunks = (vocab + cl - 1) / cl;
  p.total = 0;
  for (int c = 0; c < p.n_chunks; ++c) p.total += std::min(k, std::min(cl, vocab - c * cl));
  p.sort_len = 1;
  while (p.sort_len < k) p.sort_len <<= 1;
  p.sort_len = std::max(p.sort_len, 32);  // a k-element bitonic network, not a 256-element one
  const size_t cand = static_cast<size_t>(rows) * p.n_chunks * k;
  p.ws_key = 0;
  p.ws_idx = align_up(cand * 4, 256);
  p.ws_lse = p.ws_idx + align_up(cand * 4, 256);
  p.ws_total = p.ws_lse + align_up(static_cast<size_t>(rows) * p.n_chunks * 16, 256);
  p.smem1 = static_cast<size_t>(cl) * 4;
  p.smem2 = align_up(static_cast<size_t>(p.total) * 8, 16) + static_cast<size_t>(p.sort_len) * 8;
  return p;
}

}  // namespace rt

using namespace rt;

extern "C" size_t rt_draft_topk_workspace_size(int rows, int vocab, int k) {
  if (rows <= 0 || vocab <= 0 || k <= 0 || k > vocab || k > 1024) return 0;
  return topk_plan(rows, vocab, k).ws_total;
}

extern "C" int rt_draft_topk(const void* logits, int dtype, int64_t ld, int rows, int vocab, int k, float* top_logp,
                             int64_t* top_ids, float* log_z, void* workspace, size_t workspace_bytes,
                             rt_stream_t stream) {
  if (rows < 0 || vocab <= 0 || k <= 0 || ld < vocab) return RT_ERR_INVALID_ARGUMENT;
  if (k > vocab || k > 1024) return RT_ERR_UNSUPPORTED;
  if (rows == 0) return RT_OK;
  if (!logits || !top_logp || !top_ids) return RT_ERR_INVALID_ARGUMENT;
  const TopkPlan p = topk_plan(rows, vocab, k);
  if (workspace == nullptr || workspace_bytes < p.ws_total) return RT_ERR_WORKSPACE;
  if (p.smem2 > 220 * 1024 || p.smem1 > 220 * 1024) return RT_ERR_UNSUPPORTED;
  char* ws = static_cast<char*>(workspace);
  uint32_t* ck = reinterpret_cast<uint32_t*>(ws + p.ws_key);
  int* ci = reinterpret_cast<int*>(ws + p.ws_idx);
  double2* lse = reinterpret_cast<double2*>(ws + p.ws_lse);
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  const dim3 g1(p.n_chunks, rows);
  switch (dtype) {
    case 0:
      set_smem_limit(topk_chunk_kernel<float>, p.smem1);
      topk_chunk_kernel<float><<<g1, kTopkThreads, p.smem1, s>>>(static_cast<const float*>(logits), ld, vocab, k,
                                                                 p.chunk_len, p.n_chunks, ck, ci, lse);
      break;
    case 1:
      set_smem_limit(topk_chunk_kernel<__nv_bfloat16>, p.smem1);
      topk_chunk_kernel<__nv_bfloat16><<<g1, kTopkThreads, p.smem1, s>>>(
          static_cast<const __nv_bfloat16*>(logits), ld, vocab, k, p.chunk_len, p.n_chunks, ck, ci, lse);
      break;
    case 2:
      set_smem_limit(topk_chunk_kernel<__half>, p.smem1);
      topk_chunk_kernel<__half><<<g1, kTopkThreads, p.smem1, s>>>(static_cast<const __half*>(logits), ld, vocab,
                                                                  k, p.chunk_len, p.n_chunks, ck, ci, lse);
      break;
    default:
      return RT_ERR_INVALID_ARGUMENT;
  }
  int rc = check_launch();
  if (rc != RT_OK) return rc;
  set_smem_limit(topk_merge_kernel, p.smem2);
  const int passes = dtype == 0 ? key_passes<float>() : dtype == 1 ? key_passes<__nv_bfloat16>() : key_passes<__half>();
  topk_merge_kernel<<<rows, kTopkThreads, p.smem2, s>>>(vocab, k, p.chunk_len, p.n_chunks, passes, ck, ci, lse,
                                                        top_logp, top_ids, log_z, p.sort_len);
  return check_launch();
}
