// Draft-logit top-k and log-normaliser on the device (ddtree.py:361-370).
//
// Two launches:
//   1. topk_chunk_kernel: the rows are cut into chunks so that the chunk CTAs
//      form one wave where the shapes allow.  A CTA (512 threads) loads its
//      chunk with coalesced 16-byte loads (scalar ones where the row is not
//      16-byte aligned), widens the logits to fp32 and keeps them as
//      order-preserving uint32 keys in shared memory, reduces the chunk's
//      (max, binary64 sum of fp32 expf(x - max)) partial for logsumexp, and
//      selects the chunk's top min(k, len): a radix select over 12-bit digits
//      (key bits 31-20, 19-8, 7-0; two digits decide keys widened from bf16 or
//      fp16, whose lower bits are fixed by the sign) with one shared-memory
//      histogram of 4096 bins per digit and plain shared-memory atomics, then a
//      compaction in index order (each warp a contiguous segment, ballots for
//      the output slots).
//   2. topk_merge_kernel: one CTA per row selects the row's top k from the
//      chunks' survivors (concatenated in chunk order, hence in index order, so
//      equal values still resolve to the smaller index) with the same select,
//      ranks the k survivors by counting -- (value desc, index asc) gives each
//      its output position, no sorting network -- merges the logsumexp
//      partials and writes logp = fp32(top - log_z).
#include <cuda_fp16.h>

#include <algorithm>
#include <cstring>
#include <type_traits>

#include "common.cuh"
#include "host_util.h"

namespace rt {

constexpr int kTkThreads = 512;
constexpr int kTkWarps = kTkThreads / 32;
constexpr int kBins = 4096;            // one 12-bit digit
constexpr int kMaxCandidates = 16384;  // survivors a row's merge holds in shared memory (8 B each)
constexpr int kMaxChunk = 32768;       // keys a chunk CTA holds in shared memory (4 B each)
constexpr int kWave = 148;             // CTAs of one wave (one per SM)

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

// 12-bit digit passes that decide a key widened from T: bf16 and fp16 keep
// their significant bits in key bits 31-8, fp32 needs all 32.
template <typename T>
__host__ __device__ constexpr int key_passes() {
  return sizeof(T) == 4 ? 3 : 2;
}

template <typename T>
__device__ __forceinline__ float to_float(T x);
template <>
__device__ __forceinline__ float to_float<float>(float x) { return x; }
template <>
__device__ __forceinline__ float to_float<__nv_bfloat16>(__nv_bfloat16 x) { return __bfloat162float(x); }
template <>
__device__ __forceinline__ float to_float<__half>(__half x) { return __half2float(x); }

struct SelectShared {
  uint32_t hist[kBins];
  int warp_tot[kTkWarps];
  uint32_t prefix;
  int need;
};

// Exclusive scan of one int per thread over the block; every thread calls it.
__device__ __forceinline__ int block_scan_excl(int v, int* warp_tot) {
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
    int t = lane < kTkWarps ? warp_tot[lane] : 0;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int y = __shfl_up_sync(0xFFFFFFFFu, t, o);
      if (lane >= o) t += y;
    }
    if (lane < kTkWarps) warp_tot[lane] = t;  // inclusive
  }
  __syncthreads();
  const int before = (warp == 0 ? 0 : warp_tot[warp - 1]) + x - v;
  __syncthreads();
  return before;
}

// The kk-th largest of keys[0, len) (1 <= kk <= len) and, in *eq_take, how
// many keys equal to it belong to the top kk.  Every thread of the block calls it.
__device__ uint32_t select_kth(const uint32_t* keys, int len, int kk, int passes, SelectShared& sh, int* eq_take) {
  const int tid = threadIdx.x;
  if (tid == 0) {
    sh.prefix = 0;
    sh.need = kk;
  }
  uint32_t himask = 0;
  for (int pass = 0; pass < passes; ++pass) {
    const int shift = pass == 0 ? 20 : (pass == 1 ? 8 : 0);
    const int nbins = pass < 2 ? kBins : 256;
    const uint32_t mask = static_cast<uint32_t>(nbins - 1);
    for (int b = tid; b < nbins; b += kTkThreads) sh.hist[b] = 0u;
    __syncthreads();
    const uint32_t prefix = sh.prefix;
    const int need = sh.need;
    for (int i = tid; i < len; i += kTkThreads) {
      const uint32_t key = keys[i];
      if (((key ^ prefix) & himask) == 0) atomicAdd(&sh.hist[(key >> shift) & mask], 1u);
    }
    __syncthreads();
    // thread t owns the bins nbins-1-8t .. nbins-8-8t (largest digit first)
    int c[8];
    int s = 0;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const int bin = nbins - 1 - (tid * 8 + j);
      c[j] = bin >= 0 ? static_cast<int>(sh.hist[bin]) : 0;
      s += c[j];
    }
    int p = block_scan_excl(s, sh.warp_tot);
    if (p < need && need <= p + s) {  // exactly one thread: the bin of the need-th key
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        if (p + c[j] >= need) {
          sh.prefix = prefix | (static_cast<uint32_t>(nbins - 1 - (tid * 8 + j)) << shift);
          sh.need = need - p;
          break;
        }
        p += c[j];
      }
    }
    himask |= mask << shift;
    __syncthreads();
  }
  // below the decided digits a key's bits are fixed by its sign; a key whose
  // decided bits are all ones is a NaN (its key is all ones)
  const uint32_t low = passes >= 3 ? 0u : 0xFFu;
  const uint32_t pre = sh.prefix;
  const uint32_t kth = (pre | low) == 0xFFFFFFFFu ? 0xFFFFFFFFu : (pre | ((pre & 0x80000000u) ? 0u : low));
  *eq_take = sh.need;
  __syncthreads();
  return kth;
}

// Writes the top kk of keys[0, len) -- the keys above kth and the first
// eq_take equal to it -- in index order to out_key / out_idx (index
// idx_in[i] when idx_in is given, else idx_base + i).  Each warp takes a
// contiguous segment; a first pass counts, a second places by ballots.
__device__ void compact_top(const uint32_t* keys, const int* idx_in, int idx_base, int len, int kk, uint32_t kth,
                            int eq_take, uint32_t* out_key, int* out_idx, SelectShared& sh) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const uint32_t below = (1u << lane) - 1u;
  const int seg = (((len + kTkWarps - 1) / kTkWarps) + 31) & ~31;
  const int lo = min(len, warp * seg), hi = min(len, lo + seg);
  int gt = 0, eq = 0;
  for (int base = lo; base < hi; base += 32) {
    const int i = base + lane;
    const uint32_t key = i < hi ? keys[i] : 0u;
    gt += __popc(__ballot_sync(0xFFFFFFFFu, i < hi && key > kth));
    eq += __popc(__ballot_sync(0xFFFFFFFFu, i < hi && key == kth));
  }
  if (lane == 0) sh.warp_tot[warp] = (gt << 16) | eq;  // both below 2^15
  __syncthreads();
  int gt_before = 0, eq_before = 0;
  for (int w = 0; w < warp; ++w) {
    gt_before += sh.warp_tot[w] >> 16;
    eq_before += sh.warp_tot[w] & 0xFFFF;
  }
  int taken = gt_before + min(eq_before, eq_take);
  int eq_seen = eq_before;
  for (int base = lo; base < hi; base += 32) {
    const int i = base + lane;
    const uint32_t key = i < hi ? keys[i] : 0u;
    const bool g = i < hi && key > kth, e = i < hi && key == kth;
    const uint32_t eb = __ballot_sync(0xFFFFFFFFu, e);
    const bool take = g || (e && eq_seen + __popc(eb & below) < eq_take);
    const uint32_t tb = __ballot_sync(0xFFFFFFFFu, take);
    const int slot = taken + __popc(tb & below);
    if (take && slot < kk) {  // slot < kk always holds; the check keeps every write in bounds
      out_key[slot] = key;
      out_idx[slot] = idx_in != nullptr ? idx_in[i] : idx_base + i;
    }
    taken += __popc(tb);
    eq_seen += __popc(eb);
  }
  __syncthreads();
}

template <typename T>
__global__ void __launch_bounds__(kTkThreads) topk_chunk_kernel(const T* __restrict__ logits, int64_t ld,
                                                                int vocab, int k, int chunk_len, int n_chunks,
                                                                uint32_t* __restrict__ cand_key,
                                                                int* __restrict__ cand_idx,
                                                                double2* __restrict__ lse_part) {
  extern __shared__ __align__(16) unsigned char smem_raw[];
  uint32_t* keys = reinterpret_cast<uint32_t*>(smem_raw);
  __shared__ SelectShared sh;
  __shared__ float red_f[kTkWarps];
  __shared__ double red_d[kTkWarps];
  const int chunk = blockIdx.x, row = blockIdx.y, tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int c0 = chunk * chunk_len;
  const int len = min(chunk_len, vocab - c0);
  const T* src = logits + row * ld + c0;

  // ---- keys, chunk max, NaN flag ----
  float m = -INFINITY;
  bool nan = false;
  constexpr int V = 16 / static_cast<int>(sizeof(T));  // elements per 16-byte load
  int done = 0;
  if ((reinterpret_cast<uintptr_t>(src) & 15u) == 0) {
    const int nv = len / V;
    const uint4* src4 = reinterpret_cast<const uint4*>(src);
    for (int v = tid; v < nv; v += kTkThreads) {
      const uint4 raw = __ldg(src4 + v);
      T e[V];
      memcpy(e, &raw, 16);
      uint32_t kv[V];
#pragma unroll
      for (int j = 0; j < V; ++j) {
        const float x = to_float<T>(e[j]);
        kv[j] = order_key(x);
        nan |= (x != x);
        m = fmaxf(m, x);
      }
#pragma unroll
      for (int j = 0; j < V; j += 4)
        *reinterpret_cast<uint4*>(keys + v * V + j) = make_uint4(kv[j], kv[j + 1], kv[j + 2], kv[j + 3]);
    }
    done = nv * V;
  }
  for (int i = done + tid; i < len; i += kTkThreads) {
    const float x = to_float<T>(src[i]);
    keys[i] = order_key(x);
    nan |= (x != x);
    m = fmaxf(m, x);
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xFFFFFFFFu, m, o));
  if (lane == 0) red_f[warp] = m;
  nan = __syncthreads_or(nan) != 0;
  m = red_f[0];
#pragma unroll
  for (int w = 1; w < kTkWarps; ++w) m = fmaxf(m, red_f[w]);

  // ---- sum of exp(x - m): each term in fp32 (expf, within 2 ulp; x - m is
  // exact whenever x is within a factor of two of m, which covers every term
  // that carries weight), summed in binary64, so the rounded log_z stays
  // within an ulp of the all-binary64 one ----
  double s = 0.0;
  if (m > -INFINITY && m < INFINITY) {
    float f[4] = {0.f, 0.f, 0.f, 0.f};
    double d = 0.0;
    int c = 0;
    for (int i = tid; i < len; i += kTkThreads, ++c) {
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
  if (lane == 0) red_d[warp] = s;
  __syncthreads();
  if (tid == 0) {
    double t = 0.0;
    for (int w = 0; w < kTkWarps; ++w) t += red_d[w];
    lse_part[row * n_chunks + chunk] = make_double2(nan ? static_cast<double>(NAN) : static_cast<double>(m), t);
  }

  // ---- the chunk's top min(k, len), in index order ----
  const int kk = min(k, len);
  int eq_take;
  const uint32_t kth = select_kth(keys, len, kk, key_passes<T>(), sh, &eq_take);
  const int64_t base = (static_cast<int64_t>(row) * n_chunks + chunk) * k;
  compact_top(keys, nullptr, c0, len, kk, kth, eq_take, cand_key + base, cand_idx + base, sh);
}

__global__ void __launch_bounds__(kTkThreads) topk_merge_kernel(int vocab, int k, int chunk_len, int n_chunks,
                                                                int passes,
                                                                const uint32_t* __restrict__ cand_key,
                                                                const int* __restrict__ cand_idx,
                                                                const double2* __restrict__ lse_part,
                                                                float* __restrict__ top_logp,
                                                                int64_t* __restrict__ top_ids,
                                                                float* __restrict__ log_z_out) {
  extern __shared__ __align__(16) unsigned char smem_raw[];
  __shared__ SelectShared sh;
  __shared__ float log_z_sh;
  const int row = blockIdx.x, tid = threadIdx.x;
  // layout: keys[total] | idx[total] | sel_key[k] | sel_idx[k]
  int total = 0;
  for (int c = 0; c < n_chunks; ++c) total += min(k, min(chunk_len, vocab - c * chunk_len));
  uint32_t* keys = reinterpret_cast<uint32_t*>(smem_raw);
  int* idx = reinterpret_cast<int*>(keys + total);
  uint32_t* sel_key = reinterpret_cast<uint32_t*>(idx + total);
  int* sel_idx = reinterpret_cast<int*>(sel_key + k);
  // every chunk but the last contributed exactly k survivors, in chunk order
  for (int j = tid; j < total; j += kTkThreads) {
    const int c = j / k, i = j - c * k;
    const int64_t g = (static_cast<int64_t>(row) * n_chunks + c) * k + i;
    keys[j] = cand_key[g];
    idx[j] = cand_idx[g];
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
  int eq_take;
  const uint32_t kth = select_kth(keys, total, k, passes, sh, &eq_take);
  compact_top(keys, idx, 0, total, k, kth, eq_take, sel_key, sel_idx, sh);
  // output position of survivor i = survivors before it in (key desc, index
  // asc) order; the survivors are in index order, so an equal key ranks
  // before i exactly when it sits before i
  const float lz = log_z_sh;
  for (int i = tid; i < k; i += kTkThreads) {
    const uint32_t ki = sel_key[i];
    int r = 0;
    for (int j = 0; j < k; ++j) {
      const uint32_t kj = sel_key[j];
      r += (kj > ki || (kj == ki && j < i)) ? 1 : 0;
    }
    top_logp[static_cast<int64_t>(row) * k + r] = __fsub_rn(key_value(ki), lz);
    top_ids[static_cast<int64_t>(row) * k + r] = static_cast<int64_t>(sel_idx[i]);
  }
  if (tid == 0 && log_z_out != nullptr) log_z_out[row] = lz;
}

struct TopkPlan {
  int chunk_len, n_chunks, total;
  size_t ws_key, ws_idx, ws_lse, ws_total, smem1, smem2;
};

// Chunks: one wave of CTAs over all rows where the survivor budget of the
// merge and the chunk size allow; chunks hold whole 512-key strides (so
// every chunk start keeps the row's 16-byte alignment) and at least k keys.
static int topk_plan(int rows, int vocab, int k, TopkPlan* p) {
  int n_chunks = std::max(1, std::min(kWave / std::max(rows, 1), kMaxCandidates / k));
  n_chunks = std::max(n_chunks, (vocab + kMaxChunk - 1) / kMaxChunk);
  int cl = (vocab + n_chunks - 1) / n_chunks;
  cl = std::max(cl, k);
  cl = (cl + kTkThreads - 1) / kTkThreads * kTkThreads;
  p->chunk_len = cl;
  p->n_chunks = (vocab + cl - 1) / cl;
  p->total = 0;
  for (int c = 0; c < p->n_chunks; ++c) p->total += std::min(k, std::min(cl, vocab - c * cl));
  if (cl > kMaxChunk || p->total > kMaxCandidates) return RT_ERR_UNSUPPORTED;
  const size_t cand = static_cast<size_t>(rows) * p->n_chunks * k;
  p->ws_key = 0;
  p->ws_idx = align_up(cand * 4, 256);
  p->ws_lse = p->ws_idx + align_up(cand * 4, 256);
  p->ws_total = p->ws_lse + align_up(static_cast<size_t>(rows) * p->n_chunks * 16, 256);
  p->smem1 = static_cast<size_t>(cl) * 4;
  p->smem2 = static_cast<size_t>(p->total) * 8 + static_cast<size_t>(k) * 8;
  return RT_OK;
}

}  // namespace rt

using namespace rt;

extern "C" size_t rt_draft_topk_workspace_size(int rows, int vocab, int k) {
  if (rows <= 0 || vocab <= 0 || k <= 0 || k > vocab || k > 1024) return 0;
  TopkPlan p;
  if (topk_plan(rows, vocab, k, &p) != RT_OK) return 0;
  return p.ws_total;
}

extern "C" int rt_draft_topk(const void* logits, int dtype, int64_t ld, int rows, int vocab, int k, float* top_logp,
                             int64_t* top_ids, float* log_z, void* workspace, size_t workspace_bytes,
                             rt_stream_t stream) {
  if (rows < 0 || vocab <= 0 || k <= 0 || ld < vocab) return RT_ERR_INVALID_ARGUMENT;
  if (k > vocab || k > 1024) return RT_ERR_UNSUPPORTED;
  if (rows == 0) return RT_OK;
  if (!logits || !top_logp || !top_ids) return RT_ERR_INVALID_ARGUMENT;
  if (dtype < 0 || dtype > 2) return RT_ERR_INVALID_ARGUMENT;
  TopkPlan p;
  const int prc = topk_plan(rows, vocab, k, &p);
  if (prc != RT_OK) return prc;
  if (workspace == nullptr || workspace_bytes < p.ws_total) return RT_ERR_WORKSPACE;
  char* ws = static_cast<char*>(workspace);
  uint32_t* ck = reinterpret_cast<uint32_t*>(ws + p.ws_key);
  int* ci = reinterpret_cast<int*>(ws + p.ws_idx);
  double2* lse = reinterpret_cast<double2*>(ws + p.ws_lse);
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  const dim3 g1(p.n_chunks, rows);
  int passes = 0;
  switch (dtype) {
    case 0:
      passes = key_passes<float>();
      set_smem_limit(topk_chunk_kernel<float>, p.smem1);
      topk_chunk_kernel<float><<<g1, kTkThreads, p.smem1, s>>>(static_cast<const float*>(logits), ld, vocab, k,
                                                               p.chunk_len, p.n_chunks, ck, ci, lse);
      break;
    case 1:
      passes = key_passes<__nv_bfloat16>();
      set_smem_limit(topk_chunk_kernel<__nv_bfloat16>, p.smem1);
      topk_chunk_kernel<__nv_bfloat16><<<g1, kTkThreads, p.smem1, s>>>(
          static_cast<const __nv_bfloat16*>(logits), ld, vocab, k, p.chunk_len, p.n_chunks, ck, ci, lse);
      break;
    default:
      passes = key_passes<__half>();
      set_smem_limit(topk_chunk_kernel<__half>, p.smem1);
      topk_chunk_kernel<__half><<<g1, kTkThreads, p.smem1, s>>>(static_cast<const __half*>(logits), ld, vocab, k,
                                                                p.chunk_len, p.n_chunks, ck, ci, lse);
      break;
  }
  int rc = check_launch();
  if (rc != RT_OK) return rc;
  set_smem_limit(topk_merge_kernel, p.smem2);
  topk_merge_kernel<<<rows, kTkThreads, p.smem2, s>>>(vocab, k, p.chunk_len, p.n_chunks, passes, ck, ci, lse,
                                                      top_logp, top_ids, log_z);
  return check_launch();
}
