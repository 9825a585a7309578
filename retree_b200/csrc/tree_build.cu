// Budgeted best-first tree expansion on the device (one CTA per request).
//
// Prologue (whole CTA): copy the context window to shared memory and sort the
// (token, position) pairs of every "next" position, so the n-gram count of
// any (tail, token) is a search for the token's run plus a scan of its
// occurrences.  Expansion (warp 0): the frontier lives in shared memory as a
// struct of arrays; each pop is a warp-wide arg-max over it, followed by the
// reference's sibling/child pushes.  Scores use binary64 with the reference's
// operation order (fp32 log-probs widened exactly, no fused multiply-adds), and
// the arg-max breaks ties exactly as the reference's heap tuples do, so the
// emitted tree is bit-identical.
#include "common.cuh"
#include "host_util.h"

namespace rt {

constexpr int kBuildThreads = 256;
constexpr int kMaxTail = 7;       // max_n - 1 for max_n <= 8
constexpr int kMaxRows = 64;      // depth limit (draft rows)
constexpr int kMaxBudget = 1024;
constexpr int kMaxWindow = 8192;

struct BuildArgs {
  const float* lp;
  const int64_t* ids;
  int rows, k, budget, strategy;
  const int64_t* ctx;
  int64_t ctx_len;
  const int64_t* ctx_len_dev;
  int ctx_window, win_cap, max_n;
  double beta;
  int rank_cap, min_count, use_log_count;
  double ow[kMaxTail];
  double max_bonus;
  const double* log1p_table;
  int table_len;
  int64_t* node_tokens;
  int64_t* node_depths;
  int32_t* parents;
  uint32_t* mask;
  int mask_words;
  int32_t* count_out;
  int64_t* verify_ids;
  int64_t* verify_pos;
  int64_t root;
  const int64_t* root_dev;
  int64_t start;
  const int64_t* start_dev;
  int* status;
};

struct Frontier {
  double* aug;
  double* logw;
  double* bonus;
  double* inc;
  int* parent;  // -1 once popped
  int* rank;
  int* depth;
};

struct Nodes {
  int* tail;   // [nn][8]: tokens then length in slot 7
  int* rank;
  int* depth;
  int* parent;
};

// Candidate comparison key carried through the warp arg-max.
struct Key {
  double score;
  int parent, rank, depth, slot;
};

__device__ __forceinline__ Key shfl_key(const Key& a, int src_lane_xor) {
  Key b;
  b.score = __shfl_xor_sync(0xFFFFFFFFu, a.score, src_lane_xor);
  b.parent = __shfl_xor_sync(0xFFFFFFFFu, a.parent, src_lane_xor);
  b.rank = __shfl_xor_sync(0xFFFFFFFFu, a.rank, src_lane_xor);
  b.depth = __shfl_xor_sync(0xFFFFFFFFu, a.depth, src_lane_xor);
  b.slot = __shfl_xor_sync(0xFFFFFFFFu, a.slot, src_lane_xor);
  return b;
}

// Rank path of a candidate (parent node p, own rank r, depth d): the ranks of
// its ancestors at depths 1..d-1 followed by r -- the tuple the original heap
// compares after the score (ddtree.py:241-243, :265, :284).
__device__ bool path_less(const Nodes& nd, const Key& a, const Key& b) {
  int pa[kMaxRows + 1], pb[kMaxRows + 1];
  pa[a.depth] = a.rank;
  for (int t = a.depth - 1, node = a.parent; t >= 1; --t) {
    pa[t] = nd.rank[node];
    node = nd.parent[node];
  }
  pb[b.depth] = b.rank;
  for (int t = b.depth - 1, node = b.parent; t >= 1; --t) {
    pb[t] = nd.rank[node];
    node = nd.parent[node];
  }
  const int m = min(a.depth, b.depth);
  for (int t = 1; t <= m; ++t)
    if (pa[t] != pb[t]) return pa[t] < pb[t];
  return a.depth < b.depth;
}

// True if candidate a is popped before b.  slot < 0 marks "no candidate".
__device__ __forceinline__ bool better(const Nodes& nd, bool heap_order, const Key& a, const Key& b) {
  if (a.slot < 0) return false;
  if (b.slot < 0) return true;
  if (a.score != b.score) return a.score > b.score;
  if (heap_order) return path_less(nd, a, b);
  if (a.parent != b.parent) return a.parent < b.parent;  // ddtree.py:432-434 tuple order
  return a.rank < b.rank;
}

struct Ngram {
  const int* ctx;                        // window, shared memory
  const unsigned long long* pairs;       // sorted (token << 32 | position), shared memory
  int len;                               // window length
  int npairs;                            // len - 1
};

// First index in pairs[0..n) whose value >= target (warp-cooperative).
__device__ __forceinline__ int warp_lower_bound(const unsigned long long* pairs, int n, unsigned long long target) {
  const int lane = threadIdx.x & 31;
  int lo = 0, hi = n;
  while (hi - lo > 31) {
    const int step = (hi - lo + 31) >> 5;
    const int p = lo + lane * step;
    const bool pred = (p >= hi) || (pairs[p] >= target);
    const unsigned b = __ballot_sync(0xFFFFFFFFu, pred);
    if (b == 0u) {
      lo = lo + 31 * step + 1;
      continue;
    }
    const int f = __ffs(b) - 1;
    if (f == 0) return lo;
    const int nlo = lo + (f - 1) * step + 1;
    hi = min(hi, lo + f * step);
    lo = nlo;
  }
  const int p = lo + lane;
  const bool pred = (p >= hi) || (pairs[p] >= target);
  const unsigned b = __ballot_sync(0xFFFFFFFFu, pred);
  return lo + __ffs(b) - 1;
}

// Continuity bonus of appending `token` after `tail` (ddtree.py:154-186),
// computed by warp 0; every lane returns the same value.
__device__ double ngram_bonus(const BuildArgs& a, const Ngram& g, const int* tail, int tail_len, int64_t token) {
  if (g.len < 2) return 0.0;  // empty table (ddtree.py:165)
  const int lane = threadIdx.x & 31;
  const unsigned long long t = static_cast<unsigned long long>(token);
  const int lo = warp_lower_bound(g.pairs, g.npairs, t << 32);
  const int hi = warp_lower_bound(g.pairs, g.npairs, (t + 1) << 32);
  const int maxp = min(a.max_n - 1, tail_len);
  int cnt[kMaxTail];
#pragma unroll
  for (int p = 0; p < kMaxTail; ++p) cnt[p] = 0;
  for (int i = lo + lane; i < hi; i += 32) {
    const int j = static_cast<int>(g.pairs[i] & 0xFFFFFFFFull);
    int m = 0;
    while (m < maxp && m < j && g.ctx[j - 1 - m] == tail[tail_len - 1 - m]) ++m;
#pragma unroll
    for (int p = 0; p < kMaxTail; ++p) cnt[p] += (m >= p + 1);
  }
  double total = 0.0;
  for (int n = 2; n <= a.max_n; ++n) {
    const int p = n - 1;
    const int c = __reduce_add_sync(0xFFFFFFFFu, cnt[p - 1]);
    if (tail_len < p) continue;
    if (c < a.min_count) continue;
    const double base = a.use_log_count ? a.log1p_table[min(c, a.table_len - 1)] : 1.0;
    total = __dadd_rn(total, __dmul_rn(a.ow[n - 2], base));
  }
  if (a.max_bonus > 0.0) total = (a.max_bonus < total) ? a.max_bonus : total;
  return total;
}

// beta * bonus, gated by rank for the rank-gated strategy (ddtree.py:412-420).
__device__ __forceinline__ double weighted_inc(const BuildArgs& a, const Ngram& g, const int* tail, int tail_len,
                                               int64_t token, int rank) {
  if (a.strategy == 2 && rank > a.rank_cap) return 0.0;
  const double b = ngram_bonus(a, g, tail, tail_len, token);
  if (b <= 0.0) return 0.0;
  return __dmul_rn(a.beta, b);
}

__global__ void __launch_bounds__(kBuildThreads) tree_build_kernel(BuildArgs a) {
  extern __shared__ __align__(16) unsigned char smem[];
  const int tid = threadIdx.x, lane = tid & 31;
  const int B = a.budget, FC = 2 * B + 2, NN = B + 1;
  // ---- shared-memory carve-up (must match tree_build_smem) ----
  size_t off = 0;
  auto take = [&](size_t bytes) {
    unsigned char* p = smem + off;
    off += (bytes + 15) & ~static_cast<size_t>(15);
    return p;
  };
  Frontier f;
  f.aug = reinterpret_cast<double*>(take(sizeof(double) * FC));
  f.logw = reinterpret_cast<double*>(take(sizeof(double) * FC));
  f.bonus = reinterpret_cast<double*>(take(sizeof(double) * FC));
  f.inc = reinterpret_cast<double*>(take(sizeof(double) * FC));
  f.parent = reinterpret_cast<int*>(take(sizeof(int) * FC));
  f.rank = reinterpret_cast<int*>(take(sizeof(int) * FC));
  f.depth = reinterpret_cast<int*>(take(sizeof(int) * FC));
  Nodes nd;
  nd.tail = reinterpret_cast<int*>(take(sizeof(int) * 8 * NN));
  nd.rank = reinterpret_cast<int*>(take(sizeof(int) * NN));
  nd.depth = reinterpret_cast<int*>(take(sizeof(int) * NN));
  nd.parent = reinterpret_cast<int*>(take(sizeof(int) * NN));
  const bool use_ngram = a.strategy != 0;
  int win = 0;
  int64_t L = 0;
  const int64_t* ctx_src = nullptr;
  if (a.ctx != nullptr) {
    L = a.ctx_len_dev != nullptr ? a.ctx_len_dev[0] + a.ctx_len : a.ctx_len;
    L = L > 0 ? L : 0;
  }
  if (use_ngram && L > 0) {
    // the window of ddtree.py:135-136, bounded by the shared memory sized on the host
    const int64_t w = (a.ctx_window > 0 && L > a.ctx_window) ? a.ctx_window : L;
    win = static_cast<int>(w < a.win_cap ? w : static_cast<int64_t>(a.win_cap));
    if (w > a.win_cap && tid == 0) set_status(a.status, RT_DEV_OVERFLOW);
    ctx_src = a.ctx + (L - win);
  }
  int sort_len = 1;
  while (sort_len < max(win - 1, 1)) sort_len <<= 1;
  int* ctx = reinterpret_cast<int*>(take(sizeof(int) * max(win, 1)));
  unsigned long long* pairs = reinterpret_cast<unsigned long long*>(take(sizeof(unsigned long long) * sort_len));

  // ---- prologue: context window and sorted (token, next-position) pairs ----
  for (int i = tid; i < win; i += kBuildThreads) ctx[i] = static_cast<int>(ctx_src[i]);
  __syncthreads();
  for (int i = tid; i < sort_len; i += kBuildThreads) {
    const int j = i + 1;  // "next" positions 1..win-1
    pairs[i] = j < win ? ((static_cast<unsigned long long>(static_cast<uint32_t>(ctx[j])) << 32) | static_cast<uint32_t>(j))
                       : ~0ull;
  }
  __syncthreads();
  for (int size = 2; size <= sort_len; size <<= 1) {
    for (int stride = size >> 1; stride > 0; stride >>= 1) {
      for (int i = tid; i < sort_len; i += kBuildThreads) {
        const int j = i ^ stride;
        if (j > i) {
          const bool asc = (i & size) == 0;
          const unsigned long long x = pairs[i], y = pairs[j];
          if (asc ? (x > y) : (x < y)) {
            pairs[i] = y;
            pairs[j] = x;
          }
        }
      }
      __syncthreads();
    }
  }
  if (tid >= 32) return;

  // ---- expansion (warp 0) ----
  Ngram g{ctx, pairs, win, max(win - 1, 0)};
  const int tail_size = a.max_n - 1;
  const bool heap_order = a.strategy == 0;
  int64_t root = a.root_dev != nullptr ? a.root_dev[0] : a.root;
  if (a.root_dev == nullptr && a.root < 0) root = L > 0 ? a.ctx[L - 1] : 0;
  const int64_t start = a.start_dev != nullptr ? a.start_dev[0] : a.start;
  const int W = a.mask_words;
  // root node 0: tail = last tail_size window ids; mask row 0 = {0}
  if (lane == 0) {
    int tl = use_ngram ? min(tail_size, win) : 0;
    for (int q = 0; q < tl; ++q) nd.tail[q] = ctx[win - tl + q];
    nd.tail[7] = tl;
    nd.rank[0] = 0;
    nd.depth[0] = 0;
    nd.parent[0] = -1;
    a.parents[0] = -1;
    if (a.verify_ids) a.verify_ids[0] = root;
    if (a.verify_pos) a.verify_pos[0] = start;
  }
  for (int w = lane; w < W; w += 32) a.mask[w] = (w == 0) ? 1u : 0u;
  __syncwarp();
  int nfront = 0, count = 0;
  if (B > 0 && a.rows > 0) {
    const int64_t tok0 = a.ids[0];
    const double w0 = static_cast<double>(a.lp[0]);
    double b0 = 0.0;
    if (use_ngram) b0 = weighted_inc(a, g, nd.tail, nd.tail[7], tok0, 0);
    if (lane == 0) {
      f.aug[0] = __dadd_rn(w0, b0);
      f.logw[0] = w0;
      f.bonus[0] = b0;
      f.inc[0] = b0;
      f.parent[0] = 0;
      f.rank[0] = 0;
      f.depth[0] = 1;
    }
    nfront = 1;
    __syncwarp();
  }
  while (count < B && nfront > 0) {
    // arg-max over the live frontier
    Key best{0.0, 0, 0, 0, -1};
    for (int e = lane; e < nfront; e += 32) {
      if (f.parent[e] < 0) continue;
      Key c{f.aug[e], f.parent[e], f.rank[e], f.depth[e], e};
      if (better(nd, heap_order, c, best)) best = c;
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const Key other = shfl_key(best, o);
      if (better(nd, heap_order, other, best)) best = other;
    }
    if (best.slot < 0) break;  // frontier empty
    const int e = best.slot;
    const int parent = best.parent, rank = best.rank, depth = best.depth;
    const double logw = f.logw[e], bonus = f.bonus[e], inc_self = f.inc[e];
    const int me = count + 1;
    const int64_t tok = a.ids[static_cast<int64_t>(depth - 1) * a.k + rank];
    __syncwarp();
    if (lane == 0) {
      f.parent[e] = -1;
      a.node_tokens[count] = tok;
      a.node_depths[count] = depth;
      a.parents[me] = parent;
      if (a.verify_ids) a.verify_ids[me] = tok;
      if (a.verify_pos) a.verify_pos[me] = start + depth;
      nd.rank[me] = rank;
      nd.depth[me] = depth;
      nd.parent[me] = parent;
      // own tail = parent's tail + token, keeping the last tail_size ids
      const int* pt = nd.tail + 8 * parent;
      int* mt = nd.tail + 8 * me;
      const int pl = pt[7];
      if (pl < tail_size) {
        for (int q = 0; q < pl; ++q) mt[q] = pt[q];
        mt[pl] = static_cast<int>(tok);
        mt[7] = pl + 1;
      } else {
        for (int q = 0; q + 1 < tail_size; ++q) mt[q] = pt[q + 1];
        if (tail_size > 0) mt[tail_size - 1] = static_cast<int>(tok);
        mt[7] = tail_size;
      }
    }
    // ancestor mask row = parent's row | own bit
    for (int w = lane; w < W; w += 32) {
      uint32_t v = a.mask[static_cast<int64_t>(parent) * W + w];
      if (w == (me >> 5)) v |= 1u << (me & 31);
      a.mask[static_cast<int64_t>(me) * W + w] = v;
    }
    __syncwarp();
    count = me;
    // sibling: next rank in the same row (ddtree.py:464-490 / :264-281)
    if (rank + 1 < a.k) {
      const int r2 = rank + 1;
      const int64_t row = static_cast<int64_t>(depth - 1) * a.k;
      const double w2 = __dadd_rn(__dsub_rn(logw, static_cast<double>(a.lp[row + rank])),
                                  static_cast<double>(a.lp[row + r2]));
      double inc2 = 0.0, b2 = 0.0;
      if (use_ngram) {
        const int* pt = nd.tail + 8 * parent;
        inc2 = weighted_inc(a, g, pt, pt[7], a.ids[row + r2], r2);
        b2 = __dadd_rn(__dsub_rn(bonus, inc_self), inc2);
      }
      if (lane == 0) {
        f.aug[nfront] = use_ngram ? __dadd_rn(w2, b2) : w2;
        f.logw[nfront] = w2;
        f.bonus[nfront] = b2;
        f.inc[nfront] = inc2;
        f.parent[nfront] = parent;
        f.rank[nfront] = r2;
        f.depth[nfront] = depth;
      }
      ++nfront;
    }
    // first child: rank 0 of the next row (ddtree.py:492-516 / :283-289)
    if (depth < a.rows) {
      const int64_t row = static_cast<int64_t>(depth) * a.k;
      const double w2 = __dadd_rn(logw, static_cast<double>(a.lp[row]));
      double inc2 = 0.0, b2 = 0.0;
      if (use_ngram) {
        __syncwarp();
        const int* mt = nd.tail + 8 * me;
        inc2 = weighted_inc(a, g, mt, mt[7], a.ids[row], 0);
        b2 = __dadd_rn(bonus, inc2);
      }
      if (lane == 0) {
        f.aug[nfront] = use_ngram ? __dadd_rn(w2, b2) : w2;
        f.logw[nfront] = w2;
        f.bonus[nfront] = b2;
        f.inc[nfront] = inc2;
        f.parent[nfront] = me;
        f.rank[nfront] = 0;
        f.depth[nfront] = depth + 1;
      }
      ++nfront;
    }
    __syncwarp();
    if (nfront > FC) {
      if (lane == 0) set_status(a.status, RT_DEV_OVERFLOW);
      break;
    }
  }
  if (lane == 0) *a.count_out = count;
}

static size_t tree_build_smem(int budget, int win) {
  const size_t FC = 2 * static_cast<size_t>(budget) + 2, NN = budget + 1;
  auto al = [](size_t x) { return (x + 15) & ~static_cast<size_t>(15); };
  size_t s = 4 * al(8 * FC) + 3 * al(4 * FC) + al(32 * NN) + 3 * al(4 * NN);
  size_t sort_len = 1;
  while (sort_len < static_cast<size_t>(std::max(win - 1, 1))) sort_len <<= 1;
  s += al(4 * static_cast<size_t>(std::max(win, 1))) + al(8 * sort_len);
  return s;
}

}  // namespace rt

using namespace rt;

extern "C" int rt_tree_build(const float* top_logp, const int64_t* top_ids, int rows, int k, int budget,
                             int strategy, const int64_t* ctx, int64_t ctx_len, const int64_t* ctx_len_dev,
                             int ctx_window, int max_n, double beta, int rank_cap, int min_count,
                             int use_log_count, const double* order_weight, double max_token_bonus,
                             const double* log1p_table, int table_len, int64_t* node_tokens, int64_t* node_depths,
                             int32_t* parents, uint32_t* mask, int mask_words, int32_t* count, int64_t* verify_ids,
                             int64_t* verify_pos, int64_t root, const int64_t* root_dev, int64_t start,
                             const int64_t* start_dev, int* status, rt_stream_t stream) {
  if (rows < 0 || k <= 0 || budget < 0 || strategy < 0 || strategy > 2) return RT_ERR_INVALID_ARGUMENT;
  if (budget > kMaxBudget || rows > kMaxRows) return RT_ERR_UNSUPPORTED;
  if (!parents || !mask || !count || !node_tokens || !node_depths) return RT_ERR_INVALID_ARGUMENT;
  if (mask_words < (budget + 1 + 31) / 32) return RT_ERR_INVALID_ARGUMENT;
  if (budget > 0 && rows > 0 && (!top_logp || !top_ids)) return RT_ERR_INVALID_ARGUMENT;
  if (strategy != 0 && (max_n < 2 || max_n > kMaxTail + 1)) return RT_ERR_UNSUPPORTED;
  if (ctx != nullptr && ctx_len_dev == nullptr && ctx_len < 0) return RT_ERR_INVALID_ARGUMENT;
  // Largest window the kernel may see; shared memory is sized for it.
  int64_t win_cap = 0;
  if (strategy != 0 && ctx != nullptr) {
    if (ctx_len_dev == nullptr)
      win_cap = ctx_window > 0 ? std::min<int64_t>(ctx_len, ctx_window) : ctx_len;
    else
      win_cap = ctx_window > 0 ? ctx_window : kMaxWindow;
    if (win_cap > kMaxWindow) return RT_ERR_UNSUPPORTED;
    if (use_log_count && (log1p_table == nullptr || table_len < win_cap + 1)) return RT_ERR_INVALID_ARGUMENT;
    if (order_weight == nullptr) return RT_ERR_INVALID_ARGUMENT;
  }
  BuildArgs a{};
  a.lp = top_logp;
  a.ids = top_ids;
  a.rows = rows;
  a.k = k;
  a.budget = budget;
  a.strategy = strategy;
  a.ctx = ctx;
  a.ctx_len = ctx_len;
  a.ctx_len_dev = ctx_len_dev;
  a.ctx_window = ctx_window;
  a.win_cap = static_cast<int>(win_cap);
  a.max_n = strategy != 0 ? max_n : 2;
  a.beta = beta;
  a.rank_cap = rank_cap;
  a.min_count = min_count;
  a.use_log_count = use_log_count;
  for (int i = 0; i < kMaxTail; ++i) a.ow[i] = (order_weight && i < a.max_n - 1) ? order_weight[i] : 0.0;
  a.max_bonus = max_token_bonus;
  a.log1p_table = log1p_table;
  a.table_len = table_len;
  a.node_tokens = node_tokens;
  a.node_depths = node_depths;
  a.parents = parents;
  a.mask = mask;
  a.mask_words = mask_words;
  a.count_out = count;
  a.verify_ids = verify_ids;
  a.verify_pos = verify_pos;
  a.root = root;
  a.root_dev = root_dev;
  a.start = start;
  a.start_dev = start_dev;
  a.status = status;
  const size_t smem = tree_build_smem(budget, static_cast<int>(win_cap));
  if (smem > 227 * 1024) return RT_ERR_UNSUPPORTED;
  set_smem_limit(tree_build_kernel, smem);
  tree_build_kernel<<<1, kBuildThreads, smem, reinterpret_cast<cudaStream_t>(stream)>>>(a);
  return check_launch();
}
