// Budgeted best-first tree expansion on the device (one CTA per request).
//
// Prologue (whole CTA): the context window goes to shared memory and every
// n-gram of it (orders 2..max_n) is counted into a shared-memory open-addressing
// hash table, so the count of any (tail, token) is one short probe sequence per
// order.  The draft top-k (log-probs and ids) is staged in shared memory when
// it fits.
//
// Expansion (warp 0): the frontier is a compact struct of arrays in shared
// memory (a popped entry is replaced by the last one).  Each pop is a warp
// arg-max over it, then the reference's sibling / child pushes; the continuity
// bonuses of the two pushes are looked up at the same time on different lanes
// (one lane per n-gram order).  Scores use binary64 in the reference's
// operation order (fp32 log-probs widened exactly, explicit round-to-nearest
// adds/multiplies, no contraction) and the arg-max breaks ties as the
// reference's heap tuples do, so the tree is bit-identical.
#include "common.cuh"
#include "host_util.h"

namespace rt {

constexpr int kBuildThreads = 1024;  // the prologue's table build; the expansion is warp 0
constexpr int kMaxTail = 7;        // max_n - 1 for max_n <= 8
constexpr int kMaxRows = 64;       // depth limit (draft rows)
constexpr int kMaxBudget = 1024;
constexpr int kMaxWindow = 8192;
constexpr int kMaxHashSlots = 32768;
constexpr uint32_t kEmpty = 0xFFFFFFFFu;
constexpr uint32_t kNoCand = 0xFFFFFFFFu;

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
  int hash_slots;    // power of two (>= 64) when there is an n-gram table, else 0
  int stage_topk;    // top-k staged in shared memory
  int log1p_staged;  // leading log1p-table entries copied to shared memory
  int mask_in_smem;  // ancestor rows kept in shared memory
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

// ---------------------------------------------------------------------------
// n-gram hash table: slot = [count:16][order-2:3][window position:13]
// ---------------------------------------------------------------------------
__device__ __forceinline__ uint32_t mix32(uint32_t h) {
  h ^= h >> 16;
  h *= 0x7FEB352Du;
  h ^= h >> 15;
  h *= 0x846CA68Bu;
  h ^= h >> 16;
  return h;
}

// hash of n = p+1 tokens: p prefix tokens then `next`
__device__ __forceinline__ uint32_t ngram_hash(const int* prefix, int p, int next) {
  uint32_t h = 0x811C9DC5u ^ static_cast<uint32_t>(p);
  for (int q = 0; q < p; ++q) h = (h ^ static_cast<uint32_t>(prefix[q])) * 0x01000193u;
  h = (h ^ static_cast<uint32_t>(next)) * 0x01000193u;
  return mix32(h);
}

__device__ __forceinline__ bool ngram_at(const int* ctx, int pos, const int* prefix, int p, int next) {
  for (int q = 0; q < p; ++q)
    if (ctx[pos + q] != prefix[q]) return false;
  return ctx[pos + p] == next;
}

// Count the n-gram starting at window position i (prefix length p).
__device__ void ngram_insert(uint32_t* table, int mask, const int* ctx, int i, int p) {
  const int* pre = ctx + i;
  const int next = ctx[i + p];
  uint32_t s = ngram_hash(pre, p, next) & static_cast<uint32_t>(mask);
  const uint32_t mine = (1u << 16) | (static_cast<uint32_t>(p - 1) << 13) | static_cast<uint32_t>(i);
  for (int probe = 0; probe <= mask; ++probe) {
    uint32_t cur = table[s];
    if (cur == kEmpty) {
      cur = atomicCAS(&table[s], kEmpty, mine);
      if (cur == kEmpty) return;
    }
    if (((cur >> 13) & 7u) == static_cast<uint32_t>(p - 1) && ngram_at(ctx, cur & 0x1FFFu, pre, p, next)) {
      atomicAdd(&table[s], 1u << 16);
      return;
    }
    s = (s + 1) & static_cast<uint32_t>(mask);
  }
}

// Occurrences of (tail[tail_len-p .. tail_len), token) in the window.
__device__ int ngram_count(const uint32_t* table, int mask, const int* ctx, const int* tail, int tail_len, int p,
                           int token) {
  const int* pre = tail + (tail_len - p);
  uint32_t s = ngram_hash(pre, p, token) & static_cast<uint32_t>(mask);
  for (int probe = 0; probe <= mask; ++probe) {
    const uint32_t cur = table[s];
    if (cur == kEmpty) return 0;
    if (((cur >> 13) & 7u) == static_cast<uint32_t>(p - 1) && ngram_at(ctx, cur & 0x1FFFu, pre, p, token))
      return static_cast<int>(cur >> 16);
    s = (s + 1) & static_cast<uint32_t>(mask);
  }
  return 0;
}

// ---------------------------------------------------------------------------
// Shared-memory layout (identical on host and device)
// ---------------------------------------------------------------------------
struct Layout {
  size_t f_aug, f_logw, f_bonus, f_inc, f_tok, f_parent, f_rank, f_depth;
  size_t n_tail, n_rank, n_depth, n_parent, n_mask;
  size_t ctx, table, s_lp, s_ids, s_log1p, total;
};

__host__ __device__ inline size_t al16(size_t x) { return (x + 15) & ~static_cast<size_t>(15); }

__host__ __device__ inline Layout make_layout(int budget, int win, int hash_slots, int rows, int k, int words,
                                              bool stage, bool mask_smem, int log1p_staged) {
  Layout L{};
  const size_t FC = static_cast<size_t>(budget) + 2, NN = static_cast<size_t>(budget) + 1;
  size_t o = 0;
  auto put = [&](size_t bytes) {
    const size_t at = o;
    o += al16(bytes);
    return at;
  };
  L.f_aug = put(8 * FC);
  L.f_logw = put(8 * FC);
  L.f_bonus = put(8 * FC);
  L.f_inc = put(8 * FC);
  L.f_tok = put(8 * FC);
  L.f_parent = put(4 * FC);
  L.f_rank = put(4 * FC);
  L.f_depth = put(4 * FC);
  L.n_tail = put(32 * NN);
  L.n_rank = put(4 * NN);
  L.n_depth = put(4 * NN);
  L.n_parent = put(4 * NN);
  L.n_mask = mask_smem ? put(4 * NN * static_cast<size_t>(words)) : 0;
  L.ctx = put(4 * static_cast<size_t>(win > 0 ? win : 1));
  L.table = put(4 * static_cast<size_t>(hash_slots > 0 ? hash_slots : 1));
  L.s_lp = stage ? put(4 * static_cast<size_t>(rows) * k) : 0;
  L.s_ids = stage ? put(8 * static_cast<size_t>(rows) * k) : 0;
  L.s_log1p = log1p_staged > 0 ? put(8 * static_cast<size_t>(log1p_staged)) : 0;
  L.total = o;
  return L;
}

// Rank path of a candidate (parent node p, own rank r, depth d): the ranks of
// its ancestors at depths 1..d-1 followed by r -- the tuple the original heap
// compares after the score (ddtree.py:241-243, :265, :284).
__device__ bool path_less(const int* nrank, const int* nparent, int pa_node, int ra, int da, int pb_node, int rb,
                          int db) {
  int pa[kMaxRows + 1], pb[kMaxRows + 1];
  pa[da] = ra;
  for (int t = da - 1, node = pa_node; t >= 1; --t) {
    pa[t] = nrank[node];
    node = nparent[node];
  }
  pb[db] = rb;
  for (int t = db - 1, node = pb_node; t >= 1; --t) {
    pb[t] = nrank[node];
    node = nparent[node];
  }
  const int m = min(da, db);
  for (int t = 1; t <= m; ++t)
    if (pa[t] != pb[t]) return pa[t] < pb[t];
  return da < db;
}

__global__ void __launch_bounds__(kBuildThreads) tree_build_kernel(BuildArgs a) {
  extern __shared__ __align__(16) unsigned char smem[];
  const int tid = threadIdx.x, lane = tid & 31;
  const int B = a.budget;
  const bool use_ngram = a.strategy != 0;

  // ---- context window (ddtree.py:127-138) ----
  int win = 0;
  int64_t Lctx = 0;
  const int64_t* ctx_src = nullptr;
  if (a.ctx != nullptr) {
    Lctx = a.ctx_len_dev != nullptr ? a.ctx_len_dev[0] + a.ctx_len : a.ctx_len;
    Lctx = Lctx > 0 ? Lctx : 0;
  }
  if (use_ngram && Lctx > 0) {
    const int64_t w = (a.ctx_window > 0 && Lctx > a.ctx_window) ? a.ctx_window : Lctx;
    win = static_cast<int>(w < a.win_cap ? w : static_cast<int64_t>(a.win_cap));
    if (w > a.win_cap && tid == 0) set_status(a.status, RT_DEV_OVERFLOW);
    ctx_src = a.ctx + (Lctx - win);
  }
  const Layout Ly = make_layout(B, a.win_cap, a.hash_slots, a.rows, a.k, a.mask_words, a.stage_topk != 0,
                                a.mask_in_smem != 0, a.log1p_staged);
  double* f_aug = reinterpret_cast<double*>(smem + Ly.f_aug);
  double* f_logw = reinterpret_cast<double*>(smem + Ly.f_logw);
  double* f_bonus = reinterpret_cast<double*>(smem + Ly.f_bonus);
  double* f_inc = reinterpret_cast<double*>(smem + Ly.f_inc);
  int64_t* f_tok = reinterpret_cast<int64_t*>(smem + Ly.f_tok);
  int* f_parent = reinterpret_cast<int*>(smem + Ly.f_parent);
  int* f_rank = reinterpret_cast<int*>(smem + Ly.f_rank);
  int* f_depth = reinterpret_cast<int*>(smem + Ly.f_depth);
  int* n_tail = reinterpret_cast<int*>(smem + Ly.n_tail);  // [node][8]: tokens, length in slot 7
  int* n_rank = reinterpret_cast<int*>(smem + Ly.n_rank);
  int* n_depth = reinterpret_cast<int*>(smem + Ly.n_depth);
  int* n_parent = reinterpret_cast<int*>(smem + Ly.n_parent);
  const int W = a.mask_words;
  uint32_t* rows_mask = a.mask_in_smem ? reinterpret_cast<uint32_t*>(smem + Ly.n_mask) : a.mask;
  int* ctx = reinterpret_cast<int*>(smem + Ly.ctx);
  uint32_t* table = reinterpret_cast<uint32_t*>(smem + Ly.table);
  const float* lp = a.stage_topk ? reinterpret_cast<const float*>(smem + Ly.s_lp) : a.lp;
  const int64_t* ids = a.stage_topk ? reinterpret_cast<const int64_t*>(smem + Ly.s_ids) : a.ids;
  double* s_log1p = reinterpret_cast<double*>(smem + Ly.s_log1p);
  for (int i = tid; i < a.log1p_staged; i += kBuildThreads) s_log1p[i] = a.log1p_table[i];

  // ---- prologue: window, n-gram counts, staged top-k ----
  const int hmask = a.hash_slots - 1;
  for (int i = tid; i < win; i += kBuildThreads) ctx[i] = static_cast<int>(ctx_src[i]);
  for (int i = tid; i < a.hash_slots; i += kBuildThreads) table[i] = kEmpty;
  if (a.stage_topk) {
    float* slp = reinterpret_cast<float*>(smem + Ly.s_lp);
    int64_t* sids = reinterpret_cast<int64_t*>(smem + Ly.s_ids);
    for (int i = tid; i < a.rows * a.k; i += kBuildThreads) {
      slp[i] = a.lp[i];
      sids[i] = a.ids[i];
    }
  }
  __syncthreads();
  // the table of ddtree.py:141-149: for n in 2..max_n, every window position i < win-(n-1)
  const bool have_table = use_ngram && win >= 2 && a.hash_slots > 0;  // else the table is empty (:165)
  if (have_table) {
    for (int p = 1; p <= a.max_n - 1; ++p)
      for (int i = tid; i < win - p; i += kBuildThreads) ngram_insert(table, hmask, ctx, i, p);
  }
  __syncthreads();
  if (tid >= 32) return;

  // ---- expansion (warp 0) ----
  const int tail_size = a.max_n - 1;
  const bool heap_order = a.strategy == 0;
  const bool gated = a.strategy == 2;
  int64_t root = a.root_dev != nullptr ? a.root_dev[0] : a.root;
  if (a.root_dev == nullptr && a.root < 0) root = Lctx > 0 ? a.ctx[Lctx - 1] : 0;
  const int64_t start = a.start_dev != nullptr ? a.start_dev[0] : a.start;
  if (lane == 0) {
    const int tl = use_ngram ? min(tail_size, win) : 0;  // initial tail = last ids of the window
    for (int q = 0; q < tl; ++q) n_tail[q] = ctx[win - tl + q];
    n_tail[7] = tl;
    n_rank[0] = 0;
    n_depth[0] = 0;
    n_parent[0] = -1;
    a.parents[0] = -1;
    if (a.verify_ids) a.verify_ids[0] = root;
    if (a.verify_pos) a.verify_pos[0] = start;
  }
  for (int w = lane; w < W; w += 32) {
    const uint32_t v = (w == 0) ? 1u : 0u;
    rows_mask[w] = v;
    if (a.mask_in_smem) a.mask[w] = v;
  }
  __syncwarp();

  // beta * min(sum_n w^(n-2) * log1p(count_n), cap) of up to two queries at once
  // (ddtree.py:154-186, :412-420): query 0 on lanes 0..15 (one lane per order),
  // query 1 on lanes 16..31; every lane returns both results.
  // this lane's order weight longer_weight^(n-2) for n = (lane % 16) + 2
  const double lane_ow = (lane & 15) < kMaxTail ? a.ow[lane & 15] : 0.0;
  auto bonus_pair = [&](const int* t0, int64_t tok0, bool on0, const int* t1, int64_t tok1, bool on1,
                        double& inc0, double& inc1) {
    const bool q1 = lane >= 16;
    const int* tl_ptr = q1 ? t1 : t0;
    const int p = (lane & 15) + 1;
    const bool order_on = p <= tail_size && p <= tl_ptr[7];
    int c = 0;
    if ((q1 ? on1 : on0) && order_on)
      c = ngram_count(table, hmask, ctx, tl_ptr, tl_ptr[7], p, static_cast<int>(q1 ? tok1 : tok0));
    // each lane forms its own order's term w^(n-2) * log1p(count) (0 where the
    // reference adds nothing: adding +0.0 to the non-negative sum changes no bit)
    const int ci = min(c, a.table_len - 1);
    const double base = !a.use_log_count ? 1.0 : (ci < a.log1p_staged ? s_log1p[ci] : a.log1p_table[ci]);
    const double term = (order_on && c >= a.min_count) ? __dmul_rn(lane_ow, base) : 0.0;
    // summed over n = 2..max_n in ascending order, as the reference adds them
    double sa = 0.0, sb = 0.0;
    for (int n = 2; n <= a.max_n; ++n) {
      sa = __dadd_rn(sa, __shfl_sync(0xFFFFFFFFu, term, n - 2));
      sb = __dadd_rn(sb, __shfl_sync(0xFFFFFFFFu, term, 16 + n - 2));
    }
    if (a.max_bonus > 0.0) {
      sa = (a.max_bonus < sa) ? a.max_bonus : sa;
      sb = (a.max_bonus < sb) ? a.max_bonus : sb;
    }
    inc0 = (!on0 || sa <= 0.0) ? 0.0 : __dmul_rn(a.beta, sa);
    inc1 = (!on1 || sb <= 0.0) ? 0.0 : __dmul_rn(a.beta, sb);
  };

  int nfront = 0, count = 0;
  if (B > 0 && a.rows > 0) {
    const int64_t tok0 = ids[0];
    const double w0 = static_cast<double>(lp[0]);
    double b0 = 0.0, unused = 0.0;
    if (use_ngram) bonus_pair(n_tail, tok0, have_table && !(gated && 0 > a.rank_cap), n_tail, 0, false, b0, unused);
    if (lane == 0) {
      f_aug[0] = __dadd_rn(w0, b0);
      f_logw[0] = w0;
      f_bonus[0] = b0;
      f_inc[0] = b0;
      f_tok[0] = tok0;
      f_parent[0] = 0;
      f_rank[0] = 0;
      f_depth[0] = 1;
    }
    nfront = 1;
    __syncwarp();
  }
  while (count < B && nfront > 0) {
    // ---- arg-max: (score desc, then the heap tuple's tie order) ----
    double bs = -INFINITY;
    uint32_t bk = kNoCand;  // (parent << 21) | (rank << 11) | slot
    if (!heap_order) {
      // n-gram heaps: tuples (-aug, parent, rank), so the winner is the largest
      // score, then the smallest (parent, rank).  Scores become order-preserving
      // 64-bit keys (-0.0 as +0.0, equal doubles equal keys) and the warp
      // reduces them with three redux operations instead of a shuffle tree.
      uint64_t bo = 0;
      for (int e = lane; e < nfront; e += 32) {
        const double s = f_aug[e];
        const int64_t bits = s == 0.0 ? 0 : __double_as_longlong(s);
        const uint64_t o = bits < 0 ? ~static_cast<uint64_t>(bits) : (static_cast<uint64_t>(bits) | (1ull << 63));
        const uint32_t key = (static_cast<uint32_t>(f_parent[e]) << 21) | (static_cast<uint32_t>(f_rank[e]) << 11) |
                             static_cast<uint32_t>(e);
        if (bk == kNoCand || o > bo || (o == bo && key < bk)) {
          bo = o;
          bk = key;
        }
      }
      const uint32_t hi = static_cast<uint32_t>(bo >> 32), lo = static_cast<uint32_t>(bo);
      const uint32_t m_hi = __reduce_max_sync(0xFFFFFFFFu, hi);
      const uint32_t m_lo = __reduce_max_sync(0xFFFFFFFFu, hi == m_hi ? lo : 0u);
      const bool top = bk != kNoCand && hi == m_hi && lo == m_lo;
      bk = __reduce_min_sync(0xFFFFFFFFu, top ? bk : kNoCand);
    } else {
      for (int e = lane; e < nfront; e += 32) {
        const double s = f_aug[e];
        const uint32_t key = (static_cast<uint32_t>(f_parent[e]) << 21) | (static_cast<uint32_t>(f_rank[e]) << 11) |
                             static_cast<uint32_t>(e);
        bool take = bk == kNoCand || s > bs;
        if (!take && s == bs) {
          const int eb = bk & 0x7FF;
          take = path_less(n_rank, n_parent, f_parent[e], f_rank[e], f_depth[e], f_parent[eb], f_rank[eb],
                           f_depth[eb]);
        }
        if (take) {
          bs = s;
          bk = key;
        }
      }
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) {
        const double os = __shfl_xor_sync(0xFFFFFFFFu, bs, o);
        const uint32_t ok = __shfl_xor_sync(0xFFFFFFFFu, bk, o);
        bool take = ok != kNoCand && (bk == kNoCand || os > bs);
        if (!take && ok != kNoCand && os == bs) {
          const int ea = ok & 0x7FF, eb = bk & 0x7FF;
          take = path_less(n_rank, n_parent, f_parent[ea], f_rank[ea], f_depth[ea], f_parent[eb], f_rank[eb],
                           f_depth[eb]);
        }
        if (take) {
          bs = os;
          bk = ok;
        }
      }
    }
    if (bk == kNoCand) break;
    const int e = static_cast<int>(bk & 0x7FF);
    const int parent = static_cast<int>(bk >> 21), rank = static_cast<int>((bk >> 11) & 0x3FF);
    const int depth = f_depth[e];
    const double logw = f_logw[e], bonus = f_bonus[e], inc_self = f_inc[e];
    const int64_t tok = f_tok[e];
    const int me = count + 1;
    // operands of the two pushes
    const int64_t row = static_cast<int64_t>(depth - 1) * a.k;
    const bool has_sib = rank + 1 < a.k;
    const bool has_child = depth < a.rows;
    const float lp_cur = lp[row + rank];
    const float lp_sib = has_sib ? lp[row + rank + 1] : 0.f;
    const int64_t tok_sib = has_sib ? ids[row + rank + 1] : 0;
    const float lp_child = has_child ? lp[row + a.k] : 0.f;
    const int64_t tok_child = has_child ? ids[row + a.k] : 0;
    __syncwarp();
    if (lane == 0) {
      // emit node `me`; the frontier's last entry fills the popped slot
      a.node_tokens[count] = tok;
      a.node_depths[count] = depth;
      a.parents[me] = parent;
      if (a.verify_ids) a.verify_ids[me] = tok;
      if (a.verify_pos) a.verify_pos[me] = start + depth;
      n_rank[me] = rank;
      n_depth[me] = depth;
      n_parent[me] = parent;
      const int* pt = n_tail + 8 * parent;  // own tail = parent's tail + token, last tail_size ids
      int* mt = n_tail + 8 * me;
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
      const int last = nfront - 1;
      if (e != last) {
        f_aug[e] = f_aug[last];
        f_logw[e] = f_logw[last];
        f_bonus[e] = f_bonus[last];
        f_inc[e] = f_inc[last];
        f_tok[e] = f_tok[last];
        f_parent[e] = f_parent[last];
        f_rank[e] = f_rank[last];
        f_depth[e] = f_depth[last];
      }
    }
    // ancestor row = parent's row | own bit (visibility of ddtree.py:520-528)
    for (int w = lane; w < W; w += 32) {
      uint32_t v = rows_mask[static_cast<int64_t>(parent) * W + w];
      if (w == (me >> 5)) v |= 1u << (me & 31);
      rows_mask[static_cast<int64_t>(me) * W + w] = v;
      if (a.mask_in_smem) a.mask[static_cast<int64_t>(me) * W + w] = v;
    }
    --nfront;
    count = me;
    __syncwarp();
    // bonuses of both pushes at once: the sibling's tail is the parent's, the child's is `me`'s
    double inc_sib = 0.0, inc_child = 0.0;
    if (use_ngram && (has_sib || has_child)) {
      const bool on_sib = has_sib && have_table && !(gated && rank + 1 > a.rank_cap);
      const bool on_child = has_child && have_table && !(gated && 0 > a.rank_cap);
      bonus_pair(n_tail + 8 * parent, tok_sib, on_sib, n_tail + 8 * me, tok_child, on_child, inc_sib, inc_child);
    }
    if (lane == 0) {
      if (has_sib) {  // next rank in the same row (ddtree.py:464-490 / :264-281)
        const double w2 = __dadd_rn(__dsub_rn(logw, static_cast<double>(lp_cur)), static_cast<double>(lp_sib));
        const double b2 = use_ngram ? __dadd_rn(__dsub_rn(bonus, inc_self), inc_sib) : 0.0;
        const int s = nfront;
        f_aug[s] = use_ngram ? __dadd_rn(w2, b2) : w2;
        f_logw[s] = w2;
        f_bonus[s] = b2;
        f_inc[s] = inc_sib;
        f_tok[s] = tok_sib;
        f_parent[s] = parent;
        f_rank[s] = rank + 1;
        f_depth[s] = depth;
      }
      if (has_child) {  // rank 0 of the next row (ddtree.py:492-516 / :283-289)
        const double w2 = __dadd_rn(logw, static_cast<double>(lp_child));
        const double b2 = use_ngram ? __dadd_rn(bonus, inc_child) : 0.0;
        const int s = nfront + static_cast<int>(has_sib);
        f_aug[s] = use_ngram ? __dadd_rn(w2, b2) : w2;
        f_logw[s] = w2;
        f_bonus[s] = b2;
        f_inc[s] = inc_child;
        f_tok[s] = tok_child;
        f_parent[s] = me;
        f_rank[s] = 0;
        f_depth[s] = depth + 1;
      }
    }
    nfront += static_cast<int>(has_sib) + static_cast<int>(has_child);
    __syncwarp();
  }
  if (lane == 0) *a.count_out = count;
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
  if (budget > kMaxBudget || rows > kMaxRows || k > 1024) return RT_ERR_UNSUPPORTED;
  if (!parents || !mask || !count || !node_tokens || !node_depths) return RT_ERR_INVALID_ARGUMENT;
  if (mask_words < (budget + 1 + 31) / 32) return RT_ERR_INVALID_ARGUMENT;
  if (budget > 0 && rows > 0 && (!top_logp || !top_ids)) return RT_ERR_INVALID_ARGUMENT;
  if (strategy != 0 && (max_n < 2 || max_n > kMaxTail + 1)) return RT_ERR_UNSUPPORTED;
  if (ctx != nullptr && ctx_len_dev == nullptr && ctx_len < 0) return RT_ERR_INVALID_ARGUMENT;
  // Largest window the kernel may see; shared memory is sized for it.
  int64_t win_cap = 0;
  int slots = 0;
  if (strategy != 0 && ctx != nullptr) {
    if (ctx_len_dev == nullptr)
      win_cap = ctx_window > 0 ? std::min<int64_t>(ctx_len, ctx_window) : ctx_len;
    else
      win_cap = ctx_window > 0 ? ctx_window : kMaxWindow;
    if (win_cap > kMaxWindow) return RT_ERR_UNSUPPORTED;
    if (use_log_count && (log1p_table == nullptr || table_len < win_cap + 1)) return RT_ERR_INVALID_ARGUMENT;
    if (order_weight == nullptr) return RT_ERR_INVALID_ARGUMENT;
    const int64_t keys = static_cast<int64_t>(max_n - 1) * win_cap;
    if (keys > (kMaxHashSlots * 4) / 5) return RT_ERR_UNSUPPORTED;  // keep the table under 80 % full
    slots = 64;
    while (slots < 2 * keys + 1 && slots < kMaxHashSlots) slots <<= 1;
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
  a.hash_slots = slots;
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
  // optional shared-memory residents: the staged top-k, then the ancestor rows
  constexpr size_t kSmemBudget = 220 * 1024;
  const int stage_rows = rows > 0 ? rows : 1;
  a.mask_in_smem = 1;
  a.stage_topk = 1;
  a.log1p_staged = 0;
  if (make_layout(budget, a.win_cap, slots, stage_rows, k, mask_words, true, true, 0).total > kSmemBudget)
    a.stage_topk = 0;
  if (make_layout(budget, a.win_cap, slots, stage_rows, k, mask_words, a.stage_topk, true, 0).total > kSmemBudget)
    a.mask_in_smem = 0;
  // then the log1p table (one lookup per bonus, on the expansion's critical
  // path): all of it when it fits, else its head (small counts are the common case)
  if (use_log_count) {
    for (int want : {table_len, 256}) {
      want = want < table_len ? want : table_len;
      if (make_layout(budget, a.win_cap, slots, stage_rows, k, mask_words, a.stage_topk, a.mask_in_smem, want)
              .total <= kSmemBudget) {
        a.log1p_staged = want;
        break;
      }
    }
  }
  const size_t smem = make_layout(budget, a.win_cap, slots, stage_rows, k, mask_words, a.stage_topk,
                                  a.mask_in_smem, a.log1p_staged)
                          .total;
  if (smem > kSmemBudget) return RT_ERR_UNSUPPORTED;
  if (rows == 0) a.stage_topk = 0;
  set_smem_limit(tree_build_kernel, smem);
  tree_build_kernel<<<1, kBuildThreads, smem, reinterpret_cast<cudaStream_t>(stream)>>>(a);
  return check_launch();
}
