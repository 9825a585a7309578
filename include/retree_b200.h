/*
 * retree_b200 — C ABI of the B200 (sm_100a) kernels behind ReTree's
 * tree-verification path.
 *
 * Conventions (every entry point):
 *   - Plain device pointers, sizes and strides; no framework types.  Strides
 *     are in BYTES unless a name says otherwise.
 *   - Work is enqueued on `stream` (a cudaStream_t; NULL = legacy default
 *     stream).  Nothing here allocates device memory: scratch ("workspace") is
 *     passed in by the caller, sized by the matching *_workspace_size call.
 *   - The return value is an RT_* code checked on the host before launch
 *     (arguments, shapes, launch errors).  Kernels report data-dependent
 *     errors (an index out of range, a wait that ran out) by writing an
 *     RT_DEV_* code into the optional device word `status` (first error wins;
 *     the caller zeroes it).
 *   - Results are bit-for-bit deterministic run to run.
 *
 * Each declaration names the reference interface (Adamlong3/ReTree, or the
 * transformers 5.5.0 code the reference calls) that it replaces.
 */
#ifndef RETREE_B200_H
#define RETREE_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef struct CUstream_st* rt_stream_t;

/* Host-side return codes. */
#define RT_OK 0
#define RT_ERR_INVALID_ARGUMENT 1 /* null pointer, negative size, misaligned stride */
#define RT_ERR_UNSUPPORTED 2      /* valid but outside what the kernels implement */
#define RT_ERR_WORKSPACE 3        /* workspace missing or smaller than required */
#define RT_ERR_CUDA 4             /* launch or driver error (see rt_last_cuda_error) */

/* Device status codes written to `status`. */
#define RT_DEV_WAIT_TIMEOUT 100 /* a bounded wait ran out; the kernel exited early */
#define RT_DEV_BAD_INDEX 101    /* an index read from device memory was out of range */
#define RT_DEV_OVERFLOW 102     /* a device-side capacity was exceeded */

/* ABI version of this library (bumped on any signature change). */
int rt_abi_version(void);

/* Last CUDA error seen by an entry point on this thread (cudaError_t value). */
int rt_last_cuda_error(void);

/* Human-readable text for an RT_* or RT_DEV_* code. */
const char* rt_status_string(int code);

/* Programmatic dependent launch between the kernels of the verify forward
 * (rt_add_rmsnorm, rt_embed_rmsnorm, rt_qk_norm_rope_append, rt_silu_mul,
 * rt_linear, rt_tree_attn): each may start its prologue (and its weight or
 * prefix-KV loads) while the previous kernel in the stream finishes.  On by
 * default (RETREE_B200_PDL=0 in the environment turns the default off).
 * Turn it off in processes whose streams also carry NCCL collectives: with
 * them on the same stream, multi-process rounds were observed to slow down by
 * orders of magnitude.  Affects launches made after the call. */
void rt_set_pdl(int enabled);
int rt_pdl_enabled(void);

/* ------------------------------------------------------------------------
 * KV-cache compaction after a commit.
 * Replaces compact_tail_inplace / _compact_appended_window
 * (ddtree.py:37-65, ddtree.py:666-686) applied to every layer's K and V by
 * compact_dynamic_cache (ddtree.py:689-731), in ONE launch.
 *
 * The cache is `n_slabs` slabs (one per layer and per K/V).  Slab s starts at
 * slabs[s] (a DEVICE array of n_slabs pointers) or, when slabs is NULL, at
 * base + s * slab_stride.  Each slab holds n_heads heads of rows of
 * `row_bytes` bytes at head_stride / row_stride.  Within each head the window
 * of cur_len rows after past_len is compacted in place:
 *     row[past_len + i] = old row[past_len + keep[i]],  i < n_keep
 * with gather-then-scatter semantics (any order of keep is allowed).  As in
 * the reference, nothing moves when n_keep == 0 or n_keep == cur_len.
 * keep (int64, DEVICE) holds window-relative indices in [0, cur_len).  When
 * n_keep_dev is non-NULL the count is read from it (<= n_keep) at run time;
 * when past_len_dev is non-NULL past_len is read from it (int64, DEVICE) and
 * the host past_len is ignored.  Limit: n_keep * row_bytes <= 200 KiB.
 * ---------------------------------------------------------------------- */
int rt_kv_compact(void* const* slabs, void* base, int n_slabs, int64_t slab_stride, int n_heads,
                  int64_t head_stride, int64_t row_stride, int row_bytes, int64_t past_len,
                  const int64_t* past_len_dev, int64_t cur_len, const int64_t* keep, int n_keep,
                  const int32_t* n_keep_dev, int* status, rt_stream_t stream);

/* ------------------------------------------------------------------------
 * In-place KV append into a preallocated cache.
 * Replaces DynamicLayer.update's torch.cat of the whole cache
 * (transformers/cache_utils.py:102-121, called from
 * models/qwen3/modeling_qwen3.py:270-271) for one layer's K and V.
 *
 * Writes n_new rows per head of k_new / v_new (row r of head h at
 * h*new_head_stride + r*new_row_stride) to rows [offset, offset+n_new) of
 * k_cache / v_cache.  offset is read from offset_dev (int64, DEVICE) when
 * non-NULL.  Rows past `capacity` are not written (RT_DEV_OVERFLOW).
 * ---------------------------------------------------------------------- */
int rt_kv_append(void* k_cache, void* v_cache, int64_t cache_head_stride, int64_t cache_row_stride,
                 const void* k_new, const void* v_new, int64_t new_head_stride, int64_t new_row_stride,
                 int n_heads, int n_new, int row_bytes, int64_t capacity, int64_t offset,
                 const int64_t* offset_dev, int* status, rt_stream_t stream);

/* ------------------------------------------------------------------------
 * Tree-verify attention (bf16, GQA, head_dim 128).
 * Replaces sdpa_attention_forward with a tree mask
 * (transformers/integrations/sdpa_attention.py:40-104: repeat_kv at :57-60,
 * F.scaled_dot_product_attention at :92-101), as reached from
 * models/qwen3/modeling_qwen3.py:273-286 with the mask that
 * compile_ddtree_tree writes (ddtree.py:629-640).
 *
 * Query row (node i, head h) is at q + i*q_tok_stride + h*q_head_stride
 * (bf16[128]).  Keys/values of kv head g are rows [0, prefix_len + n) of
 * k/v + g*kv_head_stride (row stride kv_row_stride, bf16[128]); the cache
 * holds kv_capacity rows per head.  Every prefix key is visible; tree key j
 * (row prefix_len + j) is visible to node i iff bit (j % 32) of word
 * mask[i*mask_words + j/32] is set.  out row (i, h) is written at
 * out + i*out_tok_stride + h*out_head_stride (bf16[128]), normalised by the
 * softmax sum.  scale multiplies QK^T (HF passes head_dim**-0.5).
 * prefix_len is read from prefix_len_dev (int64, DEVICE) when non-NULL; then
 * prefix_len is only an upper bound used to size the launch.
 *
 * Keys are split into num_splits ranges (0 = choose).  On the tcgen05 path
 * the ranges of one (kv head, 128-row tile) run as one thread-block cluster
 * (2..16 CTAs, when every cluster of the launch fits on the GPU at once) and
 * are merged inside the kernel through distributed shared memory; otherwise
 * their partial results go through the workspace to a second kernel.
 * workspace must hold rt_tree_attn_workspace_size(...) bytes (alignment 256;
 * rt_tree_attn_plan says whether a launch uses it).  Requires
 * num_q_heads % num_kv_heads == 0, head_dim == 128, all strides multiples of
 * 16 bytes, q/k/v/out 16-byte aligned.  n * (num_q_heads/num_kv_heads) >= 64
 * runs on tcgen05 (TMEM accumulators, TMA-fed K/V); smaller trees run a
 * warp-level kernel.  `path` (0 = choose, 1 = tcgen05, 2 = warp-level)
 * forces one of them.
 * ---------------------------------------------------------------------- */
size_t rt_tree_attn_workspace_size(int n, int num_q_heads, int num_kv_heads, int head_dim,
                                   int64_t prefix_len, int num_splits);
int rt_tree_attn(const void* q, int64_t q_tok_stride, int64_t q_head_stride, const void* k, const void* v,
                 int64_t kv_head_stride, int64_t kv_row_stride, int64_t kv_capacity, void* out,
                 int64_t out_tok_stride, int64_t out_head_stride, const uint32_t* mask, int mask_words, int n,
                 int64_t prefix_len, const int64_t* prefix_len_dev, int num_q_heads, int num_kv_heads,
                 int head_dim, float scale, int num_splits, int path, void* workspace, size_t workspace_bytes,
                 int* status, rt_stream_t stream);

/* ------------------------------------------------------------------------
 * Attention-output exchange of a KV-head split over NVLink peer memory.
 * Replaces the NCCL all-gather of the attention outputs before o_proj when
 * one long request is split by KV head over several GPUs
 * (retree_b200/headsplit.py; the reference runs one request on one GPU and
 * has no counterpart).  Buffers are shared between the ranks' processes with
 * CUDA IPC (plain peer mappings, no multicast).
 *
 * rt_ipc_alloc: cudaMalloc'd, zeroed device buffer of `bytes` and its 64-byte
 *   IPC handle; rt_ipc_free releases it.  rt_ipc_open maps a peer's handle
 *   (peer access enabled lazily), rt_ipc_close unmaps it.
 * rt_peer_epoch_step: *epoch_dev += add on the stream (one per forward).
 * rt_peer_signal: after this rank's attention rows are in its buffer, stores
 *   *epoch_dev + epoch_add into slot `rank` of every rank's int64 flag array
 *   (peer_flags[p] = rank p's array as mapped here), release at system scope.
 * rt_peer_gather: for every source rank s, waits (bounded; RT_DEV_WAIT_TIMEOUT
 *   in *status, rows not copied) until flags_local[s] >= *epoch_dev +
 *   epoch_add, then copies rows [0, rows) of peer_bufs[s] (row stride src_ld
 *   bytes, row_bytes each) to out + s*row_bytes (row stride out_ld).  Sizes
 *   and strides are multiples of 16 bytes, pointers 16-byte aligned,
 *   world <= 8.
 * ---------------------------------------------------------------------- */
int rt_ipc_alloc(size_t bytes, void** ptr, void* handle);
int rt_ipc_free(void* ptr);
int rt_ipc_open(const void* handle, void** ptr);
int rt_ipc_close(void* ptr);
int rt_peer_epoch_step(int64_t* epoch_dev, int64_t add, rt_stream_t stream);
int rt_peer_signal(void* const* peer_flags, int world, int rank, const int64_t* epoch_dev, int64_t epoch_add,
                   rt_stream_t stream);
int rt_peer_gather(void* const* peer_bufs, int world, int rows, int64_t row_bytes, int64_t src_ld, void* out,
                   int64_t out_ld, const int64_t* flags_local, const int64_t* epoch_dev, int64_t epoch_add,
                   int* status, rt_stream_t stream);

/* Number of key splits rt_tree_attn chooses for this shape (num_splits = 0). */
int rt_tree_attn_default_splits(int n, int num_q_heads, int num_kv_heads, int64_t prefix_len);

/* How rt_tree_attn runs a shape (no counterpart in the reference; a query
 * for hosts that size buffers or count launches): *splits_out = key splits,
 * *merged_out = 1 when they are merged inside the kernel (one launch, no
 * workspace) and 0 when a workspace and a second (combine) launch are used,
 * *tcgen05_out = 1 on the tcgen05 path.  Outputs may be NULL. */
int rt_tree_attn_plan(int n, int num_q_heads, int num_kv_heads, int64_t prefix_len, int num_splits, int path,
                      int* splits_out, int* merged_out, int* tcgen05_out);

/* ------------------------------------------------------------------------
 * Tree-verify attention that allocates nothing.
 * No counterpart in the reference: an addition for callers that cannot
 * allocate device memory at the call -- code running during CUDA stream
 * capture (cudaMalloc is not allowed there), serving runtimes whose device
 * memory is all pre-reserved by their own pool, and C hosts with no allocator
 * to supply rt_tree_attn's workspace.
 *
 * Same arguments and results as rt_tree_attn without the workspace: the split
 * partials go to a fixed 16 MiB device array inside this library
 * (rt_tree_attn_noalloc_max_bytes()), held by every GPU that loads the
 * library until the process exits.  A shape whose rt_tree_attn_workspace_size
 * exceeds it returns RT_ERR_WORKSPACE.  The first call on a device looks the
 * array's address up for that device (that device must be current), so it
 * must come before any stream capture.  The looked-up address is kept for
 * the life of the process: after cudaDeviceReset (or anything else that
 * destroys the device's primary context) it is stale, and this entry point
 * must not be called on that device again.  Every call shares the one array:
 * calls that overlap on the GPU race on it.
 * ---------------------------------------------------------------------- */
size_t rt_tree_attn_noalloc_max_bytes(void);
int rt_tree_attn_noalloc(const void* q, int64_t q_tok_stride, int64_t q_head_stride, const void* k, const void* v,
                         int64_t kv_head_stride, int64_t kv_row_stride, int64_t kv_capacity, void* out,
                         int64_t out_tok_stride, int64_t out_head_stride, const uint32_t* mask, int mask_words,
                         int n, int64_t prefix_len, const int64_t* prefix_len_dev, int num_q_heads,
                         int num_kv_heads, int head_dim, float scale, int num_splits, int path, int* status,
                         rt_stream_t stream);

/* ------------------------------------------------------------------------
 * Packed ancestor bitmask from a dense additive mask.
 * Replaces reading the tree block of the mask compile_ddtree_tree writes
 * (ddtree.py:629-640): bit j of row i is set iff
 * dense[i*ld + col0 + j] == 0 (0 = visible, finfo.min = hidden).
 * dtype: 0 = fp32, 1 = bf16, 2 = fp16.  ld in elements.
 * ---------------------------------------------------------------------- */
int rt_mask_from_dense(const void* dense, int dtype, int64_t ld, int64_t col0, int n, uint32_t* mask,
                       int mask_words, rt_stream_t stream);

/* ------------------------------------------------------------------------
 * Draft top-k and log-normaliser.
 * Replaces torch.topk + torch.logsumexp + the subtraction of
 * ddtree.py:228-233 / :361-366, on the device and without the host copy.
 *
 * logits: rows x vocab, row stride `ld` elements, dtype 0 = fp32, 1 = bf16,
 * 2 = fp16 (values are widened to fp32 exactly, as .float() does).
 * Outputs: top_logp[r*k + j] = fp32(top_logit - log_z[r]), top_ids[r*k + j]
 * (int64), log_z[r].  Order: value descending, NaN first, equal values by
 * ascending vocabulary index.  1 <= k <= min(vocab, 1024).
 * ---------------------------------------------------------------------- */
size_t rt_draft_topk_workspace_size(int rows, int vocab, int k);
int rt_draft_topk(const void* logits, int dtype, int64_t ld, int rows, int vocab, int k, float* top_logp,
                  int64_t* top_ids, float* log_z, void* workspace, size_t workspace_bytes, rt_stream_t stream);

/* ------------------------------------------------------------------------
 * Budgeted best-first tree expansion (one CTA per request).
 * Replaces _build_ddtree_tree_original_heap (ddtree.py:200-308) and
 * _build_ddtree_tree_ngram (ddtree.py:311-535, with the n-gram table of
 * :113-151 and bonus of :154-197), i.e. build_ddtree_tree
 * (ddtree.py:538-589) after the top-k, plus the visibility of :520-528 as a
 * packed bitmask and the ids/positions of compile_ddtree_tree
 * (ddtree.py:618-627).
 *
 * strategy: 0 = original heap, 1 = n-gram, 2 = rank-gated n-gram (the
 * caller applies the reference's beta == 0 -> heap rule).  Scores are
 * accumulated in binary64 in the reference's order, so the tree is
 * bit-identical to the reference's for the same top_logp / top_ids.
 * ctx: context ids (int64, DEVICE) read only by the n-gram strategies; its
 * length is ctx_len, or ctx_len_dev[0] + ctx_len when ctx_len_dev is
 * non-NULL; the last min(length, ctx_window) ids form the window
 * (ddtree.py:135-136).
 * log1p_table (binary64, DEVICE): log1p(c) for c = 0..table_len-1,
 * table_len > window length.  order_weight (HOST array of max_n-1 doubles):
 * order_weight[n-2] = longer_weight**(n-2) for n = 2..max_n.  Outputs (DEVICE): node_tokens[budget], node_depths[budget]
 * (int64), parents[budget+1] (int32, parents[0] = -1), mask
 * [(budget+1) x mask_words] ancestor bits, count (int32, nodes emitted).
 * When verify_ids / verify_pos are non-NULL they receive
 * [root, node tokens] and start + [0, depths]; root is root_dev[0] when
 * root_dev is non-NULL, else the last context id when root < 0, else root;
 * start is start_dev[0] when start_dev is non-NULL, else start.
 * Limits: budget <= 1024, rows <= 64, max_n <= 8, ctx window <= 8192.
 * ---------------------------------------------------------------------- */
int rt_tree_build(const float* top_logp, const int64_t* top_ids, int rows, int k, int budget, int strategy,
                  const int64_t* ctx, int64_t ctx_len, const int64_t* ctx_len_dev, int ctx_window, int max_n,
                  double beta, int rank_cap, int min_count, int use_log_count, const double* order_weight,
                  double max_token_bonus, const double* log1p_table, int table_len, int64_t* node_tokens,
                  int64_t* node_depths, int32_t* parents, uint32_t* mask, int mask_words, int32_t* count,
                  int64_t* verify_ids, int64_t* verify_pos, int64_t root, const int64_t* root_dev,
                  int64_t start, const int64_t* start_dev, int* status, rt_stream_t stream);

/* ------------------------------------------------------------------------
 * Exact tree walk and commit bookkeeping.
 * Replaces follow_verified_tree (ddtree.py:650-663) and the commit of
 * ddtree.py:906-914 / retree.py:395-403 on the device.
 *
 * From the root, follow the child whose token equals posterior[current]
 * (int64[n]) while one exists (the highest-numbered such child when tokens
 * repeat, as a dict keyed by token keeps the last).  Writes accepted node
 * indices to accepted[0..len) (int64, accepted[0] = 0; directly usable as the
 * `keep` of rt_kv_compact), the length to accepted_len (int32) and
 * the target's next token to next_token.  When output_ids is non-NULL it
 * also writes the accepted tokens (verify_ids[accepted[i]]) to
 * output_ids[start + i] and next_token to output_ids[start + len], advances
 * start_dev[0] by len and keeps the start before the commit in start_dev[1]
 * (start_dev then holds two int64; start is read from start_dev[0]).
 * The tree is given by parents (int32[count+1]) and node tokens
 * (int64[count]); count from count_dev when non-NULL, else `count`.
 * ---------------------------------------------------------------------- */
int rt_tree_walk(const int32_t* parents, const int64_t* node_tokens, int count, const int32_t* count_dev,
                 const int64_t* posterior, int64_t* accepted, int32_t* accepted_len, int64_t* next_token,
                 const int64_t* verify_ids, int64_t* output_ids, int64_t output_len, int64_t* start_dev,
                 int* status, rt_stream_t stream);

/* ------------------------------------------------------------------------
 * Target-gated sibling-recovery walk on the device.
 * Replaces follow_verified_tree_with_recovery (retree.py:57-190) with the
 * RecoveryMemory reads and online updates it makes (model/recovery.py:35-298,
 * the gate :283-298, the stop check :269-280); no host syncs.
 *
 * The tree is given as in rt_tree_walk (parents int32[count+1], node tokens
 * int64[count], count from count_dev when non-NULL, <= the host count, which
 * is at most 1023).  posterior int64[count+1]; logits [count+1, >= vocab]
 * (row stride logits_ld elements, dtype 0 fp32 / 1 bf16: the gate
 * logit[draft] - logit[target] >= log(gate_threshold) is evaluated in that
 * dtype; gate_threshold <= 0 turns it off).  Walk: follow the child whose
 * token is the target's; at a mismatch (target not a stop id) rank the
 * children by target logit (ties in first-occurrence order), snapshot the
 * pair frequencies (prior + online) of the first rescue_top_k, add one online
 * count for each of the first record_top_k ranked children that differ from
 * the target (when online_update; stop pairs skipped), then move to the first
 * candidate whose snapshot frequency is >= freq_threshold and that passes the
 * gate; stop when none does.  stop_ids (int64[n_stop], DEVICE) is the
 * reference's disallow_rescue_target_ids; NULL means none.
 *
 * Recovery memory: open-addressing table of table_capacity (a power of two)
 * slots, key uint64 = draft << 32 | target (all ones = empty), slot =
 * splitmix64-mix(key) & (capacity - 1) with linear probing, prior / online
 * int32 counts per slot (retree_b200/recovery_device.py builds it).  Each
 * online increment is also appended as (draft, target) int32 to log_pairs at
 * *log_count (both may be NULL), up to log_capacity (RT_DEV_OVERFLOW beyond).
 * Outputs accepted / accepted_len / next_token as rt_tree_walk, rescued =
 * number of sibling rescues; output_ids / start_dev commit as in
 * rt_tree_walk when non-NULL.
 * ---------------------------------------------------------------------- */
int rt_recovery_walk(const int32_t* parents, const int64_t* node_tokens, int count, const int32_t* count_dev,
                     const int64_t* posterior, const void* logits, int64_t logits_ld, int logits_dtype,
                     int64_t vocab, double gate_threshold, int64_t freq_threshold, int rescue_top_k,
                     int record_top_k, int online_update, const int64_t* stop_ids, int n_stop, void* table_keys,
                     int32_t* table_prior, int32_t* table_online, int64_t table_capacity, int32_t* log_pairs,
                     int32_t* log_count, int log_capacity, int64_t* accepted, int32_t* accepted_len,
                     int64_t* next_token, int32_t* rescued, const int64_t* verify_ids, int64_t* output_ids,
                     int64_t output_len, int64_t* start_dev, int* status, rt_stream_t stream);

/* ------------------------------------------------------------------------
 * Elementwise stages of the target's verify forward (bf16, row-major,
 * contiguous, 16-byte aligned rows).  Each reproduces the bf16 rounding
 * points of the transformers ops it replaces; the projections between them
 * stay library GEMMs.
 *
 * rt_embed_rmsnorm: residual[r] = table[ids[r]] (table bf16[vocab, hidden]),
 *   out[r] = weight * bf16(residual[r] * rsqrt(mean(residual[r]^2) + eps)).
 *   Replaces the embedding lookup of Qwen3Model.forward plus the first
 *   Qwen3RMSNorm.forward (models/qwen3/modeling_qwen3.py:59-64).  An id
 *   outside [0, vocab) gives a zero row and RT_DEV_BAD_INDEX.
 * rt_add_rmsnorm: residual = bf16(residual + delta) (delta may be NULL: the
 *   norm of residual alone), out = weight * bf16(norm(residual)).  Replaces
 *   the residual adds of Qwen3DecoderLayer.forward (modeling_qwen3.py:327,
 *   :333) with the RMSNorm that follows each.  hidden % 8 == 0, <= 16384.
 * rt_qk_norm_rope_append: qkv is bf16[n, (Hq + 2 Hkv) * 128] ([q | k | v]
 *   heads).  Query and key heads get their per-head RMSNorm (weights
 *   bf16[128]; both NULL for models without one, modeling_qwen3.py:269-270)
 *   and the rotary embedding with cos/sin rows cos_table[positions[i]]
 *   (bf16[table_len, 128], :151-181); queries go to q_out bf16[n, Hq, 128],
 *   keys/values to row offset + i of k_cache/v_cache (+ g*cache_head_stride
 *   bytes for kv head g, cache_row_stride bytes per row), offset read from
 *   offset_dev (DEVICE) when non-NULL (cache_utils.py:102-121).  A row
 *   past `capacity` is not written (RT_DEV_OVERFLOW); a position outside the
 *   table gives RT_DEV_BAD_INDEX.
 * rt_silu_mul: out[r] = bf16(bf16(silu(gate)) * up) with gate_up[r] =
 *   [gate (inter) | up (inter)] (Qwen3MLP.forward, modeling_qwen3.py:81-83).
 * ---------------------------------------------------------------------- */
int rt_embed_rmsnorm(const int64_t* ids, const void* table, int64_t vocab, void* residual, const void* weight,
                     void* out, int rows, int hidden, float eps, int* status, rt_stream_t stream);
int rt_add_rmsnorm(const void* delta, void* residual, const void* weight, void* out, int rows, int hidden,
                   float eps, rt_stream_t stream);
int rt_qk_norm_rope_append(const void* qkv, int n, int num_q_heads, int num_kv_heads, int head_dim,
                           const void* q_norm_weight, const void* k_norm_weight, float eps, const void* cos_table,
                           const void* sin_table, int64_t table_len, const int64_t* positions, void* q_out,
                           void* k_cache, void* v_cache, int64_t cache_head_stride, int64_t cache_row_stride,
                           int64_t capacity, int64_t offset, const int64_t* offset_dev, int* status,
                           rt_stream_t stream);
int rt_silu_mul(const void* gate_up, void* out, int rows, int inter, rt_stream_t stream);

/* ------------------------------------------------------------------------
 * Projections of the verify forward on tcgen05 (bf16 in, fp32 accumulate):
 * Y[m, n_out] = X[m, k] . W[n_out, k]^T for m <= 512 tree nodes, with W
 * row-major contiguous (the nn.Linear weights of Qwen3Attention / Qwen3MLP,
 * models/qwen3/modeling_qwen3.py:236-247 and :70-83, and the lm_head).
 * X rows are ld_x elements apart.  n_out % 128 == 0, k % 8 == 0, X / W /
 * out 16-byte aligned, ld_x and ld_out multiples of 8.
 *
 * epilogue:
 *   RT_EPI_STORE     out[i, :n_out] = bf16(Y[i]) (row stride ld_out);
 *   RT_EPI_SILU_MUL  W = [gate; up] (n_out = 2 * inter): out[i, :inter] =
 *                    bf16(bf16(silu(bf16(Y[i, :inter]))) * bf16(Y[i, inter:]))
 *                    (Qwen3MLP.forward, modeling_qwen3.py:81-83);
 *   RT_EPI_QKV_ROPE  W = [Wq; Wk; Wv] (n_out = (Hq + 2 Hkv) * 128): what
 *                    rt_qk_norm_rope_append does with the bf16 result, with
 *                    the arguments of *qkv (out / ld_out unused);
 * When 128-row tiles alone do not cover the GPU, K is split over a cluster
 * of up to 8 CTAs whose partial sums are added in a fixed order over
 * distributed shared memory: no workspace, results independent of timing.
 * rt_linear_check returns RT_OK when rt_linear takes the shape.
 * ---------------------------------------------------------------------- */
#define RT_EPI_STORE 0
#define RT_EPI_SILU_MUL 1
#define RT_EPI_QKV_ROPE 2

typedef struct rt_qkv_epilogue {
  int num_q_heads;
  int num_kv_heads;
  const void* q_norm_weight; /* bf16[128] or NULL (no head norm; then k_norm_weight NULL too) */
  const void* k_norm_weight;
  float eps;
  const void* cos_table; /* bf16[table_len, 128] */
  const void* sin_table;
  int64_t table_len;
  const int64_t* positions; /* [m] */
  void* q_out;              /* bf16[m, Hq, 128] */
  void* k_cache;            /* + g*cache_head_stride + row*cache_row_stride bytes */
  void* v_cache;
  int64_t cache_head_stride;
  int64_t cache_row_stride;
  int64_t capacity;
  int64_t offset;
  const int64_t* offset_dev; /* DEVICE; added to offset when non-NULL */
} rt_qkv_epilogue;

int rt_linear_check(int m, int n_out, int k, int epilogue);
/* The launch rt_linear makes for this shape on the current device: K splits
 * (cluster size), ring stages and shared memory per CTA (diagnostics). */
int rt_linear_plan(int m, int n_out, int k, int epilogue, int* splits, int* stages, int* smem_bytes);
int rt_linear(const void* x, int64_t ld_x, int m, int k, const void* w, int n_out, int epilogue, void* out,
              int64_t ld_out, const rt_qkv_epilogue* qkv, int* status, rt_stream_t stream);

/* ------------------------------------------------------------------------
 * rt_linear (RT_EPI_STORE) that also returns each token's argmax over the
 * n_out outputs: index[t] = the first row of the largest bf16 value of out[t]
 * (NaN counts as the largest, -0.0 equals +0.0) -- sample(logits) at
 * temperature 0, model/utils.py:52-54, without a second pass over the
 * [m, n_out] logits.  keys is device scratch of m 8-byte words (zeroed here on
 * the stream); index is int64[m] on the device.
 * ---------------------------------------------------------------------- */
int rt_linear_argmax(const void* x, int64_t ld_x, int m, int k, const void* w, int n_out, void* out, int64_t ld_out,
                     void* keys, int64_t* index, int* status, rt_stream_t stream);

/* ------------------------------------------------------------------------
 * rt_linear (RT_EPI_STORE) whose X is gathered from the ranks of a KV-head
 * split as the K loop reaches it: rank r's columns [r*cols_per_rank,
 * (r+1)*cols_per_rank) of X are rows of x_ranks[r] (row stride ld_x
 * elements; peer memory for the other ranks, read with plain TMA loads), and
 * each CTA waits (bounded; RT_DEV_WAIT_TIMEOUT in *status) until
 * flags_local[r] >= *epoch_dev + epoch_add before its first load from rank r
 * -- the announcement rt_peer_signal makes.  Replaces the all-gather + o_proj
 * pair of the split with one launch whose transfers overlap the weight
 * stream.  cols_per_rank is a multiple of 64, k == world * cols_per_rank,
 * world <= 8; results equal rt_linear's on the gathered X.
 * ---------------------------------------------------------------------- */
int rt_linear_gather(const void* const* x_ranks, int world, int cols_per_rank, int64_t ld_x, int m, const void* w,
                     int n_out, int k, void* out, int64_t ld_out, const int64_t* flags_local, const int64_t* epoch_dev,
                     int64_t epoch_add, int* status, rt_stream_t stream);

#ifdef __cplusplus
}
#endif

#endif /* RETREE_B200_H */
