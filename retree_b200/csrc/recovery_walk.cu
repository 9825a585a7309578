// On-device target-gated sibling-recovery walk (retree.py:57-190 with the
// recovery memory of model/recovery.py:35-298): the walk of
// recovery_walk.cuh on one thread, its scratch in shared memory, the recovery
// memory as a device hash table that the walk reads (pre-update snapshot) and
// updates (online counts) in place, plus an optional log of the online
// increments for the cross-rank delta exchange.  Optionally commits the
// accepted tokens like rt_tree_walk.  Replaces the per-child .item() syncs of
// the reference's host walk.
#include "common.cuh"
#include "host_util.h"
#include "recovery_walk.cuh"

#include <math.h>

namespace rt {
namespace {

constexpr int kMaxWalkNodes = 1024;

size_t walk_scratch_bytes(int cap) { return align_up(static_cast<size_t>(21) * cap, 16); }

__global__ void recovery_walk_kernel(rec::WalkArgs a, int count, const int32_t* count_dev,
                                     const int64_t* verify_ids, int64_t* output_ids, int64_t output_len,
                                     int64_t* start_dev, int* status) {
  extern __shared__ __align__(16) unsigned char scratch[];
  if (threadIdx.x != 0) return;
  const int cap = count + 1;  // scratch is sized for the host's node bound
  const int cnt = count_dev != nullptr ? min(max(*count_dev, 0), count) : count;
  a.n = cnt + 1;
  a.child_tok = reinterpret_cast<int64_t*>(scratch);
  a.child_node = reinterpret_cast<int32_t*>(scratch + 8 * cap);
  a.child_score = reinterpret_cast<float*>(scratch + 12 * cap);
  a.order = reinterpret_cast<int32_t*>(scratch + 16 * cap);
  a.used = scratch + 20 * cap;
  int code = 0;
  a.status_code = &code;
  rec::recovery_walk(a);
  if (code != 0) set_status(status, code == 3 ? RT_DEV_BAD_INDEX : RT_DEV_OVERFLOW);
  if (output_ids != nullptr) {
    const int len = *a.accepted_len;
    const int64_t start = *start_dev;
    if (start < 0 || start + len >= output_len) {
      set_status(status, RT_DEV_OVERFLOW);
      return;
    }
    for (int i = 0; i < len; ++i) output_ids[start + i] = verify_ids[a.accepted[i]];
    output_ids[start + len] = *a.next_token;
    start_dev[1] = start;
    start_dev[0] = start + len;
  }
}

}  // namespace
}  // namespace rt

using namespace rt;

extern "C" int rt_recovery_walk(const int32_t* parents, const int64_t* node_tokens, int count,
                                const int32_t* count_dev, const int64_t* posterior, const void* logits,
                                int64_t logits_ld, int logits_dtype, int64_t vocab, double gate_threshold,
                                int64_t freq_threshold, int rescue_top_k, int record_top_k, int online_update,
                                const int64_t* stop_ids, int n_stop, void* table_keys, int32_t* table_prior,
                                int32_t* table_online, int64_t table_capacity, int32_t* log_pairs,
                                int32_t* log_count, int log_capacity, int64_t* accepted, int32_t* accepted_len,
                                int64_t* next_token, int32_t* rescued, const int64_t* verify_ids,
                                int64_t* output_ids, int64_t output_len, int64_t* start_dev, int* status,
                                rt_stream_t stream) {
  if (count < 0 || count + 1 > kMaxWalkNodes || !parents || !posterior || !logits || !accepted ||
      !accepted_len || !next_token || !rescued)
    return RT_ERR_INVALID_ARGUMENT;
  if (count > 0 && node_tokens == nullptr) return RT_ERR_INVALID_ARGUMENT;
  if ((logits_dtype != 0 && logits_dtype != 1) || vocab <= 0 || logits_ld < vocab) return RT_ERR_INVALID_ARGUMENT;
  if (!table_keys || !table_prior || !table_online || table_capacity <= 0 ||
      (table_capacity & (table_capacity - 1)) != 0)
    return RT_ERR_INVALID_ARGUMENT;
  if ((log_pairs == nullptr) != (log_count == nullptr) || log_capacity < 0) return RT_ERR_INVALID_ARGUMENT;
  if (stop_ids != nullptr && n_stop < 0) return RT_ERR_INVALID_ARGUMENT;
  if (output_ids != nullptr && (verify_ids == nullptr || start_dev == nullptr)) return RT_ERR_INVALID_ARGUMENT;
  rec::WalkArgs a{};
  a.parents = parents;
  a.tokens = node_tokens;
  a.posterior = posterior;
  a.logits = logits;
  a.ld = logits_ld;
  a.dtype = logits_dtype;
  a.vocab = vocab;
  a.gate_on = gate_threshold > 0.0 ? 1 : 0;
  float lt = a.gate_on ? static_cast<float>(log(gate_threshold)) : 0.f;
  a.log_thr = logits_dtype == 1 ? rec::round_to_bf16(lt) : lt;
  a.freq_threshold = freq_threshold;
  a.rescue_top_k = rescue_top_k;
  a.record_top_k = record_top_k;
  a.online_update = online_update;
  a.stop = stop_ids;
  a.n_stop = stop_ids != nullptr ? n_stop : 0;
  a.table = rec::Table{static_cast<unsigned long long*>(table_keys), table_prior, table_online, table_capacity};
  a.log_pairs = log_pairs;
  a.log_count = log_count;
  a.log_capacity = log_capacity;
  a.accepted = accepted;
  a.accepted_len = accepted_len;
  a.next_token = next_token;
  a.rescued = rescued;
  const size_t smem = walk_scratch_bytes(count + 1);
  recovery_walk_kernel<<<1, 32, smem, reinterpret_cast<cudaStream_t>(stream)>>>(
      a, count, count_dev, verify_ids, output_ids, output_len, start_dev, status);
  return check_launch();
}
