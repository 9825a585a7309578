// Host build of the recovery walk (retree_b200/csrc/recovery_walk.cuh) for the
// CPU tests: the same code the GPU kernel runs, called through ctypes.
#include <stdlib.h>

#include <vector>

#include "../../retree_b200/csrc/recovery_walk.cuh"

extern "C" int host_recovery_walk(int n, const int32_t* parents, const int64_t* tokens, const int64_t* posterior,
                                  const void* logits, int64_t ld, int dtype, int64_t vocab, int gate_on, float log_thr,
                                  int64_t freq_threshold, int rescue_top_k, int record_top_k, int online_update,
                                  const int64_t* stop, int n_stop, unsigned long long* keys, int32_t* prior,
                                  int32_t* online, int64_t capacity, int32_t* log_pairs, int32_t* log_count,
                                  int log_capacity, int64_t* accepted, int32_t* accepted_len, int64_t* next_token,
                                  int32_t* rescued) {
  std::vector<int64_t> tok(n);
  std::vector<int32_t> node(n), order(n);
  std::vector<float> score(n);
  std::vector<uint8_t> used(n);
  int code = 0;
  rt::rec::WalkArgs a{};
  a.n = n;
  a.parents = parents;
  a.tokens = tokens;
  a.posterior = posterior;
  a.logits = logits;
  a.ld = ld;
  a.dtype = dtype;
  a.vocab = vocab;
  a.gate_on = gate_on;
  a.log_thr = log_thr;
  a.freq_threshold = freq_threshold;
  a.rescue_top_k = rescue_top_k;
  a.record_top_k = record_top_k;
  a.online_update = online_update;
  a.stop = stop;
  a.n_stop = n_stop;
  a.table = rt::rec::Table{keys, prior, online, capacity};
  a.log_pairs = log_pairs;
  a.log_count = log_count;
  a.log_capacity = log_capacity;
  a.accepted = accepted;
  a.accepted_len = accepted_len;
  a.next_token = next_token;
  a.rescued = rescued;
  a.status_code = &code;
  a.child_tok = tok.data();
  a.child_node = node.data();
  a.child_score = score.data();
  a.order = order.data();
  a.used = used.data();
  rt::rec::recovery_walk(a);
  return code;
}

extern "C" float host_round_to_bf16(float x) { return rt::rec::round_to_bf16(x); }
