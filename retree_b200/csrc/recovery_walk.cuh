// ReTree's target-gated sibling-recovery walk (retree.py:57-190 with
// model/recovery.py:35-298), written once for the device and the host.
//
// The walk is sequential (one step per accepted node, at most one mismatch
// handled per step), so it runs on a single thread on the GPU; the host build
// of the same code is what the CPU tests check against the reference's Python.
//
// Recovery memory: an open-addressing hash table of (draft token, target token)
// pairs with separate prior and online counts (the two tables of
// RecoveryMemory), linear probing, key = draft << 32 | target, empty slot =
// all ones.  Only the walk (and the host) write it, one thread at a time.
#pragma once

#include <stdint.h>

#ifdef __CUDACC__
#define RT_HD __host__ __device__ __forceinline__
#else
#define RT_HD inline
#endif

namespace rt {
namespace rec {

constexpr unsigned long long kEmptyKey = ~0ull;
constexpr int kMaxRescue = 64;  // rescue_top_k is clamped to this

RT_HD unsigned long long pair_key(int64_t draft, int64_t target) {
  return (static_cast<unsigned long long>(static_cast<uint32_t>(draft)) << 32) | static_cast<uint32_t>(target);
}

// splitmix64's output mix (Steele, Lea, Flood 2014)
RT_HD unsigned long long mix64(unsigned long long x) {
  x ^= x >> 30;
  x *= 0xbf58476d1ce4e5b9ull;
  x ^= x >> 27;
  x *= 0x94d049bb133111ebull;
  x ^= x >> 31;
  return x;
}

struct Table {
  unsigned long long* keys;  // [capacity]
  int32_t* prior;            // [capacity]
  int32_t* online;           // [capacity]
  int64_t capacity;          // a power of two
};

RT_HD int64_t table_find(const Table& t, unsigned long long key) {
  const int64_t mask = t.capacity - 1;
  int64_t s = static_cast<int64_t>(mix64(key) & static_cast<unsigned long long>(mask));
  for (int64_t i = 0; i < t.capacity; ++i) {
    const unsigned long long k = t.keys[s];
    if (k == key) return s;
    if (k == kEmptyKey) return -1;
    s = (s + 1) & mask;
  }
  return -1;
}

// Slot of `key`, inserted with zero counts if absent; -1 when the table is full.
RT_HD int64_t table_insert(const Table& t, unsigned long long key) {
  const int64_t mask = t.capacity - 1;
  int64_t s = static_cast<int64_t>(mix64(key) & static_cast<unsigned long long>(mask));
  for (int64_t i = 0; i < t.capacity; ++i) {
    const unsigned long long k = t.keys[s];
    if (k == key) return s;
    if (k == kEmptyKey) {
      t.keys[s] = key;
      t.prior[s] = 0;
      t.online[s] = 0;
      return s;
    }
    s = (s + 1) & mask;
  }
  return -1;
}

// prior + online count of a pair (RecoveryMemory.get_frequency)
RT_HD int64_t table_frequency(const Table& t, int64_t draft, int64_t target) {
  const int64_t s = table_find(t, pair_key(draft, target));
  return s < 0 ? 0 : static_cast<int64_t>(t.prior[s]) + t.online[s];
}

RT_HD float bf16_bits_to_float(uint16_t b) {
  union {
    uint32_t u;
    float f;
  } v;
  v.u = static_cast<uint32_t>(b) << 16;
  return v.f;
}

// Round-to-nearest-even of a float to bf16 precision, returned as a float
// (NaN stays NaN).
RT_HD float round_to_bf16(float x) {
  union {
    uint32_t u;
    float f;
  } v;
  v.f = x;
  if ((v.u & 0x7F800000u) == 0x7F800000u && (v.u & 0x007FFFFFu)) return x;
  const uint32_t lsb = (v.u >> 16) & 1u;
  v.u = (v.u + 0x7FFFu + lsb) & 0xFFFF0000u;
  return v.f;
}

struct WalkArgs {
  int n;                     // tree nodes, root included (<= 1024)
  const int32_t* parents;    // [n]; parents[0] unused
  const int64_t* tokens;     // [n - 1]: token of node i is tokens[i - 1]
  const int64_t* posterior;  // [n] target token at each node
  const void* logits;        // [n, >= vocab] target logits, row stride ld elements
  int64_t ld;
  int dtype;                 // 0 fp32, 1 bf16 (the gate's arithmetic follows it)
  int64_t vocab;
  int gate_on;               // gate_threshold > 0
  float log_thr;             // log(gate_threshold) rounded to the logits dtype
  int64_t freq_threshold;
  int rescue_top_k, record_top_k, online_update;
  const int64_t* stop;       // stop token ids (disallow_rescue_target_ids) or NULL for none
  int n_stop;
  Table table;
  int32_t* log_pairs;        // online increments, (draft, target) per entry; may be NULL
  int32_t* log_count;        // entries written (read and advanced)
  int log_capacity;
  // outputs
  int64_t* accepted;         // [n]
  int32_t* accepted_len;
  int64_t* next_token;
  int32_t* rescued;
  int* status_code;          // first error: 1 table full, 2 log full, 3 token outside the logits
  // scratch, n entries each
  int64_t* child_tok;
  int32_t* child_node;
  float* child_score;
  int32_t* order;
  uint8_t* used;
};

RT_HD bool is_stop(const WalkArgs& a, int64_t tok) {
  if (a.stop == nullptr) return false;
  for (int i = 0; i < a.n_stop; ++i)
    if (a.stop[i] == tok) return true;
  return false;
}

RT_HD void set_code(const WalkArgs& a, int code) {
  if (a.status_code != nullptr && *a.status_code == 0) *a.status_code = code;
}

RT_HD float logit_at(const WalkArgs& a, int row, int64_t tok, bool* ok) {
  if (tok < 0 || tok >= a.vocab) {
    *ok = false;
    return 0.f;
  }
  *ok = true;
  const int64_t idx = static_cast<int64_t>(row) * a.ld + tok;
  if (a.dtype == 0) return static_cast<const float*>(a.logits)[idx];
  return bf16_bits_to_float(static_cast<const uint16_t*>(a.logits)[idx]);
}

// logit[draft] - logit[target] >= log(threshold), evaluated in the logits'
// dtype like the reference's tensor expression (model/recovery.py:283-298):
// the difference is rounded to that dtype, and so is the python-float bound.
RT_HD bool gate_passes(const WalkArgs& a, int row, int64_t draft, int64_t target) {
  if (draft == target || !a.gate_on) return true;
  bool ok1, ok2;
  const float x = logit_at(a, row, draft, &ok1);
  const float y = logit_at(a, row, target, &ok2);
  if (!ok1 || !ok2) {
    set_code(a, 3);
    return false;
  }
  float d = x - y;
  if (a.dtype == 1) d = round_to_bf16(d);
  return d >= a.log_thr;
}

RT_HD void recovery_walk(const WalkArgs& a) {
  int len = 0;
  a.accepted[len++] = 0;
  int cur = 0;
  int64_t nxt = a.posterior[0];
  int rescued = 0;
  const int rescue_k = a.rescue_top_k < kMaxRescue ? a.rescue_top_k : kMaxRescue;
  int64_t snap[kMaxRescue];
  for (int step = 0; step < a.n; ++step) {
    // children of cur as the reference's dict {token: node}: first occurrence
    // fixes the order, the last node with a token wins
    int nc = 0;
    for (int i = 1; i < a.n; ++i) {
      if (a.parents[i] != cur) continue;
      const int64_t t = a.tokens[i - 1];
      int j = 0;
      while (j < nc && a.child_tok[j] != t) ++j;
      if (j == nc) {
        a.child_tok[nc] = t;
        a.child_node[nc] = i;
        ++nc;
      } else {
        a.child_node[j] = i;
      }
    }
    int hit = -1;
    for (int j = 0; j < nc && hit < 0; ++j)
      if (a.child_tok[j] == nxt) hit = j;
    // every accepted node lies one level below the previous one, so a tree of
    // n nodes accepts at most n; a parent array with a cycle stops here
    if (len >= a.n) break;
    if (hit >= 0) {  // exact accept
      cur = a.child_node[hit];
      a.accepted[len++] = cur;
      nxt = a.posterior[cur];
      continue;
    }
    if (nc == 0) break;
    if (a.stop != nullptr && is_stop(a, nxt)) break;
    const int64_t target = nxt;
    for (int j = 0; j < nc; ++j) {
      bool ok;
      a.child_score[j] = logit_at(a, cur, a.child_tok[j], &ok);
      if (!ok) set_code(a, 3);
      a.used[j] = 0;
    }
    // children by descending target logit (NaN above every number, as a
    // descending sort puts it), ties in dict order, produced on demand
    int have = 0;
    auto ranked = [&](int r) -> int {
      while (have <= r) {
        int best = -1;
        for (int j = 0; j < nc; ++j) {
          if (a.used[j]) continue;
          if (best < 0) {
            best = j;
            continue;
          }
          const float sj = a.child_score[j], sb = a.child_score[best];
          if ((sj != sj && sb == sb) || sj > sb) best = j;
        }
        a.used[best] = 1;
        a.order[have++] = best;
      }
      return a.order[r];
    };
    const int ncand = rescue_k < nc ? (rescue_k > 0 ? rescue_k : 0) : nc;
    // pre-update snapshot of the candidates' frequencies (stop pairs are never frequent)
    for (int r = 0; r < ncand; ++r) {
      const int64_t c = a.child_tok[ranked(r)];
      snap[r] = (is_stop(a, c) || is_stop(a, target)) ? -1 : table_frequency(a.table, c, target);
    }
    // causal online update: up to record_top_k ranked children that differ from the target
    if (a.online_update && a.record_top_k > 0) {
      int recorded = 0;
      for (int r = 0; r < nc && recorded < a.record_top_k; ++r) {
        const int64_t c = a.child_tok[ranked(r)];
        if (c == target || is_stop(a, c) || is_stop(a, target)) continue;
        const int64_t s = table_insert(a.table, pair_key(c, target));
        if (s < 0) {
          set_code(a, 1);
        } else {
          a.table.online[s] += 1;
          if (a.log_pairs != nullptr && a.log_count != nullptr) {
            const int e = *a.log_count;
            if (e < a.log_capacity) {
              a.log_pairs[2 * e] = static_cast<int32_t>(c);
              a.log_pairs[2 * e + 1] = static_cast<int32_t>(target);
              *a.log_count = e + 1;
            } else {
              set_code(a, 2);
            }
          }
        }
        ++recorded;
      }
    }
    bool moved = false;
    for (int r = 0; r < ncand && !moved; ++r) {
      const int j = ranked(r);
      const int64_t c = a.child_tok[j];
      if (snap[r] < 0 || snap[r] < a.freq_threshold) continue;
      if (!gate_passes(a, cur, c, target)) continue;
      cur = a.child_node[j];
      a.accepted[len++] = cur;
      ++rescued;
      nxt = a.posterior[cur];
      moved = true;
    }
    if (!moved) break;
  }
  *a.accepted_len = len;
  *a.next_token = nxt;
  *a.rescued = rescued;
}

}  // namespace rec
}  // namespace rt
