"""Recovery memory and the target-gated sibling-recovery walk
(test infrastructure only; see ``oracle/__init__.py``).

Restates ``RecoveryMemory`` (model/recovery.py:35-266), the stop-pair and
logit-consistency gates (model/recovery.py:269-298) and
``follow_verified_tree_with_recovery`` (retree.py:25-190).
"""

from __future__ import annotations

import math
from collections import defaultdict

import numpy as np


class Memory:
    """Prior and online ``(draft, target) -> count`` tables (model/recovery.py:35-207)."""

    def __init__(self, freq_threshold: int = 6):
        if freq_threshold < 0:
            raise ValueError("freq_threshold must be non-negative")
        self.freq_threshold = int(freq_threshold)
        self.prior: dict = defaultdict(int)
        self.online: dict = defaultdict(int)

    def record_prior(self, d, t, count=1):
        if count < 0:
            raise ValueError("Recovery-memory updates must be non-negative")
        if count > 0:
            self.prior[(int(d), int(t))] += int(count)

    def record_online(self, d, t, count=1):
        if count < 0:
            raise ValueError("Recovery-memory updates must be non-negative")
        if count > 0:
            self.online[(int(d), int(t))] += int(count)

    def frequency(self, d, t) -> int:
        key = (int(d), int(t))
        return self.prior.get(key, 0) + self.online.get(key, 0)

    def record_online_divergences(self, ranked_children, target, top_k, stop_ids) -> int:
        """model/recovery.py:74-130: skip exact and stop pairs, record at most ``top_k``."""
        if top_k <= 0:
            return 0
        n = 0
        for c in ranked_children:
            c = int(c)
            if c == int(target) or pair_has_stop(c, target, stop_ids):
                continue
            self.record_online(c, target)
            n += 1
            if n >= top_k:
                break
        return n


def pair_has_stop(d, t, stop_ids) -> bool:
    """model/recovery.py:269-280."""
    return stop_ids is not None and (int(d) in stop_ids or int(t) in stop_ids)


def logit_gate(logits_row: np.ndarray, d: int, t: int, threshold: float) -> bool:
    """``logit[d] - logit[t] >= log(threshold)`` in fp32 (model/recovery.py:283-298)."""
    if int(d) == int(t) or threshold <= 0:
        return True
    diff = np.float32(logits_row[int(d)]) - np.float32(logits_row[int(t)])
    return bool(diff >= np.float32(math.log(threshold)))


def follow_with_recovery(maps, posterior, logits: np.ndarray, memory: Memory,
                         gate_threshold=0.01, online_update=True, record_top_k=8,
                         rescue_top_k=8, stop_ids=None):
    """ReTree's verifier walk (retree.py:57-190).

    Exact accept while the target's argmax is a child; at a mismatch, rank
    the children by target logit (descending), snapshot pair frequencies,
    optionally record the online divergences, then accept the first
    non-stop child whose pre-update frequency reaches the threshold and whose
    logit passes the consistency gate.  Returns ``(accepted, next, rescued)``.
    """
    post = [int(x) for x in np.asarray(posterior).reshape(-1)]
    logits = np.asarray(logits, dtype=np.float32)
    accepted = [0]
    cur = 0
    nxt = post[0]
    rescued = 0
    while True:
        children = maps[cur]
        if nxt in children:
            cur = children[nxt]
            accepted.append(cur)
            nxt = post[cur]
            continue
        if not children:
            break
        if stop_ids is not None and int(nxt) in stop_ids:
            break
        toks = list(children.keys())
        scores = logits[cur, toks]
        order = sorted(range(len(toks)), key=lambda j: -float(scores[j]))
        ranked = [(toks[j], children[toks[j]]) for j in order]
        candidates = ranked[:rescue_top_k]
        target = int(nxt)
        frequent = {c: memory.frequency(c, target) >= memory.freq_threshold
                    for c, _ in candidates if not pair_has_stop(c, target, stop_ids)}
        if online_update:
            memory.record_online_divergences([c for c, _ in ranked], target, record_top_k, stop_ids)
        moved = False
        for c, idx in candidates:
            if pair_has_stop(c, target, stop_ids) or not frequent.get(c, False):
                continue
            if not logit_gate(logits[cur], c, target, gate_threshold):
                continue
            cur = idx
            accepted.append(cur)
            rescued += 1
            nxt = post[cur]
            moved = True
            break
        if not moved:
            break
    return accepted, nxt, rescued
