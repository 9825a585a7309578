"""Recovery memory for ReTree's target-gated sibling recovery.

Host-side state with the reference's interface and file formats
(model/recovery.py:13-298): a fixed offline prior and a causally updated
online table of ``(draft_token, target_token) -> count``, pre-update frequency
snapshots, online deltas for cross-rank synchronisation, and the two JSON
layouts (``retree-recovery-state-v1`` runtime state and the legacy flat prior).
"""

from __future__ import annotations

import json
import math
import os
from collections import defaultdict
from collections.abc import Iterable, Mapping

TokenPair = tuple[int, int]
STATE_FORMAT = "retree-recovery-state-v1"


def _encode(counts: Mapping[TokenPair, int]) -> dict[str, int]:
    return {f"{d},{t}": int(c) for (d, t), c in counts.items() if int(c) > 0}


def _decode(serialized: Mapping[str, int]) -> dict[TokenPair, int]:
    out: dict[TokenPair, int] = {}
    for key, value in serialized.items():
        parts = str(key).split(",")
        if len(parts) != 2:
            raise ValueError(f"Invalid recovery-memory key: {key!r}")
        c = int(value)
        if c < 0:
            raise ValueError(f"Recovery-memory counts must be non-negative: {key!r}")
        if c > 0:
            out[(int(parts[0]), int(parts[1]))] = c
    return out


class RecoveryMemory:
    """Two-stage recovery memory with a fixed prior and causal online counts (model/recovery.py:35)."""

    def __init__(self, freq_threshold: int = 6):
        if freq_threshold < 0:
            raise ValueError("freq_threshold must be non-negative")
        self.freq_threshold = int(freq_threshold)
        self._prior_counts: dict[TokenPair, int] = defaultdict(int)
        self._online_counts: dict[TokenPair, int] = defaultdict(int)

    @staticmethod
    def _add(table, draft_token, target_token, count=1):
        count = int(count)
        if count < 0:
            raise ValueError("Recovery-memory updates must be non-negative")
        if count > 0:
            table[(int(draft_token), int(target_token))] += count

    def record_prior(self, draft_token: int, target_token: int, count: int = 1) -> None:
        self._add(self._prior_counts, draft_token, target_token, count)

    def record_online(self, draft_token: int, target_token: int, count: int = 1) -> None:
        self._add(self._online_counts, draft_token, target_token, count)

    def _record_ranked(self, ranked_child_tokens: Iterable[int], target_token: int, top_k: int,
                       stop_token_ids, online: bool) -> int:
        if top_k <= 0:
            return 0
        target_token = int(target_token)
        n = 0
        for child in ranked_child_tokens:
            child = int(child)
            if child == target_token or token_pair_has_stop(child, target_token, stop_token_ids):
                continue
            (self.record_online if online else self.record_prior)(child, target_token)
            n += 1
            if n >= top_k:
                break
        return n

    def record_prior_divergences(self, ranked_child_tokens, target_token, top_k, stop_token_ids) -> int:
        return self._record_ranked(ranked_child_tokens, target_token, top_k, stop_token_ids, online=False)

    def record_online_divergences(self, ranked_child_tokens, target_token, top_k, stop_token_ids) -> int:
        return self._record_ranked(ranked_child_tokens, target_token, top_k, stop_token_ids, online=True)

    def get_prior_frequency(self, draft_token: int, target_token: int) -> int:
        return self._prior_counts.get((int(draft_token), int(target_token)), 0)

    def get_online_frequency(self, draft_token: int, target_token: int) -> int:
        return self._online_counts.get((int(draft_token), int(target_token)), 0)

    def get_frequency(self, draft_token: int, target_token: int) -> int:
        key = (int(draft_token), int(target_token))
        return self._prior_counts.get(key, 0) + self._online_counts.get(key, 0)

    def snapshot_frequencies(self, pairs: Iterable[TokenPair]) -> dict[TokenPair, int]:
        return {(int(d), int(t)): self.get_frequency(d, t) for d, t in pairs}

    def is_frequent(self, draft_token: int, target_token: int) -> bool:
        return self.get_frequency(draft_token, target_token) >= self.freq_threshold

    def prior_counts(self) -> dict[TokenPair, int]:
        return dict(self._prior_counts)

    def online_counts(self) -> dict[TokenPair, int]:
        return dict(self._online_counts)

    def online_delta_since(self, snapshot: Mapping[TokenPair, int]) -> dict[TokenPair, int]:
        delta: dict[TokenPair, int] = {}
        for pair, current in self._online_counts.items():
            change = int(current) - int(snapshot.get(pair, 0))
            if change < 0:
                raise ValueError("Online recovery-memory counts cannot decrease")
            if change > 0:
                delta[pair] = change
        return delta

    def apply_online_delta(self, delta: Mapping[TokenPair, int]) -> None:
        for (d, t), c in delta.items():
            self.record_online(d, t, count=int(c))

    def clear_online(self) -> None:
        self._online_counts = defaultdict(int)

    def _combined(self) -> dict[TokenPair, int]:
        out = dict(self._prior_counts)
        for pair, c in self._online_counts.items():
            out[pair] = out.get(pair, 0) + c
        return out

    def top_k_pairs(self, k: int = 20) -> list[tuple[TokenPair, int]]:
        return sorted(self._combined().items(), key=lambda it: it[1], reverse=True)[:k]

    def prior_total_pairs(self) -> int:
        return len(self._prior_counts)

    def online_total_pairs(self) -> int:
        return len(self._online_counts)

    def total_pairs(self) -> int:
        return len(self._combined())

    def prior_total_events(self) -> int:
        return sum(self._prior_counts.values())

    def online_total_events(self) -> int:
        return sum(self._online_counts.values())

    def total_rejections(self) -> int:
        return self.prior_total_events() + self.online_total_events()

    def save_prior(self, path: str) -> None:
        """The prior alone, in the legacy flat ``{"d,t": count}`` layout."""
        _atomic_json(path, _encode(self._prior_counts))

    def save_runtime_state(self, path: str) -> None:
        """Prior and online tables kept apart (``retree-recovery-state-v1``)."""
        _atomic_json(path, {
            "format": STATE_FORMAT,
            "freq_threshold": self.freq_threshold,
            "prior_counts": _encode(self._prior_counts),
            "online_counts": _encode(self._online_counts),
        })

    def load(self, path: str, load_online: bool = False) -> None:
        with open(path, "r", encoding="utf-8") as f:
            payload = json.load(f)
        if not isinstance(payload, dict):
            raise TypeError("Recovery-memory files must contain a JSON object")
        if "prior_counts" in payload:
            prior = payload["prior_counts"]
            online = payload.get("online_counts", {}) if load_online else {}
        elif "rescue_pairs" in payload:
            prior, online = payload["rescue_pairs"], {}
        else:
            prior, online = payload, {}
        if not isinstance(prior, dict) or not isinstance(online, dict):
            raise TypeError("Recovery-memory count tables must be JSON objects")
        self._prior_counts = defaultdict(int, _decode(prior))
        self._online_counts = defaultdict(int, _decode(online))

    @staticmethod
    def from_file(path: str, freq_threshold: int = 6, load_online: bool = False) -> "RecoveryMemory":
        m = RecoveryMemory(freq_threshold=freq_threshold)
        m.load(path, load_online=load_online)
        return m


def _atomic_json(path: str, payload) -> None:
    directory = os.path.dirname(path) or "."
    os.makedirs(directory, exist_ok=True)
    tmp = f"{path}.tmp.{os.getpid()}"
    try:
        with open(tmp, "w", encoding="utf-8") as f:
            json.dump(payload, f, sort_keys=True)
        os.replace(tmp, path)
    finally:
        if os.path.exists(tmp):
            os.remove(tmp)


def token_pair_has_stop(draft_token: int, target_token: int, stop_token_ids) -> bool:
    """Either side of the pair is a stop token (model/recovery.py:269-280)."""
    if stop_token_ids is None:
        return False
    return int(draft_token) in stop_token_ids or int(target_token) in stop_token_ids


def target_logit_consistency_gate(target_logits, draft_token_id: int, target_top_token_id: int,
                                  position: int, threshold: float = 0.01) -> bool:
    """``logit[draft] - logit[target] >= log(threshold)`` in the logits' dtype (model/recovery.py:283-298)."""
    if int(draft_token_id) == int(target_top_token_id) or threshold <= 0:
        return True
    a = target_logits[position, int(draft_token_id)]
    b = target_logits[position, int(target_top_token_id)]
    return bool((a - b >= math.log(threshold)).item())
