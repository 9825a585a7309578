"""Recovery memory for ReTree's target-gated sibling recovery.

The caller-facing API and the two JSON file layouts are those of the
reference's ``RecoveryMemory`` (model/recovery.py:35-266): an offline prior
and a causally updated online count per ``(draft_token, target_token)`` pair,
pre-update frequency snapshots, online deltas for the cross-rank exchange, the
flat prior file ``{"d,t": count}`` and the ``retree-recovery-state-v1``
runtime state.

Storage is one pair table instead of two dictionaries: pair ``(d, t)`` gets a
row the first time either count of it is touched, and the row holds both
counts side by side (``int64[rows, 2]``: column 0 the prior, column 1 the
online count).  The device table of ``recovery_device`` is filled from these
rows directly.  A pair is *present* in a column while its count there is
positive (counts only grow, except ``clear_online``), and each column also
keeps the order in which its pairs became present, which is the order the
reference's dictionaries iterate in (``prior_counts``, ``online_counts`` and
the tie order of ``top_k_pairs``).
"""

from __future__ import annotations

import json
import math
import os
from collections.abc import Iterable, Iterator, Mapping

import numpy as np

TokenPair = tuple[int, int]
STATE_FORMAT = "retree-recovery-state-v1"
PRIOR, ONLINE = 0, 1


def _key(draft: int, target: int) -> TokenPair:
    return int(draft), int(target)


def _pairs_to_json(items: Iterable[tuple[TokenPair, int]]) -> dict[str, int]:
    """``{"d,t": count}`` for the positive counts."""
    return {f"{d},{t}": int(c) for (d, t), c in items if int(c) > 0}


def _pairs_from_json(table: Mapping) -> list[tuple[TokenPair, int]]:
    """The ``(pair, count)`` entries of a ``{"d,t": count}`` object, file order, zero counts dropped."""
    out = []
    for text, value in table.items():
        fields = str(text).split(",")
        if len(fields) != 2:
            raise ValueError(f"recovery-memory pair {text!r} is not of the form 'draft,target'")
        count = int(value)
        if count < 0:
            raise ValueError(f"recovery-memory pair {text!r} has a negative count")
        if count:
            out.append(((int(fields[0]), int(fields[1])), count))
    return out


def _write_json_atomically(path: str, payload) -> None:
    """Write ``payload`` (sorted keys) to a temporary file beside ``path`` and rename it into place."""
    folder = os.path.dirname(path) or "."
    os.makedirs(folder, exist_ok=True)
    partial = f"{path}.tmp.{os.getpid()}"
    try:
        with open(partial, "w", encoding="utf-8") as f:
            json.dump(payload, f, sort_keys=True)
        os.replace(partial, path)
    finally:
        if os.path.exists(partial):
            os.remove(partial)


class RecoveryMemory:
    """Prior and online recovery counts of ``(draft_token, target_token)`` pairs (model/recovery.py:35-266)."""

    def __init__(self, freq_threshold: int = 6):
        if freq_threshold < 0:
            raise ValueError("freq_threshold cannot be negative")
        self.freq_threshold = int(freq_threshold)
        self._reset()

    # ---- the pair table ----------------------------------------------------
    def _reset(self) -> None:
        self._index: dict[TokenPair, int] = {}       # pair -> row
        self._pair_of: list[TokenPair] = []          # row -> pair
        self._counts = np.zeros((64, 2), dtype=np.int64)
        self._since = np.zeros((64, 2), dtype=np.int64)  # when the pair became present in each column
        self._clock = 0

    def _row(self, pair: TokenPair, create: bool) -> int:
        r = self._index.get(pair, -1)
        if r >= 0 or not create:
            return r
        r = len(self._pair_of)
        if r == len(self._counts):
            self._counts = np.concatenate([self._counts, np.zeros_like(self._counts)])
            self._since = np.concatenate([self._since, np.zeros_like(self._since)])
        self._index[pair] = r
        self._pair_of.append(pair)
        return r

    def _add(self, column: int, draft: int, target: int, count: int) -> None:
        count = int(count)
        if count < 0:
            raise ValueError("a recovery-memory count can only grow (negative increment)")
        if count == 0:
            return
        r = self._row(_key(draft, target), True)
        if self._counts[r, column] == 0:
            self._clock += 1
            self._since[r, column] = self._clock
        self._counts[r, column] += count

    def _count(self, column: int, draft: int, target: int) -> int:
        r = self._row(_key(draft, target), False)
        return 0 if r < 0 else int(self._counts[r, column])

    def _present(self, column: int) -> list[int]:
        """Rows whose count in ``column`` is positive, in the order they became so."""
        n = len(self._pair_of)
        rows = np.flatnonzero(self._counts[:n, column] > 0)
        return rows[np.argsort(self._since[rows, column], kind="stable")].tolist()

    def rows(self) -> Iterator[tuple[int, int, int, int]]:
        """``(draft, target, prior, online)`` for every pair with a positive count."""
        for r, (d, t) in enumerate(self._pair_of):
            p, o = int(self._counts[r, PRIOR]), int(self._counts[r, ONLINE])
            if p or o:
                yield d, t, p, o

    # ---- recording -----------------------------------------------------------
    def record_prior(self, draft_token: int, target_token: int, count: int = 1) -> None:
        """One offline calibration event (or ``count`` of them)."""
        self._add(PRIOR, draft_token, target_token, count)

    def record_online(self, draft_token: int, target_token: int, count: int = 1) -> None:
        """One event observed during this run's decoding (or ``count`` of them)."""
        self._add(ONLINE, draft_token, target_token, count)

    def _record_divergent_children(self, column: int, ranked_child_tokens: Iterable[int], target_token: int,
                                   top_k: int, stop_token_ids) -> int:
        """Count ``(child, target)`` for the first ``top_k`` ranked children that are neither the target
        nor part of a stop pair; returns how many were counted."""
        if top_k <= 0:
            return 0
        target = int(target_token)
        done = 0
        for child in map(int, ranked_child_tokens):
            if child == target or token_pair_has_stop(child, target, stop_token_ids):
                continue
            self._add(column, child, target, 1)
            done += 1
            if done == top_k:
                break
        return done

    def record_prior_divergences(self, ranked_child_tokens, target_token, top_k, stop_token_ids) -> int:
        return self._record_divergent_children(PRIOR, ranked_child_tokens, target_token, top_k, stop_token_ids)

    def record_online_divergences(self, ranked_child_tokens, target_token, top_k, stop_token_ids) -> int:
        return self._record_divergent_children(ONLINE, ranked_child_tokens, target_token, top_k, stop_token_ids)

    # ---- queries -----------------------------------------------------------
    def get_prior_frequency(self, draft_token: int, target_token: int) -> int:
        return self._count(PRIOR, draft_token, target_token)

    def get_online_frequency(self, draft_token: int, target_token: int) -> int:
        return self._count(ONLINE, draft_token, target_token)

    def get_frequency(self, draft_token: int, target_token: int) -> int:
        r = self._row(_key(draft_token, target_token), False)
        return 0 if r < 0 else int(self._counts[r].sum())

    def snapshot_frequencies(self, pairs: Iterable[TokenPair]) -> dict[TokenPair, int]:
        """Combined frequencies of ``pairs`` now (taken before the current mismatch is recorded)."""
        return {_key(*p): self.get_frequency(*p) for p in pairs}

    def is_frequent(self, draft_token: int, target_token: int) -> bool:
        return self.get_frequency(draft_token, target_token) >= self.freq_threshold

    def prior_counts(self) -> dict[TokenPair, int]:
        return {self._pair_of[r]: int(self._counts[r, PRIOR]) for r in self._present(PRIOR)}

    def online_counts(self) -> dict[TokenPair, int]:
        return {self._pair_of[r]: int(self._counts[r, ONLINE]) for r in self._present(ONLINE)}

    def top_k_pairs(self, k: int = 20) -> list[tuple[TokenPair, int]]:
        """The ``k`` pairs of largest combined count; ties in the order prior pairs, then online-only ones."""
        prior_rows = self._present(PRIOR)
        seen = set(prior_rows)
        order = prior_rows + [r for r in self._present(ONLINE) if r not in seen]
        items = [(self._pair_of[r], int(self._counts[r].sum())) for r in order]
        return sorted(items, key=lambda it: -it[1])[:k]

    def prior_total_pairs(self) -> int:
        return int((self._counts[:len(self._pair_of), PRIOR] > 0).sum())

    def online_total_pairs(self) -> int:
        return int((self._counts[:len(self._pair_of), ONLINE] > 0).sum())

    def total_pairs(self) -> int:
        return int((self._counts[:len(self._pair_of)].sum(axis=1) > 0).sum())

    def prior_total_events(self) -> int:
        return int(self._counts[:, PRIOR].sum())

    def online_total_events(self) -> int:
        return int(self._counts[:, ONLINE].sum())

    def total_rejections(self) -> int:
        return int(self._counts.sum())

    # ---- cross-rank exchange -------------------------------------------------
    def online_delta_since(self, snapshot: Mapping[TokenPair, int]) -> dict[TokenPair, int]:
        """Online counts gained since ``snapshot`` (an earlier ``online_counts()``), positive changes only."""
        delta: dict[TokenPair, int] = {}
        for r in self._present(ONLINE):
            pair = self._pair_of[r]
            gained = int(self._counts[r, ONLINE]) - int(snapshot.get(pair, 0))
            if gained < 0:
                raise ValueError(f"online count of {pair} is below the snapshot's")
            if gained:
                delta[pair] = gained
        return delta

    def apply_online_delta(self, delta: Mapping[TokenPair, int]) -> None:
        for (d, t), c in delta.items():
            self._add(ONLINE, d, t, c)

    def clear_online(self) -> None:
        self._counts[:, ONLINE] = 0
        self._since[:, ONLINE] = 0

    # ---- files ---------------------------------------------------------------
    def save_prior(self, path: str) -> None:
        """The prior alone, flat ``{"d,t": count}`` (the legacy layout)."""
        _write_json_atomically(path, _pairs_to_json(self.prior_counts().items()))

    def save_runtime_state(self, path: str) -> None:
        """Prior and online counts side by side (``retree-recovery-state-v1``)."""
        _write_json_atomically(path, {"format": STATE_FORMAT, "freq_threshold": self.freq_threshold,
                                      "prior_counts": _pairs_to_json(self.prior_counts().items()),
                                      "online_counts": _pairs_to_json(self.online_counts().items())})

    def load(self, path: str, load_online: bool = False) -> None:
        """Replace both tables from a file of either layout (or a legacy ``rescue_pairs`` one);
        online counts only when ``load_online``."""
        with open(path, "r", encoding="utf-8") as f:
            doc = json.load(f)
        if not isinstance(doc, dict):
            raise TypeError(f"{path}: a recovery-memory file holds one JSON object")
        online: object = {}
        if "prior_counts" in doc:
            prior = doc["prior_counts"]
            if load_online:
                online = doc.get("online_counts", {})
        else:
            prior = doc.get("rescue_pairs", doc)
        if not isinstance(prior, dict) or not isinstance(online, dict):
            raise TypeError(f"{path}: the count tables must be JSON objects")
        prior_items, online_items = _pairs_from_json(prior), _pairs_from_json(online)
        self._reset()
        for (d, t), c in prior_items:
            self._add(PRIOR, d, t, c)
        for (d, t), c in online_items:
            self._add(ONLINE, d, t, c)

    @staticmethod
    def from_file(path: str, freq_threshold: int = 6, load_online: bool = False) -> "RecoveryMemory":
        m = RecoveryMemory(freq_threshold=freq_threshold)
        m.load(path, load_online=load_online)
        return m


def token_pair_has_stop(draft_token: int, target_token: int, stop_token_ids) -> bool:
    """Whether either token of the pair is a stop token (model/recovery.py:269-280)."""
    return stop_token_ids is not None and (int(draft_token) in stop_token_ids or int(target_token) in stop_token_ids)


def target_logit_consistency_gate(target_logits, draft_token_id: int, target_top_token_id: int,
                                  position: int, threshold: float = 0.01) -> bool:
    """``exp(logit[draft] - logit[target]) >= threshold``, evaluated as a difference of logits in their own
    dtype against ``log(threshold)`` (model/recovery.py:283-298); always true for the target itself or a
    non-positive threshold."""
    if threshold <= 0 or int(draft_token_id) == int(target_top_token_id):
        return True
    row = target_logits[position]
    return bool((row[int(draft_token_id)] - row[int(target_top_token_id)] >= math.log(threshold)).item())
