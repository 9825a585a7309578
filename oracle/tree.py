"""CPU restatement of ReTree's tree construction, mask compile, exact walk and
KV compaction (test infrastructure only; see ``oracle/__init__.py``).

Every function names the reference code it restates as ``file:line`` inside
Adamlong3/ReTree.  Arithmetic that decides tree structure is done exactly as the
reference does it: fp32 log-probs widened to Python floats (IEEE binary64) and
combined in the same order, and candidates ordered by the same tuple keys that
``heapq`` compares in the reference.
"""

from __future__ import annotations

import dataclasses
import heapq
import os
from typing import Sequence

import numpy as np

# ---------------------------------------------------------------------------
# Strategy names (ddtree.py:564-589)
# ---------------------------------------------------------------------------
STRATEGY_HEAP = "heap"
STRATEGY_NGRAM = "ngram"
STRATEGY_RANK_GATED = "rank_gated_ngram"

_STRATEGY_ALIASES = {
    "heap": STRATEGY_HEAP,
    "original": STRATEGY_HEAP,
    "default": STRATEGY_HEAP,
    "ngram": STRATEGY_NGRAM,
    "ngram_continuity": STRATEGY_NGRAM,
    "continuity": STRATEGY_NGRAM,
    "rank_gated_ngram": STRATEGY_RANK_GATED,
    "fast_rank_gated_ngram": STRATEGY_RANK_GATED,
}


def canonical_strategy(name: str) -> str:
    """Map a ``DDTREE_TREE_STRATEGY`` value to its builder (ddtree.py:564-589)."""
    key = name.strip().lower()
    if key not in _STRATEGY_ALIASES:
        raise ValueError(
            f"Unknown DDTREE_TREE_STRATEGY={key}. Use one of: heap, ngram, rank_gated_ngram."
        )
    return _STRATEGY_ALIASES[key]


@dataclasses.dataclass(frozen=True)
class NgramParams:
    """The n-gram knobs read by ddtree.py:346-354 (defaults are the reference's)."""

    max_n: int = 4
    beta: float = 0.15
    rank_cap: int = 8
    min_count: int = 1
    context_window: int = 2048
    use_log_count: bool = True
    longer_weight: float = 1.5
    max_token_bonus: float = 6.0
    exact_beta0: bool = True

    @staticmethod
    def from_env(env: dict | None = None) -> "NgramParams":
        e = os.environ if env is None else env
        return NgramParams(
            max_n=max(2, int(e.get("DDTREE_NGRAM_MAX_N", "4"))),
            beta=float(e.get("DDTREE_NGRAM_BETA", "0.15")),
            rank_cap=int(e.get("DDTREE_NGRAM_RANK_CAP", "8")),
            min_count=int(e.get("DDTREE_NGRAM_MIN_COUNT", "1")),
            context_window=int(e.get("DDTREE_NGRAM_CONTEXT_WINDOW", "2048")),
            use_log_count=e.get("DDTREE_NGRAM_USE_LOG_COUNT", "1") != "0",
            longer_weight=float(e.get("DDTREE_NGRAM_LONGER_WEIGHT", "1.5")),
            max_token_bonus=float(e.get("DDTREE_NGRAM_MAX_TOKEN_BONUS", "6.0")),
            exact_beta0=e.get("DDTREE_NGRAM_EXACT_BETA0", "1") != "0",
        )


# ---------------------------------------------------------------------------
# Top-k and log-normaliser (ddtree.py:228-237, :361-370)
# ---------------------------------------------------------------------------
def topk_logz(logits: np.ndarray, k: int):
    """Row-wise top-k of fp32 logits plus logsumexp, as ddtree.py:362-365 uses them.

    Order: value descending; NaN above everything (torch.topk's order); equal
    values by ascending vocabulary index.  ``torch.topk`` leaves the order of
    equal values unspecified, so this index rule is the contract the device
    kernel is held to.  ``log_z`` is computed in binary64 and rounded to fp32;
    torch's fp32 reduction agrees with it to a few ulp.

    Returns ``(top_logp f32[R,k], top_ids i64[R,k], log_z f32[R], top_logits f32[R,k])``
    with ``top_logp = fp32(top_logits - log_z)`` (ddtree.py:365).
    """
    x = np.ascontiguousarray(logits, dtype=np.float32)
    rows, vocab = x.shape
    k = int(min(k, vocab))
    ids = np.empty((rows, k), dtype=np.int64)
    for r in range(rows):
        row = x[r]
        nan = np.isnan(row)
        neg = np.where(nan, -np.inf, -row.astype(np.float64))
        order = np.lexsort((np.arange(vocab), neg, ~nan))
        ids[r] = order[:k]
    top = np.take_along_axis(x, ids, axis=1)
    x64 = x.astype(np.float64)
    has_nan = np.isnan(x64).any(axis=1)
    m = np.where(has_nan, np.nan, np.nanmax(np.where(np.isnan(x64), -np.inf, x64), axis=1))
    with np.errstate(invalid="ignore", over="ignore"):
        lse = m + np.log(np.exp(x64 - m[:, None]).sum(axis=1))
    # torch.logsumexp: +inf if any +inf (and no NaN), -inf if all -inf, NaN if any NaN
    lse = np.where(np.isinf(m), m, lse)
    log_z = lse.astype(np.float32)
    with np.errstate(invalid="ignore"):
        top_logp = (top - log_z[:, None]).astype(np.float32)
    return top_logp, ids, log_z, top


# ---------------------------------------------------------------------------
# Online n-gram continuity bonus (ddtree.py:113-197, :372-420)
# ---------------------------------------------------------------------------
def context_window(context_ids, window: int) -> list[int]:
    """The request-local context the n-gram table is built from (ddtree.py:127-138)."""
    if context_ids is None:
        return []
    ctx = np.asarray(context_ids).reshape(-1).astype(np.int64).tolist()
    if window > 0 and len(ctx) > window:
        ctx = ctx[-window:]
    return [int(t) for t in ctx]


class NgramCounter:
    """Counts of ``(prefix of 1..max_n-1 tokens) -> next`` over a context window.

    Restates the table of ddtree.py:113-151 by direct search over the window:
    ``count(prefix, token)`` is the number of positions ``i`` with
    ``ctx[i:i+len(prefix)] == prefix`` and ``ctx[i+len(prefix)] == token``.
    """

    def __init__(self, ctx: Sequence[int], max_n: int):
        self.ctx = np.asarray(ctx, dtype=np.int64)
        self.max_n = max_n
        self._views = {}

    def count(self, prefix: tuple[int, ...], token: int) -> int:
        p = len(prefix)
        if len(self.ctx) <= p:
            return 0
        if p not in self._views:
            self._views[p] = np.lib.stride_tricks.sliding_window_view(self.ctx, p + 1)
        pattern = np.asarray(prefix + (int(token),), dtype=np.int64)
        return int(np.all(self._views[p] == pattern, axis=1).sum())


def ngram_bonus(counter: NgramCounter, parent_tail: tuple[int, ...], token: int,
                params: NgramParams) -> float:
    """``min(sum_n w^(n-2) * log1p(count_n), cap)`` of ddtree.py:154-186.

    Accumulated in ascending ``n`` in binary64, term by term, as the reference does.
    """
    # The reference's table is empty (bonus 0) unless the window holds a pair.
    if counter is None or len(counter.ctx) < 2 or params.max_n < 2:
        return 0.0
    total = 0.0
    for n in range(2, params.max_n + 1):
        p = n - 1
        if len(parent_tail) < p:
            continue
        c = counter.count(tuple(parent_tail[-p:]), token)
        if c < params.min_count:
            continue
        base = float(np.log1p(c)) if params.use_log_count else 1.0
        weight = float(params.longer_weight ** max(0, n - 2))
        total += weight * base
    if params.max_token_bonus > 0:
        total = min(total, params.max_token_bonus)
    return float(total)


def _extend_tail(tail: tuple[int, ...], token: int, size: int) -> tuple[int, ...]:
    """Last ``size`` tokens after appending ``token`` (ddtree.py:189-197)."""
    if size <= 0:
        return ()
    return (tail + (int(token),))[-size:]


# ---------------------------------------------------------------------------
# Tree builders
# ---------------------------------------------------------------------------
@dataclasses.dataclass
class Tree:
    tokens: np.ndarray      # int64 [count]      node token ids (node i+1)
    depths: np.ndarray      # int64 [count]      node depths (root depth 0 excluded)
    parents: list[int]      # [count+1]          parents[0] == -1
    ranks: list[int]        # [count+1]          draft rank of each node (root 0)

    @property
    def count(self) -> int:
        return int(self.tokens.shape[0])


def _empty_tree() -> Tree:
    return Tree(np.empty(0, np.int64), np.empty(0, np.int64), [-1], [0])


def build_tree_heap(top_logp: np.ndarray, top_ids: np.ndarray, budget: int) -> Tree:
    """Best-first DDTree expansion by cumulative draft log-prob (ddtree.py:200-308).

    Candidate order: ``(-logw, rank path from the root)``, ascending; the rank
    path is the tuple that breaks ties in the reference's heap tuple
    (ddtree.py:241-243, :271-289).
    """
    rows, k = top_logp.shape
    if budget <= 0 or rows == 0:
        return _empty_tree()
    lp = top_logp.astype(np.float32)
    first = float(lp[0, 0])
    # heap entries: (-score, rank_path, parent, depth, rank, score)
    frontier = [(-first, (0,), 0, 1, 0, first)]
    tokens, depths, parents, ranks = [], [], [-1], [0]
    while frontier and len(tokens) < budget:
        _, path, parent, depth, rank, score = heapq.heappop(frontier)
        me = len(tokens) + 1
        tokens.append(int(top_ids[depth - 1, rank]))
        depths.append(depth)
        parents.append(parent)
        ranks.append(rank)
        if rank + 1 < k:
            s = score - float(lp[depth - 1, rank]) + float(lp[depth - 1, rank + 1])
            heapq.heappush(frontier, (-s, path[:-1] + (rank + 1,), parent, depth, rank + 1, s))
        if depth < rows:
            s = score + float(lp[depth, 0])
            heapq.heappush(frontier, (-s, path + (0,), me, depth + 1, 0, s))
    return Tree(np.asarray(tokens, np.int64), np.asarray(depths, np.int64), parents, ranks)


def build_tree_ngram(top_logp: np.ndarray, top_ids: np.ndarray, budget: int,
                     context_ids, params: NgramParams, rank_gated: bool) -> Tree:
    """Online n-gram DDTree (ddtree.py:311-535): score = sum logp + beta * bonus.

    Candidate order: ``(-aug, parent index, rank)`` ascending — the leading
    fields of the reference's heap tuple (ddtree.py:432-434, :478-516), which
    already identify a candidate uniquely.  Score updates follow the
    reference's operation order: sibling ``(logw - lp[r]) + lp[r+1]`` and
    ``(bonus - inc_self) + inc_sibling``; child ``logw + lp[d, 0]`` and
    ``bonus + inc_child``; ``aug = logw + bonus``.
    """
    rows, k = top_logp.shape
    if budget <= 0 or rows == 0:
        return _empty_tree()
    if abs(params.beta) < 1e-12 and params.exact_beta0:
        return build_tree_heap(top_logp, top_ids, budget)
    lp = top_logp.astype(np.float32)
    tail_size = params.max_n - 1
    ctx = context_window(context_ids, params.context_window)
    counter = NgramCounter(ctx, params.max_n) if ctx else None
    root_tail = tuple(ctx[-tail_size:]) if (ctx and tail_size > 0) else ()

    memo: dict = {}

    def inc(tail, token, rank):
        if rank_gated and rank > params.rank_cap:
            return 0.0
        key = (tail, token)
        if key not in memo:
            memo[key] = ngram_bonus(counter, tail, token, params)
        b = memo[key]
        return 0.0 if b <= 0.0 else float(params.beta * b)

    t0 = int(top_ids[0, 0])
    w0 = float(lp[0, 0])
    b0 = inc(root_tail, t0, 0)
    # heap entries: (-aug, parent, depth, rank, logw, bonus, parent_tail, own_tail)
    frontier = [(-(w0 + b0), 0, 1, 0, w0, b0, root_tail, _extend_tail(root_tail, t0, tail_size))]
    tokens, depths, parents, ranks = [], [], [-1], [0]
    while frontier and len(tokens) < budget:
        _, parent, depth, rank, logw, bonus, ptail, own_tail = heapq.heappop(frontier)
        me = len(tokens) + 1
        tok = int(top_ids[depth - 1, rank])
        tokens.append(tok)
        depths.append(depth)
        parents.append(parent)
        ranks.append(rank)
        if rank + 1 < k:
            r2 = rank + 1
            tok2 = int(top_ids[depth - 1, r2])
            w2 = logw - float(lp[depth - 1, rank]) + float(lp[depth - 1, r2])
            b2 = bonus - inc(ptail, tok, rank) + inc(ptail, tok2, r2)
            heapq.heappush(frontier, (-(w2 + b2), parent, depth, r2, w2, b2, ptail,
                                      _extend_tail(ptail, tok2, tail_size)))
        if depth < rows:
            tok2 = int(top_ids[depth, 0])
            w2 = logw + float(lp[depth, 0])
            b2 = bonus + inc(own_tail, tok2, 0)
            heapq.heappush(frontier, (-(w2 + b2), me, depth + 1, 0, w2, b2, own_tail,
                                      _extend_tail(own_tail, tok2, tail_size)))
    return Tree(np.asarray(tokens, np.int64), np.asarray(depths, np.int64), parents, ranks)


def build_tree(top_logp, top_ids, budget: int, strategy: str, context_ids=None,
               params: NgramParams | None = None) -> Tree:
    """Dispatch of ddtree.py:538-589 given precomputed top-k log-probs and ids."""
    params = params or NgramParams()
    s = canonical_strategy(strategy)
    if s == STRATEGY_HEAP:
        return build_tree_heap(top_logp, top_ids, budget)
    return build_tree_ngram(top_logp, top_ids, budget, context_ids, params,
                            rank_gated=(s == STRATEGY_RANK_GATED))


def build_tree_from_logits(draft_logits: np.ndarray, budget: int, strategy: str,
                           context_ids=None, params: NgramParams | None = None) -> Tree:
    """``build_ddtree_tree`` end to end (ddtree.py:538-589): top-k then the builder."""
    x = np.asarray(draft_logits, dtype=np.float32)
    if budget <= 0 or x.shape[0] == 0:
        return _empty_tree()
    params = params or NgramParams()
    s = canonical_strategy(strategy)
    if s != STRATEGY_HEAP and abs(params.beta) < 1e-12 and params.exact_beta0:
        s = STRATEGY_HEAP
    top_logp, top_ids, _, _ = topk_logz(x, min(budget, x.shape[1]))
    return build_tree(top_logp, top_ids, budget, s, context_ids, params)


# ---------------------------------------------------------------------------
# Visibility, packed ancestor bitmask, compile (ddtree.py:520-528, :592-647)
# ---------------------------------------------------------------------------
def visibility(parents: Sequence[int]) -> np.ndarray:
    """Ancestor closure ``vis[i] = vis[parent[i]] | {i}`` (ddtree.py:520-528)."""
    n = len(parents)
    vis = np.zeros((n, n), dtype=np.bool_)
    vis[0, 0] = True
    for i in range(1, n):
        vis[i, :i] = vis[parents[i], :i]
        vis[i, i] = True
    return vis


def pack_bits(vis: np.ndarray, words: int | None = None) -> np.ndarray:
    """Packed ancestor bitmask: bit ``j%32`` of word ``j//32`` in row ``i`` is ``vis[i, j]``."""
    n = vis.shape[0]
    w = (n + 31) // 32 if words is None else words
    out = np.zeros((n, w), dtype=np.uint32)
    for j in range(n):
        out[vis[:, j], j // 32] |= np.uint32(1 << (j % 32))
    return out


def unpack_bits(bits: np.ndarray, n: int) -> np.ndarray:
    bits = np.asarray(bits, dtype=np.uint32)
    j = np.arange(n)
    return ((bits[:n, j // 32] >> (j % 32).astype(np.uint32)) & 1).astype(np.bool_)


def compile_tree(root_token: int, start: int, tokens, depths, parents, past_length: int,
                 dtype_min: float = float(np.finfo(np.float32).min)):
    """Verify ids, positions and the additive mask of ddtree.py:592-647.

    Returns ``ids i64[n]``, ``pos i64[n]`` and ``mask f32[n, past_length+n]``
    (0 where visible, ``dtype_min`` where not; the prefix is fully visible).
    """
    tokens = np.asarray(tokens, np.int64)
    n = 1 + tokens.shape[0]
    ids = np.concatenate([[int(root_token)], tokens]).astype(np.int64)
    pos = (start + np.concatenate([[0], np.asarray(depths, np.int64)])).astype(np.int64)
    vis = visibility(parents)
    mask = np.zeros((n, past_length + n), dtype=np.float32)
    mask[:, past_length:] = np.where(vis, 0.0, dtype_min)
    return ids, pos, mask


# ---------------------------------------------------------------------------
# Exact walk (ddtree.py:650-663)
# ---------------------------------------------------------------------------
def child_maps(parents: Sequence[int], tokens: Sequence[int]) -> list[dict[int, int]]:
    """``child_maps[p][token] = node`` as built during expansion (ddtree.py:460-461)."""
    maps: list[dict[int, int]] = [dict() for _ in range(len(parents))]
    for i in range(1, len(parents)):
        maps[parents[i]][int(tokens[i - 1])] = i
    return maps


def follow_tree(maps: list[dict[int, int]], posterior: Sequence[int]):
    """Longest path whose every step is the target's argmax (ddtree.py:650-663)."""
    post = [int(t) for t in np.asarray(posterior).reshape(-1)]
    accepted = [0]
    cur = 0
    nxt = post[0]
    while nxt in maps[cur]:
        cur = maps[cur][nxt]
        accepted.append(cur)
        nxt = post[cur]
    return accepted, nxt


# ---------------------------------------------------------------------------
# Commit-time KV compaction (ddtree.py:666-731 and the C++ of :37-65)
# ---------------------------------------------------------------------------
def compact_tensor(t: np.ndarray, past_length: int, keep: Sequence[int]) -> None:
    """In place: rows ``past+keep[i]`` -> ``past+i`` along axis -2 (ddtree.py:666-686).

    Skips when the appended window is empty, when nothing is kept, and when the
    keep count equals the window length (ddtree.py:669-675).
    """
    cur = t.shape[-2] - past_length
    if cur <= 0:
        return
    kc = len(keep)
    if kc == 0 or kc == cur:
        return
    idx = past_length + np.asarray(keep, dtype=np.int64)
    gathered = np.take(t, idx, axis=-2).copy()
    sl = [slice(None)] * t.ndim
    sl[-2] = slice(past_length, past_length + kc)
    t[tuple(sl)] = gathered


def compact_cache(layers: list[tuple[np.ndarray, np.ndarray]], past_length: int,
                  keep: Sequence[int]) -> list[tuple[np.ndarray, np.ndarray]]:
    """``compact_dynamic_cache`` (ddtree.py:689-731): compact K and V, then crop.

    Returns the cropped ``(keys, values)`` per layer (crop keeps the first
    ``past+len(keep)`` rows, or ``past`` when ``keep`` is empty; a layer shorter
    than that is left as is, as ``DynamicLayer.crop`` does).
    """
    out = []
    new_len = past_length + len(keep)
    for k, v in layers:
        if len(keep) > 0:
            compact_tensor(k, past_length, keep)
            compact_tensor(v, past_length, keep)
        if k.shape[-2] > new_len:
            k = k[..., :new_len, :]
            v = v[..., :new_len, :]
        out.append((k, v))
    return out


def log1p_table(n: int) -> np.ndarray:
    """``np.log1p(c)`` for ``c = 0..n`` in binary64 (the base of ddtree.py:180)."""
    return np.log1p(np.arange(n + 1, dtype=np.float64))


__all__ = [
    "NgramParams", "Tree", "canonical_strategy", "topk_logz", "context_window",
    "NgramCounter", "ngram_bonus", "build_tree_heap", "build_tree_ngram", "build_tree",
    "build_tree_from_logits", "visibility", "pack_bits", "unpack_bits", "compile_tree",
    "child_maps", "follow_tree", "compact_tensor", "compact_cache", "log1p_table",
    "STRATEGY_HEAP", "STRATEGY_NGRAM", "STRATEGY_RANK_GATED",
]
