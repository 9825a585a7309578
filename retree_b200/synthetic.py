"""Seeded synthetic workloads for the verification path.

There are no datasets or checkpoints on the machines this runs on, so draft
logits, contexts, trees and KV caches are drawn from fixed-seed generators
with the shapes and value distributions of the workloads being measured:

* draft logits: ``[rows, vocab]`` N(0,1) plus a Zipf(s) boost ``amp / r**s``
  (r = 1..n_boost) on ``n_boost`` distinct random token ids per row;
* context ids: uniform ids, or a short-alphabet Markov walk so that n-grams
  repeat and the continuity bonus fires;
* random trees: BFS trees, depth <= ``max_depth``, each node with a
  Geometric(p) number of children, numbered so that parents precede children.

numpy's ``default_rng`` (PCG64) is platform independent, so the same seed
gives the same inputs on every host.
"""

from __future__ import annotations

import numpy as np

#: Zipf boost amplitude used for the Zipf-peaked draft logits (chosen so that
#: the top-1 draft token carries ~40% of the mass at vocab 151936).
DEFAULT_ZIPF_AMP = 12.0


def draft_logits(seed: int, rows: int, vocab: int, amp: float = DEFAULT_ZIPF_AMP,
                 n_boost: int = 32, s: float = 1.1) -> np.ndarray:
    """N(0,1) logits plus ``amp / r**s`` on ``n_boost`` distinct ids per row (fp32)."""
    rng = np.random.default_rng(seed)
    x = rng.standard_normal((rows, vocab), dtype=np.float32)
    nb = min(n_boost, vocab)
    boost = (amp / np.arange(1, nb + 1, dtype=np.float64) ** s).astype(np.float32)
    for r in range(rows):
        ids = rng.choice(vocab, size=nb, replace=False)
        x[r, ids] += boost
    return x


def context_ids(seed: int, length: int, vocab: int, alphabet: int | None = None) -> np.ndarray:
    """Uniform ids in ``[0, vocab)``; with ``alphabet``, a Markov walk over that many ids.

    The walk repeats short patterns (each id has three likely successors), so
    2-, 3- and 4-grams recur inside the window.
    """
    rng = np.random.default_rng(seed)
    if alphabet is None:
        return rng.integers(0, vocab, size=length, dtype=np.int64)
    a = min(alphabet, vocab)
    succ = rng.integers(0, a, size=(a, 3))
    out = np.empty(length, dtype=np.int64)
    cur = int(rng.integers(0, a))
    for i in range(length):
        out[i] = cur
        cur = int(succ[cur, rng.integers(0, 3)]) if rng.random() < 0.9 else int(rng.integers(0, a))
    return out


def random_tree_parents(seed: int, budget: int, max_depth: int = 16, p: float = 0.5) -> np.ndarray:
    """Parent array ``[budget+1]`` (root first, parent[0] = -1) of a BFS tree.

    Each node gets ``Geometric(p)`` (>= 1) children until ``budget`` nodes are
    placed; nodes at ``max_depth`` get none.
    """
    rng = np.random.default_rng(seed)
    parents = [-1]
    depth = [0]
    queue = [0]
    qi = 0
    while len(parents) < budget + 1 and qi < len(queue):
        node = queue[qi]
        qi += 1
        if depth[node] >= max_depth:
            continue
        for _ in range(int(rng.geometric(p))):
            if len(parents) >= budget + 1:
                break
            parents.append(node)
            depth.append(depth[node] + 1)
            queue.append(len(parents) - 1)
    return np.asarray(parents, dtype=np.int64)


def depths_from_parents(parents) -> np.ndarray:
    parents = np.asarray(parents, dtype=np.int64)
    d = np.zeros(len(parents), dtype=np.int64)
    for i in range(1, len(parents)):
        d[i] = d[parents[i]] + 1
    return d


def accepted_path(seed: int, parents, length: int | None = None) -> list[int]:
    """A root-to-node path: from the root, step to a uniformly chosen child.

    Stops at a leaf, or after ``length`` nodes (root included) when given.
    """
    rng = np.random.default_rng(seed)
    parents = np.asarray(parents, dtype=np.int64)
    kids: list[list[int]] = [[] for _ in range(len(parents))]
    for i in range(1, len(parents)):
        kids[parents[i]].append(i)
    path = [0]
    while kids[path[-1]] and (length is None or len(path) < length):
        path.append(int(rng.choice(kids[path[-1]])))
    return path
