"""Recovery-memory files written by the reference's own RecoveryMemory (model/recovery.py:209-256).

Fills a memory from a seeded stream of prior and online records, then saves
its legacy flat prior (``save_prior``) and its ``retree-recovery-state-v1``
runtime state (``save_runtime_state``) next to this script:

    python tests/golden/make_recovery_files.py --reference /path/to/ReTree
"""

from __future__ import annotations

import argparse
import os
import sys
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent


def records(seed: int = 0):
    """The seeded (kind, draft, target, count) stream the files are made from."""
    rng = np.random.default_rng(seed)
    out = []
    for _ in range(60):
        kind = "prior" if rng.random() < 0.6 else "online"
        out.append((kind, int(rng.integers(0, 50)), int(rng.integers(0, 50)), int(rng.integers(0, 4))))
    return out


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", default=os.environ.get("RETREE_REFERENCE"),
                    help="checkout of the reference repository (or set RETREE_REFERENCE)")
    args = ap.parse_args()
    if not args.reference:
        ap.error("--reference (or RETREE_REFERENCE) must name the reference checkout")
    sys.path.insert(0, args.reference)
    from model.recovery import RecoveryMemory  # type: ignore

    mem = RecoveryMemory(freq_threshold=4)
    for kind, d, t, c in records():
        (mem.record_prior if kind == "prior" else mem.record_online)(d, t, c)
    mem.save_prior(str(HERE / "recovery_prior.json"))
    mem.save_runtime_state(str(HERE / "recovery_state.json"))
    print(mem.prior_total_pairs(), mem.online_total_pairs())


if __name__ == "__main__":
    main()
