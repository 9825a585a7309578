"""CPU oracle for the ReTree tree-verification path.

TEST INFRASTRUCTURE ONLY. This package is a CPU restatement (numpy / plain
Python, torch CPU only for the fp32 attention reference) of the reference
algorithms on the verification hot path of Adamlong3/ReTree, used to check the
kernels: only ``tests/``, ``__graft_entry__.smoke()`` and the CPU-baseline leg of
``bench.py`` import it. The product (``retree_b200``) never imports, links or
calls anything here, and has no CPU fallback.

Parity of the restatement itself is pinned by golden vectors generated from the
reference's own functions (``tests/golden/make_golden.py``, committed with its
outputs under ``tests/golden/``).

Modules:
  tree       top-k/log-normaliser, the three tree builders, visibility, mask
             compile, exact walk, KV compaction       (ddtree.py)
  attention  fp32 tree-verify attention as HF SDPA computes it
             (transformers/integrations/sdpa_attention.py)
  recovery   recovery memory and the target-gated sibling-recovery walk
             (model/recovery.py, retree.py)
  dflash     the DFlash block-draft forward with its cache crop
             (model/dflash.py), golden outputs from the reference module
             (tests/golden/make_dflash_golden.py)
"""
