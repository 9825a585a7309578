"""fp32 tree-verify attention as the reference's SDPA path computes it
(test infrastructure only; see ``oracle/__init__.py``).

The reference verifies a tree with HF ``sdpa_attention_forward``
(transformers/integrations/sdpa_attention.py:40-104, transformers 5.5.0): with a
mask present it expands K/V to every query head with ``repeat_kv`` (:57-60) and
calls ``F.scaled_dot_product_attention`` with the additive float mask that
``compile_ddtree_tree`` writes (ddtree.py:629-640): 0 where a key is visible,
``finfo(dtype).min`` where not; every prefix key is visible.  This restatement
computes the same softmax(QK^T*scale + mask)V in fp32 with explicit matmuls.
"""

from __future__ import annotations

import numpy as np
import torch


def tree_attention(q, k, v, past_length: int, visible_tree: np.ndarray,
                   scale: float | None = None) -> torch.Tensor:
    """Masked GQA attention over ``[prefix ; tree block]`` in fp32.

    q: ``[Hq, n, D]`` (or ``[1, Hq, n, D]``); k, v: ``[Hkv, S, D]`` (or with a
    leading batch of 1) with ``S >= past_length + n``; keys past
    ``past_length + n`` are ignored.  ``visible_tree``: bool ``[n, n]``, row i =
    tree nodes node i attends to.  Returns ``[n, Hq, D]`` fp32 (the layout HF
    returns after ``transpose(1, 2)``, sdpa_attention.py:102).
    """
    q = torch.as_tensor(q).float()
    k = torch.as_tensor(k).float()
    v = torch.as_tensor(v).float()
    if q.dim() == 4:
        q = q[0]
    if k.dim() == 4:
        k, v = k[0], v[0]
    hq, n, d = q.shape
    hkv = k.shape[0]
    groups = hq // hkv
    s = past_length + n
    k = k[:, :s].repeat_interleave(groups, dim=0)
    v = v[:, :s].repeat_interleave(groups, dim=0)
    scale = d ** -0.5 if scale is None else scale
    mask = torch.zeros((n, s), dtype=torch.float32)
    vis = torch.as_tensor(np.asarray(visible_tree, dtype=np.bool_))
    mask[:, past_length:] = torch.where(vis, 0.0, torch.finfo(torch.float32).min)
    scores = torch.matmul(q, k.transpose(-1, -2)) * scale + mask
    probs = torch.softmax(scores, dim=-1)
    out = torch.matmul(probs, v)           # [Hq, n, D]
    return out.transpose(0, 1).contiguous()
