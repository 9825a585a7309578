"""Drop-in for the reference's ``retree.py``: ReTree decoding with target-gated sibling recovery.

``follow_verified_tree_with_recovery`` keeps the reference's semantics
(retree.py:57-190): exact accept while the target's argmax is a child; at a
mismatch, rank the children by target logit, snapshot the pair frequencies,
optionally record the online divergences, and accept the first non-stop child
whose pre-update frequency reaches the threshold and whose target logit passes
the consistency gate.  ``retree_generate`` runs the decode loop of
retree.py:193-444 on ``TreeVerifier`` with that walk.
"""

from __future__ import annotations

import torch

from .ddtree import follow_verified_tree  # noqa: F401  (re-exported like the reference's import list)
from .recovery import RecoveryMemory, target_logit_consistency_gate, token_pair_has_stop


def _rank_children_by_target_logits(children: dict[int, int], logits_2d: torch.Tensor, position: int):
    """Children ``(token, node)`` by descending target logit at ``position`` (retree.py:25-54).

    Equal logits keep the children's dict order (a stable sort; the reference's
    unstable argsort leaves their order to the sort implementation).
    """
    if not children:
        return []
    toks = torch.tensor([int(t) for t in children.keys()], dtype=torch.long, device=logits_2d.device)
    scores = logits_2d[position].index_select(0, toks)
    order = torch.argsort(scores, descending=True, stable=True).tolist()
    toks_host = toks.tolist()
    return [(toks_host[j], children[toks_host[j]]) for j in order]


def follow_verified_tree_with_recovery(child_maps, posterior, target_logits, recovery_memory: RecoveryMemory,
                                       gate_threshold: float = 0.01, online_update: bool = True,
                                       record_top_k: int = 8, rescue_top_k: int = 8,
                                       disallow_rescue_target_ids=None):
    """ReTree's verifier walk; returns ``(accepted_indices, next_token, num_rescued)``."""
    post = posterior[0].tolist()
    logits_2d = target_logits[0]
    accepted = [0]
    cur = 0
    nxt = int(post[0])
    rescued = 0
    while True:
        children = child_maps[cur]
        if nxt in children:
            cur = children[nxt]
            accepted.append(cur)
            nxt = int(post[cur])
            continue
        if not children:
            break
        if disallow_rescue_target_ids is not None and int(nxt) in disallow_rescue_target_ids:
            break
        ranked = _rank_children_by_target_logits(children, logits_2d, cur)
        candidates = ranked[:rescue_top_k]
        target_tok = int(nxt)
        pairs = [(int(c), target_tok) for c, _ in candidates
                 if not token_pair_has_stop(int(c), target_tok, disallow_rescue_target_ids)]
        snap = recovery_memory.snapshot_frequencies(pairs)
        frequent = {int(c): (int(c), target_tok) in snap and snap[(int(c), target_tok)] >= recovery_memory.freq_threshold
                    for c, _ in candidates}
        if online_update:
            recovery_memory.record_online_divergences((c for c, _ in ranked), target_token=target_tok,
                                                      top_k=record_top_k, stop_token_ids=disallow_rescue_target_ids)
        moved = False
        for c, idx in candidates:
            c = int(c)
            if token_pair_has_stop(c, target_tok, disallow_rescue_target_ids) or not frequent.get(c, False):
                continue
            if not target_logit_consistency_gate(logits_2d, c, target_tok, cur, gate_threshold):
                continue
            cur = idx
            accepted.append(cur)
            rescued += 1
            nxt = int(post[cur])
            moved = True
            break
        if not moved:
            break
    return accepted, nxt, rescued


@torch.inference_mode()
def retree_generate(model, target, input_ids, mask_token_id, max_new_tokens, block_size, stop_token_ids,
                    temperature: float = 0.0, tree_budget: int | None = None,
                    recovery_memory: RecoveryMemory | None = None, gate_threshold: float = 0.01,
                    recovery_online_update: bool = True, recovery_record_top_k: int = 8,
                    recovery_rescue_top_k: int = 8, draft_fn=None, device_recovery: bool = True,
                    fused: bool | None = None, fused_draft: bool = False):
    """ReTree decode loop (retree.py:193-444); ``total_rescued`` counts sibling rescues.

    ``device_recovery`` (the default) runs the recovery walk on the GPU
    (rt_recovery_walk) over a device copy of ``recovery_memory``, so a round
    is one graph replay with no per-candidate host round trip; its online
    counts are applied to ``recovery_memory`` when the request ends.  False
    walks on the host with the reference's control flow.  ``fused`` /
    ``fused_draft`` as in ``ddtree_generate``.
    """
    from .verify import TreeVerifier

    if block_size <= 1:  # retree.py:210-219: the linear path
        from .ddtree import dflash_generate
        out = dflash_generate(model, target, input_ids, mask_token_id, max_new_tokens, block_size, stop_token_ids,
                              temperature=temperature, draft_fn=draft_fn, fused=fused, fused_draft=fused_draft)
        out.total_rescued = 0
        return out
    stop_set = None if stop_token_ids is None else {int(t) for t in stop_token_ids if t is not None}
    rescued = [0]

    def walk(maps, posterior, logits):
        acc, nxt, r = follow_verified_tree_with_recovery(
            maps, posterior, logits, recovery_memory, gate_threshold=gate_threshold,
            online_update=recovery_online_update, record_top_k=recovery_record_top_k,
            rescue_top_k=recovery_rescue_top_k, disallow_rescue_target_ids=stop_set)
        rescued[0] += r
        return acc, nxt

    verifier = TreeVerifier(target, tree_budget=(block_size - 1) if tree_budget is None else max(tree_budget, 0),
                            max_length=input_ids.shape[1] + max_new_tokens + 2 * block_size + 8,
                            draft_horizon=block_size - 1, temperature=temperature,
                            target_layer_ids=None if (model is None or draft_fn is not None)
                            else list(model.target_layer_ids), fused=fused, fused_draft=fused_draft)
    if device_recovery and recovery_memory is not None:
        from .recovery_device import DeviceRecoveryMemory
        dm = DeviceRecoveryMemory(recovery_memory, verifier.device, stop_ids=stop_set)
        verifier.enable_recovery(dm, gate_threshold=gate_threshold, rescue_top_k=recovery_rescue_top_k,
                                 record_top_k=recovery_record_top_k, online_update=recovery_online_update)
        out = verifier.generate(input_ids, mask_token_id, max_new_tokens, block_size, stop_token_ids,
                                draft_model=model, draft_fn=draft_fn)
        dm.sync()
        out.total_rescued = int(verifier.rescued_total.item())
        return out
    out = verifier.generate(input_ids, mask_token_id, max_new_tokens, block_size, stop_token_ids,
                            draft_model=model, draft_fn=draft_fn,
                            host_walk=None if recovery_memory is None else walk)
    out.total_rescued = rescued[0]
    return out
