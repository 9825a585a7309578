"""Drop-in for the reference's ``ddtree.py`` tree-verification entry points.

Same names, arguments and return values as Adamlong3/ReTree ddtree.py, with
the work done by the sm_100a kernels:

  build_ddtree_tree      device top-k + best-first expansion      (ddtree.py:538-589)
  compile_ddtree_tree    verify ids / positions + packed tree mask (ddtree.py:592-647)
  follow_verified_tree   host walk over child_maps                 (ddtree.py:650-663)
  compact_dynamic_cache  one-launch KV compaction                  (ddtree.py:689-731)
  maybe_enable_cpp_compact                                        (ddtree.py:84-88)
  ddtree_generate        the DDTree decode loop                    (ddtree.py:734-968)

The CPU-list outputs (``parents``, ``child_maps``, the visibility matrix) are
still returned for callers such as recovery and calibration; the device
results of the last build stay available as ``last_device_tree()``.
"""

from __future__ import annotations

import os
import time
from types import SimpleNamespace

import numpy as np
import torch

from . import _lib, kernels
from .attention import attach
from .cache import TreeKVCache

DDTREE_STAGE_ORDER = ("draft", "tree_build", "tree_compile", "verify", "commit")
DDTREE_TREE_BUILD_STAGE_ORDER = ("tree_build_copy", "tree_build_heap", "tree_build_visibility")

_STRATEGIES = {
    "heap": "heap", "original": "heap", "default": "heap",
    "ngram": "ngram", "ngram_continuity": "ngram", "continuity": "ngram",
    "rank_gated_ngram": "rank_gated_ngram", "fast_rank_gated_ngram": "rank_gated_ngram",
}

_CPP_COMPACT_ENABLED = False
_LAST_TREE: dict | None = None


def cuda_time() -> float:
    """Synchronise the device and read the host clock (dflash.py:163-165)."""
    torch.cuda.synchronize()
    return time.perf_counter()


def empty_stage_times(stage_names) -> dict[str, float]:
    return {name: 0.0 for name in stage_names}


def maybe_enable_cpp_compact(enabled: bool) -> None:
    """Kept for the reference's API (ddtree.py:84-88).

    Compaction always runs the CUDA kernel here; enabling it only checks that
    the kernel library loads (it raises if it does not).
    """
    global _CPP_COMPACT_ENABLED
    _CPP_COMPACT_ENABLED = bool(enabled)
    if enabled:
        _lib.load()


class NgramParams(SimpleNamespace):
    """The ``DDTREE_NGRAM_*`` knobs, read per build as ddtree.py:346-354 does."""

    @staticmethod
    def from_env(env=None) -> "NgramParams":
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


def resolve_strategy(env=None) -> tuple[str, NgramParams]:
    """Builder selected by ``DDTREE_TREE_STRATEGY`` (ddtree.py:564-589), beta==0 rule applied."""
    e = os.environ if env is None else env
    name = e.get("DDTREE_TREE_STRATEGY", "heap").strip().lower()
    if name not in _STRATEGIES:
        raise ValueError(f"Unknown DDTREE_TREE_STRATEGY={name}. Use one of: heap, ngram, rank_gated_ngram.")
    strategy = _STRATEGIES[name]
    params = NgramParams.from_env(e)
    if strategy != "heap" and abs(params.beta) < 1e-12 and params.exact_beta0:
        strategy = "heap"  # ddtree.py:356-359
    return strategy, params


def _device_context(context_ids, device):
    if context_ids is None:
        return None
    if isinstance(context_ids, torch.Tensor):
        ctx = context_ids.reshape(-1)
        if ctx.device != device or ctx.dtype != torch.int64:
            ctx = ctx.to(device=device, dtype=torch.int64)
        return ctx
    arr = np.asarray(context_ids, dtype=np.int64).reshape(-1)
    return torch.from_numpy(arr).to(device)


def build_tree_device(draft_logits: torch.Tensor, budget: int, context_ids=None, strategy: str | None = None,
                      params: NgramParams | None = None, out: dict | None = None, k: int | None = None,
                      **kw) -> dict:
    """Top-k + tree expansion on the device; returns the device tensors of ``kernels.tree_build``.

    ``k`` candidates per draft row (default min(budget, vocab), the reference's
    top-k; 1 gives the chain of the rows' argmax tokens).
    """
    if strategy is None or params is None:
        strategy, params = resolve_strategy()
    if not draft_logits.is_cuda:
        raise RuntimeError("build_ddtree_tree runs on the device: pass CUDA draft logits")
    logits = draft_logits if draft_logits.stride(-1) == 1 else draft_logits.contiguous()
    k = min(max(int(budget), 1) if k is None else max(int(k), 1), logits.shape[-1])
    top_logp, top_ids, _ = kernels.draft_topk(logits, k)
    ctx = _device_context(context_ids, logits.device)
    return kernels.tree_build(top_logp, top_ids, int(budget), strategy, params, ctx=ctx, out=out, **kw)


def last_device_tree() -> dict | None:
    """Device tensors of the most recent ``build_ddtree_tree`` call."""
    return _LAST_TREE


def _host_tree(parents: list[int], tokens: list[int]):
    maps: list[dict[int, int]] = [dict() for _ in range(len(parents))]
    for i in range(1, len(parents)):
        maps[parents[i]][int(tokens[i - 1])] = i
    return maps


def build_ddtree_tree(draft_logits: torch.Tensor, budget: int, context_ids=None):
    """``(node_token_ids, node_depths, parents, child_maps, visibility, subtimes)`` as ddtree.py:538-549."""
    global _LAST_TREE
    subtimes = empty_stage_times(DDTREE_TREE_BUILD_STAGE_ORDER)
    strategy, params = resolve_strategy()
    if budget <= 0 or draft_logits.shape[0] == 0:
        vis = torch.zeros((1, 1), dtype=torch.bool)
        vis[0, 0] = True
        return (torch.empty(0, dtype=torch.long), torch.empty(0, dtype=torch.long), [-1], [dict()], vis, subtimes)
    t0 = cuda_time()
    tree = build_tree_device(draft_logits, budget, context_ids, strategy, params)
    _LAST_TREE = tree
    # one device->host transfer of the small tree arrays
    count = int(tree["count"].item())
    packed = torch.cat([tree["tokens"][:count], tree["depths"][:count],
                        tree["parents"][: count + 1].to(torch.int64)]).cpu()
    t1 = time.perf_counter()
    subtimes["tree_build_copy"] = 0.0
    subtimes["tree_build_heap"] = t1 - t0
    tokens = packed[:count]
    depths = packed[count: 2 * count]
    parents = packed[2 * count:].tolist()
    maps = _host_tree(parents, tokens.tolist())
    n = count + 1
    vis = np.zeros((n, n), dtype=np.bool_)
    vis[0, 0] = True
    for i in range(1, n):
        vis[i, :i] = vis[parents[i], :i]
        vis[i, i] = True
    subtimes["tree_build_visibility"] = time.perf_counter() - t1
    return tokens, depths, parents, maps, torch.from_numpy(vis), subtimes


def _pack_visibility(vis: torch.Tensor, words: int) -> np.ndarray:
    v = np.asarray(vis.cpu().numpy(), dtype=np.bool_)
    n = v.shape[0]
    padded = np.zeros((n, words * 32), dtype=np.bool_)
    padded[:, : v.shape[1]] = v
    return np.packbits(padded, axis=1, bitorder="little").view("<u4").view(np.int32)


def compile_ddtree_tree(root_token_id, start: int, node_token_ids, node_depths, visibility_cpu, past_length: int,
                        dtype, device, verify_input_ids_buffer, verify_position_ids_buffer, attention_mask_buffer,
                        tree_visibility_buffer, previous_tree_start: int, previous_tree_length: int):
    """``(verify_ids, verify_pos, mask, past_length, n)`` as ddtree.py:592-647.

    With an int32 ``attention_mask_buffer`` (``[max_nodes, W]``, what
    ``allocate_tree_buffers`` returns) the mask is the packed ancestor bitmask.
    With the reference's dense ``[1, 1, max_nodes, L]`` float buffer the dense
    additive mask is written exactly as the reference writes it and the packed
    bits ride along on the returned view, so either attention backend can
    consume it.
    """
    n = 1 + int(node_token_ids.numel())
    ids = verify_input_ids_buffer[:, :n]
    ids[0, 0] = root_token_id
    if n > 1:
        ids[0, 1:n].copy_(node_token_ids, non_blocking=False)
    pos = verify_position_ids_buffer[:, :n]
    pos[0, 0] = start
    if n > 1:
        pos[0, 1:n].copy_(node_depths, non_blocking=False)
        pos[0, 1:n].add_(start)
    if attention_mask_buffer.dtype == torch.int32:
        words = attention_mask_buffer.shape[-1]
        bits = torch.from_numpy(_pack_visibility(visibility_cpu, words))
        buf = attention_mask_buffer[:n]
        buf.copy_(bits, non_blocking=False)
        mask = attach(buf.view(1, 1, n, words), buf)
        return ids, pos, mask, past_length, n
    if previous_tree_length > 0:
        attention_mask_buffer[0, 0, :previous_tree_length,
                              previous_tree_start: previous_tree_start + previous_tree_length] = 0
    vis = tree_visibility_buffer[:n, :n]
    vis.copy_(visibility_cpu, non_blocking=False)
    block = attention_mask_buffer[0, 0, :n, past_length: past_length + n]
    block.fill_(torch.finfo(dtype).min)
    block.masked_fill_(vis, 0)
    mask = attention_mask_buffer[:, :, :n, : past_length + n]
    words = (n + 31) // 32
    bits = torch.from_numpy(_pack_visibility(visibility_cpu, words)).to(attention_mask_buffer.device)
    return ids, pos, attach(mask, bits), past_length, n


def follow_verified_tree(child_maps, posterior: torch.Tensor):
    """Longest path of target-argmax steps through the tree (ddtree.py:650-663)."""
    post = posterior[0].tolist()
    accepted = [0]
    cur = 0
    nxt = int(post[0])
    while nxt in child_maps[cur]:
        cur = child_maps[cur][nxt]
        accepted.append(cur)
        nxt = int(post[cur])
    return accepted, nxt


def compact_dynamic_cache(past_key_values, past_length: int, keep_current_indices) -> None:
    """Move the accepted rows of the appended window to ``past_length..`` and crop (ddtree.py:689-731).

    A ``TreeKVCache`` is compacted in one launch over its slab; a
    ``DynamicCache`` (``layers[i].keys/.values`` or the older
    ``key_cache/value_cache`` lists) with one launch per tensor.
    ``keep_current_indices`` may be a list or an int64 CUDA tensor.
    """
    nkeep = int(keep_current_indices.numel()) if isinstance(keep_current_indices, torch.Tensor) \
        else len(keep_current_indices)
    if nkeep == 0:
        past_key_values.crop(past_length)
        return
    keep_by_device: dict = {}

    def keep_on(device):
        if device not in keep_by_device:
            if isinstance(keep_current_indices, torch.Tensor):
                keep_by_device[device] = keep_current_indices.to(device=device, dtype=torch.long)
            else:
                keep_by_device[device] = torch.tensor(list(keep_current_indices), dtype=torch.long, device=device)
        return keep_by_device[device]

    if isinstance(past_key_values, TreeKVCache):
        cur = past_key_values.length - past_length
        if cur > 0:
            kernels.kv_compact(past_key_values.slab[:, :, : past_key_values.length, :], past_length,
                               keep_on(past_key_values.device))
        past_key_values.crop(past_length + nkeep)
        return
    if hasattr(past_key_values, "key_cache") and hasattr(past_key_values, "value_cache"):
        for k, v in zip(past_key_values.key_cache, past_key_values.value_cache):
            kernels.kv_compact([k, v], past_length, keep_on(k.device))
        past_key_values.crop(past_length + nkeep)
        return
    if hasattr(past_key_values, "layers"):
        for layer in past_key_values.layers:
            if getattr(layer, "keys", None) is None or layer.keys.numel() == 0:
                continue
            kernels.kv_compact([layer.keys, layer.values], past_length, keep_on(layer.keys.device))
        past_key_values.crop(past_length + nkeep)
        return
    raise RuntimeError("Unsupported DynamicCache layout for DDTree cache compaction.")


def sample(logits: torch.Tensor, temperature: float = 0.0) -> torch.Tensor:
    """Posterior tokens (model/utils.py:52-59): argmax at T=0, else multinomial."""
    if temperature < 1e-5:
        return torch.argmax(logits, dim=-1)
    bsz, seq_len, vocab = logits.shape
    probs = torch.softmax(logits.view(-1, vocab) / temperature, dim=-1)
    return torch.multinomial(probs, num_samples=1).view(bsz, seq_len)


def allocate_tree_buffers(tree_budget: int, device):
    """Verify-id / position buffers and the packed int32 tree-mask buffer for ``compile_ddtree_tree``."""
    n = 1 + max(int(tree_budget), 0)
    words = (n + 31) // 32
    return (torch.empty((1, n), dtype=torch.long, device=device),
            torch.empty((1, n), dtype=torch.long, device=device),
            torch.zeros((n, words), dtype=torch.int32, device=device),
            torch.empty((n, n), dtype=torch.bool, device=device))


@torch.inference_mode()
def ddtree_generate(model, target, input_ids: torch.Tensor, mask_token_id: int, max_new_tokens: int,
                    block_size: int, stop_token_ids, temperature: float = 0.0, tree_budget: int | None = None,
                    save_tree_traces: bool = False, draft_fn=None, fused: bool | None = None,
                    fused_draft: bool = False) -> SimpleNamespace:
    """The DDTree decode loop of ddtree.py:734-968 on the device kernels.

    ``target`` is a causal LM whose attention backend is ``"retree_tree"``.
    ``model`` is the block draft model (a DFlash module), called as in
    ddtree.py:832-844 on the target's layer outputs ``model.target_layer_ids``
    (ddtree.py:811-812, :917-918); a ``draft_fn(output_ids, start, round) ->
    [block_size-1, vocab]`` logits callable may replace it.  ``fused`` picks
    the verify forward (None: the fused stages when the model allows them and
    no hidden states are needed), ``fused_draft`` runs the draft module on the
    fused stages (``retree_b200.draft.FusedDraft``).
    """
    from .verify import TreeVerifier

    if block_size <= 1:  # ddtree.py:747-757: the linear path
        return dflash_generate(model, target, input_ids, mask_token_id, max_new_tokens, block_size, stop_token_ids,
                               temperature=temperature, draft_fn=draft_fn, fused=fused, fused_draft=fused_draft)
    layer_ids = None if (model is None or draft_fn is not None) else list(model.target_layer_ids)
    verifier = TreeVerifier(target, tree_budget=(block_size - 1) if tree_budget is None else max(tree_budget, 0),
                            max_length=input_ids.shape[1] + max_new_tokens + 2 * block_size + 8,
                            draft_horizon=block_size - 1, temperature=temperature, target_layer_ids=layer_ids,
                            fused=fused, fused_draft=fused_draft)
    return verifier.generate(input_ids, mask_token_id, max_new_tokens, block_size, stop_token_ids,
                             draft_model=model, draft_fn=draft_fn, save_tree_traces=save_tree_traces)


@torch.inference_mode()
def dflash_generate(model, target, input_ids: torch.Tensor, mask_token_id: int, max_new_tokens: int,
                    block_size: int, stop_token_ids, temperature: float = 0.0, draft_fn=None,
                    fused: bool | None = None, fused_draft: bool = False) -> SimpleNamespace:
    """The linear DFlash decode loop of dflash.py:14-162 on the device kernels.

    Each round verifies the chain of the draft rows' argmax tokens (a tree with
    one candidate per row; the exact walk accepts its longest matching
    prefix, dflash.py:108-118); ``block_size <= 1`` decodes one target token
    per round without a draft.  Arguments as in ``ddtree_generate``.
    """
    from .verify import TreeVerifier

    chain = max(int(block_size) - 1, 0)
    layer_ids = None if (chain == 0 or model is None or draft_fn is not None) else list(model.target_layer_ids)
    verifier = TreeVerifier(target, tree_budget=chain,
                            max_length=input_ids.shape[1] + max_new_tokens + 2 * max(block_size, 1) + 8,
                            draft_horizon=max(chain, 1), temperature=temperature, target_layer_ids=layer_ids,
                            fused=fused, fused_draft=fused_draft, chain=True)
    return verifier.generate(input_ids, mask_token_id, max_new_tokens, max(int(block_size), 1), stop_token_ids,
                             draft_model=model, draft_fn=draft_fn)
