"""Split one long request's attention by KV head across ranks.

For a target whose KV cache is too large or too slow for one GPU (e.g. the
Qwen3-8B geometry with a 32768-token prefix and a 256-node tree), rank g of G keeps
KV heads ``[g*Hkv/G, (g+1)*Hkv/G)`` and their ``group`` query heads:

* ``shard_attention_heads`` slices every layer's q/k/v projections to the
  rank's heads (the MLP, norms, embeddings and lm_head stay replicated), so
  the rank computes, caches and attends over its heads only -- the KV cache and
  its HBM traffic shrink by G;
* the attention backend runs on the local heads and all-gathers the outputs
  ``[n, Hq/G * head_dim]`` of every rank into head order before ``o_proj``
  (one NCCL all-gather per layer over NVLink; the result lands in local HBM).

``headsplit_backend(inner)`` wraps any HF attention function with the
gather; ``register()`` installs ``retree_tree_headsplit`` (the sm_100a kernel
inside) and ``sdpa_headsplit`` (HF SDPA inside, for CPU checks of the host
logic).
"""

from __future__ import annotations

import torch
import torch.distributed as dist
from torch import nn

NAME = "retree_tree_headsplit"
SDPA_NAME = "sdpa_headsplit"


def head_range(total: int, rank: int, world: int) -> tuple[int, int]:
    if total % world:
        raise ValueError(f"{total} heads do not split over {world} ranks")
    per = total // world
    return rank * per, (rank + 1) * per


def _slice_linear(lin: nn.Linear, rows: slice) -> nn.Linear:
    out = nn.Linear(lin.in_features, rows.stop - rows.start, bias=lin.bias is not None,
                    device=lin.weight.device, dtype=lin.weight.dtype)
    with torch.no_grad():
        out.weight.copy_(lin.weight[rows])
        if lin.bias is not None:
            out.bias.copy_(lin.bias[rows])
    return out.requires_grad_(False)


def shard_attention_heads(model, rank: int, world: int, group=None):
    """Keep only this rank's attention heads in every layer (in place); returns the model."""
    cfg = model.config
    hd = getattr(cfg, "head_dim", None) or cfg.hidden_size // cfg.num_attention_heads
    q0, q1 = head_range(cfg.num_attention_heads, rank, world)
    k0, k1 = head_range(cfg.num_key_value_heads, rank, world)
    for layer in model.model.layers:
        attn = layer.self_attn
        attn.q_proj = _slice_linear(attn.q_proj, slice(q0 * hd, q1 * hd))
        attn.k_proj = _slice_linear(attn.k_proj, slice(k0 * hd, k1 * hd))
        attn.v_proj = _slice_linear(attn.v_proj, slice(k0 * hd, k1 * hd))
        attn._rt_head_split = (group, world, rank)
    model._rt_local_kv_heads = k1 - k0
    if world > 1 and torch.cuda.is_available():
        # the forward all-gathers attention outputs on the compute stream: no
        # programmatic dependent launch around those collectives (rt_set_pdl)
        from . import kernels
        kernels.set_pdl(False)
    return model


def gather_heads(out_local: torch.Tensor, group, world: int) -> torch.Tensor:
    """``[1, n, Hq/G, D]`` on every rank -> ``[1, n, Hq, D]`` in head order."""
    _, n, hl, d = out_local.shape
    send = out_local.reshape(n * hl * d).contiguous()
    recv = torch.empty((world * n * hl * d,), dtype=send.dtype, device=send.device)
    dist.all_gather_into_tensor(recv, send, group=group)
    return recv.view(world, n, hl, d).permute(1, 0, 2, 3).reshape(1, n, world * hl, d)


def headsplit_backend(inner):
    def forward(module, query, key, value, attention_mask, **kwargs):
        out, w = inner(module, query, key, value, attention_mask, **kwargs)
        split = getattr(module, "_rt_head_split", None)
        if split is None:
            return out, w
        group, world, _ = split
        return gather_heads(out, group, world), None
    return forward


def register() -> tuple[str, str]:
    from transformers import AttentionInterface
    from transformers.integrations.sdpa_attention import sdpa_attention_forward

    from . import attention

    AttentionInterface.register(NAME, headsplit_backend(attention.tree_attention_forward))
    AttentionInterface.register(SDPA_NAME, headsplit_backend(sdpa_attention_forward))
    return NAME, SDPA_NAME
