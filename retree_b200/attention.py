"""Tree-verify attention as a transformers attention backend.

``register()`` adds ``"retree_tree"`` to ``transformers.AttentionInterface``;
a model loaded with ``attn_implementation="retree_tree"`` then calls
``tree_attention_forward`` from ``Qwen3Attention.forward``
(models/qwen3/modeling_qwen3.py:273-286) with the arguments HF's SDPA backend
receives (integrations/sdpa_attention.py:40-50) and gets the same
``(out [B, n, Hq, D], None)`` back (:102-104).  Every call runs the sm_100a
kernel; there is no repeat_kv and no fallback.

Masks understood (the 4-D mask is passed through untouched by HF,
masking_utils.py:827-829):
  * a ``TreeMask`` from ``retree_b200.ddtree.compile_ddtree_tree``: packed
    ancestor bits of the tree block (and, in device-length mode, the device
    word holding the prefix length);
  * the dense additive mask the reference's ``compile_ddtree_tree`` writes
    (ddtree.py:629-640): its tree block is packed to bits on the device;
  * no mask (prefill / plain decode): causal attention of the new tokens over
    the cache, run as a chain-shaped tree -- unless the caller asks for
    ``is_causal=False`` (the DFlash draft's attention, model/dflash.py:47 and
    its callers' kwargs), which the SDPA backend honours the same way
    (sdpa_attention.py:64-77): then every new token sees every key.
"""

from __future__ import annotations

import numpy as np
import torch

from . import kernels

NAME = "retree_tree"

_CAUSAL_BITS: dict = {}

#: when a list, every call appends (start event, end event, prefix_len, n, q heads, kv heads)
PROFILE: list | None = None


class TreeMask:
    """Marker carried as attributes on the 4-D mask tensor handed to the model."""

    BITS_ATTR = "_rt_bits"           # int32 [n, W] packed ancestor bits
    PREFIX_DEV_ATTR = "_rt_prefix_dev"  # int64[1] device prefix length (device-length mode) or None


def attach(mask4d: torch.Tensor, bits: torch.Tensor, prefix_dev: torch.Tensor | None = None) -> torch.Tensor:
    setattr(mask4d, TreeMask.BITS_ATTR, bits)
    setattr(mask4d, TreeMask.PREFIX_DEV_ATTR, prefix_dev)
    return mask4d


def causal_bits(n: int, device) -> torch.Tensor:
    """Lower-triangular packed mask: node i sees nodes 0..i (a chain), int32 ``[n, ceil(n/32)]``."""
    key = (torch.device(device).index, n)
    b = _CAUSAL_BITS.get(key)
    if b is None:
        w = (n + 31) // 32
        vis = np.arange(w * 32)[None, :] <= np.arange(n)[:, None]
        words = np.packbits(vis, axis=1, bitorder="little").view("<u4").view(np.int32)
        b = torch.from_numpy(np.ascontiguousarray(words)).to(device)
        _CAUSAL_BITS[key] = b
    return b


def full_bits(n: int, device) -> torch.Tensor:
    """Every node sees every node of the block, int32 ``[n, ceil(n/32)]`` (bits past n are ignored)."""
    key = ("full", torch.device(device).index, n)
    b = _CAUSAL_BITS.get(key)
    if b is None:
        b = torch.full((n, (n + 31) // 32), -1, dtype=torch.int32, device=device)
        _CAUSAL_BITS[key] = b
    return b


def _bits_for(mask, n: int, key_len: int, device, causal: bool = True):
    if mask is None:
        return (causal_bits(n, device) if causal else full_bits(n, device)), None
    bits = getattr(mask, TreeMask.BITS_ATTR, None)
    if bits is not None:
        return bits, getattr(mask, TreeMask.PREFIX_DEV_ATTR, None)
    if mask.dim() != 4:
        raise RuntimeError("retree_tree attention takes a 4-D tree mask")
    if mask.dtype == torch.int32:
        return mask[0, 0, :n], None
    # dense additive mask (0 visible / finfo.min hidden): pack its tree block
    if mask.shape[-1] < key_len:
        raise RuntimeError("dense tree mask narrower than the key length")
    m2 = mask[0, 0, :n, :key_len]
    if m2.stride(-1) != 1:
        m2 = m2.contiguous()
    return kernels.mask_from_dense(m2, key_len - n, n), None


def tree_attention_forward(module, query: torch.Tensor, key: torch.Tensor, value: torch.Tensor,
                           attention_mask, dropout: float = 0.0, scaling: float | None = None,
                           sliding_window=None, **kwargs):
    """HF attention backend: ``query [1, Hq, n, D]``, ``key/value [1, Hkv, S, D]``."""
    if dropout and module.training:
        raise RuntimeError("retree_tree attention is inference-only")
    if sliding_window is not None:
        raise RuntimeError("retree_tree attention has no sliding-window mode")
    if query.shape[0] != 1:
        raise RuntimeError("retree_tree attention verifies one sequence (batch 1)")
    n = query.shape[2]
    # the SDPA backend's rule: the call's is_causal, else the module's (default causal)
    causal = kwargs.get("is_causal", None)
    if causal is None:
        causal = getattr(module, "is_causal", True)
    bits, prefix_dev = _bits_for(attention_mask, n, key.shape[2], query.device, causal=bool(causal))
    if PROFILE is not None:
        ev0 = torch.cuda.Event(enable_timing=True)
        ev1 = torch.cuda.Event(enable_timing=True)
        ev0.record()
    # rows allocated per head: the launch (and its split of the keys) is sized
    # for the cache's capacity, so host-length and device-length rounds over the
    # same cache run the identical launch
    cap = key.shape[2]
    if key.stride(-1) == 1 and key.stride(2) > 0 and key.stride(1) % key.stride(2) == 0:
        cap = max(cap, key.stride(1) // key.stride(2))
    splits = kernels.default_splits(n, query.shape[1], key.shape[1], cap - n)
    if prefix_dev is not None:
        # full-capacity K/V views; the real prefix length lives on the device
        out = kernels.tree_attention(query, key, value, bits, prefix_len=cap - n, scale=scaling,
                                     prefix_len_dev=prefix_dev, kv_capacity=cap, num_splits=splits)
    else:
        out = kernels.tree_attention(query, key, value, bits, prefix_len=key.shape[2] - n, scale=scaling,
                                     kv_capacity=cap, num_splits=splits)
    if PROFILE is not None:
        ev1.record()
        PROFILE.append((ev0, ev1, key.shape[2] - n, n, query.shape[1], key.shape[1]))
    return out.unsqueeze(0), None


def register() -> str:
    """Register the backend with transformers and return its name."""
    from transformers import AttentionInterface

    AttentionInterface.register(NAME, tree_attention_forward)
    return NAME
