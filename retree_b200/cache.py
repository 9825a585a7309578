"""Preallocated KV cache for tree verification (a ``transformers.Cache``).

Replaces ``DynamicCache``'s per-round ``torch.cat`` of every layer
(transformers/cache_utils.py:102-121) with one HBM slab

    slab[2*layer + {0: K, 1: V}, kv_head, position, head_dim]   (bf16, zeroed)

written in place by the ``rt_kv_append`` kernel.  ``layers[i].keys`` /
``.values`` are views ``[1, kv_heads, length, head_dim]`` of the slab, so code
written against ``DynamicCache`` (the reference's ``compact_dynamic_cache``,
ddtree.py:717-729) keeps working, and the slab as a whole is compacted in ONE
launch by ``retree_b200.ddtree.compact_dynamic_cache``.

Positions past a layer's length are never garbage: the slab starts zeroed and
only ever holds K/V rows, so the attention kernel may read whole 128-key
blocks past the end (they are masked, and finite).

Device-length mode (``use_device_length(True)``): appends land at the offset
held in ``length_dev`` (int64[1] on the device) and ``update`` returns views of
the full capacity, so a verify forward can be captured once in a CUDA graph
and replayed at any prefix length; the attention plugin then reads the prefix
length from the same device word.
"""

from __future__ import annotations

import torch
from transformers.cache_utils import Cache, CacheLayerMixin

from . import kernels


class TreeKVLayer(CacheLayerMixin):
    is_sliding = False
    is_compileable = False

    def __init__(self, cache: "TreeKVCache", index: int):
        super().__init__()
        self._cache = cache
        self.index = index
        self.length = 0
        self.is_initialized = True
        self.dtype = cache.dtype
        self.device = cache.device

    # views of the slab -----------------------------------------------------
    def _view(self, kv: int, length: int) -> torch.Tensor:
        return self._cache.slab[2 * self.index + kv, :, :length, :].unsqueeze(0)

    @property
    def keys(self) -> torch.Tensor:  # type: ignore[override]
        return self._view(0, self.length)

    @keys.setter
    def keys(self, value):
        if value is not None:
            raise AttributeError("TreeKVLayer keys are views of the preallocated slab")

    @property
    def values(self) -> torch.Tensor:  # type: ignore[override]
        return self._view(1, self.length)

    @values.setter
    def values(self, value):
        if value is not None:
            raise AttributeError("TreeKVLayer values are views of the preallocated slab")

    # CacheLayerMixin ---------------------------------------------------------
    def lazy_initialization(self, key_states, value_states) -> None:
        return None

    def update(self, key_states: torch.Tensor, value_states: torch.Tensor, *args, **kwargs):
        c = self._cache
        n = key_states.shape[-2]
        kc = c.slab[2 * self.index]
        vc = c.slab[2 * self.index + 1]
        if c.device_length:
            kernels.kv_append(kc, vc, key_states, value_states, offset_dev=c.length_dev)
            self.length = c.capacity
            return self._view(0, c.capacity), self._view(1, c.capacity)
        if self.length + n > c.capacity:
            raise RuntimeError(f"TreeKVCache capacity {c.capacity} exceeded ({self.length} + {n})")
        kernels.kv_append(kc, vc, key_states, value_states, offset=self.length)
        self.length += n
        return self.keys, self.values

    def get_mask_sizes(self, query_length: int) -> tuple[int, int]:
        return self.length + query_length, 0

    def get_seq_length(self) -> int:
        return self.length

    def get_max_cache_shape(self) -> int:
        return self._cache.capacity

    def crop(self, max_length: int) -> None:
        if max_length < 0:
            max_length = self.length - abs(max_length)
        self.length = max(0, min(self.length, max_length))

    def reset(self) -> None:
        self.length = 0

    def offload(self):
        raise NotImplementedError("TreeKVCache stays resident in HBM")

    def prefetch(self):
        return None

    def reorder_cache(self, beam_idx):
        raise NotImplementedError("TreeKVCache holds one sequence")


class TreeKVCache(Cache):
    """One bf16 slab for all layers' K and V, appended and compacted in place."""

    def __init__(self, num_layers: int, num_kv_heads: int, head_dim: int, capacity: int,
                 dtype=torch.bfloat16, device=None):
        self.num_layers = int(num_layers)
        self.num_kv_heads = int(num_kv_heads)
        self.head_dim = int(head_dim)
        self.capacity = int(capacity)
        self.dtype = dtype
        self.device = torch.device(device if device is not None else "cuda")
        if self.device.type != "cuda":
            raise RuntimeError("TreeKVCache lives on a CUDA device")
        self.slab = torch.zeros((2 * self.num_layers, self.num_kv_heads, self.capacity, self.head_dim),
                                dtype=dtype, device=self.device)
        self.length_dev = torch.zeros(1, dtype=torch.int64, device=self.device)
        self.device_length = False
        super().__init__(layers=[TreeKVLayer(self, i) for i in range(self.num_layers)])

    @classmethod
    def for_model(cls, config, capacity: int, dtype=torch.bfloat16, device=None) -> "TreeKVCache":
        head_dim = getattr(config, "head_dim", None) or config.hidden_size // config.num_attention_heads
        return cls(config.num_hidden_layers, config.num_key_value_heads, head_dim, capacity, dtype, device)

    # host / device length ----------------------------------------------------
    @property
    def length(self) -> int:
        return self.layers[0].length

    def set_length(self, n: int) -> None:
        for layer in self.layers:
            layer.length = int(n)
        self.length_dev.fill_(int(n))

    def use_device_length(self, enabled: bool) -> None:
        """Append at ``length_dev`` and hand out full-capacity views (for graph capture)."""
        self.device_length = bool(enabled)

    # Cache API ---------------------------------------------------------------
    def get_seq_length(self, layer_idx: int = 0) -> int:
        return self.layers[layer_idx].length

    def get_mask_sizes(self, query_length: int, layer_idx: int = 0) -> tuple[int, int]:
        return self.layers[layer_idx].get_mask_sizes(query_length)

    def get_max_cache_shape(self, layer_idx: int = 0) -> int:
        return self.capacity

    def crop(self, max_length: int) -> None:
        for layer in self.layers:
            layer.crop(max_length)

    def reset(self) -> None:
        self.set_length(0)

    @property
    def is_compileable(self) -> bool:
        return False

    def batch_repeat_interleave(self, repeats: int):
        raise NotImplementedError("TreeKVCache holds one sequence")

    def batch_select_indices(self, indices):
        raise NotImplementedError("TreeKVCache holds one sequence")
