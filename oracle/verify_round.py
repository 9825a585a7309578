"""The reference's verify round on the host CPU (test / baseline infrastructure only).

Restates one round of ``ddtree_generate`` (ddtree.py:853-924) with the
reference's own building blocks: the tree from ``oracle.tree`` (top-k on the
fp32 draft logits, best-first expansion, visibility), the dense additive mask
of ``compile_ddtree_tree`` (ddtree.py:629-640), one HF ``Qwen3ForCausalLM``
forward with ``attn_implementation="sdpa"`` over a ``DynamicCache``
(transformers 5.5.0), argmax, the exact walk, and the index_select + copy
compaction of ``_compact_appended_window`` (ddtree.py:683-686) on every
layer, then ``crop``.  bench.py times it on the machine's host cores as the
CPU baseline; nothing in the product calls it.

The prefix KV cache is filled with seeded random values instead of running a
prompt prefill (a 2048-token CPU prefill of a 4B model would dominate the
sample); the round's work does not depend on the values.
"""

from __future__ import annotations

import math

import numpy as np
import torch
from transformers import DynamicCache, Qwen3ForCausalLM
from transformers.models.qwen3.modeling_qwen3 import Qwen3RotaryEmbedding

from . import tree as ot


def _fill_(t: torch.Tensor, base: torch.Tensor) -> None:
    flat = t.view(-1)
    reps = math.ceil(flat.numel() / base.numel())
    flat.copy_(base.repeat(reps)[: flat.numel()])


def cpu_target(config, dtype=torch.bfloat16, seed: int = 0) -> Qwen3ForCausalLM:
    """The target on the host with random-pattern weights (cheap to materialise)."""
    config._attn_implementation = "sdpa"
    prev = torch.get_default_dtype()
    torch.set_default_dtype(dtype)
    try:
        with torch.device("meta"):
            model = Qwen3ForCausalLM(config)
    finally:
        torch.set_default_dtype(prev)
    model = model.to_empty(device="cpu")
    g = torch.Generator().manual_seed(seed)
    base = (torch.randn(1 << 20, generator=g) * 0.02).to(dtype)
    with torch.no_grad():
        for p in model.parameters():
            _fill_(p, base)
        for m in model.modules():
            if m.__class__.__name__.endswith("RMSNorm"):
                m.weight.fill_(1.0)
    model.model.rotary_emb = Qwen3RotaryEmbedding(config=config)
    model.config._attn_implementation = "sdpa"
    return model.eval().requires_grad_(False)


class CpuVerifyRound:
    def __init__(self, config, prompt_len: int, budget: int, strategy: str = "rank_gated_ngram",
                 params: ot.NgramParams | None = None, seed: int = 0, dtype=torch.bfloat16):
        self.model = cpu_target(config, dtype=dtype, seed=seed)
        self.config = config
        self.budget = budget
        self.strategy = strategy
        self.params = params or ot.NgramParams()
        self.dtype = dtype
        hkv = config.num_key_value_heads
        hd = getattr(config, "head_dim", None) or config.hidden_size // config.num_attention_heads
        g = torch.Generator().manual_seed(seed + 1)
        self.cache = DynamicCache()
        for li in range(config.num_hidden_layers):
            k = torch.randn((1, hkv, prompt_len, hd), generator=g).to(dtype)
            v = torch.randn((1, hkv, prompt_len, hd), generator=g).to(dtype)
            self.cache.update(k, v, li)
        rng = np.random.default_rng(seed)
        self.output_ids = list(rng.integers(0, config.vocab_size, size=prompt_len + 1))
        self.start = prompt_len

    @torch.inference_mode()
    def round(self, draft_logits: np.ndarray) -> int:
        start = self.start
        tree = ot.build_tree_from_logits(np.asarray(draft_logits, np.float32), self.budget, self.strategy,
                                         self.output_ids[: start + 1], self.params)
        ids, pos, mask = ot.compile_tree(self.output_ids[start], start, tree.tokens, tree.depths, tree.parents,
                                         start, float(torch.finfo(self.dtype).min))
        n = ids.shape[0]
        out = self.model(torch.from_numpy(ids)[None], position_ids=torch.from_numpy(pos)[None],
                         attention_mask=torch.from_numpy(mask).to(self.dtype)[None, None],
                         past_key_values=self.cache, use_cache=True)
        posterior = out.logits[0].argmax(-1).numpy()
        acc, nxt = ot.follow_tree(ot.child_maps(tree.parents, tree.tokens), posterior)
        self.output_ids[start: start + len(acc)] = [int(ids[i]) for i in acc]
        self.output_ids[start + len(acc): start + len(acc) + 1] = [int(nxt)]
        if 0 < len(acc) < n:
            keep = torch.tensor(acc, dtype=torch.long)
            for layer in self.cache.layers:
                for t in (layer.keys, layer.values):
                    kept = t.narrow(-2, start, n).index_select(-2, keep)
                    t.narrow(-2, start, len(acc)).copy_(kept)
        self.cache.crop(start + len(acc))
        self.start = start + len(acc)
        return len(acc)
