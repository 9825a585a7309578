"""Random-initialised Qwen3 targets for the verify benchmarks and tests.

No checkpoints are available offline, so the target is an HF
``Qwen3ForCausalLM`` with the published Qwen3-4B / Qwen3-8B geometry
(36 layers, 32 query / 8 KV heads, head_dim 128, RoPE theta 1e6, vocab 151936)
and seeded random weights, built directly on the GPU in bf16 with the
``retree_tree`` attention backend (or any other backend name, e.g. ``"sdpa"``
for the reference's path).
"""

from __future__ import annotations

import torch
from transformers import Qwen3Config, Qwen3ForCausalLM

from . import attention

GEOMETRY = {
    # name: hidden, ffn, layers, q heads, kv heads, tied embeddings
    "qwen3-4b": dict(hidden_size=2560, intermediate_size=9728, num_hidden_layers=36, num_attention_heads=32,
                     num_key_value_heads=8, tie_word_embeddings=True),
    "qwen3-8b": dict(hidden_size=4096, intermediate_size=12288, num_hidden_layers=36, num_attention_heads=32,
                     num_key_value_heads=8, tie_word_embeddings=False),
}


def qwen3_config(name: str = "qwen3-4b", **overrides) -> Qwen3Config:
    g = dict(GEOMETRY[name]) if name in GEOMETRY else {}
    g.update(overrides)
    return Qwen3Config(vocab_size=g.pop("vocab_size", 151936), head_dim=128, hidden_act="silu",
                       max_position_embeddings=g.pop("max_position_embeddings", 40960), rms_norm_eps=1e-6,
                       rope_parameters={"rope_theta": 1_000_000.0, "rope_type": "default"},
                       attention_bias=False, use_sliding_window=False, **g)


def build_target(config: Qwen3Config, device="cuda", seed: int = 0, attn_implementation: str | None = None,
                 dtype=torch.bfloat16) -> Qwen3ForCausalLM:
    """An eval-mode ``Qwen3ForCausalLM`` with seeded random weights on ``device``."""
    name = attn_implementation or attention.register()
    config._attn_implementation = name
    torch.manual_seed(seed)
    prev = torch.get_default_dtype()
    torch.set_default_dtype(dtype)
    try:
        with torch.device(device):
            model = Qwen3ForCausalLM(config)
    finally:
        torch.set_default_dtype(prev)
    model.config._attn_implementation = name
    return model.eval().requires_grad_(False)
