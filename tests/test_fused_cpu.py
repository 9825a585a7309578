"""Host logic of the fused verify forward that needs no GPU: which models it takes, and the packed
projection weights (the HF modules keep row-block views, so the module forward is unchanged)."""

import torch

from retree_b200 import fused
from retree_b200.target import build_target, qwen3_config


def _small(**kw):
    base = dict(hidden_size=256, intermediate_size=512, num_hidden_layers=2, num_attention_heads=4,
                num_key_value_heads=2, vocab_size=300, tie_word_embeddings=False)
    base.update(kw)
    return qwen3_config("small", **base)


def test_supports_qwen3_geometry_and_refuses_others():
    m = build_target(_small(), device="cpu", seed=0, attn_implementation="sdpa")
    assert fused.supports(m)
    m32 = build_target(_small(), device="cpu", seed=0, attn_implementation="sdpa", dtype=torch.float32)
    assert not fused.supports(m32)                        # bf16 weights only
    odd = build_target(_small(), device="cpu", seed=0, attn_implementation="sdpa")
    odd.config.head_dim = 64
    assert not fused.supports(odd)                        # head_dim 128 only
    gelu = build_target(_small(), device="cpu", seed=0, attn_implementation="sdpa")
    gelu.config.hidden_act = "gelu"
    assert not fused.supports(gelu)


@torch.inference_mode()
def test_packed_projection_weights_leave_the_module_forward_unchanged():
    m = build_target(_small(), device="cpu", seed=3, attn_implementation="sdpa", dtype=torch.float32)
    ids = torch.randint(0, 300, (1, 9), generator=torch.Generator().manual_seed(1))
    before = m(ids).logits.clone()
    layer = m.model.layers[0]
    q0, k0, v0 = (layer.self_attn.q_proj.weight.clone(), layer.self_attn.k_proj.weight.clone(),
                  layer.self_attn.v_proj.weight.clone())
    g0, u0 = layer.mlp.gate_proj.weight.clone(), layer.mlp.up_proj.weight.clone()
    packed = {}
    for i, L in enumerate(m.model.layers):
        packed[i] = (fused._pack([L.self_attn.q_proj, L.self_attn.k_proj, L.self_attn.v_proj])[0],
                     fused._pack([L.mlp.gate_proj, L.mlp.up_proj])[0])
    qkv, gu = packed[0]
    assert torch.equal(qkv, torch.cat([q0, k0, v0])) and torch.equal(gu, torch.cat([g0, u0]))
    # the modules now hold views of the packed tensors (no second copy of the weights)
    assert layer.self_attn.q_proj.weight.data_ptr() == qkv.data_ptr()
    assert layer.self_attn.k_proj.weight.data_ptr() == qkv.data_ptr() + q0.numel() * qkv.element_size()
    assert layer.mlp.up_proj.weight.data_ptr() == gu.data_ptr() + g0.numel() * gu.element_size()
    assert torch.equal(m(ids).logits, before)
