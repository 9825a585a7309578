"""The DFlash block-draft forward restated in torch (test infrastructure only).

Restates ``DFlashDraftModel.forward`` (model/dflash.py:212-238) with its
decoder layer (:154-174) and attention (:76-124):

  target_hidden = hidden_norm(fc(concat of the target's layer outputs))
  h = noise embedding of the block ``[root, mask, mask, ...]``
  per layer:
      x = input_layernorm(h)
      q = q_norm(q_proj(x))                     (noise rows only)
      k = k_norm(k_proj([target_hidden ; x]))   (context rows, then noise rows)
      v = v_proj([target_hidden ; x])
      rotary at the positions [cache length, start + block)  -- q takes the
        last ``block`` positions (:23-29)
      K/V appended to the draft cache, then attention of the noise rows over
        every cached row, no causal mask (``is_causal=False``, :47 and the
        callers' ``is_causal=False`` kwarg: sdpa_attention.py:65-77)
      h = h + o_proj(attn);  h = h + mlp(post_attention_layernorm(h))
  out = norm(h)

The caller crops the draft cache back to ``start`` after each call, so the
noise rows never stay cached (ddtree.py:832-846, retree.py:300-315).

``DraftModule`` carries the reference's attribute layout (``layers[i].self_attn
.q_proj`` ... ``fc``, ``hidden_norm``, ``norm``, ``rotary_emb``) so the fused
draft forward reads it like the reference's module; its ``forward`` is the
restatement, built from transformers' Qwen3 RMSNorm / MLP / rotary modules as
the reference's is.  ``seeded_weights`` makes the weights from a seed so the
golden vectors (tests/golden/make_dflash_golden.py, written by the reference's
own module) and the tests agree without storing weights.
"""

from __future__ import annotations

from types import SimpleNamespace

import torch
import torch.nn.functional as F
from torch import nn
from transformers import Qwen3Config
from transformers.models.qwen3.modeling_qwen3 import Qwen3MLP, Qwen3RMSNorm, Qwen3RotaryEmbedding, rotate_half


def small_config(hidden: int = 256, layers: int = 2, heads: int = 4, kv_heads: int = 2, inter: int = 512,
                 target_layers: int = 2, block_size: int = 8, rope_theta: float = 1_000_000.0,
                 max_positions: int = 4096) -> Qwen3Config:
    """A small DFlash draft configuration (head_dim 128, the fused kernels' head size)."""
    cfg = Qwen3Config(vocab_size=1024, hidden_size=hidden, intermediate_size=inter, num_hidden_layers=layers,
                      num_attention_heads=heads, num_key_value_heads=kv_heads, head_dim=128, rms_norm_eps=1e-6,
                      max_position_embeddings=max_positions, rope_theta=rope_theta, tie_word_embeddings=False)
    cfg.num_target_layers = 2 * target_layers + 4
    cfg.block_size = block_size
    cfg.dflash_config = {"mask_token_id": 3, "target_layer_ids": list(range(1, 1 + 2 * target_layers, 2))}
    cfg._attn_implementation = "sdpa"
    return cfg


def weight_shapes(cfg) -> dict[str, tuple[int, ...]]:
    """Parameter names (the reference module's state_dict keys) and shapes."""
    h, d = cfg.hidden_size, cfg.head_dim
    hq, hkv, inter = cfg.num_attention_heads, cfg.num_key_value_heads, cfg.intermediate_size
    nt = len(cfg.dflash_config["target_layer_ids"])
    shapes = {}
    for i in range(cfg.num_hidden_layers):
        p = f"layers.{i}."
        shapes[p + "self_attn.q_proj.weight"] = (hq * d, h)
        shapes[p + "self_attn.k_proj.weight"] = (hkv * d, h)
        shapes[p + "self_attn.v_proj.weight"] = (hkv * d, h)
        shapes[p + "self_attn.o_proj.weight"] = (h, hq * d)
        shapes[p + "self_attn.q_norm.weight"] = (d,)
        shapes[p + "self_attn.k_norm.weight"] = (d,)
        shapes[p + "input_layernorm.weight"] = (h,)
        shapes[p + "post_attention_layernorm.weight"] = (h,)
        shapes[p + "mlp.gate_proj.weight"] = (inter, h)
        shapes[p + "mlp.up_proj.weight"] = (inter, h)
        shapes[p + "mlp.down_proj.weight"] = (h, inter)
    shapes["fc.weight"] = (h, nt * h)
    shapes["hidden_norm.weight"] = (h,)
    shapes["norm.weight"] = (h,)
    return shapes


def seeded_weights(cfg, seed: int = 0) -> dict[str, torch.Tensor]:
    """fp32 weights from a CPU generator: N(0, 1/fan_in) projections, 1 + N(0, 0.1^2) norm scales."""
    g = torch.Generator().manual_seed(seed)
    out = {}
    for name, shape in weight_shapes(cfg).items():
        if len(shape) == 2:
            out[name] = torch.randn(shape, generator=g) * shape[1] ** -0.5
        else:
            out[name] = 1.0 + 0.1 * torch.randn(shape, generator=g)
    return out


def seeded_inputs(cfg, seed: int, ctx_rows: int, block: int | None = None) -> tuple[torch.Tensor, torch.Tensor]:
    """(target_hidden ``[ctx_rows, n_target_layers * hidden]``, noise embedding ``[block, hidden]``), fp32 N(0,1)."""
    g = torch.Generator().manual_seed(seed)
    block = cfg.block_size if block is None else block
    nt = len(cfg.dflash_config["target_layer_ids"])
    th = torch.randn((ctx_rows, nt * cfg.hidden_size), generator=g)
    noise = torch.randn((block, cfg.hidden_size), generator=g)
    return th, noise


class _Attention(nn.Module):
    def __init__(self, cfg, layer_idx: int):
        super().__init__()
        h, d = cfg.hidden_size, cfg.head_dim
        self.layer_idx = layer_idx
        self.head_dim = d
        self.num_key_value_groups = cfg.num_attention_heads // cfg.num_key_value_heads
        self.scaling = d ** -0.5
        self.is_causal = False
        bias = bool(getattr(cfg, "attention_bias", False))
        self.q_proj = nn.Linear(h, cfg.num_attention_heads * d, bias=bias)
        self.k_proj = nn.Linear(h, cfg.num_key_value_heads * d, bias=bias)
        self.v_proj = nn.Linear(h, cfg.num_key_value_heads * d, bias=bias)
        self.o_proj = nn.Linear(cfg.num_attention_heads * d, h, bias=bias)
        self.q_norm = Qwen3RMSNorm(d, eps=cfg.rms_norm_eps)
        self.k_norm = Qwen3RMSNorm(d, eps=cfg.rms_norm_eps)

    def forward(self, x, target_hidden, cos, sin, cache):
        # model/dflash.py:76-124 (batch 1)
        b, n = x.shape[:2]
        c = target_hidden.shape[1]
        d = self.head_dim
        q = self.q_norm(self.q_proj(x).view(b, n, -1, d)).transpose(1, 2)
        k = torch.cat([self.k_proj(target_hidden), self.k_proj(x)], dim=1).view(b, c + n, -1, d)
        v = torch.cat([self.v_proj(target_hidden), self.v_proj(x)], dim=1).view(b, c + n, -1, d)
        k = self.k_norm(k).transpose(1, 2)
        v = v.transpose(1, 2)
        cos, sin = cos.unsqueeze(1), sin.unsqueeze(1)
        q = q * cos[..., -n:, :] + rotate_half(q) * sin[..., -n:, :]
        k = k * cos + rotate_half(k) * sin
        if cache is not None:
            k, v = cache.update(k, v, self.layer_idx)
        groups = self.num_key_value_groups
        out = F.scaled_dot_product_attention(q, k.repeat_interleave(groups, dim=1), v.repeat_interleave(groups, dim=1),
                                             scale=self.scaling, is_causal=False)
        return self.o_proj(out.transpose(1, 2).reshape(b, n, -1))


class _Layer(nn.Module):
    def __init__(self, cfg, layer_idx: int):
        super().__init__()
        self.self_attn = _Attention(cfg, layer_idx)
        self.mlp = Qwen3MLP(cfg)
        self.input_layernorm = Qwen3RMSNorm(cfg.hidden_size, eps=cfg.rms_norm_eps)
        self.post_attention_layernorm = Qwen3RMSNorm(cfg.hidden_size, eps=cfg.rms_norm_eps)

    def forward(self, h, target_hidden, cos, sin, cache):
        # model/dflash.py:154-174
        h = h + self.self_attn(self.input_layernorm(h), target_hidden, cos, sin, cache)
        return h + self.mlp(self.post_attention_layernorm(h))


class DraftModule(nn.Module):
    """The reference draft's module layout with the restated forward (model/dflash.py:176-238)."""

    def __init__(self, cfg):
        super().__init__()
        self.config = cfg
        self.layers = nn.ModuleList([_Layer(cfg, i) for i in range(cfg.num_hidden_layers)])
        self.target_layer_ids = list(cfg.dflash_config["target_layer_ids"])
        self.norm = Qwen3RMSNorm(cfg.hidden_size, eps=cfg.rms_norm_eps)
        self.rotary_emb = Qwen3RotaryEmbedding(cfg)
        self.fc = nn.Linear(len(self.target_layer_ids) * cfg.hidden_size, cfg.hidden_size, bias=False)
        self.hidden_norm = Qwen3RMSNorm(cfg.hidden_size, eps=cfg.rms_norm_eps)
        self.block_size = cfg.block_size
        self.mask_token_id = cfg.dflash_config["mask_token_id"]

    def forward(self, position_ids, attention_mask=None, noise_embedding=None, target_hidden=None,
                past_key_values=None, use_cache=False, **kwargs):
        if attention_mask is not None:
            raise NotImplementedError("the draft runs without a mask")
        h = noise_embedding
        target_hidden = self.hidden_norm(self.fc(target_hidden))
        cos, sin = self.rotary_emb(h, position_ids)
        for layer in self.layers:
            h = layer(h, target_hidden, cos, sin, past_key_values)
        return self.norm(h)


def build_module(cfg, weights: dict[str, torch.Tensor], dtype=torch.float32, device="cpu") -> DraftModule:
    m = DraftModule(cfg)
    missing, unexpected = m.load_state_dict(weights, strict=False)
    if unexpected or [k for k in missing if not k.endswith("inv_freq")]:
        raise RuntimeError(f"weights do not match the draft layout: {missing} {unexpected}")
    return m.to(device=device, dtype=dtype).eval()


def run_calls(module: DraftModule, calls, device="cpu", dtype=torch.float32) -> list[torch.Tensor]:
    """Consecutive draft calls over one draft cache, cropped after each as the decode loops do.

    ``calls``: list of (target_hidden ``[c, nT*H]``, noise ``[block, H]``);
    call j's positions run from the cache length to ``start_j + block`` where
    ``start_j`` = the context rows seen so far.  Returns each call's ``[block, H]``.
    """
    from transformers import DynamicCache

    cache = DynamicCache()
    outs, start = [], 0
    with torch.no_grad():
        for th, noise in calls:
            c, blk = th.shape[0], noise.shape[0]
            past = cache.get_seq_length()
            start = past + c
            pos = torch.arange(past, start + blk, device=device).unsqueeze(0)
            out = module(position_ids=pos, noise_embedding=noise.to(device, dtype).unsqueeze(0),
                         target_hidden=th.to(device, dtype).unsqueeze(0), past_key_values=cache, use_cache=True,
                         is_causal=False)
            cache.crop(start)
            outs.append(out[0])
    return outs


GOLDEN_CALLS = SimpleNamespace(seed=0, input_seeds=(11, 12, 13), ctx_rows=(40, 5, 9))
