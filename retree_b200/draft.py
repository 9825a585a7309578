"""The DFlash block-draft forward as fused stages over preallocated buffers.

``FusedDraft(draft, target, capacity)`` runs ``DFlashDraftModel.forward``
(model/dflash.py:212-238) followed by the target's ``lm_head`` -- the draft
call of the decode loops (ddtree.py:828-846, retree.py:300-315) -- on this
package's kernels, with the draft's KV cache in one slab.  Per call:

  context rows (the target's layer outputs of the tokens committed since the
  last call; the whole prompt on the first call), in chunks:
      fc projection + ``hidden_norm``       cuBLAS + rt_add_rmsnorm
      per layer: packed q|k|v projection    cuBLAS (or rt_linear)
                 k head norm + rotary, K/V appended at the cache length
                                            rt_qk_norm_rope_append
  the block's rows (root token + mask tokens), per layer:
      rt_embed_rmsnorm / rt_add_rmsnorm     residual stream + input norm
      q|k|v projection + head norms + rotary + append after the context
      rt_tree_attn                          every cached row visible (the
                                            draft attends without a causal
                                            mask: an all-ones block mask)
      o projection, rt_add_rmsnorm, gate|up projection + rt_silu_mul, down
  final norm, the target's lm_head over the last ``horizon`` rows.

The reference projects the context rows and the block's rows with separate
``k_proj``/``v_proj`` calls and normalises/rotates both (dflash.py:93-107);
here the context rows go through the same packed projection (their q heads
are computed and dropped).  After the call the cache is cropped back to
``start`` (the block's rows are never kept), as ``past_key_values_draft.crop
(start)`` does.

The draft module is read through the reference's attribute layout
(``layers[i].self_attn.q_proj`` ..., ``fc``, ``hidden_norm``, ``norm``,
``rotary_emb``); its q/k/v and gate/up weights are packed like the target's
(the modules keep views).
"""

from __future__ import annotations

import torch

from . import kernels
from .cache import TreeKVCache
from .fused import _Layer, _pack, rope_tables


def supports(draft, target=None) -> bool:
    """Whether ``FusedDraft`` can run this draft module (and target)."""
    need = ("layers", "fc", "hidden_norm", "norm", "rotary_emb", "config")
    if not all(hasattr(draft, a) for a in need):
        return False
    cfg = draft.config
    hd = getattr(cfg, "head_dim", None) or cfg.hidden_size // cfg.num_attention_heads
    if hd != 128 or cfg.hidden_size % 8 or cfg.intermediate_size % 8:
        return False
    if getattr(cfg, "hidden_act", "silu") != "silu" or getattr(cfg, "mlp_bias", False):
        return False
    if any(t == "sliding_attention" for t in (getattr(cfg, "layer_types", None) or [])):
        return False
    for attr in ("rope_parameters", "rope_scaling"):
        rs = getattr(cfg, attr, None) or {}
        if isinstance(rs, dict) and rs.get("rope_type", rs.get("type")) in ("dynamic", "longrope"):
            return False
    try:
        for layer in draft.layers:
            a = layer.self_attn
            if getattr(a, "q_norm", None) is None or getattr(a, "k_norm", None) is None:
                return False
    except (AttributeError, TypeError):
        return False
    if next(draft.parameters()).dtype != torch.bfloat16:
        return False
    if target is not None:
        if target.config.hidden_size != cfg.hidden_size:
            return False
        if next(target.parameters()).dtype != torch.bfloat16:
            return False
    return True


class FusedDraft:
    """DFlash draft forward + the target's lm_head on the fused stages (one request)."""

    def __init__(self, draft, target, capacity: int, block_size: int | None = None, ctx_chunk: int = 1024,
                 gemm: str = "cublas"):
        if not supports(draft, target):
            raise RuntimeError("FusedDraft does not support this draft module")
        if gemm not in ("cublas", "tcgen05"):
            raise ValueError("gemm must be 'cublas' or 'tcgen05'")
        cfg = draft.config
        dev = next(draft.parameters()).device
        self.device = dev
        self.gemm = gemm
        self.head_dim = getattr(cfg, "head_dim", None) or cfg.hidden_size // cfg.num_attention_heads
        self.hidden = cfg.hidden_size
        self.inter = cfg.intermediate_size
        self.block = int(block_size if block_size is not None else getattr(draft, "block_size", cfg.block_size))
        self.capacity = int(capacity)
        self.ctx_chunk = int(ctx_chunk)
        self.embed = target.model.embed_tokens.weight
        self.lm_head = target.lm_head.weight
        self.vocab = self.lm_head.shape[0]
        self.eps = float(getattr(draft.norm, "variance_epsilon", cfg.rms_norm_eps))
        self.final_norm = draft.norm.weight
        self.fc_w = draft.fc.weight
        self.fc_b = draft.fc.bias
        self.hidden_norm = draft.hidden_norm.weight
        self.eps_hidden = float(getattr(draft.hidden_norm, "variance_epsilon", cfg.rms_norm_eps))
        self.ctx_width = self.fc_w.shape[1]
        self.layers = []
        with torch.no_grad():
            for i, layer in enumerate(draft.layers):
                a, m = layer.self_attn, layer.mlp
                L = _Layer()
                L.index = i
                L.in_norm = layer.input_layernorm.weight
                L.post_norm = layer.post_attention_layernorm.weight
                L.eps_in = float(getattr(layer.input_layernorm, "variance_epsilon", cfg.rms_norm_eps))
                L.eps_post = float(getattr(layer.post_attention_layernorm, "variance_epsilon", cfg.rms_norm_eps))
                L.qkv_w, L.qkv_b = _pack([a.q_proj, a.k_proj, a.v_proj])
                L.gate_up_w, _ = _pack([m.gate_proj, m.up_proj])
                L.o_w, L.o_b = a.o_proj.weight, a.o_proj.bias
                L.down_w = m.down_proj.weight
                L.hq = a.q_proj.weight.shape[0] // self.head_dim
                L.hkv = a.k_proj.weight.shape[0] // self.head_dim
                L.q_norm, L.k_norm = a.q_norm.weight, a.k_norm.weight
                L.eps_qk = float(getattr(a.q_norm, "variance_epsilon", cfg.rms_norm_eps))
                L.scale = float(getattr(a, "scaling", self.head_dim ** -0.5))
                self.layers.append(L)
        self.hq, self.hkv = self.layers[0].hq, self.layers[0].hkv
        self.cache = TreeKVCache(len(self.layers), self.hkv, self.head_dim, self.capacity, device=dev)
        self.cos, self.sin = rope_tables(draft.rotary_emb, dev, self.capacity)
        self.positions = torch.arange(self.capacity, dtype=torch.int64, device=dev)
        b, d, e = self.block, self.head_dim, dict(dtype=torch.bfloat16, device=dev)
        ch = self.ctx_chunk
        self.ctx = torch.empty((ch, self.hidden), **e)
        self.ctx_norm = torch.empty((ch, self.hidden), **e)
        self.ctx_qkv = torch.empty((ch, (self.hq + 2 * self.hkv) * d), **e)
        self.ctx_q = torch.empty((ch, self.hq, d), **e)
        self.residual = torch.empty((b, self.hidden), **e)
        self.xnorm = torch.empty((b, self.hidden), **e)
        self.qkv = torch.empty((b, (self.hq + 2 * self.hkv) * d), **e)
        self.q = torch.empty((b, self.hq, d), **e)
        self.attn = torch.empty((b, self.hq, d), **e)
        self.o = torch.empty((b, self.hidden), **e)
        self.gate_up = torch.empty((b, 2 * self.inter), **e)
        self.act = torch.empty((b, self.inter), **e)
        self.mlp_out = torch.empty((b, self.hidden), **e)
        self.logits = torch.empty((b, self.vocab), **e)
        # every block row sees every cached row and every block row
        self.visible = torch.full((b, (b + 31) // 32), -1, dtype=torch.int32, device=dev)
        self.length = 0  # rows kept in the draft cache (the reference's get_seq_length())

    def reset(self) -> None:
        self.length = 0

    def crop(self, length: int) -> None:
        if length < 0 or length > self.length:
            raise ValueError("crop past the cached rows")
        self.length = int(length)

    def _mm(self, x, w, b, out):
        if self.gemm == "tcgen05" and b is None and kernels.linear_supported(x.shape[0], w.shape[0], x.shape[1], 0):
            return kernels.linear(x, w, out=out)
        if b is None:
            return torch.mm(x, w.t(), out=out)
        return torch.addmm(b, x, w.t(), out=out)

    def _context(self, target_hidden: torch.Tensor) -> None:
        """fc + hidden_norm of the new context rows and their K/V in every layer (appended at the cache length)."""
        c = target_hidden.shape[0]
        for c0 in range(0, c, self.ctx_chunk):
            rows = min(self.ctx_chunk, c - c0)
            at = self.length + c0
            th = self._mm(target_hidden[c0: c0 + rows], self.fc_w, self.fc_b, self.ctx[:rows])
            xn = kernels.add_rmsnorm(None, th, self.hidden_norm, self.eps_hidden, self.ctx_norm[:rows])
            pos = self.positions[at: at + rows]
            for L in self.layers:
                kc, vc = self.cache.slab[2 * L.index], self.cache.slab[2 * L.index + 1]
                qkv = self._mm(xn, L.qkv_w, L.qkv_b, self.ctx_qkv[:rows])
                kernels.qk_norm_rope_append(qkv, L.hq, L.hkv, L.q_norm, L.k_norm, L.eps_qk, self.cos, self.sin, pos,
                                            self.ctx_q[:rows], kc, vc, offset=at)

    @torch.inference_mode()
    def forward(self, block_ids: torch.Tensor, target_hidden: torch.Tensor, start: int,
                horizon: int | None = None, return_hidden: bool = False) -> torch.Tensor:
        """Draft logits ``[horizon, vocab]`` (bf16 view of a reused buffer) for one block.

        ``block_ids``: int64 ``[block]`` (the committed token at ``start``, then
        mask tokens); ``target_hidden``: ``[c, n_target_layers * hidden]``, the
        target's layer outputs at positions ``[cache length, start)``.
        ``horizon`` (default ``block - 1``) trailing rows go through the
        lm_head; ``return_hidden`` returns the draft's normed ``[block, hidden]``
        output instead.  The cache is cropped to ``start`` on return.
        """
        block_ids = block_ids.reshape(-1)
        b = block_ids.numel()
        if b != self.block:
            raise RuntimeError(f"block of {b} ids, the draft runs blocks of {self.block}")
        if target_hidden.dim() == 3:
            target_hidden = target_hidden[0]
        c = target_hidden.shape[0]
        if target_hidden.shape[1] != self.ctx_width or target_hidden.dtype != torch.bfloat16:
            raise RuntimeError("target_hidden must be bf16 [c, n_target_layers * hidden]")
        if self.length + c != start:
            raise RuntimeError(f"draft cache holds {self.length} rows + {c} context rows != start {start}")
        if start + b > self.capacity:
            raise RuntimeError("draft cache capacity exceeded")
        horizon = b - 1 if horizon is None else int(horizon)
        if not 0 < horizon <= b:
            raise ValueError("horizon must be in [1, block]")
        target_hidden = target_hidden.contiguous()
        if c > 0:
            self._context(target_hidden)
        pos = self.positions[start: start + b]
        res, xn = self.residual, self.xnorm
        splits = kernels.default_splits(b, self.hq, self.hkv, start)
        for L in self.layers:
            if L.index == 0:
                kernels.embed_rmsnorm(block_ids, self.embed, L.in_norm, L.eps_in, res, xn)
            else:
                kernels.add_rmsnorm(self.mlp_out, res, L.in_norm, L.eps_in, xn)
            kc, vc = self.cache.slab[2 * L.index], self.cache.slab[2 * L.index + 1]
            qkv = self._mm(xn, L.qkv_w, L.qkv_b, self.qkv)
            kernels.qk_norm_rope_append(qkv, L.hq, L.hkv, L.q_norm, L.k_norm, L.eps_qk, self.cos, self.sin, pos,
                                        self.q, kc, vc, offset=start)
            kernels.tree_attention(self.q, kc[:, : start + b], vc[:, : start + b], self.visible, start,
                                   scale=L.scale, out=self.attn, num_splits=splits, kv_capacity=self.capacity)
            self._mm(self.attn.view(b, -1), L.o_w, L.o_b, self.o)
            kernels.add_rmsnorm(self.o, res, L.post_norm, L.eps_post, xn)
            kernels.silu_mul(self._mm(xn, L.gate_up_w, None, self.gate_up), self.act)
            self._mm(self.act, L.down_w, None, self.mlp_out)
        kernels.add_rmsnorm(self.mlp_out, res, self.final_norm, self.eps, xn)
        self.length = start  # crop(start): the block's rows are not kept
        if return_hidden:
            return xn
        return torch.mm(xn[b - horizon:], self.lm_head.t(), out=self.logits[:horizon])


class _DraftAttention(torch.nn.Module):
    pass


class _DraftLayer(torch.nn.Module):
    pass


class DraftLayout(torch.nn.Module):
    """A DFlash draft's parameters under the reference module's names (model/dflash.py:33-75, :127-139,
    :176-209), with no forward of its own: what ``FusedDraft`` reads.  For synthetic-weight benchmarks."""


def random_draft(hidden: int, layers: int, heads: int, kv_heads: int, inter: int, block_size: int,
                 target_layer_ids, device, seed: int = 0, rope_theta: float = 1_000_000.0,
                 max_positions: int = 40960) -> DraftLayout:
    """A bf16 draft with the reference's layout and N(0, 1/fan_in) projections (norm scales 1)."""
    from torch import nn
    from transformers import Qwen3Config
    from transformers.models.qwen3.modeling_qwen3 import Qwen3RMSNorm, Qwen3RotaryEmbedding

    cfg = Qwen3Config(hidden_size=hidden, intermediate_size=inter, num_hidden_layers=layers,
                      num_attention_heads=heads, num_key_value_heads=kv_heads, head_dim=128, rms_norm_eps=1e-6,
                      max_position_embeddings=max_positions, rope_theta=rope_theta)
    cfg.block_size = block_size
    g = torch.Generator(device="cpu").manual_seed(seed)

    def lin(i, o):
        m = nn.Linear(i, o, bias=False, device="meta")
        m.weight = nn.Parameter((torch.randn((o, i), generator=g) * i ** -0.5).to(torch.bfloat16).to(device),
                                requires_grad=False)
        return m

    def norm(n):
        return Qwen3RMSNorm(n, eps=cfg.rms_norm_eps).to(device=device, dtype=torch.bfloat16).requires_grad_(False)

    d = DraftLayout()
    d.config = cfg
    d.block_size = block_size
    d.target_layer_ids = list(target_layer_ids)
    d.layers = nn.ModuleList()
    for _ in range(layers):
        L = _DraftLayer()
        a = _DraftAttention()
        a.q_proj, a.k_proj, a.v_proj = lin(hidden, heads * 128), lin(hidden, kv_heads * 128), lin(hidden, kv_heads * 128)
        a.o_proj = lin(heads * 128, hidden)
        a.q_norm, a.k_norm = norm(128), norm(128)
        a.scaling = 128 ** -0.5
        L.self_attn = a
        L.mlp = nn.Module()
        L.mlp.gate_proj, L.mlp.up_proj, L.mlp.down_proj = lin(hidden, inter), lin(hidden, inter), lin(inter, hidden)
        L.input_layernorm, L.post_attention_layernorm = norm(hidden), norm(hidden)
        d.layers.append(L)
    d.fc = lin(len(d.target_layer_ids) * hidden, hidden)
    d.hidden_norm, d.norm = norm(hidden), norm(hidden)
    d.rotary_emb = Qwen3RotaryEmbedding(cfg, device=device)
    return d
