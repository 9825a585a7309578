"""The target's tree-verify forward as fused stages over preallocated buffers.

``FusedTarget(model, cache, n_max)`` runs the decoder stack of a
transformers Qwen3 / Qwen2 / Llama causal LM (pre-norm, rotary, GQA, SiLU
MLP) for one verify round of ``n <= n_max`` tree nodes without going through
the module tree.  Per layer the HF forward (models/qwen3/modeling_qwen3.py:
305-334 with Qwen3Attention.forward :252-299 and Qwen3MLP.forward :81-83)
issues about forty kernels -- casts, the four RMSNorm steps, rotary slicing
and concatenation, residual adds, the cache ``torch.cat`` -- around seven
projections.  Here a layer is seven launches:

  rt_add_rmsnorm     residual += mlp_out; x = rmsnorm(residual) * w_in
  rt_linear QKV      x @ [Wq;Wk;Wv]^T, epilogue: q/k head norms + rotary,
                     q out, k/v into the cache
  rt_tree_attn       the tree-masked attention kernel (+ split combine)
  rt_linear          attn @ Wo^T
  rt_add_rmsnorm     residual += o; x = rmsnorm(residual) * w_post
  rt_linear SILU     x @ [Wg;Wu]^T, epilogue: silu(gate) * up
  rt_linear          act @ Wd^T

and the stack opens with ``rt_embed_rmsnorm`` (embedding lookup + first norm)
and closes with the final norm and the lm_head projection.  The projections
are the tcgen05 kernel of ``csrc/linear.cu`` (``gemm="tcgen05"``) or cuBLAS
followed by the standalone stage kernels (``gemm="cublas"``; also used for
shapes ``rt_linear`` does not take and for biased projections); the default
``gemm="auto"`` times both per projection kind on the model's own weights at
construction and keeps the faster.
The packed projection weights are single tensors whose row blocks the HF
modules keep as views, so the model's memory does not grow and the HF
forward stays usable (prefill runs through it).

The rotary tables are the model's own ``rotary_emb`` outputs for positions
``[0, max_positions)`` (bf16, what HF computes per forward), so positions are
device-side indices.  Numerics follow the HF ops' bf16 rounding points (see
``csrc/layer_ops.cu``); the projections accumulate in fp32 and round to bf16
like the library GEMM, in their own summation order.
"""

from __future__ import annotations

import torch
from torch import nn

from . import kernels
from .headsplit import gather_heads

SUPPORTED_MODEL_TYPES = ("qwen3", "qwen2", "llama")

_AUTOTUNE: dict = {}


def supports(model) -> bool:
    """Whether ``FusedTarget`` can run this model's verify forward."""
    cfg = model.config
    if getattr(cfg, "model_type", None) not in SUPPORTED_MODEL_TYPES:
        return False
    if getattr(cfg, "hidden_act", "silu") != "silu" or getattr(cfg, "mlp_bias", False):
        return False
    hd = getattr(cfg, "head_dim", None) or cfg.hidden_size // cfg.num_attention_heads
    if hd != 128 or cfg.hidden_size % 8 or cfg.intermediate_size % 8:
        return False
    if getattr(cfg, "sliding_window", None) and getattr(cfg, "use_sliding_window", False):
        return False
    # the rotary tables are precomputed per position: rope types whose
    # frequencies depend on the sequence length are out
    for attr in ("rope_parameters", "rope_scaling"):
        rs = getattr(cfg, attr, None) or {}
        if isinstance(rs, dict) and rs.get("rope_type", rs.get("type")) in ("dynamic", "longrope"):
            return False
    return next(model.parameters()).dtype == torch.bfloat16


def rope_tables(rot, device, max_positions: int) -> tuple[torch.Tensor, torch.Tensor]:
    """bf16 ``cos, sin [max_positions, head_dim]``: a rotary module's outputs for positions ``[0, max_positions)``.

    The HF rotary modules compute each position's angles independently
    (fp32 outer product, then cos/sin cast to the activations' dtype), so the
    table rows equal what a forward at those positions computes.
    """
    cos_parts, sin_parts = [], []
    dummy = torch.empty((1, 1), dtype=torch.bfloat16, device=device)
    step = 8192
    with torch.no_grad():
        for p0 in range(0, max_positions, step):
            pos = torch.arange(p0, min(max_positions, p0 + step), device=device).unsqueeze(0)
            c, s = rot(dummy, pos)
            cos_parts.append(c[0])
            sin_parts.append(s[0])
    return torch.cat(cos_parts).contiguous(), torch.cat(sin_parts).contiguous()


def _pack(linears) -> tuple[torch.Tensor, torch.Tensor | None]:
    """One weight (and bias) for several nn.Linear; the modules keep row-block views of it."""
    w = torch.cat([lin.weight.detach() for lin in linears], dim=0).contiguous()
    has_bias = [lin.bias is not None for lin in linears]
    if any(has_bias) and not all(has_bias):
        raise RuntimeError("packed projections must all have a bias or none")
    b = torch.cat([lin.bias.detach() for lin in linears]).contiguous() if all(has_bias) else None
    r = 0
    for lin in linears:
        rows = lin.weight.shape[0]
        lin.weight = nn.Parameter(w[r: r + rows], requires_grad=False)
        if b is not None:
            lin.bias = nn.Parameter(b[r: r + rows], requires_grad=False)
        r += rows
    return w, b


class _Layer:
    pass


class FusedTarget:
    def __init__(self, model, cache, n_max: int, max_positions: int | None = None, gemm: str = "auto",
                 capture_layers=None, exchange: str = "nccl", argmax: bool = False):
        if not supports(model):
            raise RuntimeError(f"FusedTarget does not support this model ({model.config.model_type})")
        cfg = model.config
        inner = model.model
        dev = next(model.parameters()).device
        kernels.pdl_guard()  # no dependent launch beside NCCL collectives
        self.device = dev
        self.cache = cache
        self.n_max = int(n_max)
        self.head_dim = getattr(cfg, "head_dim", None) or cfg.hidden_size // cfg.num_attention_heads
        self.hidden = cfg.hidden_size
        self.inter = cfg.intermediate_size
        self.vocab = cfg.vocab_size
        self.eps = float(cfg.rms_norm_eps)
        self.embed = inner.embed_tokens.weight
        self.final_norm = inner.norm.weight
        self.lm_head = model.lm_head.weight
        self.layers = []
        with torch.no_grad():
            for i, layer in enumerate(inner.layers):
                a, m = layer.self_attn, layer.mlp
                L = _Layer()
                L.index = i
                L.in_norm = layer.input_layernorm.weight
                L.post_norm = layer.post_attention_layernorm.weight
                L.eps_in = float(getattr(layer.input_layernorm, "variance_epsilon", self.eps))
                L.eps_post = float(getattr(layer.post_attention_layernorm, "variance_epsilon", self.eps))
                L.qkv_w, L.qkv_b = _pack([a.q_proj, a.k_proj, a.v_proj])
                L.gate_up_w, _ = _pack([m.gate_proj, m.up_proj])
                L.o_w, L.o_b = a.o_proj.weight, a.o_proj.bias
                L.down_w = m.down_proj.weight
                L.hq = a.q_proj.weight.shape[0] // self.head_dim
                L.hkv = a.k_proj.weight.shape[0] // self.head_dim
                qn, kn = getattr(a, "q_norm", None), getattr(a, "k_norm", None)
                L.q_norm = None if qn is None else qn.weight
                L.k_norm = None if kn is None else kn.weight
                L.eps_qk = float(getattr(qn, "variance_epsilon", self.eps)) if qn is not None else self.eps
                L.scale = float(getattr(a, "scaling", self.head_dim ** -0.5))
                L.split = getattr(a, "_rt_head_split", None)
                self.layers.append(L)
        hq = self.layers[0].hq
        hkv = self.layers[0].hkv
        if cache.num_kv_heads != hkv:
            raise RuntimeError("cache KV heads do not match the model's (local) KV heads")
        self.hq, self.hkv = hq, hkv
        self.max_positions = int(max_positions or cache.capacity)
        self.cos, self.sin = self._rope_tables(model, self.max_positions)
        n, d = self.n_max, self.head_dim
        e = dict(dtype=torch.bfloat16, device=dev)
        self.residual = torch.empty((n, self.hidden), **e)
        self.xnorm = torch.empty((n, self.hidden), **e)
        self.qkv = torch.empty((n, (hq + 2 * hkv) * d), **e)
        self.q = torch.empty((n, hq, d), **e)
        self.attn = torch.empty((n, hq, d), **e)
        self.o = torch.empty((n, self.hidden), **e)
        self.gate_up = torch.empty((n, 2 * self.inter), **e)
        self.act = torch.empty((n, self.inter), **e)
        self.mlp_out = torch.empty((n, self.hidden), **e)
        self.logits = torch.empty((n, self.vocab), **e)
        # layer outputs the caller wants (HF hidden_states[i + 1] for i in capture_layers),
        # side by side in one [n, len * hidden] buffer (model/utils.py:40-49)
        self.capture_layers = None if capture_layers is None else [int(i) for i in capture_layers]
        self.hidden_out = None
        if self.capture_layers is not None:
            if not self.capture_layers or any(i < 0 or i >= len(self.layers) for i in self.capture_layers):
                raise ValueError(f"capture_layers must name layers in [0, {len(self.layers)})")
            self.hidden_out = torch.empty((n, len(self.capture_layers) * self.hidden), **e)
        # the lm_head projection also returns each node's argmax (rt_linear_argmax):
        # the temperature-0 posterior without a pass over the logits
        self.argmax = bool(argmax)
        self.posterior = torch.empty(self.n_max, dtype=torch.int64, device=dev) if self.argmax else None
        self.last_posterior = None
        # under a KV-head split: the attention outputs' all-gather before o_proj,
        # NCCL ("nccl"), this package's peer-memory exchange ("p2p", retree_b200.peer),
        # or that exchange pulled by the o_proj kernel itself ("p2p_fused")
        if exchange not in ("nccl", "p2p", "p2p_fused"):
            raise ValueError("exchange must be 'nccl', 'p2p' or 'p2p_fused'")
        self.exchange = exchange
        self.peer = None
        split = self.layers[0].split
        if exchange != "nccl" and split is not None and split[1] > 1:
            from .peer import PeerExchange
            if len(self.layers) % 2:
                raise RuntimeError("the peer exchange alternates two slots by layer: it needs an even layer count")
            group, world, rank = split
            self.peer = PeerExchange(group, rank, world, self.n_max, hq * self.head_dim, len(self.layers), dev)
            self.attn_full = torch.empty((self.n_max, world * hq * self.head_dim), dtype=torch.bfloat16, device=dev)
        if gemm not in ("auto", "tcgen05", "cublas"):
            raise ValueError("gemm must be 'auto', 'tcgen05' or 'cublas'")
        self.gemm = gemm
        # projection kind -> use rt_linear (True) or cuBLAS (False)
        kinds = ("qkv", "o", "gate_up", "down", "lm_head")
        self.use_rt = {kd: gemm == "tcgen05" for kd in kinds}
        if gemm == "auto":
            # one decision per process and shape, so every verifier of a model computes alike
            key = (dev.index, self.n_max, self.hidden, self.inter, hq, hkv, self.vocab, len(self.layers))
            if key not in _AUTOTUNE:
                _AUTOTUNE[key] = self._agree(self._autotune(self.n_max))
            self.use_rt = dict(_AUTOTUNE[key])

    @staticmethod
    def _rope_tables(model, max_positions: int):
        return rope_tables(model.model.rotary_emb, next(model.parameters()).device, max_positions)

    def _splits(self, n: int) -> int:
        return kernels.default_splits(n, self.hq, self.hkv, self.cache.capacity - n)

    @torch.inference_mode()
    def _autotune(self, n: int) -> dict:
        """Per projection kind, whether rt_linear beats cuBLAS (+ the stage kernel) at n rows.

        Each candidate runs over every layer's weights back to back (so the
        weights stream from HBM as in a round), K/V going to scratch rows.
        """
        dev = self.device
        widest = max(w.shape[1] for w in (self.layers[0].qkv_w, self.layers[0].o_w, self.layers[0].down_w))
        x = torch.randn((n, max(widest, self.hidden)), device=dev).to(torch.bfloat16)
        pos = torch.zeros(n, dtype=torch.int64, device=dev)
        kv = torch.zeros((2, self.hkv, n, self.head_dim), dtype=torch.bfloat16, device=dev)
        choice = {}

        def timed(fn):
            fn()
            torch.cuda.synchronize(dev)
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            for _ in range(3):
                fn()
            e1.record()
            torch.cuda.synchronize(dev)
            return e0.elapsed_time(e1)

        # (weights, epilogue, bias-free); the input width is the weights' (o_proj
        # stays full width under a KV-head split)
        specs = {
            "qkv": ([L.qkv_w for L in self.layers], 2, all(L.qkv_b is None for L in self.layers)),
            "o": ([L.o_w for L in self.layers], 0, all(L.o_b is None for L in self.layers)),
            "gate_up": ([L.gate_up_w for L in self.layers], 1, True),
            "down": ([L.down_w for L in self.layers], 0, True),
            "lm_head": ([self.lm_head], 0, True),
        }
        for kind, (ws, epi, no_bias) in specs.items():
            k = ws[0].shape[1]
            xk = x[:, :k]
            if not no_bias or not kernels.linear_supported(n, ws[0].shape[0], k, epi):
                choice[kind] = False
                continue
            L0 = self.layers[0]
            qkv = dict(num_q_heads=self.hq, num_kv_heads=self.hkv, q_norm=L0.q_norm, k_norm=L0.k_norm,
                       eps=L0.eps_qk, cos=self.cos, sin=self.sin, positions=pos, q_out=self.q[:n], k_cache=kv[0],
                       v_cache=kv[1])
            width = ws[0].shape[0] // 2 if epi == 1 else ws[0].shape[0]
            out = self.logits[:n] if kind == "lm_head" else torch.empty((n, width), dtype=torch.bfloat16, device=dev)

            def ours():
                for w in ws:
                    kernels.linear(xk, w, out=None if epi == 2 else out, epilogue=epi, qkv=qkv if epi == 2 else None)

            def library():
                for w in ws:
                    if epi == 1:
                        kernels.silu_mul(torch.mm(xk, w.t(), out=self.gate_up[:n]), out)
                    elif epi == 2:
                        y = torch.mm(xk, w.t(), out=self.qkv[:n])
                        kernels.qk_norm_rope_append(y, self.hq, self.hkv, L0.q_norm, L0.k_norm, L0.eps_qk, self.cos,
                                                    self.sin, pos, self.q[:n], kv[0], kv[1])
                    else:
                        torch.mm(xk, w.t(), out=out)

            choice[kind] = timed(ours) < timed(library)
        kernels.check_device_status(dev)
        return choice

    def _agree(self, choice: dict) -> dict:
        """Under a KV-head split the ranks hold replicated activations: take rank 0's choice everywhere."""
        split = self.layers[0].split
        if split is None:
            return choice
        import torch.distributed as dist
        group = split[0]
        kinds = sorted(choice)
        t = torch.tensor([int(choice[kd]) for kd in kinds], dtype=torch.int32, device=self.device)
        src = dist.get_global_rank(group, 0) if group is not None else 0
        dist.broadcast(t, src=src, group=group)
        return {kd: bool(v) for kd, v in zip(kinds, t.tolist())}

    def _linear(self, x, w, b, out, epilogue: int = 0, kind: str = ""):
        """One projection: rt_linear (tcgen05, fused epilogue) when chosen for this kind, else cuBLAS."""
        m, k = x.shape
        if self.use_rt.get(kind, False) and b is None and kernels.linear_supported(m, w.shape[0], k, epilogue):
            return kernels.linear(x, w, out=out, epilogue=epilogue)
        if epilogue == 1:
            y = torch.mm(x, w.t(), out=self.gate_up[:m])
            return kernels.silu_mul(y, out)
        if b is None:
            return torch.mm(x, w.t(), out=out)
        return torch.addmm(b, x, w.t(), out=out)

    def _qkv(self, L, xn, positions, offset, offset_dev):
        """Packed q/k/v projection + head norms + rotary + cache append."""
        n = xn.shape[0]
        kc, vc = self.cache.slab[2 * L.index], self.cache.slab[2 * L.index + 1]
        if self.use_rt["qkv"] and L.qkv_b is None and kernels.linear_supported(n, L.qkv_w.shape[0], xn.shape[1], 2):
            kernels.linear(xn, L.qkv_w, epilogue=2,
                           qkv=dict(num_q_heads=L.hq, num_kv_heads=L.hkv, q_norm=L.q_norm, k_norm=L.k_norm,
                                    eps=L.eps_qk, cos=self.cos, sin=self.sin, positions=positions, q_out=self.q[:n],
                                    k_cache=kc, v_cache=vc, offset=offset, offset_dev=offset_dev))
            return
        self._linear(xn, L.qkv_w, L.qkv_b, self.qkv[:n], kind="qkv")
        kernels.qk_norm_rope_append(self.qkv[:n], L.hq, L.hkv, L.q_norm, L.k_norm, L.eps_qk, self.cos, self.sin,
                                    positions, self.q[:n], kc, vc, offset=offset, offset_dev=offset_dev)

    @torch.inference_mode()
    def forward(self, ids: torch.Tensor, positions: torch.Tensor, bits: torch.Tensor, offset: int = 0,
                offset_dev: torch.Tensor | None = None) -> torch.Tensor:
        """Logits ``[n, vocab]`` (bf16, a view of a reused buffer) of ``n`` tree nodes.

        ``ids``/``positions``: int64 ``[n]``; ``bits``: int32 ``[n, W]`` ancestor
        bits of the tree block; K/V rows are appended at ``offset`` (+
        ``offset_dev[0]``, the device prefix length, when given), and the
        attention sees every cached row before them.
        """
        n = ids.numel()
        if n > self.n_max:
            raise RuntimeError(f"{n} nodes exceed the fused forward's n_max {self.n_max}")
        last = len(self.layers) - 1
        # after the residual add that opens layer i + 1, the residual holds layer i's output
        capture = {} if self.capture_layers is None else {li: j for j, li in enumerate(self.capture_layers)}
        hid = self.hidden
        ids = ids.reshape(n)
        positions = positions.reshape(n)
        slab = self.cache.slab
        cap = self.cache.capacity
        splits = self._splits(n)
        res, xn = self.residual[:n], self.xnorm[:n]
        if self.peer is not None:
            self.peer.step()
        for L in self.layers:
            if L.index == 0:
                kernels.embed_rmsnorm(ids, self.embed, L.in_norm, L.eps_in, res, xn)
            else:
                kernels.add_rmsnorm(self.mlp_out[:n], res, L.in_norm, L.eps_in, xn)
                j = capture.get(L.index - 1)
                if j is not None:
                    self.hidden_out[:n, j * hid: (j + 1) * hid].copy_(res)
            self._qkv(L, xn, positions, offset, offset_dev)
            kc, vc = slab[2 * L.index], slab[2 * L.index + 1]
            # this rank's heads go straight into its exchange slot under the peer exchange
            attn_out = self.attn[:n] if self.peer is None else self.peer.slot(L.index, n).view(n, L.hq, -1)
            if offset_dev is not None:
                kernels.tree_attention(self.q[:n], kc, vc, bits, cap - n, scale=L.scale, out=attn_out,
                                       num_splits=splits, prefix_len_dev=offset_dev, kv_capacity=cap)
            else:
                kernels.tree_attention(self.q[:n], kc[:, : offset + n], vc[:, : offset + n], bits, offset,
                                       scale=L.scale, out=attn_out, num_splits=splits, kv_capacity=cap)
            attn = attn_out
            fused_pull = False
            if self.peer is not None:
                self.peer.signal(L.index)
                fused_pull = (self.exchange == "p2p_fused" and L.o_b is None
                              and kernels.linear_supported(n, L.o_w.shape[0], L.o_w.shape[1], 0))
                if not fused_pull:
                    attn = self.peer.gather(L.index, n, self.attn_full[:n])
            elif L.split is not None:
                group, world, _ = L.split
                attn = gather_heads(attn.unsqueeze(0), group, world)[0]
            if fused_pull:
                self.peer.linear(L.index, n, L.o_w, self.o[:n])
            else:
                self._linear(attn.reshape(n, -1), L.o_w, L.o_b, self.o[:n], kind="o")
            kernels.add_rmsnorm(self.o[:n], res, L.post_norm, L.eps_post, xn)
            self._linear(xn, L.gate_up_w, None, self.act[:n], epilogue=1, kind="gate_up")
            self._linear(self.act[:n], L.down_w, None, self.mlp_out[:n], kind="down")
        kernels.add_rmsnorm(self.mlp_out[:n], res, self.final_norm, self.eps, xn)
        j = capture.get(last)
        if j is not None:
            # HF's last hidden state is the final norm's output (utils/output_capturing.py:253-258)
            self.hidden_out[:n, j * hid: (j + 1) * hid].copy_(xn)
        self.last_posterior = None
        if self.argmax and kernels.linear_supported(n, self.lm_head.shape[0], self.lm_head.shape[1], 0):
            logits = self.logits[:n]
            self.last_posterior = kernels.linear_argmax(xn, self.lm_head, logits, self.posterior[:n])
        else:
            logits = self._linear(xn, self.lm_head, None, self.logits[:n], kind="lm_head")
        return logits
