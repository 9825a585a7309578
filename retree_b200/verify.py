"""Device-resident tree-verify rounds over a transformers causal LM.

``TreeVerifier`` holds what the reference's decode loops keep between rounds
(ddtree.py:765-795, retree.py:228-264): the output-id buffer, the target KV
cache (a ``TreeKVCache`` here), the tree buffers, and the stage timers.  One
``round(draft_logits)`` is the verification hot path:

  1. draft top-k + best-first expansion   (kernels: rt_draft_topk, rt_tree_build)
     -> node tokens / depths / parents, packed ancestor mask, verify ids and
        positions, all on the device (no host copy of the draft logits);
  2. one target forward over the 1+budget nodes (``retree_tree`` attention,
     in-place cache append);
  3. posterior = argmax (temperature 0) or multinomial sample;
  4. exact walk + commit to the output ids (rt_tree_walk), or a host walk
     callback (ReTree's sibling recovery);
  5. compaction of the accepted rows of every layer in one launch
     (rt_kv_compact) and the cache length update.

The host reads back one small vector per round (accepted count, committed
tokens) -- the reference syncs several times per round (ddtree.py:361-367,
:653, :939-942).
"""

from __future__ import annotations

from types import SimpleNamespace

import torch

from . import fused as fused_mod
from . import kernels
from .attention import NAME as ATTN_NAME
from .headsplit import NAME as HEADSPLIT_NAME
from .attention import attach
from .cache import TreeKVCache
from .ddtree import (DDTREE_STAGE_ORDER, DDTREE_TREE_BUILD_STAGE_ORDER, build_tree_device, cuda_time,
                     empty_stage_times, resolve_strategy, sample)


def expected_tree_size(budget: int, rows: int, vocab: int, k: int | None = None) -> int:
    """Nodes the best-first expansion emits: ``budget`` unless the tree runs out of candidates
    (``k`` candidates per draft row; default min(budget, vocab))."""
    k = min(max(budget, 1), vocab) if k is None else min(k, vocab)
    total, level = 0, 1
    for _ in range(rows):
        level *= k
        total += level
        if total >= budget:
            return budget
    return min(budget, total)


def extract_context_feature(hidden_states, layer_ids):
    """Concatenate the selected target hidden states (model/utils.py:40-49)."""
    return torch.cat([hidden_states[i + 1] for i in layer_ids], dim=-1)


class TreeVerifier:
    def __init__(self, target, tree_budget: int, max_length: int, draft_horizon: int = 15,
                 temperature: float = 0.0, target_layer_ids=None, device=None, fused: bool | None = None,
                 gemm: str = "auto", fused_draft: bool = False, exchange: str = "nccl", chain: bool = False,
                 fused_argmax: bool = False):
        cfg = target.config
        if getattr(cfg, "_attn_implementation", None) not in (ATTN_NAME, HEADSPLIT_NAME):
            raise RuntimeError(f"target must use attn_implementation={ATTN_NAME!r} (retree_b200.attention.register())")
        self.target = target
        self.device = torch.device(device) if device is not None else next(target.parameters()).device
        kernels.pdl_guard()  # no dependent launch beside NCCL collectives
        self.budget = max(int(tree_budget), 0)
        self.horizon = int(draft_horizon)
        self.temperature = float(temperature)
        self.n_max = 1 + self.budget
        self.words = (self.n_max + 31) // 32
        self.max_length = int(max_length)
        # a target split by KV head (retree_b200.headsplit) caches only its own heads
        kv_heads = getattr(target, "_rt_local_kv_heads", cfg.num_key_value_heads)
        head_dim = getattr(cfg, "head_dim", None) or cfg.hidden_size // cfg.num_attention_heads
        self.cache = TreeKVCache(cfg.num_hidden_layers, kv_heads, head_dim, self.max_length + self.n_max + 128,
                                 device=self.device)
        self.output_ids = torch.zeros(self.max_length + self.n_max + 1, dtype=torch.long, device=self.device)
        # [start, start before the last commit]; in graph mode the cache appends at start_dev[0]
        self.start_dev = torch.zeros(2, dtype=torch.int64, device=self.device)
        self.graph_mode = False
        self.graph = None
        self.static_logits = None
        self.launches_per_round = None
        self.start = 0
        self.target_layer_ids = target_layer_ids
        self.target_hidden = None
        d = self.device
        b = max(self.budget, 1)
        self.tree = dict(
            tokens=torch.zeros(b, dtype=torch.int64, device=d),
            depths=torch.zeros(b, dtype=torch.int64, device=d),
            parents=torch.zeros(self.n_max, dtype=torch.int32, device=d),
            mask=torch.zeros((self.n_max, self.words), dtype=torch.int32, device=d),
            count=torch.zeros(1, dtype=torch.int32, device=d),
            verify_ids=torch.zeros(self.n_max, dtype=torch.int64, device=d),
            verify_pos=torch.zeros(self.n_max, dtype=torch.int64, device=d),
        )
        self.walk = dict(accepted=torch.zeros(self.n_max, dtype=torch.int64, device=d),
                         accepted_len=torch.zeros(1, dtype=torch.int32, device=d),
                         next_token=torch.zeros(1, dtype=torch.int64, device=d),
                         rescued=torch.zeros(1, dtype=torch.int32, device=d))
        # ReTree's sibling recovery on the device (enable_recovery); None = exact walk
        self.recovery = None
        self.recovery_params: dict = {}
        self.rescued_total = torch.zeros(1, dtype=torch.int64, device=d)
        self.stage_times = empty_stage_times(DDTREE_STAGE_ORDER + DDTREE_TREE_BUILD_STAGE_ORDER)
        self.timed = False
        self.debug = False  # keep the posterior and the pre-compaction cache of the last round
        self.strategy, self.params = resolve_strategy()
        # chain mode (the linear DFlash baseline, dflash.py:73-118): one candidate per
        # draft row, so the best-first expansion is the chain of the rows' argmax tokens
        self.topk = 1 if chain else None
        if chain:
            self.strategy = "heap"
        # verify forward: fused stages (retree_b200.fused) unless the model is not
        # one they cover; with target_layer_ids the fused forward also writes the
        # selected layer outputs (the draft's context features)
        if fused is None:
            # (a target split by KV head keeps the module forward: the fused stages
            # with per-layer all-gathers have not been timed on several GPUs yet)
            fused = (target_layer_ids is None and fused_mod.supports(target)
                     and not hasattr(target, "_rt_local_kv_heads"))
        self.fused = (fused_mod.FusedTarget(target, self.cache, self.n_max, gemm=gemm,
                                            capture_layers=target_layer_ids, exchange=exchange,
                                            argmax=fused_argmax and self.temperature < 1e-5)
                      if fused else None)
        # draft forward: the DFlash module (reference layout) on the fused stages
        # (retree_b200.draft.FusedDraft) when asked for and supported
        self.fused_draft = bool(fused_draft)
        self._draft_runner = None
        self._draft_cache = None

    # ------------------------------------------------------------------ prefill
    @torch.inference_mode()
    def prefill(self, input_ids: torch.Tensor) -> None:
        """Prompt forward (causal, same kernel) and the first target token."""
        ids = input_ids.to(self.device)
        n = ids.shape[1]
        device_mode = self.cache.device_length
        self.cache.use_device_length(False)  # the prompt is causal over an empty cache
        self.cache.set_length(0)
        pos = torch.arange(n, device=self.device).unsqueeze(0)
        out = self.target(ids, position_ids=pos, past_key_values=self.cache, use_cache=True, logits_to_keep=1,
                          output_hidden_states=self.target_layer_ids is not None)
        self.output_ids[:n] = ids[0]
        self.output_ids[n: n + 1] = sample(out.logits, self.temperature)[0]
        if self.target_layer_ids is not None:
            self.target_hidden = extract_context_feature(out.hidden_states, self.target_layer_ids)
        self.start = n
        self.start_dev.fill_(n)
        self.graph = None
        self.cache.use_device_length(device_mode)
        # a new request: the draft's cache starts empty
        self._draft_cache = None
        if self._draft_runner is not None:
            self._draft_runner.reset()

    @torch.inference_mode()
    def prefill_random(self, length: int, seed: int = 0, vocab: int | None = None) -> None:
        """A synthetic committed prefix: N(0,1) K/V rows and uniform ids (no prompt forward).

        For long-context measurements (a 32K-token prompt forward would dominate
        and the round's work does not depend on the cached values).
        """
        vocab = vocab or self.target.config.vocab_size
        g = torch.Generator(device=self.device).manual_seed(seed)
        slab = self.cache.slab
        for i in range(slab.shape[0]):
            slab[i, :, :length].copy_(torch.randn(slab[i, :, :length].shape, device=self.device, generator=g))
        self.output_ids[: length + 1] = torch.randint(0, vocab, (length + 1,), device=self.device, generator=g)
        self.cache.set_length(length)
        self.start = length
        self.start_dev.fill_(length)
        self.graph = None

    # ------------------------------------------------------------------ one round
    def _tick(self, name, t0):
        if self.timed:
            t1 = cuda_time()
            self.stage_times[name] += t1 - t0
            return t1
        return t0

    # ------------------------------------------------------------------ graph mode
    def enable_graph(self, enabled: bool = True) -> None:
        """Run every round as one CUDA-graph replay (after a first eager round that captures it).

        The cache appends at ``start_dev[0]``, the attention reads the prefix
        length from it, the walk advances it, and compaction reads the
        pre-commit start from ``start_dev[1]``: no host value of the round
        changes between rounds, so one capture serves every prefix length.
        """
        if enabled and self.target_layer_ids is not None and self.fused is None:
            raise RuntimeError("graph mode with target_layer_ids needs the fused verify forward")
        self.graph_mode = bool(enabled)
        self.graph = None
        self.cache.use_device_length(self.graph_mode)
        if self.graph_mode:
            self.cache.length_dev = self.start_dev[:1]

    def enable_recovery(self, memory, gate_threshold: float = 0.01, rescue_top_k: int = 8, record_top_k: int = 8,
                        online_update: bool = True) -> None:
        """Walk with ReTree's target-gated sibling recovery on the device (rt_recovery_walk).

        ``memory`` is a ``recovery_device.DeviceRecoveryMemory`` (None: back to
        the exact walk); the knobs are those of follow_verified_tree_with_recovery.
        """
        self.recovery = memory
        self.recovery_params = dict(gate_threshold=gate_threshold, rescue_top_k=rescue_top_k,
                                    record_top_k=record_top_k, online_update=online_update,
                                    freq_threshold=0 if memory is None else memory.freq_threshold)
        self.graph = None

    def _posterior(self, logits: torch.Tensor) -> torch.Tensor:
        """Target token per node, ``[1, n]``: the fused lm_head's argmax when it ran, else sample(logits)."""
        if self.fused is not None and self.fused.last_posterior is not None:
            return self.fused.last_posterior.unsqueeze(0)
        return sample(logits, self.temperature)

    def _walk_and_commit(self, posterior: torch.Tensor, logits: torch.Tensor, count: int) -> None:
        """Exact or recovery walk over the round's tree; commits to the output ids and start_dev."""
        if self.recovery is None:
            kernels.tree_walk(self.tree["parents"], self.tree["tokens"], posterior, count=count, out=self.walk,
                              verify_ids=self.tree["verify_ids"], output_ids=self.output_ids,
                              start_dev=self.start_dev)
            return
        kernels.recovery_walk(self.tree["parents"], self.tree["tokens"], posterior, logits, self.recovery.table,
                              self.recovery_params, count=count, stop_ids=self.recovery.stop_ids,
                              log=self.recovery.log(), out=self.walk, verify_ids=self.tree["verify_ids"],
                              output_ids=self.output_ids, start_dev=self.start_dev)
        self.rescued_total += self.walk["rescued"]

    def _round_body(self, logits: torch.Tensor, count: int) -> None:
        """One round with every varying quantity on the device (capturable)."""
        n = 1 + count
        if self.budget > 0:
            build_tree_device(logits, self.budget, self.output_ids, self.strategy, self.params, out=self.tree, k=self.topk,
                              ctx_len=1, ctx_len_dev=self.start_dev[:1], start_dev=self.start_dev[:1])
        else:
            raise RuntimeError("graph mode needs a tree budget > 0")
        ids = self.tree["verify_ids"][:n].view(1, n)
        pos = self.tree["verify_pos"][:n].view(1, n)
        bits = self.tree["mask"][:n]
        if self.fused is not None:
            logits = self.fused.forward(ids[0], pos[0], bits, offset_dev=self.start_dev[:1]).unsqueeze(0)
        else:
            mask = attach(bits.view(1, 1, n, self.words), bits, prefix_dev=self.start_dev[:1])
            logits = self.target(ids, position_ids=pos, attention_mask=mask, past_key_values=self.cache,
                                 use_cache=True).logits
        posterior = self._posterior(logits)
        self._walk_and_commit(posterior[0], logits[0], count)
        kernels.kv_compact(self.cache.slab, 0, self.walk["accepted"], cur_length=n,
                           n_keep_dev=self.walk["accepted_len"], n_keep=n, past_len_dev=self.start_dev[1:2])

    def _graph_round(self, draft_logits: torch.Tensor) -> int:
        rows, vocab = draft_logits.shape
        count = expected_tree_size(self.budget, rows, vocab, self.topk)
        if self.start + self.n_max + 1 > self.output_ids.numel():
            raise RuntimeError("TreeVerifier max_length exceeded")
        if self.graph is None:
            self.static_logits = torch.empty_like(draft_logits).contiguous()
            self.static_logits.copy_(draft_logits)
            side = torch.cuda.Stream(self.device)
            side.wait_stream(torch.cuda.current_stream(self.device))
            with torch.cuda.stream(side):
                self._round_body(self.static_logits, count)  # real round, and warm-up for the capture
            torch.cuda.current_stream(self.device).wait_stream(side)
            acc = int(self.walk["accepted_len"].item())
            before = kernels.LAUNCHES
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g, stream=side, capture_error_mode="thread_local"):
                self._round_body(self.static_logits, count)
            self.launches_per_round = kernels.LAUNCHES - before
            self.graph = g
        else:
            self.static_logits.copy_(draft_logits, non_blocking=True)
            self.graph.replay()
            kernels._count(self.launches_per_round)
            acc = int(self.walk["accepted_len"].item())
        if self.target_layer_ids is not None:
            self.target_hidden = self.fused.hidden_out.index_select(0, self.walk["accepted"][:acc]).unsqueeze(0)
        self.start += acc
        for layer in self.cache.layers:
            layer.length = self.start
        return acc

    @torch.inference_mode()
    def round(self, draft_logits: torch.Tensor, host_walk=None) -> int:
        """Verify one tree built from ``draft_logits [horizon, vocab]``; returns the accepted length.

        ``host_walk(child_maps, posterior, logits) -> (accepted list, next token)``
        replaces the device exact walk (ReTree's recovery verifier).
        """
        if self.graph_mode and host_walk is None and not self.timed:
            return self._graph_round(draft_logits)
        if self.graph_mode:
            raise RuntimeError("graph mode runs the exact device walk without stage timers")
        start = self.start
        if start + self.n_max + 1 > self.output_ids.numel():
            raise RuntimeError("TreeVerifier max_length exceeded")
        t = cuda_time() if self.timed else 0.0
        rows, vocab = draft_logits.shape
        count = expected_tree_size(self.budget, rows, vocab, self.topk) if self.budget > 0 else 0
        n = 1 + count
        # 1. tree (context = committed ids up to and including the root)
        if self.budget > 0:
            build_tree_device(draft_logits, self.budget, self.output_ids, self.strategy, self.params,
                              out=self.tree, ctx_len=start + 1, start=start, k=self.topk)
        else:
            self.tree["verify_ids"][0] = self.output_ids[start]
            self.tree["verify_pos"][0] = start
            self.tree["mask"][0, 0] = 1
            self.tree["count"].zero_()
        t = self._tick("tree_build", t)
        ids = self.tree["verify_ids"][:n].view(1, n)
        pos = self.tree["verify_pos"][:n].view(1, n)
        bits = self.tree["mask"][:n]
        mask = attach(bits.view(1, 1, n, self.words), bits)
        t = self._tick("tree_compile", t)
        # 2. verify forward
        if self.fused is not None:
            out = SimpleNamespace(logits=self.fused.forward(ids[0], pos[0], bits, offset=start).unsqueeze(0))
        else:
            out = self.target(ids, position_ids=pos, attention_mask=mask, past_key_values=self.cache,
                              use_cache=True, output_hidden_states=self.target_layer_ids is not None)
        t = self._tick("verify", t)
        # 3.-5. posterior, walk, commit, compaction
        posterior = self._posterior(out.logits)
        if self.debug:
            self.last_posterior = posterior
            self.last_slab = self.cache.slab[:, :, : start + n, :].clone()
        if host_walk is None:
            self._walk_and_commit(posterior[0], out.logits[0], count)
            kernels.kv_compact(self.cache.slab[:, :, : start + n, :], start, self.walk["accepted"], cur_length=n,
                               n_keep_dev=self.walk["accepted_len"], n_keep=n)
            acc_len = int(self.walk["accepted_len"].item())
            accepted = None
        else:
            host = torch.cat([self.tree["parents"][:n].to(torch.int64), self.tree["tokens"][:count]]).cpu().tolist()
            parents, tokens = host[:n], host[n:]
            maps = [dict() for _ in range(n)]
            for i in range(1, n):
                maps[parents[i]][int(tokens[i - 1])] = i
            accepted, nxt = host_walk(maps, posterior, out.logits)
            acc_len = len(accepted)
            keep = torch.tensor(accepted, dtype=torch.long, device=self.device)
            self.output_ids[start: start + acc_len] = self.tree["verify_ids"].index_select(0, keep)
            self.output_ids[start + acc_len] = int(nxt)
            kernels.kv_compact(self.cache.slab[:, :, : start + n, :], start, keep, cur_length=n)
            self.start_dev.fill_(start + acc_len)
        self.cache.crop(start)
        for layer in self.cache.layers:
            layer.length = start + acc_len
        if self.target_layer_ids is not None:
            keep_idx = self.walk["accepted"][:acc_len] if accepted is None else keep
            if self.fused is not None:
                self.target_hidden = self.fused.hidden_out[:n].index_select(0, keep_idx).unsqueeze(0)
            else:
                self.target_hidden = extract_context_feature(out.hidden_states, self.target_layer_ids).index_select(
                    1, keep_idx)
        self.start = start + acc_len
        self._tick("commit", t)
        return acc_len

    # ------------------------------------------------------------------ decode loop
    def _draft(self, draft_model, draft_fn, round_idx, block_size):
        start = self.start
        if draft_fn is not None:
            return draft_fn(self.output_ids, start, round_idx)
        if self.target_hidden is None:
            raise RuntimeError("the draft model needs the target's hidden states: pass target_layer_ids")
        if self.fused_draft:
            if self._draft_runner is None:
                from .draft import FusedDraft
                self._draft_runner = FusedDraft(draft_model, self.target, capacity=self.max_length + block_size + 8,
                                                block_size=block_size)
            return self._draft_runner.forward(self.output_ids[start: start + block_size], self.target_hidden, start,
                                              horizon=block_size - 1)
        # the reference's draft call (ddtree.py:828-845)
        block = self.output_ids[start: start + block_size].clone().unsqueeze(0)
        noise = self.target.model.embed_tokens(block)
        if self._draft_cache is None:
            from transformers import DynamicCache
            self._draft_cache = DynamicCache()
            self._positions = torch.arange(self.output_ids.numel(), device=self.device).unsqueeze(0)
        dc = self._draft_cache
        hidden = draft_model(target_hidden=self.target_hidden, noise_embedding=noise,
                             position_ids=self._positions[:, dc.get_seq_length(): start + block_size],
                             past_key_values=dc, use_cache=True, is_causal=False)[:, -(block_size - 1):, :]
        logits = self.target.lm_head(hidden)
        dc.crop(start)
        return logits[0]

    @torch.inference_mode()
    def generate(self, input_ids, mask_token_id, max_new_tokens, block_size, stop_token_ids, draft_model=None,
                 draft_fn=None, save_tree_traces=False, host_walk=None) -> SimpleNamespace:
        """The decode loop of ddtree.py:827-968 / retree.py:296-444 on this verifier."""
        self.timed = True
        num_input = input_ids.shape[1]
        max_length = num_input + max_new_tokens
        self.output_ids.fill_(mask_token_id)
        stop = None if stop_token_ids is None else torch.tensor(stop_token_ids, device=self.device)
        t0 = cuda_time()
        self.prefill(input_ids)
        ttft = cuda_time() - t0
        decode_start = cuda_time()
        acceptance, stamps, traces = [], [], ([] if save_tree_traces else None)
        r = 0
        while self.start < max_length:
            ts = cuda_time()
            if self.budget == 0:  # no draft: one target token per round (dflash.py with block_size <= 1)
                logits = torch.empty((0, self.target.config.vocab_size), dtype=torch.bfloat16, device=self.device)
            else:
                logits = self._draft(draft_model, draft_fn, r, block_size)
            if r > 0:
                self.stage_times["draft"] += cuda_time() - ts
            else:
                decode_start = cuda_time()
            acc = self.round(logits, host_walk=host_walk)
            acceptance.append(acc)
            stamps.append(cuda_time() - decode_start)
            if save_tree_traces:
                cnt = int(self.tree["count"].item())
                traces.append(dict(
                    accepted_indices=[] if self.walk is None else self.walk["accepted"][:acc].tolist(),
                    tree=dict(node_token_ids=self.tree["tokens"][:cnt].tolist(),
                              node_depths=self.tree["depths"][:cnt].tolist(),
                              parents=self.tree["parents"][: cnt + 1].tolist())))
            r += 1
            if stop is not None:
                new = self.output_ids[self.start - acc: self.start + 1]
                if torch.isin(new, stop).any():
                    break
        out = self.output_ids[:max_length]
        out = out[out != mask_token_id].unsqueeze(0)
        if stop is not None:
            hits = torch.isin(out[0][num_input:], stop).nonzero(as_tuple=True)[0]
            if hits.numel() > 0:
                out = out[:, : num_input + int(hits[0]) + 1]
        n_out = out.shape[1] - num_input
        total = cuda_time() - decode_start
        self.timed = False
        return SimpleNamespace(output_ids=out.cpu(), num_input_tokens=num_input, num_output_tokens=n_out,
                               time_to_first_token=ttft, time_per_output_token=total / max(n_out, 1),
                               acceptance_lengths=acceptance, decode_rounds=len(acceptance),
                               stage_times=self.stage_times, round_timestamps=stamps, round_trees=traces)
