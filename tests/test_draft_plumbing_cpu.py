"""Host-side plumbing of the fused draft and of the fused verify forward's layer capture, on the CPU.

The stage kernels are replaced, inside these tests only, by torch stand-ins
that compute the same math in fp32 and round like the kernels (bf16 outputs).
What is checked is the orchestration around them: context chunks, cache
offsets and positions, the residual stream, the crop after each call, the
layer-output capture -- against the restated draft forward (``oracle.dflash``,
pinned to the reference's module) and the HF forward's hidden states.  The
kernels themselves are compared with the same references on the GPU.
"""

import numpy as np
import pytest
import torch
import torch.nn.functional as F

from oracle import dflash as od
from retree_b200 import draft as draft_mod
from retree_b200 import fused as fused_mod
from retree_b200 import kernels

BF = torch.bfloat16


def _norm(x, w, eps):
    x = x.float()
    y = (x * torch.rsqrt(x.pow(2).mean(-1, keepdim=True) + eps)).to(BF)
    return (w.to(BF) * y).to(BF)


def _rope(x, cos, sin):
    half = x.shape[-1] // 2
    rot = torch.cat([-x[..., half:], x[..., :half]], dim=-1)
    return (x * cos + rot * sin).to(BF)


class FakeCache:
    def __init__(self, layers, hkv, d, cap):
        self.slab = torch.zeros((2 * layers, hkv, cap, d), dtype=BF)
        self.capacity = cap
        self.num_kv_heads = hkv


@pytest.fixture
def fake_kernels(monkeypatch):
    def add_rmsnorm(delta, residual, weight, eps, out):
        if delta is not None:
            residual.copy_((residual.float() + delta.float()).to(BF))
        out.copy_(_norm(residual, weight, eps))
        return out

    def embed_rmsnorm(ids, table, weight, eps, residual, out):
        residual.copy_(table[ids])
        out.copy_(_norm(residual, weight, eps))
        return out

    def qk_norm_rope_append(qkv, hq, hkv, qn, kn, eps, cos, sin, positions, q_out, k_cache, v_cache, offset=0,
                            offset_dev=None):
        n = positions.numel()
        off = offset + (0 if offset_dev is None else int(offset_dev[0]))
        x = qkv.view(n, hq + 2 * hkv, 128)
        c, s = cos[positions][:, None, :], sin[positions][:, None, :]
        q = _rope(_norm(x[:, :hq], qn, eps), c, s)
        k = _rope(_norm(x[:, hq: hq + hkv], kn, eps), c, s)
        q_out.copy_(q)
        k_cache[:, off: off + n] = k.transpose(0, 1)
        v_cache[:, off: off + n] = x[:, hq + hkv:].transpose(0, 1)
        return q_out

    def tree_attention(q, k, v, bits, prefix_len, scale=None, out=None, num_splits=0, path=0, prefix_len_dev=None,
                       kv_capacity=None):
        if q.dim() == 4:  # HF's [1, Hq, n, D] / [1, Hkv, S, D], as the real wrapper takes them
            q, k, v = q[0].transpose(0, 1), k[0], v[0]
        n, hq, d = q.shape
        if out is None:
            out = torch.empty((n, hq, d), dtype=BF)
        L = int(prefix_len) + (0 if prefix_len_dev is None else int(prefix_len_dev[0]))
        hkv = k.shape[0]
        words = bits.numpy().view(np.uint32)
        vis = np.unpackbits(words.view(np.uint8), axis=1, bitorder="little")[:, :n].astype(bool)
        mask = torch.zeros((n, L + n))
        mask[:, L:] = torch.where(torch.from_numpy(vis), 0.0, float("-inf"))
        kk = k[:, : L + n].float().repeat_interleave(hq // hkv, 0)
        vv = v[:, : L + n].float().repeat_interleave(hq // hkv, 0)
        o = F.scaled_dot_product_attention(q.float().transpose(0, 1), kk, vv, attn_mask=mask, scale=scale)
        out.copy_(o.transpose(0, 1).to(BF))
        return out

    def silu_mul(gate_up, out):
        inter = out.shape[-1]
        g, u = gate_up.view(-1, 2 * inter).float().split(inter, dim=-1)
        out.copy_((F.silu(g).to(BF).float() * u).to(BF).view_as(out))
        return out

    monkeypatch.setattr(kernels, "add_rmsnorm", add_rmsnorm)
    monkeypatch.setattr(kernels, "embed_rmsnorm", embed_rmsnorm)
    monkeypatch.setattr(kernels, "qk_norm_rope_append", qk_norm_rope_append)
    monkeypatch.setattr(kernels, "tree_attention", tree_attention)
    monkeypatch.setattr(kernels, "silu_mul", silu_mul)
    monkeypatch.setattr(kernels, "default_splits", lambda *a: 1)
    monkeypatch.setattr(kernels, "linear_supported", lambda *a: False)
    monkeypatch.setattr(draft_mod, "TreeKVCache",
                        lambda layers, hkv, d, cap, device=None: FakeCache(layers, hkv, d, cap))


class _Target(torch.nn.Module):
    """Embedding table and lm_head of a target (what the draft call uses of it)."""

    def __init__(self, hidden, vocab, seed):
        super().__init__()
        g = torch.Generator().manual_seed(seed)
        self.config = type("C", (), {"hidden_size": hidden})()
        self.model = torch.nn.Module()
        self.model.embed_tokens = torch.nn.Embedding(vocab, hidden)
        self.lm_head = torch.nn.Linear(hidden, vocab, bias=False)
        with torch.no_grad():
            self.model.embed_tokens.weight.copy_(torch.randn((vocab, hidden), generator=g))
            self.lm_head.weight.copy_(torch.randn((vocab, hidden), generator=g) * hidden ** -0.5)
        self.to(BF)


@torch.inference_mode()
@pytest.mark.parametrize("ctx_chunk", [1024, 16])
def test_fused_draft_plumbing_matches_restated_forward(fake_kernels, ctx_chunk):
    cfg = od.small_config()
    w = {k: v.to(BF) for k, v in od.seeded_weights(cfg, 0).items()}
    d16 = od.build_module(cfg, w, dtype=BF)
    ref = od.build_module(cfg, {k: v.float() for k, v in w.items()})
    target = _Target(cfg.hidden_size, 500, seed=1)
    fd = draft_mod.FusedDraft(d16, target, capacity=256, ctx_chunk=ctx_chunk)
    assert fd.layers[0].qkv_w.shape[0] == (cfg.num_attention_heads + 2 * cfg.num_key_value_heads) * 128
    calls, got, start = [], [], 0
    for j, c in enumerate((40, 5, 9)):
        th, _ = od.seeded_inputs(cfg, 20 + j, c)
        ids = torch.full((cfg.block_size,), 3, dtype=torch.int64)
        ids[0] = 10 + j
        calls.append((th.to(BF), ids))
        start += c
        got.append(fd.forward(ids, th.to(BF), start, return_hidden=True).clone())
        assert fd.length == start
    embed = target.model.embed_tokens.weight
    want = od.run_calls(ref, [(th.float(), embed[ids].float()) for th, ids in calls])
    for j in range(3):
        rel = float((got[j].float() - want[j]).norm() / want[j].norm())
        assert rel < 2e-2, (j, rel)
    # the cache holds exactly the context rows: rows past start were never kept
    assert fd.cache.slab[:, :, start + cfg.block_size:].abs().sum() == 0
    logits = fd.forward(calls[-1][1], calls[-1][0][:0], start, horizon=4)
    assert logits.shape == (4, 500)
    ref_logits = want[-1][-4:] @ target.lm_head.weight.float().t()
    assert float((logits.float() - ref_logits).norm() / ref_logits.norm()) < 2e-2
    with pytest.raises(RuntimeError):
        fd.forward(calls[-1][1][:5], calls[-1][0][:0], start)  # not a whole block
    with pytest.raises(RuntimeError):
        fd.forward(calls[-1][1], calls[-1][0][:0], start + 1)  # context does not end at start


@torch.inference_mode()
def test_fused_target_layer_capture_plumbing(fake_kernels):
    """The layer outputs FusedTarget writes are HF's ``hidden_states[i + 1]`` (last: the final norm's output)."""
    from transformers import DynamicCache, Qwen3Config, Qwen3ForCausalLM

    cfg = Qwen3Config(vocab_size=300, hidden_size=256, intermediate_size=512, num_hidden_layers=3,
                      num_attention_heads=4, num_key_value_heads=2, head_dim=128, tie_word_embeddings=False)
    cfg._attn_implementation = "sdpa"
    torch.manual_seed(0)
    model = Qwen3ForCausalLM(cfg).to(BF).eval()
    L, n = 20, 6
    ids = torch.randint(0, 300, (1, L + n), generator=torch.Generator().manual_seed(1))
    dc = DynamicCache()
    model(ids[:, :L], past_key_values=dc, use_cache=True)
    out = model(ids[:, L:], position_ids=torch.arange(L, L + n)[None], past_key_values=dc, use_cache=True,
                output_hidden_states=True)
    cache = FakeCache(3, 2, 128, 64)
    for i in range(3):
        cache.slab[2 * i, :, :L] = dc.layers[i].keys[0, :, :L]
        cache.slab[2 * i + 1, :, :L] = dc.layers[i].values[0, :, :L]
    ft = fused_mod.FusedTarget(model, cache, n_max=8, gemm="cublas", capture_layers=[2, 0])
    bits = torch.from_numpy(np.packbits(np.tril(np.ones((n, 32), dtype=bool)), axis=1, bitorder="little")
                            .view("<u4").view(np.int32).copy())
    logits = ft.forward(ids[0, L:], torch.arange(L, L + n), bits, offset=L)
    h = cfg.hidden_size
    for j, li in enumerate([2, 0]):
        want = out.hidden_states[li + 1][0].float()
        got = ft.hidden_out[:n, j * h: (j + 1) * h].float()
        assert float((got - want).norm() / want.norm()) < 2e-2, li
    assert float((logits.float() - out.logits[0].float()).norm() / out.logits[0].float().norm()) < 2e-2


@torch.inference_mode()
def test_synthetic_draft_layout_runs_through_the_fused_draft(fake_kernels):
    """``draft.random_draft`` (the benchmark's synthetic draft) has the layout ``FusedDraft`` reads."""
    d = draft_mod.random_draft(256, 2, 4, 2, 512, 8, [1, 3], "cpu")
    assert draft_mod.supports(d)
    fd = draft_mod.FusedDraft(d, _Target(256, 300, seed=2), capacity=128)
    th = torch.randn((12, 512)).to(BF)
    logits = fd.forward(torch.full((8,), 5, dtype=torch.int64), th, 12)
    assert logits.shape == (7, 300) and bool(torch.isfinite(logits.float()).all())


@torch.inference_mode()
@pytest.mark.parametrize("module_causal,call_causal,want_causal", [
    (True, None, True), (False, None, False), (True, False, False), (False, True, True)])
def test_attention_backend_honours_is_causal_without_a_mask(fake_kernels, module_causal, call_causal, want_causal):
    """No mask: causal unless the call (else the module) says is_causal=False, as HF's SDPA backend decides
    (the DFlash draft attends to every key, model/dflash.py:47)."""
    from retree_b200 import attention

    g = torch.Generator().manual_seed(0)
    n, S = 6, 20
    q = torch.randn((1, 4, n, 128), generator=g).to(BF)
    k = torch.randn((1, 2, S, 128), generator=g).to(BF)
    v = torch.randn((1, 2, S, 128), generator=g).to(BF)
    mod = torch.nn.Module()
    mod.is_causal = module_causal
    kw = {} if call_causal is None else {"is_causal": call_causal}
    out, _ = attention.tree_attention_forward(mod, q, k, v, None, scaling=128 ** -0.5, **kw)
    mask = torch.zeros((n, S))
    if want_causal:
        mask[:, S - n:] = torch.triu(torch.full((n, n), float("-inf")), diagonal=1)
    ref = F.scaled_dot_product_attention(q.float(), k.float().repeat_interleave(2, 1),
                                         v.float().repeat_interleave(2, 1), attn_mask=mask, scale=128 ** -0.5)
    assert float((out[0].float() - ref[0].transpose(0, 1)).abs().max()) < 2e-2


def test_chain_tree_size_is_one_node_per_draft_row():
    """The linear baseline's tree (one candidate per row) has min(budget, rows) nodes."""
    from retree_b200.verify import expected_tree_size

    assert expected_tree_size(15, 15, 151936, k=1) == 15
    assert expected_tree_size(15, 7, 151936, k=1) == 7
    assert expected_tree_size(0, 7, 151936, k=1) == 0
    assert expected_tree_size(16, 15, 151936) == 16  # the reference's top-k: budget candidates per row
