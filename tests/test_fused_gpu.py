"""Fused verify-forward stages against the transformers ops they replace.

Each layer-stage kernel is compared with the HF Qwen3 modules on the same
bf16 inputs (modeling_qwen3.py: Qwen3RMSNorm, apply_rotary_pos_emb, Qwen3MLP's
silu * up): bit-exact where the computation order is the same, and at most one
bf16 unit apart in a small fraction of elements where only the order of the
fp32 sum of squares differs.  The whole fused forward is compared with the HF
forward on the same cache, and decoding through it with greedy decoding.
"""

import numpy as np
import pytest
import torch
import torch.nn.functional as F
from transformers.models.qwen3.modeling_qwen3 import Qwen3RMSNorm, apply_rotary_pos_emb

from oracle import tree as ot
from retree_b200 import attention, fused, kernels, synthetic
from retree_b200.cache import TreeKVCache
from retree_b200.target import build_target, qwen3_config
from retree_b200.verify import TreeVerifier
from tests.gpu_util import cuda

pytestmark = pytest.mark.gpu

VOCAB = 2000


def _cfg(layers=3, **kw):
    base = dict(hidden_size=512, intermediate_size=1024, num_hidden_layers=layers, num_attention_heads=8,
                num_key_value_heads=2, vocab_size=VOCAB, tie_word_embeddings=False)
    base.update(kw)
    return qwen3_config("small", **base)


def _ulps_apart(a, b):
    """Per-element distance in bf16 units of the larger magnitude (0 where equal)."""
    a, b = a.float(), b.float()
    scale = torch.maximum(a.abs(), b.abs()).clamp_min(1e-30)
    ulp = torch.exp2(torch.floor(torch.log2(scale)) - 7)
    return ((a - b).abs() / ulp).round()


def _near_equal(got, want, max_frac=2e-3):
    d = _ulps_apart(got, want)
    assert float(d.max()) <= 1.0, f"max {float(d.max())} bf16 units apart"
    assert float((d > 0).float().mean()) <= max_frac


@torch.inference_mode()
def test_embed_and_add_rmsnorm_match_hf():
    dev = cuda()
    g = torch.Generator(device=dev).manual_seed(0)
    hidden, vocab, rows = 2560, 5000, 37
    table = (torch.randn((vocab, hidden), device=dev, generator=g) * 0.05).to(torch.bfloat16)
    norm = Qwen3RMSNorm(hidden, eps=1e-6).to(dev).to(torch.bfloat16)
    norm.weight.copy_((1 + 0.1 * torch.randn(hidden, device=dev, generator=g)).to(torch.bfloat16))
    ids = torch.randint(0, vocab, (rows,), device=dev, generator=g)
    res = torch.empty((rows, hidden), dtype=torch.bfloat16, device=dev)
    out = torch.empty_like(res)
    kernels.embed_rmsnorm(ids, table, norm.weight, 1e-6, res, out)
    emb = F.embedding(ids, table)
    assert torch.equal(res, emb)
    _near_equal(out, norm(emb))
    delta = (torch.randn((rows, hidden), device=dev, generator=g) * 3).to(torch.bfloat16)
    want_res = emb + delta
    kernels.add_rmsnorm(delta, res, norm.weight, 1e-6, out)
    assert torch.equal(res, want_res)
    _near_equal(out, norm(want_res))
    kernels.add_rmsnorm(None, res, norm.weight, 1e-6, out)   # norm only
    assert torch.equal(res, want_res)
    _near_equal(out, norm(want_res))
    # an out-of-range id: zero row and a device status
    bad = ids.clone()
    bad[3] = vocab + 7
    kernels.embed_rmsnorm(bad, table, norm.weight, 1e-6, res, out)
    assert not res[3].any()
    with pytest.raises(RuntimeError):
        kernels.check_device_status(dev)


@torch.inference_mode()
def test_qk_norm_rope_append_matches_hf():
    dev = cuda()
    model = build_target(_cfg(1), device=dev, seed=1)
    attn = model.model.layers[0].self_attn
    with torch.no_grad():
        attn.q_norm.weight.copy_((1 + 0.2 * torch.randn(128, device=dev)).to(torch.bfloat16))
        attn.k_norm.weight.copy_((1 + 0.2 * torch.randn(128, device=dev)).to(torch.bfloat16))
    hq, hkv, n, cap, off = 8, 2, 45, 300, 211
    g = torch.Generator(device=dev).manual_seed(2)
    qkv = torch.randn((n, (hq + 2 * hkv) * 128), device=dev, generator=g).to(torch.bfloat16)
    pos = torch.randint(0, 4000, (n,), device=dev, generator=g)
    cos_t, sin_t = fused.FusedTarget._rope_tables(model, 4096)
    q_out = torch.empty((n, hq, 128), dtype=torch.bfloat16, device=dev)
    kc = torch.zeros((hkv, cap, 128), dtype=torch.bfloat16, device=dev)
    vc = torch.zeros_like(kc)
    off_dev = torch.tensor([off - 11], dtype=torch.int64, device=dev)
    kernels.qk_norm_rope_append(qkv, hq, hkv, attn.q_norm.weight, attn.k_norm.weight, 1e-6, cos_t, sin_t, pos,
                                q_out, kc, vc, offset=11, offset_dev=off_dev)
    kernels.check_device_status(dev)
    # HF: q_norm / k_norm on [1, n, H, D], transpose, rotary with the model's cos/sin for these positions
    q = attn.q_norm(qkv[:, : hq * 128].view(1, n, hq, 128)).transpose(1, 2)
    k = attn.k_norm(qkv[:, hq * 128: (hq + hkv) * 128].view(1, n, hkv, 128)).transpose(1, 2)
    v = qkv[:, (hq + hkv) * 128:].view(1, n, hkv, 128).transpose(1, 2)
    cos, sin = model.model.rotary_emb(qkv[None], pos[None])
    qe, ke = apply_rotary_pos_emb(q, k, cos, sin)
    _near_equal(q_out, qe[0].transpose(0, 1))
    _near_equal(kc[:, off: off + n], ke[0])
    assert torch.equal(vc[:, off: off + n], v[0])
    assert not kc[:, :off].any() and not kc[:, off + n:].any()
    # rows past the capacity are refused, not written
    kernels.qk_norm_rope_append(qkv, hq, hkv, attn.q_norm.weight, attn.k_norm.weight, 1e-6, cos_t, sin_t, pos,
                                q_out, kc, vc, offset=cap - 5)
    with pytest.raises(RuntimeError):
        kernels.check_device_status(dev)


@torch.inference_mode()
def test_silu_mul_matches_torch_bit_exact():
    dev = cuda()
    g = torch.Generator(device=dev).manual_seed(4)
    rows, inter = 33, 9728
    gu = (torch.randn((rows, 2 * inter), device=dev, generator=g) * 4).to(torch.bfloat16)
    out = torch.empty((rows, inter), dtype=torch.bfloat16, device=dev)
    kernels.silu_mul(gu, out)
    assert torch.equal(out, F.silu(gu[:, :inter]) * gu[:, inter:])


def _tree(seed, n, L, dev):
    parents = synthetic.random_tree_parents(seed, n - 1).tolist()
    n = len(parents)
    depths = synthetic.depths_from_parents(parents)
    bits = torch.from_numpy(ot.pack_bits(ot.visibility(parents)).view(np.int32)).to(dev)
    pos = torch.from_numpy(L + depths).to(dev)
    return n, bits, pos


@torch.inference_mode()
@pytest.mark.parametrize("device_offset,gemm", [(False, "auto"), (True, "auto"), (False, "tcgen05"),
                                                (True, "cublas")])
def test_fused_forward_matches_hf_forward(device_offset, gemm):
    dev = cuda()
    model = build_target(_cfg(3), device=dev, seed=5)
    L = 260
    prompt = torch.randint(0, VOCAB, (1, L), device=dev, generator=torch.Generator(device=dev).manual_seed(6))
    c_hf = TreeKVCache.for_model(model.config, capacity=512, device=dev)
    model(prompt, position_ids=torch.arange(L, device=dev)[None], past_key_values=c_hf, use_cache=True)
    c_fu = TreeKVCache.for_model(model.config, capacity=512, device=dev)
    c_fu.slab.copy_(c_hf.slab)
    c_fu.set_length(L)
    n, bits, pos = _tree(8, 40, L, dev)
    tok = torch.randint(0, VOCAB, (n,), device=dev, generator=torch.Generator(device=dev).manual_seed(9))
    want = model(tok[None], position_ids=pos[None], attention_mask=attention.attach(bits.view(1, 1, n, -1), bits),
                 past_key_values=c_hf, use_cache=True).logits[0]
    ft = fused.FusedTarget(model, c_fu, n_max=64, gemm=gemm)
    if device_offset:
        got = ft.forward(tok, pos, bits, offset_dev=torch.tensor([L], dtype=torch.int64, device=dev)).clone()
    else:
        got = ft.forward(tok, pos, bits, offset=L).clone()
    kernels.check_device_status(dev)
    rel = float((got.float() - want.float()).norm() / want.float().norm())
    assert rel < 1e-2, rel
    # the K/V rows the fused forward appended
    for li in range(3):
        for kv in range(2):
            a = c_fu.slab[2 * li + kv, :, L: L + n].float()
            b = c_hf.slab[2 * li + kv, :, L: L + n].float()
            assert float((a - b).norm() / b.norm()) < 1e-2
    assert torch.equal(c_fu.slab[:, :, :L], c_hf.slab[:, :, :L])
    # argmax agrees wherever HF's top-2 margin is not a near tie
    top2 = want.float().topk(2, dim=-1).values
    clear = (top2[:, 0] - top2[:, 1]) > 0.05 * top2[:, 0].abs().clamp_min(1.0)
    assert torch.equal(got.argmax(-1)[clear], want.argmax(-1)[clear])
    # the HF modules still run on the packed weights (views)
    assert model.model.layers[0].self_attn.q_proj.weight.data_ptr() == ft.layers[0].qkv_w.data_ptr()


@torch.inference_mode()
@pytest.mark.parametrize("use_fused", [True, False])
def test_fused_and_hf_verifier_graph_rounds(monkeypatch, use_fused):
    """Graph replays equal eager rounds on both verify-forward paths."""
    monkeypatch.setenv("DDTREE_TREE_STRATEGY", "rank_gated_ngram")
    dev = cuda()
    model = build_target(_cfg(2), device=dev, seed=11)
    prompt = torch.from_numpy(synthetic.context_ids(8, 150, VOCAB, alphabet=40))[None].to(dev)
    drafts = [torch.from_numpy(synthetic.draft_logits(400 + r, 15, VOCAB, amp=6.0)).to(dev).to(torch.bfloat16)
              for r in range(5)]
    eager = TreeVerifier(model, tree_budget=40, max_length=500, fused=use_fused)
    graph = TreeVerifier(model, tree_budget=40, max_length=500, fused=use_fused)
    assert (eager.fused is not None) == use_fused
    eager.prefill(prompt)
    graph.prefill(prompt)
    graph.enable_graph(True)
    for d in drafts:
        assert eager.round(d) == graph.round(d)
    s = eager.start
    assert torch.equal(eager.output_ids[: s + 1], graph.output_ids[: s + 1])
    assert torch.equal(eager.cache.slab[:, :, :s], graph.cache.slab[:, :, :s])


@torch.inference_mode()
def test_fused_tree_decoding_equals_greedy_decoding(monkeypatch):
    """Speculative invariant on the fused forward: tree rounds commit the greedy tokens.

    The greedy reference runs the same fused stages one token per forward
    (n = 1, the warp-level attention path and M = 1 GEMMs), so two runs can
    only part at a near tie of the reference's top-2 logits; the test requires
    identity up to such a tie and a long common run before it.
    """
    monkeypatch.setenv("DDTREE_TREE_STRATEGY", "rank_gated_ngram")
    dev = cuda()
    model = build_target(_cfg(2), device=dev, seed=12)
    prompt = torch.from_numpy(synthetic.context_ids(5, 64, VOCAB, alphabet=30))[None].to(dev)
    new = 40
    cache = TreeKVCache.for_model(model.config, capacity=256, device=dev)
    out = model(prompt, position_ids=torch.arange(64, device=dev)[None], past_key_values=cache, use_cache=True)
    ft = fused.FusedTarget(model, cache, n_max=1)
    one = attention.causal_bits(1, dev)
    greedy, margins = [int(out.logits[0, -1].argmax())], []
    for i in range(new - 1):
        logits = ft.forward(torch.tensor([greedy[-1]], device=dev), torch.tensor([64 + i], device=dev), one,
                            offset=64 + i)[0].float()
        top2 = logits.topk(2).values
        margins.append(float(top2[0] - top2[1]) / max(float(top2[0].abs()), 1.0))
        greedy.append(int(logits.argmax()))
    v = TreeVerifier(model, tree_budget=24, max_length=200, fused=True)
    assert v.fused is not None
    v.prefill(prompt)
    r = 0
    while v.start < 64 + new:
        d = torch.randn((15, VOCAB), device=dev, generator=torch.Generator(device=dev).manual_seed(r))
        v.round(d)
        r += 1
    got = v.output_ids[64: 64 + new].tolist()
    if got != greedy:
        first = next(i for i, (a, b) in enumerate(zip(got, greedy)) if a != b)
        assert first >= 16 and margins[first - 1] < 1e-2, (first, margins[first - 1])
