"""The drop-in API on a real (small, random) Qwen3 target: backend vs SDPA, cache compaction,
verifier rounds stage by stage against the oracle, and tree decoding == greedy decoding."""


import numpy as np
import pytest
import torch
from transformers import DynamicCache

from oracle import tree as ot
from retree_b200 import attention, kernels, synthetic
from retree_b200.cache import TreeKVCache
from retree_b200.ddtree import build_ddtree_tree, compact_dynamic_cache, ddtree_generate
from retree_b200.target import build_target, qwen3_config
from retree_b200.verify import TreeVerifier
from tests.gpu_util import cuda

pytestmark = pytest.mark.gpu

VOCAB = 2000


def _small_cfg(layers=3):
    return qwen3_config("small", hidden_size=512, intermediate_size=1024, num_hidden_layers=layers,
                        num_attention_heads=8, num_key_value_heads=2, vocab_size=VOCAB, tie_word_embeddings=False)


@pytest.fixture(scope="module")
def models():
    dev = cuda()
    ours = build_target(_small_cfg(), device=dev, seed=3)
    ref = build_target(_small_cfg(), device=dev, seed=3, attn_implementation="sdpa")
    with torch.no_grad():
        for a, b in zip(ours.parameters(), ref.parameters()):
            assert torch.equal(a, b)
    return ours, ref


def _rel(a, b):
    return float((a.float() - b.float()).norm() / b.float().norm())


@torch.inference_mode()
def test_backend_matches_sdpa_prefill_and_tree(models):
    ours, ref = models
    dev = cuda()
    L = 300
    ids = torch.randint(0, VOCAB, (1, L), device=dev, generator=torch.Generator(device=dev).manual_seed(0))
    pos = torch.arange(L, device=dev)[None]
    c1 = TreeKVCache.for_model(ours.config, capacity=1024, device=dev)
    c2 = DynamicCache()
    o1 = ours(ids, position_ids=pos, past_key_values=c1, use_cache=True)
    o2 = ref(ids, position_ids=pos, past_key_values=c2, use_cache=True)
    assert _rel(o1.logits, o2.logits) < 2e-2
    assert torch.equal(c1.layers[0].keys, c2.layers[0].keys)   # same projections + RoPE, in place
    # tree verify forward: packed bits (ours) vs the reference's dense additive mask (sdpa)
    parents = synthetic.random_tree_parents(7, 40).tolist()
    n = len(parents)
    depths = synthetic.depths_from_parents(parents)
    tok = torch.randint(0, VOCAB, (1, n), device=dev, generator=torch.Generator(device=dev).manual_seed(1))
    tpos = torch.from_numpy(L + depths).to(dev)[None]
    _, _, dense = ot.compile_tree(0, L, tok[0, 1:].tolist(), depths[1:], parents, L,
                                  float(torch.finfo(torch.bfloat16).min))
    dense_t = torch.from_numpy(dense).to(dev).to(torch.bfloat16)[None, None]
    bits = torch.from_numpy(ot.pack_bits(ot.visibility(parents)).view(np.int32)).to(dev)
    o1 = ours(tok, position_ids=tpos, attention_mask=attention.attach(bits.view(1, 1, n, -1), bits),
              past_key_values=c1, use_cache=True)
    o2 = ref(tok, position_ids=tpos, attention_mask=dense_t, past_key_values=c2, use_cache=True)
    assert _rel(o1.logits, o2.logits) < 2e-2
    # the reference's dense mask fed to our backend gives the same result as the packed bits
    c3 = TreeKVCache.for_model(ours.config, capacity=1024, device=dev)
    ours(ids, position_ids=pos, past_key_values=c3, use_cache=True)
    o3 = ours(tok, position_ids=tpos, attention_mask=dense_t, past_key_values=c3, use_cache=True)
    assert torch.equal(o3.logits, o1.logits)


@torch.inference_mode()
def test_compact_dynamic_cache_both_layouts():
    dev = cuda()
    g = torch.Generator(device=dev).manual_seed(5)
    past, cur, keep = 50, 17, [0, 2, 3, 9, 16]
    tree = TreeKVCache(4, 2, 128, 100, device=dev)
    dyn = DynamicCache()
    for li in range(4):
        k = torch.randn((1, 2, past + cur, 128), device=dev, generator=g).to(torch.bfloat16)
        v = torch.randn((1, 2, past + cur, 128), device=dev, generator=g).to(torch.bfloat16)
        tree.update(k, v, li)
        dyn.update(k.clone(), v.clone(), li)
    want = [(l.keys.float().cpu().numpy().copy(), l.values.float().cpu().numpy().copy()) for l in dyn.layers]
    want = ot.compact_cache(want, past, keep)
    compact_dynamic_cache(tree, past, keep)
    compact_dynamic_cache(dyn, past, keep)
    for li, (wk, wv) in enumerate(want):
        for cache in (tree, dyn):
            assert cache.get_seq_length() == past + len(keep)
            assert np.array_equal(cache.layers[li].keys.float().cpu().numpy(), wk)
            assert np.array_equal(cache.layers[li].values.float().cpu().numpy(), wv)


def test_build_ddtree_tree_dropin_matches_oracle(monkeypatch):
    dev = cuda()
    logits = synthetic.draft_logits(11, 15, 151936)
    ctx = synthetic.context_ids(11, 700, 151936)
    for strategy in ("heap", "rank_gated_ngram", "ngram"):
        monkeypatch.setenv("DDTREE_TREE_STRATEGY", strategy)
        tok, dep, parents, maps, vis, sub = build_ddtree_tree(torch.from_numpy(logits).to(dev), 32,
                                                              context_ids=torch.from_numpy(ctx).to(dev))
        want = ot.build_tree_from_logits(logits, 32, strategy, ctx, ot.NgramParams())
        assert tok.tolist() == want.tokens.tolist() and parents == want.parents
        assert dep.tolist() == want.depths.tolist()
        assert maps == ot.child_maps(want.parents, want.tokens)
        assert np.array_equal(vis.numpy(), ot.visibility(want.parents))
        assert set(sub) == {"tree_build_copy", "tree_build_heap", "tree_build_visibility"}


@torch.inference_mode()
def test_verifier_round_stages_match_oracle(models, monkeypatch):
    monkeypatch.setenv("DDTREE_TREE_STRATEGY", "rank_gated_ngram")
    ours, _ = models
    dev = cuda()
    v = TreeVerifier(ours, tree_budget=32, max_length=600, draft_horizon=15)
    v.debug = True
    prompt = torch.from_numpy(synthetic.context_ids(2, 200, VOCAB, alphabet=50))[None].to(dev)
    v.prefill(prompt)
    for r in range(4):
        start = v.start
        ctx = v.output_ids[: start + 1].cpu().numpy()
        draft = torch.from_numpy(synthetic.draft_logits(100 + r, 15, VOCAB, amp=6.0)).to(dev)
        acc_len = v.round(draft)
        lp, ids, _ = kernels.draft_topk(draft, 32)
        tree = ot.build_tree(lp.cpu().numpy(), ids.cpu().numpy(), 32, "rank_gated_ngram", ctx, ot.NgramParams())
        n = tree.count + 1
        assert v.tree["parents"][:n].tolist() == tree.parents
        assert v.tree["tokens"][: tree.count].tolist() == tree.tokens.tolist()
        post = v.last_posterior[0].cpu().numpy()
        acc, nxt = ot.follow_tree(ot.child_maps(tree.parents, tree.tokens), post)
        assert acc_len == len(acc)
        vids = [int(ctx[-1])] + tree.tokens.tolist()
        assert v.output_ids[start: start + acc_len + 1].tolist() == [vids[i] for i in acc] + [nxt]
        slab = v.last_slab.float().cpu().numpy()
        ot.compact_tensor(slab, start, acc)
        got = v.cache.slab[:, :, : start + acc_len].float().cpu().numpy()
        assert np.array_equal(got, slab[:, :, : start + acc_len])
        assert v.cache.get_seq_length() == start + acc_len == v.start


@torch.inference_mode()
def test_tree_decoding_equals_greedy_decoding(monkeypatch):
    """Speculative decoding invariant at temperature 0: the committed tokens are the target's greedy tokens."""
    monkeypatch.setenv("DDTREE_TREE_STRATEGY", "rank_gated_ngram")
    dev = cuda()
    model = build_target(_small_cfg(2), device=dev, seed=9)
    with torch.no_grad():
        model.lm_head.weight.mul_(8.0)  # wide logit margins: argmax immune to bf16 reordering
    prompt = torch.from_numpy(synthetic.context_ids(4, 64, VOCAB, alphabet=30))[None].to(dev)
    new = 48
    # greedy reference with the same backend, one token per forward
    cache = TreeKVCache.for_model(model.config, capacity=256, device=dev)
    out = model(prompt, position_ids=torch.arange(64, device=dev)[None], past_key_values=cache, use_cache=True)
    greedy = [int(out.logits[0, -1].argmax())]
    margins = [1.0]
    for i in range(new - 1):
        t = torch.tensor([[greedy[-1]]], device=dev)
        out = model(t, position_ids=torch.tensor([[64 + i]], device=dev), past_key_values=cache, use_cache=True)
        top2 = out.logits[0, -1].float().topk(2).values
        margins.append(float(top2[0] - top2[1]) / max(float(top2[0].abs()), 1.0))
        greedy.append(int(out.logits[0, -1].argmax()))

    # draft: a noisy copy of the target's own next-token distribution keeps acceptance above 1
    def draft_fn(output_ids, start, r):
        g = torch.Generator(device=dev).manual_seed(r)
        return torch.randn((15, VOCAB), device=dev, generator=g)

    res = ddtree_generate(None, model, prompt, mask_token_id=VOCAB - 1, max_new_tokens=new, block_size=16,
                          stop_token_ids=None, tree_budget=24, draft_fn=draft_fn)
    got = res.output_ids[0, 64:].tolist()
    assert res.num_output_tokens >= new
    # the verify forward (fused stages, tcgen05 projections) and this one-token
    # HF forward round differently, so the runs may part only at a near tie
    # of the greedy reference's top-2 logits
    if got[: len(greedy)] != greedy[: len(got)]:
        first = next(i for i, (a, b) in enumerate(zip(got, greedy)) if a != b)
        assert first >= 8 and margins[first] < 2e-2, (first, margins[first])


@torch.inference_mode()
def test_graph_rounds_equal_eager_rounds(models, monkeypatch):
    """A CUDA-graph replay of the round is bit-identical to the eager round."""
    monkeypatch.setenv("DDTREE_TREE_STRATEGY", "rank_gated_ngram")
    ours, _ = models
    dev = cuda()
    prompt = torch.from_numpy(synthetic.context_ids(8, 150, VOCAB, alphabet=40))[None].to(dev)
    drafts = [torch.from_numpy(synthetic.draft_logits(300 + r, 15, VOCAB, amp=6.0)).to(dev).to(torch.bfloat16)
              for r in range(6)]
    eager = TreeVerifier(ours, tree_budget=24, max_length=500, draft_horizon=15)
    eager.prefill(prompt)
    graph = TreeVerifier(ours, tree_budget=24, max_length=500, draft_horizon=15)
    graph.prefill(prompt)
    graph.enable_graph(True)
    for d in drafts:
        a = eager.round(d)
        b = graph.round(d)
        assert a == b and eager.start == graph.start
    s = eager.start
    assert torch.equal(eager.output_ids[: s + 1], graph.output_ids[: s + 1])
    assert torch.equal(eager.cache.slab[:, :, :s], graph.cache.slab[:, :, :s])
    assert graph.launches_per_round and graph.graph is not None
