"""The attention launch's L2 warm-up (rt_tree_attn_ex) changes no result.

The requests only load lines into L2, so the attention output and the fused
verify forward's logits must be bit-identical with and without them, for
ranges that are shorter than, equal to, and longer than the CTAs' shares.
"""

import pytest
import torch

from retree_b200 import fused, kernels
from retree_b200.cache import TreeKVCache
from retree_b200.target import build_target, qwen3_config
from tests.gpu_util import bits_tensor, cuda, random_tree

pytestmark = [pytest.mark.gpu, pytest.mark.late]


@torch.inference_mode()
@pytest.mark.parametrize("n,prefix", [(17, 2048), (65, 700), (257, 4096)])
def test_attention_output_is_unchanged_by_l2_warm_up(n, prefix):
    dev = cuda()
    g = torch.Generator(device=dev).manual_seed(n)
    cap = prefix + n + 64
    k = torch.randn((8, cap, 128), device=dev, generator=g).to(torch.bfloat16)
    v = torch.randn((8, cap, 128), device=dev, generator=g).to(torch.bfloat16)
    q = torch.randn((n, 32, 128), device=dev, generator=g).to(torch.bfloat16)
    _, vis = random_tree(n, n - 1)
    assert vis.shape == (n, n)
    bits = bits_tensor(vis, dev)
    want = kernels.tree_attention(q, k, v, bits, prefix, kv_capacity=cap).clone()
    w1 = torch.randn((4096, 2560), device=dev, generator=g).to(torch.bfloat16)
    w2 = torch.randn((1000, 24), device=dev, generator=g).to(torch.bfloat16)
    for ranges in ([(w1, w1.numel() * 2)], [(w1, 5 << 20), (w2, w2.numel() * 2)], [(w2, 100)]):
        got = kernels.tree_attention(q, k, v, bits, prefix, kv_capacity=cap, l2_prefetch=ranges)
        torch.cuda.synchronize()
        kernels.check_device_status(dev)
        assert torch.equal(got, want)


@torch.inference_mode()
def test_fused_forward_is_unchanged_by_l2_warm_up():
    dev = cuda()
    cfg = qwen3_config("small", hidden_size=512, intermediate_size=1024, num_hidden_layers=2, num_attention_heads=8,
                       num_key_value_heads=2, vocab_size=2000, tie_word_embeddings=False)
    model = build_target(cfg, device=dev, seed=2)
    L, n = 300, 17
    outs = []
    for pf in (0, 1 << 20, 64 << 20):
        cache = TreeKVCache.for_model(model.config, capacity=512, device=dev)
        cache.slab.copy_(torch.randn(cache.slab.shape, device=dev,
                                     generator=torch.Generator(device=dev).manual_seed(1)).to(torch.bfloat16))
        ft = fused.FusedTarget(model, cache, n_max=32, gemm="cublas", attn_l2_prefetch=pf)
        tok = torch.randint(0, 2000, (n,), device=dev, generator=torch.Generator(device=dev).manual_seed(3))
        pos = torch.arange(L, L + n, device=dev)
        bits = bits_tensor(random_tree(4, n - 1)[1], dev)
        outs.append(ft.forward(tok, pos, bits, offset=L).clone())
    kernels.check_device_status(dev)
    assert torch.equal(outs[0], outs[1]) and torch.equal(outs[0], outs[2])


@torch.inference_mode()
def test_side_stream_warm_up_changes_no_round(monkeypatch):
    """FusedTarget(l2_stream=True): same logits eagerly, and graph rounds equal to eager rounds without it."""
    from retree_b200 import synthetic
    from retree_b200.verify import TreeVerifier

    monkeypatch.setenv("DDTREE_TREE_STRATEGY", "rank_gated_ngram")
    dev = cuda()
    cfg = qwen3_config("small", hidden_size=512, intermediate_size=1024, num_hidden_layers=3, num_attention_heads=8,
                       num_key_value_heads=2, vocab_size=2000, tie_word_embeddings=False)
    model = build_target(cfg, device=dev, seed=6)
    prompt = torch.from_numpy(synthetic.context_ids(2, 120, 2000, alphabet=40))[None].to(dev)
    drafts = [torch.from_numpy(synthetic.draft_logits(50 + r, 15, 2000, amp=6.0)).to(dev).to(torch.bfloat16)
              for r in range(4)]
    plain = TreeVerifier(model, tree_budget=20, max_length=400, fused=True, gemm="cublas", l2_stream=False)
    warm = TreeVerifier(model, tree_budget=20, max_length=400, fused=True, gemm="cublas", l2_stream=True,
                        attn_l2_prefetch=8 << 20)
    assert warm.fused.l2_stream and not plain.fused.l2_stream
    plain.prefill(prompt)
    warm.prefill(prompt)
    warm.enable_graph(True)
    for d in drafts:
        assert plain.round(d) == warm.round(d)
    kernels.check_device_status(dev)
    s = plain.start
    assert torch.equal(plain.output_ids[: s + 1], warm.output_ids[: s + 1])
    assert torch.equal(plain.cache.slab[:, :, :s], warm.cache.slab[:, :, :s])


@torch.inference_mode()
def test_kv_prefix_warm_up_in_the_qkv_projection_changes_nothing():
    """RT_EPI_QKV_ROPE_KV_WARM (the QKV projection also asks the L2 for the K/V prefix) writes what
    RT_EPI_QKV_ROPE writes, and a fused forward with it gives the same logits."""
    dev = cuda()
    cfg = qwen3_config("small", hidden_size=512, intermediate_size=1024, num_hidden_layers=2, num_attention_heads=8,
                       num_key_value_heads=2, vocab_size=2000, tie_word_embeddings=False)
    model = build_target(cfg, device=dev, seed=3)
    L, n = 300, 17
    outs = []
    for warm in (False, True):
        cache = TreeKVCache.for_model(model.config, capacity=512, device=dev)
        cache.slab.copy_(torch.randn(cache.slab.shape, device=dev,
                                     generator=torch.Generator(device=dev).manual_seed(1)).to(torch.bfloat16))
        ft = fused.FusedTarget(model, cache, n_max=32, gemm="tcgen05", kv_l2_prefetch=warm)
        tok = torch.randint(0, 2000, (n,), device=dev, generator=torch.Generator(device=dev).manual_seed(3))
        pos = torch.arange(L, L + n, device=dev)
        bits = bits_tensor(random_tree(4, n - 1)[1], dev)
        for offset_dev in (None, torch.tensor([L], dtype=torch.int64, device=dev)):
            if offset_dev is None:
                outs.append(ft.forward(tok, pos, bits, offset=L).clone())
            else:
                outs.append(ft.forward(tok, pos, bits, offset_dev=offset_dev).clone())
        outs.append(cache.slab[:, :, : L + n].clone())
    kernels.check_device_status(dev)
    assert all(torch.equal(a, b) for a, b in zip(outs[:3], outs[3:]))


@torch.inference_mode()
def test_weight_row_warm_up_changes_no_projection():
    """rt_set_linear_weight_warm: every rt_linear mode gives the same bits with the warm-up on."""
    dev = cuda()
    g = torch.Generator(device=dev).manual_seed(7)
    x = torch.randn((17, 2560), device=dev, generator=g).to(torch.bfloat16)
    outs = []
    for warm in (False, True):
        kernels.set_linear_weight_warm(warm)
        try:
            for n_out, k, epi in ((2560, 2560, 0), (19456, 2560, 1), (2560, 9728, 0)):
                w = (torch.randn((n_out, k), device=dev, generator=torch.Generator(device=dev).manual_seed(n_out + k))
                     * k ** -0.5).to(torch.bfloat16)
                xx = x if k == 2560 else torch.randn((17, k), device=dev,
                                                     generator=torch.Generator(device=dev).manual_seed(1)).to(
                    torch.bfloat16)
                outs.append(kernels.linear(xx, w, epilogue=epi).clone())
            torch.cuda.synchronize()
        finally:
            kernels.set_linear_weight_warm(False)
    kernels.check_device_status(dev)
    half = len(outs) // 2
    assert all(torch.equal(a, b) for a, b in zip(outs[:half], outs[half:]))
