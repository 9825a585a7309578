"""The DFlash draft forward on the fused stages, and the decode loops with a draft module.

``FusedDraft`` is compared with the restated draft forward (``oracle.dflash``,
pinned to the reference's module by tests/golden/dflash.npz) in fp32 on the
same bf16-rounded weights and inputs, over consecutive calls that share the
draft cache (first call over a whole prompt's context rows, then decode-sized
calls).  Tolerance, against the fp32 restatement: relative L2 error below 2e-2
(bf16 activations through the layers), and no more than twice the error of
the draft module's own bf16 forward on the same inputs (both round to bf16 at
every stage, in different orders: neither is the reference for the other).

The fused verify forward's layer outputs (the draft's context features,
HF ``hidden_states[i + 1]``) are compared with the HF forward's, and
``ddtree_generate`` with a draft module must commit the target's greedy
tokens on both the module and the fused paths.
"""

import pytest
import torch

from oracle import dflash as od
from retree_b200 import attention, fused, kernels, synthetic
from retree_b200.cache import TreeKVCache
from retree_b200.ddtree import ddtree_generate
from retree_b200.draft import FusedDraft, supports
from retree_b200.target import build_target, qwen3_config
from tests.gpu_util import cuda

pytestmark = [pytest.mark.gpu, pytest.mark.late]

VOCAB = 2000


def _rel(got, want):
    return float((got.float() - want.float()).norm() / want.float().norm())


def _target(hidden, layers, dev, seed=3):
    cfg = qwen3_config("small", hidden_size=hidden, intermediate_size=2 * hidden, num_hidden_layers=layers,
                       num_attention_heads=hidden // 64, num_key_value_heads=2, vocab_size=VOCAB,
                       tie_word_embeddings=False)
    return build_target(cfg, device=dev, seed=seed)


def _calls(cfg, dev, target):
    """The golden call sequence's context rows (bf16) and seeded block ids (root + mask tokens)."""
    spec = od.GOLDEN_CALLS
    out = []
    for j, (seed, c) in enumerate(zip(spec.input_seeds, spec.ctx_rows)):
        th, _ = od.seeded_inputs(cfg, seed, c)
        ids = torch.full((cfg.block_size,), cfg.dflash_config["mask_token_id"], dtype=torch.int64)
        ids[0] = 100 + 7 * j
        out.append((th.to(dev, torch.bfloat16), ids.to(dev)))
    return out


@torch.inference_mode()
@pytest.mark.parametrize("ctx_chunk", [1024, 16])
def test_fused_draft_matches_restated_forward(ctx_chunk):
    dev = cuda()
    cfg = od.small_config()
    w = {k: v.to(torch.bfloat16) for k, v in od.seeded_weights(cfg, od.GOLDEN_CALLS.seed).items()}
    draft = od.build_module(cfg, w, dtype=torch.bfloat16, device=dev)
    ref32 = od.build_module(cfg, {k: v.float() for k, v in w.items()}, dtype=torch.float32, device=dev)
    ref16 = od.build_module(cfg, w, dtype=torch.bfloat16, device=dev)
    target = _target(cfg.hidden_size, 2, dev)
    assert supports(draft, target)
    embed = target.model.embed_tokens.weight
    calls = _calls(cfg, dev, target)
    fd = FusedDraft(draft, target, capacity=256, ctx_chunk=ctx_chunk)
    got, start = [], 0
    for th, ids in calls:
        start += th.shape[0]
        got.append(fd.forward(ids, th, start, return_hidden=True).clone())
        assert fd.length == start
    kernels.check_device_status(dev)
    seq = [(th, embed[ids]) for th, ids in calls]
    want32 = od.run_calls(ref32, [(th.float(), e.float()) for th, e in seq], device=dev, dtype=torch.float32)
    want16 = od.run_calls(ref16, seq, device=dev, dtype=torch.bfloat16)
    for j in range(len(calls)):
        e_got, e_mod = _rel(got[j], want32[j]), _rel(want16[j], want32[j])
        print(f"call {j}: fused vs fp32 {e_got:.5f}, bf16 module vs fp32 {e_mod:.5f}, "
              f"fused vs bf16 module {_rel(got[j], want16[j]):.5f}")
        assert e_got < 2e-2, (j, e_got)
        assert e_got <= max(2.0 * e_mod, 5e-3), (j, e_got, e_mod)
    # crop semantics: the block's rows are not kept, so the same block at the
    # same start (no new context) gives the same output
    th, ids = calls[-1]
    again = fd.forward(ids, th[:0], start, return_hidden=True)
    assert torch.equal(again, got[-1])
    # logits: the target's lm_head over the last block - 1 rows
    logits = fd.forward(ids, th[:0], start)
    assert logits.shape == (cfg.block_size - 1, VOCAB)
    ref_logits = want32[-1][1:] @ target.lm_head.weight.float().t()
    assert _rel(logits, ref_logits) < 2e-2
    with pytest.raises(RuntimeError):
        fd.forward(ids, th, start)  # context rows that do not end at start


@torch.inference_mode()
def test_fused_forward_writes_the_selected_layer_outputs():
    dev = cuda()
    model = _target(512, 4, dev, seed=8)
    L = 200
    prompt = torch.randint(0, VOCAB, (1, L), device=dev, generator=torch.Generator(device=dev).manual_seed(4))
    c_hf = TreeKVCache.for_model(model.config, capacity=512, device=dev)
    model(prompt, position_ids=torch.arange(L, device=dev)[None], past_key_values=c_hf, use_cache=True)
    c_fu = TreeKVCache.for_model(model.config, capacity=512, device=dev)
    c_fu.slab.copy_(c_hf.slab)
    c_fu.set_length(L)
    n = 12
    bits = attention.causal_bits(n, dev)
    pos = torch.arange(L, L + n, device=dev)
    tok = torch.randint(0, VOCAB, (n,), device=dev, generator=torch.Generator(device=dev).manual_seed(5))
    out = model(tok[None], position_ids=pos[None], attention_mask=attention.attach(bits.view(1, 1, n, -1), bits),
                past_key_values=c_hf, use_cache=True, output_hidden_states=True)
    layers = [1, 3, 0]
    ft = fused.FusedTarget(model, c_fu, n_max=32, gemm="cublas", capture_layers=layers)
    ft.forward(tok, pos, bits, offset=L)
    kernels.check_device_status(dev)
    h = model.config.hidden_size
    for j, li in enumerate(layers):
        got = ft.hidden_out[:n, j * h: (j + 1) * h]
        want = out.hidden_states[li + 1][0]  # the last entry is the final norm's output
        assert _rel(got, want) < 1e-2, (li, _rel(got, want))
    with pytest.raises(ValueError):
        fused.FusedTarget(model, c_fu, n_max=32, gemm="cublas", capture_layers=[4])


@torch.inference_mode()
@pytest.mark.parametrize("fused_paths", [False, True])
def test_ddtree_generate_with_a_draft_module_commits_greedy_tokens(monkeypatch, fused_paths):
    """Speculative invariant with a real draft module: the committed tokens are the target's greedy ones.

    The draft (a DFlash module with seeded weights, context features from
    target layers 1 and 3) only changes how many tokens a round accepts.  The
    runs may part from the one-token HF greedy reference only at a near tie
    of its top-2 logits.
    """
    monkeypatch.setenv("DDTREE_TREE_STRATEGY", "rank_gated_ngram")
    dev = cuda()
    cfg = od.small_config(hidden=512, heads=4, kv_heads=2, inter=1024, target_layers=2, block_size=16)
    target = _target(512, 4, dev, seed=9)
    draft = od.build_module(cfg, od.seeded_weights(cfg, 1), dtype=torch.bfloat16, device=dev)
    prompt = torch.from_numpy(synthetic.context_ids(5, 64, VOCAB, alphabet=30))[None].to(dev)
    new = 40
    cache = TreeKVCache.for_model(target.config, capacity=256, device=dev)
    out = target(prompt, position_ids=torch.arange(64, device=dev)[None], past_key_values=cache, use_cache=True)
    greedy, margins = [int(out.logits[0, -1].argmax())], [1.0]
    for i in range(new - 1):
        o = target(torch.tensor([[greedy[-1]]], device=dev), position_ids=torch.tensor([[64 + i]], device=dev),
                   past_key_values=cache, use_cache=True)
        top2 = o.logits[0, -1].float().topk(2).values
        margins.append(float(top2[0] - top2[1]) / max(float(top2[0].abs()), 1.0))
        greedy.append(int(o.logits[0, -1].argmax()))
    res = ddtree_generate(draft, target, prompt, mask_token_id=VOCAB - 1, max_new_tokens=new, block_size=16,
                          stop_token_ids=None, fused=fused_paths, fused_draft=fused_paths)
    kernels.check_device_status(dev)
    got = res.output_ids[0, 64:].tolist()
    assert res.num_output_tokens >= new and min(res.acceptance_lengths) >= 1
    if got[: len(greedy)] != greedy[: len(got)]:
        first = next(i for i, (a, b) in enumerate(zip(got, greedy)) if a != b)
        assert margins[first] < 2e-2, (first, margins[first])  # the runs may part only at a near tie


@torch.inference_mode()
def test_attention_backend_runs_the_draft_attention_non_causal():
    """The HF backend with no mask and is_causal=False (the draft's call) matches SDPA without a mask."""
    import torch.nn.functional as F

    dev = cuda()
    g = torch.Generator(device=dev).manual_seed(3)
    n, S = 16, 300
    q = torch.randn((1, 32, n, 128), device=dev, generator=g).to(torch.bfloat16)
    k = torch.randn((1, 8, S, 128), device=dev, generator=g).to(torch.bfloat16)
    v = torch.randn((1, 8, S, 128), device=dev, generator=g).to(torch.bfloat16)
    mod = torch.nn.Module()
    mod.is_causal = False
    out, _ = attention.tree_attention_forward(mod, q, k, v, None, scaling=128 ** -0.5, is_causal=False)
    ref = F.scaled_dot_product_attention(q.float(), k.float().repeat_interleave(4, 1),
                                         v.float().repeat_interleave(4, 1), scale=128 ** -0.5)
    err = (out[0].float() - ref[0].transpose(0, 1)).abs()
    assert float(err.max()) < 2e-2 and float(err.mean()) < 1e-3


@torch.inference_mode()
@pytest.mark.parametrize("block_size", [1, 16])
def test_linear_dflash_loop_commits_greedy_tokens(monkeypatch, block_size):
    """dflash_generate (the linear baseline; block_size <= 1: no draft) commits the target's greedy tokens,
    and ddtree_generate / retree_generate hand block_size <= 1 to it as the reference does."""
    from retree_b200.ddtree import dflash_generate
    from retree_b200.retree import retree_generate

    dev = cuda()
    target = _target(512, 2, dev, seed=10)
    prompt = torch.from_numpy(synthetic.context_ids(6, 48, VOCAB, alphabet=30))[None].to(dev)
    new = 24
    cache = TreeKVCache.for_model(target.config, capacity=256, device=dev)
    out = target(prompt, position_ids=torch.arange(48, device=dev)[None], past_key_values=cache, use_cache=True)
    greedy, margins = [int(out.logits[0, -1].argmax())], [1.0]
    for i in range(new - 1):
        o = target(torch.tensor([[greedy[-1]]], device=dev), position_ids=torch.tensor([[48 + i]], device=dev),
                   past_key_values=cache, use_cache=True)
        top2 = o.logits[0, -1].float().topk(2).values
        margins.append(float(top2[0] - top2[1]) / max(float(top2[0].abs()), 1.0))
        greedy.append(int(o.logits[0, -1].argmax()))

    def draft_fn(output_ids, start, r):
        return torch.randn((15, VOCAB), device=dev, generator=torch.Generator(device=dev).manual_seed(r))

    runs = [dflash_generate(None, target, prompt, VOCAB - 1, new, block_size, None, draft_fn=draft_fn)]
    if block_size == 1:
        runs.append(ddtree_generate(None, target, prompt, VOCAB - 1, new, block_size, None))
        runs.append(retree_generate(None, target, prompt, VOCAB - 1, new, block_size, None))
    kernels.check_device_status(dev)
    for res in runs:
        got = res.output_ids[0, 48:].tolist()
        assert res.num_output_tokens >= new
        if block_size == 1:
            assert set(res.acceptance_lengths) == {1}
        if got[: len(greedy)] != greedy[: len(got)]:
            first = next(i for i, (a, b) in enumerate(zip(got, greedy)) if a != b)
            assert margins[first] < 2e-2, (first, margins[first])
