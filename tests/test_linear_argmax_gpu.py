"""rt_linear_argmax: the projection's logits and each row's argmax from one launch.

The logits must equal rt_linear's bit for bit, and the index must be
torch.argmax of those logits (first largest value; rows with exact ties are
planted by duplicating weight rows; a NaN input row makes every logit NaN and
its argmax 0, as torch's).  The fused verify forward with the argmax on gives
the same rounds as without it.
"""

import pytest
import torch

from retree_b200 import kernels, synthetic
from retree_b200.target import build_target, qwen3_config
from retree_b200.verify import TreeVerifier
from tests.gpu_util import cuda

pytestmark = [pytest.mark.gpu, pytest.mark.late]


@torch.inference_mode()
@pytest.mark.parametrize("m,n_out,k", [(1, 1024, 256), (17, 151936, 2560), (65, 4096, 512), (200, 2048, 1024)])
def test_argmax_projection_matches_store_and_torch_argmax(m, n_out, k):
    dev = cuda()
    g = torch.Generator(device=dev).manual_seed(m + n_out)
    w = (torch.randn((n_out, k), device=dev, generator=g) * k ** -0.5).to(torch.bfloat16)
    w[n_out // 3] = w[n_out // 7]  # exact ties between two output rows
    w[n_out - 1] = w[5]
    x = torch.randn((m, k), device=dev, generator=g).to(torch.bfloat16)
    if m > 1:
        x[m // 2] = float("nan")
    want = kernels.linear(x, w)
    got = torch.empty_like(want)
    idx = torch.empty(m, dtype=torch.int64, device=dev)
    kernels.linear_argmax(x, w, got, idx)
    torch.cuda.synchronize()
    kernels.check_device_status(dev)
    assert torch.equal(got.view(torch.int16), want.view(torch.int16))  # bit for bit, NaNs included
    assert torch.equal(idx, want.argmax(dim=-1))


@torch.inference_mode()
def test_fused_rounds_with_the_argmax_projection(monkeypatch):
    monkeypatch.setenv("DDTREE_TREE_STRATEGY", "rank_gated_ngram")
    dev = cuda()
    cfg = qwen3_config("small", hidden_size=512, intermediate_size=1024, num_hidden_layers=2, num_attention_heads=8,
                       num_key_value_heads=2, vocab_size=2048, tie_word_embeddings=False)
    model = build_target(cfg, device=dev, seed=14)
    prompt = torch.from_numpy(synthetic.context_ids(4, 100, 2048, alphabet=40))[None].to(dev)
    drafts = [torch.from_numpy(synthetic.draft_logits(70 + r, 15, 2048, amp=6.0)).to(dev).to(torch.bfloat16)
              for r in range(4)]
    a = TreeVerifier(model, tree_budget=24, max_length=400, fused=True, gemm="tcgen05")
    b = TreeVerifier(model, tree_budget=24, max_length=400, fused=True, gemm="tcgen05", fused_argmax=True)
    assert b.fused.argmax and not a.fused.argmax
    a.prefill(prompt)
    b.prefill(prompt)
    b.enable_graph(True)
    for d in drafts:
        assert a.round(d) == b.round(d)
    kernels.check_device_status(dev)
    s = a.start
    assert torch.equal(a.output_ids[: s + 1], b.output_ids[: s + 1])
