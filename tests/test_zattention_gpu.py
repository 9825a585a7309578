"""GPU parity of tree-verify attention against the fp32 SDPA oracle.

Tolerance (the bound this path is held to): max |err| <= 2e-2 and
mean |err| <= 1e-3 against fp32 attention on the same bf16-rounded inputs.
"""

import pytest
import torch

from oracle import attention as oatt
from oracle import tree as ot
from retree_b200 import kernels
from tests import golden_cases as gc
from tests.gpu_util import bits_tensor, cuda, random_tree

pytestmark = pytest.mark.gpu

MAX_ABS = 2e-2
MEAN_ABS = 1e-3


def _inputs(seed, n, prefix, hq=32, hkv=8, cap_extra=0, hf_q_layout=True):
    g = torch.Generator().manual_seed(seed)
    q = torch.randn((1, n, hq, 128), generator=g).to(torch.bfloat16)
    kv = torch.randn((2, hkv, prefix + n + cap_extra, 128), generator=g).to(torch.bfloat16)
    q_hf = q.transpose(1, 2)  # [1, Hq, n, D] strided, as HF hands it over
    return (q_hf if hf_q_layout else q[0]), kv[0], kv[1]


def _check(out, q, k, v, prefix, vis):
    qf = q.float() if q.dim() == 4 else q.float().transpose(0, 1)[None]
    ref = oatt.tree_attention(qf.cpu(), k.float().cpu(), v.float().cpu(), prefix, vis)
    err = (out.float().cpu() - ref).abs()
    assert float(err.max()) <= MAX_ABS, float(err.max())
    assert float(err.mean()) <= MEAN_ABS, float(err.mean())
    rel = float(torch.linalg.norm(out.float().cpu() - ref) / torch.linalg.norm(ref))
    assert rel < 1e-2, rel


def test_attention_cfg1_against_reference_sdpa_output():
    """Config 1 (prefix 512, budget-16 tree): kernel on bf16-rounded inputs vs the reference's fp32 SDPA."""
    dev = cuda()
    meta = gc.load_json("attention_cfg1.json")
    t = gc.tree_case(meta["tree"])
    n, past = meta["n"], meta["past"]
    g = torch.Generator().manual_seed(0)
    q = torch.randn((1, 32, n, 128), generator=g)
    k = torch.randn((1, 8, past + n, 128), generator=g)
    v = torch.randn((1, 8, past + n, 128), generator=g)
    vis = ot.visibility(t["parents"])
    qb, kb, vb = (x.to(torch.bfloat16) for x in (q, k, v))
    for path in ((1, 2) if n * 4 <= 64 else (1,)):
        out = kernels.tree_attention(qb.to(dev), kb.to(dev), vb.to(dev), bits_tensor(vis, dev), past, path=path)
        kernels.check_device_status(dev)
        _check(out, qb, kb[0], vb[0], past, vis)
    ref_fp32 = torch.from_numpy(gc.load_npz("attention_cfg1.npz")["out"][0])
    err = (out.float().cpu() - ref_fp32).abs()  # includes the bf16 rounding of q/k/v
    assert float(err.max()) <= MAX_ABS and float(err.mean()) <= MEAN_ABS


@pytest.mark.parametrize("n,prefix,splits", [
    (5, 0, 1), (5, 37, 1), (15, 300, 0), (16, 1000, 3), (9, 4096, 0),
])
def test_warp_path(n, prefix, splits):
    dev = cuda()
    parents, vis = random_tree(n, n - 1)
    q, k, v = _inputs(n * 7 + prefix, n, prefix, cap_extra=11)
    out = kernels.tree_attention(q.to(dev), k.to(dev), v.to(dev), bits_tensor(vis, dev), prefix,
                                 num_splits=splits, path=2)
    kernels.check_device_status(dev)
    _check(out, q, k, v, prefix, vis)


@pytest.mark.parametrize("n,prefix,splits", [
    (17, 512, 1), (17, 4096, 0), (16, 0, 1), (17, 1, 0), (33, 200, 2), (65, 1023, 0),
    (129, 4096, 0), (257, 4096, 0), (257, 130, 1), (100, 5000, 7),
])
def test_tcgen05_path(n, prefix, splits):
    dev = cuda()
    parents, vis = random_tree(1000 + n, n - 1)
    q, k, v = _inputs(n * 13 + prefix, n, prefix, cap_extra=40)
    out = kernels.tree_attention(q.to(dev), k.to(dev), v.to(dev), bits_tensor(vis, dev), prefix,
                                 num_splits=splits, path=1)
    kernels.check_device_status(dev)
    _check(out, q, k, v, prefix, vis)


def test_tcgen05_device_prefix_length_and_group_sizes():
    dev = cuda()
    for hq, hkv, n in ((32, 8, 17), (16, 8, 40), (8, 1, 9), (64, 8, 33)):
        parents, vis = random_tree(hq + n, n - 1)
        prefix = 777
        q, k, v = _inputs(hq * 3 + n, n, prefix, hq=hq, hkv=hkv, cap_extra=300)
        plen = torch.tensor([prefix], dtype=torch.int64, device=dev)
        out = kernels.tree_attention(q.to(dev), k.to(dev), v.to(dev), bits_tensor(vis, dev), prefix + 200,
                                     prefix_len_dev=plen, path=1 if n * (hq // hkv) >= 64 else 0)
        kernels.check_device_status(dev)
        _check(out, q, k, v, prefix, vis)


def _gpu_reference(q, k, v, prefix, vis, scale=128 ** -0.5):
    """fp32 masked GQA attention on the device (the same op as oracle.attention), one kv head at a time."""
    n, hq, d = q.shape
    hkv = k.shape[0]
    G = hq // hkv
    s = prefix + n
    mask = torch.zeros((n, s), dtype=torch.float32, device=q.device)
    mask[:, prefix:] = torch.where(torch.from_numpy(vis).to(q.device), 0.0, torch.finfo(torch.float32).min)
    out = torch.empty((n, hq, d), dtype=torch.float32, device=q.device)
    for h in range(hkv):
        qh = q[:, h * G:(h + 1) * G].float().transpose(0, 1)            # [G, n, D]
        sc = torch.matmul(qh, k[h, :s].float().t()) * scale + mask       # [G, n, S]
        out[:, h * G:(h + 1) * G] = torch.matmul(torch.softmax(sc, dim=-1), v[h, :s].float()).transpose(0, 1)
    return out


@pytest.mark.parametrize("hq,hkv", [(32, 8), (16, 4), (8, 2), (4, 1)])
def test_long_context_budget_256_at_split_head_counts(hq, hkv):
    """The long-context workload: prefix 32768, budget 256 (257 tree rows), with the query / kv heads one
    rank holds when Qwen3-8B's 32 / 8 heads are split by kv head over 1, 2, 4 or 8 GPUs."""
    dev = cuda()
    n, prefix = 257, 32768
    parents, vis = random_tree(5000 + hq, n - 1)
    g = torch.Generator(device=dev).manual_seed(hq * 31 + hkv)
    q = torch.randn((n, hq, 128), device=dev, generator=g).to(torch.bfloat16)
    kv = torch.randn((2, hkv, prefix + n + 64, 128), device=dev, generator=g).to(torch.bfloat16)
    out = kernels.tree_attention(q, kv[0], kv[1], bits_tensor(vis, dev), prefix)
    kernels.check_device_status(dev)
    ref = _gpu_reference(q, kv[0], kv[1], prefix, vis)
    err = (out.float() - ref).abs()
    assert float(err.max()) <= MAX_ABS, float(err.max())
    assert float(err.mean()) <= MEAN_ABS, float(err.mean())
