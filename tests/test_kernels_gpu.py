"""GPU parity of the data-movement, top-k, tree-build and walk kernels against the oracle (bit-exact)."""

import numpy as np
import pytest
import torch

from oracle import tree as ot
from retree_b200 import kernels
from tests import golden_cases as gc
from tests.gpu_util import cuda

pytestmark = pytest.mark.gpu


# ---------------------------------------------------------------- compaction
@pytest.mark.parametrize("past,cur,keep", [
    (5, 7, [0, 2, 5]), (0, 9, [0, 3, 4, 8]), (100, 17, [0, 1, 5, 9, 16]), (3, 4, [0, 1, 3]),
    (4, 6, [2, 0, 5]), (6, 3, [0, 2]), (5, 7, list(range(7))), (2, 257, list(range(0, 257, 16))),
])
def test_kv_compact_matches_oracle(past, cur, keep):
    dev = cuda()
    g = torch.Generator().manual_seed(past * 1000 + cur)
    slab = torch.randn((6, 8, past + cur + 5, 128), generator=g).to(torch.bfloat16)
    view = slab[:, :, : past + cur, :]
    want = view.float().numpy().copy()
    ot.compact_tensor(want, past, keep)
    got = slab.to(dev)
    kernels.kv_compact(got[:, :, : past + cur, :], past, torch.tensor(keep, device=dev))
    kernels.check_device_status(dev)
    assert np.array_equal(got[:, :, : past + cur].float().cpu().numpy(), want)
    # rows past the window are untouched
    assert torch.equal(got[:, :, past + cur:].cpu(), slab[:, :, past + cur:])


def test_kv_compact_golden_fp32_rows():
    dev = cuda()
    meta = gc.load_json("compact.json")
    arr = gc.load_npz("compact.npz")
    for i, c in enumerate(meta):
        for li in range(c["layers"]):
            for kv in ("k", "v"):
                t = torch.from_numpy(arr[f"c{i}_in{li}_{kv}"]).to(dev)
                if c["keep"]:
                    kernels.kv_compact(t, c["past"], torch.tensor(c["keep"], dtype=torch.long, device=dev))
                new_len = c["past"] + len(c["keep"])
                got = t[..., : min(new_len, t.shape[-2]), :].cpu().numpy()
                assert np.array_equal(got, arr[f"c{i}_out{li}_{kv}"]), (i, li, kv)


def test_kv_compact_device_count_and_bad_index():
    dev = cuda()
    slab = torch.randn((2, 4, 20, 128), device=dev).to(torch.bfloat16)
    ref = slab.clone()
    keep = torch.tensor([0, 3, 5, 7, 9], device=dev)
    n = torch.tensor([3], dtype=torch.int32, device=dev)
    kernels.kv_compact(slab, 10, keep, n_keep_dev=n)
    kernels.check_device_status(dev)
    want = ref.float().cpu().numpy().copy()
    ot.compact_tensor(want, 10, [0, 3, 5])
    assert np.array_equal(slab.float().cpu().numpy(), want)
    bad = torch.tensor([0, 11], device=dev)
    kernels.kv_compact(slab, 10, bad)
    with pytest.raises(RuntimeError, match="out of range"):
        kernels.check_device_status(dev)


def test_kv_append_matches_copy():
    dev = cuda()
    cache_k = torch.zeros((8, 64, 128), dtype=torch.bfloat16, device=dev)
    cache_v = torch.zeros_like(cache_k)
    new = torch.randn((1, 17, 8, 128), device=dev).to(torch.bfloat16).transpose(1, 2)  # HF layout, strided
    newv = torch.randn((1, 17, 8, 128), device=dev).to(torch.bfloat16).transpose(1, 2)
    kernels.kv_append(cache_k, cache_v, new, newv, offset=9)
    off = torch.tensor([30], dtype=torch.int64, device=dev)
    kernels.kv_append(cache_k, cache_v, new, newv, offset_dev=off)
    kernels.check_device_status(dev)
    assert torch.equal(cache_k[:, 9:26], new[0]) and torch.equal(cache_v[:, 9:26], newv[0])
    assert torch.equal(cache_k[:, 30:47], new[0]) and torch.equal(cache_v[:, 30:47], newv[0])
    assert int(cache_k[:, :9].abs().sum()) == 0 and int(cache_k[:, 47:].abs().sum()) == 0


# ---------------------------------------------------------------- top-k
def _check_topk(x_np, k, dev, dtype):
    x = torch.from_numpy(x_np).to(dev).to(dtype)
    logp, ids, lz = kernels.draft_topk(x, k)
    xf = x.float().cpu().numpy()
    o_logp, o_ids, o_lz, _ = ot.topk_logz(xf, k)
    assert np.array_equal(ids.cpu().numpy(), o_ids)
    lz_c = lz.cpu().numpy()
    finite = np.isfinite(o_lz)
    np.testing.assert_array_equal(lz_c[~finite], o_lz[~finite])  # +-inf / NaN exactly as torch
    assert np.all(np.abs(lz_c[finite] - o_lz[finite]) <= 2 * np.spacing(np.abs(o_lz[finite])))
    # logp is exactly fp32(top - log_z) with the kernel's own log_z
    top = np.take_along_axis(xf, o_ids, 1)
    with np.errstate(invalid="ignore"):
        np.testing.assert_array_equal(logp.cpu().numpy(), (top - lz_c[:, None]).astype(np.float32))
    return ids.cpu().numpy(), lz_c


@pytest.mark.parametrize("k", [1, 16, 64, 256, 1024])
def test_topk_fp32_matches_oracle_and_torch(k):
    dev = cuda()
    x = gc.make_logits(dict(seed=0, rows=16, vocab=151936, slice_last=15))
    ids, lz = _check_topk(x, k, dev, torch.float32)
    tv, ti = torch.topk(torch.from_numpy(x), k)
    assert np.array_equal(np.take_along_axis(x, ids, 1), tv.numpy())


@pytest.mark.parametrize("k", [16, 256])
def test_topk_bf16_ties_resolve_to_lowest_index(k):
    dev = cuda()
    x = gc.make_logits(dict(seed=5, rows=15, vocab=151936))
    xb = torch.from_numpy(x).to(torch.bfloat16).float().numpy()  # many exact ties
    _check_topk(xb, k, dev, torch.bfloat16)


@pytest.mark.parametrize("k", [16, 64])
def test_topk_fp16_matches_oracle(k):
    # fp16 logits: keys whose significant bits end at bit 13, decided by two 12-bit digits
    dev = cuda()
    x = gc.make_logits(dict(seed=7, rows=15, vocab=151936))
    xh = torch.from_numpy(x).to(torch.float16).float().numpy()  # exact in fp16, many ties
    _check_topk(xh, k, dev, torch.float16)


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_topk_rows_with_more_nans_than_k(dtype):
    # NaN ranks first (ties by index): rows with fewer NaNs than k, more NaNs than k
    # spread over the chunks, and more than k inside one chunk (its k-th key is a NaN)
    dev = cuda()
    rng = np.random.default_rng(11)
    x = rng.standard_normal((3, 151936)).astype(np.float32)
    x[0, rng.choice(151936, 5, replace=False)] = np.nan
    x[1, rng.choice(151936, 40, replace=False)] = np.nan
    x[2, 100:140] = np.nan
    if dtype == torch.bfloat16:
        x = torch.from_numpy(x).to(torch.bfloat16).float().numpy()
    for k in (16, 64):
        ids, lz = _check_topk(x, k, dev, dtype)
        assert np.all(np.isnan(lz))


def test_topk_small_vocab_and_specials():
    dev = cuda()
    x = np.random.default_rng(3).standard_normal((4, 300)).astype(np.float32)
    x[0, 5] = np.inf
    x[1, :] = -np.inf
    x[1, 7] = 0.0
    x[2, 10:20] = 2.5
    x[3, 3] = -0.0
    x[3, 4] = 0.0
    _check_topk(x, 37, dev, torch.float32)
    _check_topk(x[:, :40].copy(), 40, dev, torch.float32)


# ---------------------------------------------------------------- tree build
TREES = gc.tree_cases()


def _case_topk(case):
    x = gc.make_logits(case["logits"])
    k = min(max(case["budget"], 1), x.shape[1])
    if case.get("ref_top_ids") is not None:
        return np.asarray(case["ref_top_logp"], np.float32), np.asarray(case["ref_top_ids"], np.int64)
    lp, ids, _, _ = ot.topk_logz(x, k)
    return lp, ids


@pytest.mark.parametrize("case", TREES, ids=[c["name"] for c in TREES])
def test_tree_build_matches_golden(case):
    dev = cuda()
    params = gc.params_for(case)
    strategy = ot.canonical_strategy(case["strategy"])
    if strategy != ot.STRATEGY_HEAP and abs(params.beta) < 1e-12 and params.exact_beta0:
        strategy = ot.STRATEGY_HEAP
    lp, ids = _case_topk(case)
    ctx = gc.make_context(case["context"])
    budget = case["budget"]
    out = kernels.tree_build(torch.from_numpy(lp).to(dev), torch.from_numpy(ids).to(dev), budget, strategy, params,
                             ctx=None if ctx is None else torch.from_numpy(ctx).to(dev), root=777, start=1000)
    kernels.check_device_status(dev)
    cnt = int(out["count"].item())
    assert cnt == len(case["tokens"])
    assert out["tokens"][:cnt].tolist() == case["tokens"]
    assert out["depths"][:cnt].tolist() == case["depths"]
    assert out["parents"][: cnt + 1].tolist() == case["parents"]
    n = cnt + 1
    bits = out["mask"][:n].cpu().numpy().view(np.uint32)
    assert np.array_equal(ot.unpack_bits(bits, n), gc.bits_to_vis(case["visibility_bits"], n))
    assert out["verify_ids"][:n].tolist() == [777] + case["tokens"]
    assert out["verify_pos"][:n].tolist() == [1000] + [1000 + d for d in case["depths"]]


def test_tree_build_device_context_length_and_root():
    dev = cuda()
    case = next(c for c in TREES if c["name"] == "small_vocab_02_rank_gated_ngram_b256")
    params = gc.params_for(case)
    lp, ids = _case_topk(case)
    ctx = gc.make_context(case["context"])
    buf = torch.zeros(len(ctx) + 50, dtype=torch.int64, device=dev)
    buf[: len(ctx)] = torch.from_numpy(ctx)
    start = torch.tensor([len(ctx) - 1], dtype=torch.int64, device=dev)
    out = kernels.tree_build(torch.from_numpy(lp).to(dev), torch.from_numpy(ids).to(dev), case["budget"],
                             "rank_gated_ngram", params, ctx=buf, ctx_len_dev=start, ctx_len=1, start_dev=start)
    kernels.check_device_status(dev)
    cnt = int(out["count"].item())
    assert out["tokens"][:cnt].tolist() == case["tokens"]
    assert out["parents"][: cnt + 1].tolist() == case["parents"]
    assert int(out["verify_ids"][0]) == int(ctx[-1])


# ---------------------------------------------------------------- walk
def test_tree_walk_matches_golden():
    dev = cuda()
    trees = {c["name"]: c for c in TREES}
    for c in gc.load_json("follow.json"):
        t = trees[c["tree"]]
        parents = torch.tensor(t["parents"], dtype=torch.int32, device=dev)
        toks = torch.tensor(t["tokens"] or [0], dtype=torch.int64, device=dev)
        post = torch.tensor(c["posterior"], dtype=torch.int64, device=dev)
        res = kernels.tree_walk(parents, toks, post, count=len(t["tokens"]))
        n = int(res["accepted_len"].item())
        assert res["accepted"][:n].tolist() == c["accepted"]
        assert int(res["next_token"].item()) == c["next"]


def test_tree_walk_commits_to_output_ids():
    dev = cuda()
    t = next(c for c in TREES if c["name"] == "small_vocab_01_rank_gated_ngram_b64")
    f = next(c for c in gc.load_json("follow.json") if c["tree"] == t["name"] and len(c["accepted"]) > 1)
    parents = torch.tensor(t["parents"], dtype=torch.int32, device=dev)
    toks = torch.tensor(t["tokens"], dtype=torch.int64, device=dev)
    vids = torch.tensor([99] + t["tokens"], dtype=torch.int64, device=dev)
    out_ids = torch.full((200,), -1, dtype=torch.int64, device=dev)
    start = torch.tensor([40], dtype=torch.int64, device=dev)
    post = torch.tensor(f["posterior"], dtype=torch.int64, device=dev)
    res = kernels.tree_walk(parents, toks, post, verify_ids=vids, output_ids=out_ids, start_dev=start)
    kernels.check_device_status(dev)
    acc = f["accepted"]
    assert out_ids[40:40 + len(acc)].tolist() == [([99] + t["tokens"])[i] for i in acc]
    assert int(out_ids[40 + len(acc)]) == f["next"]
    assert int(start.item()) == 40 + len(acc)
    assert int(res["accepted_len"].item()) == len(acc)


# ---------------------------------------------------------------- dense mask bridge
@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16, torch.float16])
def test_mask_from_dense_matches_compile(dtype):
    dev = cuda()
    parents = [-1, 0, 0, 1, 2, 2, 3] + [4] * 40
    tokens = list(range(len(parents) - 1))
    depths = [0] * len(tokens)
    _, _, mask = ot.compile_tree(1, 10, tokens, depths, parents, 10, float(torch.finfo(dtype).min))
    dense = torch.from_numpy(mask).to(dtype).to(dev)
    bits = kernels.mask_from_dense(dense, 10, len(parents))
    assert np.array_equal(bits.cpu().numpy().view(np.uint32), ot.pack_bits(ot.visibility(parents)))


def test_kv_compact_depth_12_path_after_a_32k_prefix():
    """The long-context workload's commit: a seeded depth-12 accepted path (root + 12 nodes) of a budget-256
    tree, compacted after a 32768-token prefix in every layer's K and V; the prefix rows stay as they were."""
    dev = cuda()
    past, n, layers, heads = 32768, 257, 4, 8
    # a tree whose seeded chain of 12 nodes (at random increasing indices) hangs off the root; every other
    # node's parent is an earlier node
    rng = np.random.default_rng(12)
    chain = sorted(rng.choice(np.arange(1, n), size=12, replace=False).tolist())
    parents = [-1] + [int(rng.integers(0, i)) for i in range(1, n)]
    prev = 0
    for c in chain:
        parents[c], prev = prev, c
    keep = [0] + chain
    depth = [0] * n
    for i in range(1, n):
        depth[i] = depth[parents[i]] + 1
    assert depth[chain[-1]] == 12
    g = torch.Generator(device=dev).manual_seed(5)
    slab = torch.randn((2 * layers, heads, past + n + 8, 128), device=dev, generator=g).to(torch.bfloat16)
    ref = slab.clone()
    kernels.kv_compact(slab[:, :, : past + n, :], past, torch.tensor(keep, device=dev))
    kernels.check_device_status(dev)
    assert torch.equal(slab[:, :, :past], ref[:, :, :past])
    assert torch.equal(slab[:, :, past: past + len(keep)], ref[:, :, [past + i for i in keep]])
    assert torch.equal(slab[:, :, past + n:], ref[:, :, past + n:])
