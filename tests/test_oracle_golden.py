"""The CPU oracle reproduces the reference's own outputs (committed golden vectors)."""

import numpy as np
import pytest
import torch

from oracle import attention as oatt
from oracle import recovery as orec
from oracle import tree as ot
from tests import golden_cases as gc

TREES = gc.tree_cases()


@pytest.mark.parametrize("case", TREES, ids=[c["name"] for c in TREES])
def test_tree_builder_matches_reference(case):
    params = gc.params_for(case)
    if case.get("ref_top_ids") is not None:
        # tied scores: torch.topk's order of equal values is unspecified, so the
        # builder is checked on the reference's own top-k
        logp = np.asarray(case["ref_top_logp"], dtype=np.float32)
        ids = np.asarray(case["ref_top_ids"], dtype=np.int64)
        tree = ot.build_tree(logp, ids, case["budget"], case["strategy"],
                             gc.make_context(case["context"]), params)
    else:
        tree = ot.build_tree_from_logits(gc.make_logits(case["logits"]), case["budget"],
                                         case["strategy"], gc.make_context(case["context"]), params)
    assert tree.tokens.tolist() == case["tokens"]
    assert tree.depths.tolist() == case["depths"]
    assert tree.parents == case["parents"]
    n = 1 + len(case["tokens"])
    vis = ot.visibility(tree.parents)
    assert np.array_equal(vis, gc.bits_to_vis(case["visibility_bits"], n))
    maps = ot.child_maps(tree.parents, tree.tokens)
    assert [{str(t): c for t, c in m.items()} for m in maps] == case["child_maps"]


def test_topk_logz_matches_torch():
    meta = gc.load_json("topk.json")
    arr = gc.load_npz("topk.npz")
    for name, m in meta.items():
        x = gc.make_logits(m["spec"])
        logp, ids, log_z, top = ot.topk_logz(x, m["k"])
        ref_ids = arr[f"{name}__ids"]
        ref_logz = arr[f"{name}__log_z"]
        # values are unique as a multiset; ids agree wherever values are distinct
        assert np.array_equal(np.take_along_axis(x, ids, 1), np.take_along_axis(x, ref_ids, 1))
        if not m["ties"]:
            assert np.array_equal(ids, ref_ids)
        ulp = np.spacing(np.abs(ref_logz).astype(np.float32))
        assert np.all(np.abs(log_z - ref_logz) <= 4 * ulp)


def test_ngram_bonus_bit_exact():
    from retree_b200 import synthetic
    for c in gc.load_json("bonus.json"):
        ctx = synthetic.context_ids(c["ctx"]["seed"], c["ctx"]["length"], c["ctx"]["alphabet"],
                                    c["ctx"]["alphabet"])
        p = ot.NgramParams(max_n=c["max_n"], min_count=c["min_count"], use_log_count=c["use_log"],
                           longer_weight=c["longer_weight"], max_token_bonus=c["cap"])
        got = ot.ngram_bonus(ot.NgramCounter(ctx.tolist(), c["max_n"]), tuple(c["tail"]), c["token"], p)
        assert float(got).hex() == c["bonus_hex"]


def test_compile_matches_reference():
    trees = {c["name"]: c for c in TREES}
    for c in gc.load_json("compile.json"):
        t = trees[c["tree"]]
        ids, pos, mask = ot.compile_tree(c["root"], c["start"], t["tokens"], t["depths"],
                                         t["parents"], c["past"])
        assert ids.tolist() == c["ids"]
        assert pos.tolist() == c["pos"]
        assert c["prefix_all_visible"]
        n = len(ids)
        vis = mask[:, c["past"]:] == 0
        assert np.array_equal(ot.pack_bits(vis).astype(np.int64), np.asarray(c["tree_bits"]))
        assert c["prev"] == [c["past"], n]


def test_follow_matches_reference():
    trees = {c["name"]: c for c in TREES}
    for c in gc.load_json("follow.json"):
        t = trees[c["tree"]]
        acc, nxt = ot.follow_tree(ot.child_maps(t["parents"], t["tokens"]), c["posterior"])
        assert acc == c["accepted"] and nxt == c["next"]


def test_compaction_matches_reference():
    meta = gc.load_json("compact.json")
    arr = gc.load_npz("compact.npz")
    for i, c in enumerate(meta):
        layers = [(arr[f"c{i}_in{li}_k"].copy(), arr[f"c{i}_in{li}_v"].copy()) for li in range(c["layers"])]
        out = ot.compact_cache(layers, c["past"], c["keep"])
        for li, (k, v) in enumerate(out):
            assert np.array_equal(k, arr[f"c{i}_out{li}_k"]), (i, li)
            assert np.array_equal(v, arr[f"c{i}_out{li}_v"]), (i, li)


def test_attention_cfg1_matches_reference():
    meta = gc.load_json("attention_cfg1.json")
    ref = gc.load_npz("attention_cfg1.npz")["out"][0]
    t = gc.tree_case(meta["tree"])
    n, past = meta["n"], meta["past"]
    g = torch.Generator().manual_seed(0)
    q = torch.randn((1, 32, n, 128), generator=g)
    k = torch.randn((1, 8, past + n, 128), generator=g)
    v = torch.randn((1, 8, past + n, 128), generator=g)
    out = oatt.tree_attention(q, k, v, past, ot.visibility(t["parents"]))
    assert out.shape == ref.shape
    assert float((out - torch.from_numpy(ref)).abs().max()) < 2e-5


def test_recovery_walk_matches_reference():
    trees = {c["name"]: c for c in TREES}
    arr = gc.load_npz("recovery.npz")
    for i, c in enumerate(gc.load_json("recovery.json")):
        t = trees[c["tree"]]
        logits = arr[f"r{i}_logits"]
        mem = orec.Memory(c["freq_threshold"])
        for d, tt, cnt in c["prior"]:
            mem.record_prior(d, tt, cnt)
        acc, nxt, resc = orec.follow_with_recovery(
            ot.child_maps(t["parents"], t["tokens"]), logits.argmax(-1), logits, mem,
            gate_threshold=c["gate_threshold"], online_update=True, record_top_k=c["record_top_k"],
            rescue_top_k=c["rescue_top_k"], stop_ids=None if c["stop"] is None else set(c["stop"]))
        assert (acc, nxt, resc) == (c["accepted"], c["next"], c["rescued"]), i
        assert sorted([d, tt, n] for (d, tt), n in mem.online.items()) == c["online"]
