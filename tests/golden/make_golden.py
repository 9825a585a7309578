"""Generate the golden vectors that pin the CPU oracle to the reference.

Runs the reference's own functions (Adamlong3/ReTree, imported from a local
checkout) on seeded inputs and writes their outputs next to this script:

    python tests/golden/make_golden.py --reference /path/to/ReTree

Inputs are regenerated from their seeds by the tests (``retree_b200.synthetic``
and ``torch.Generator``), so only the reference's outputs are stored.  The
reference's ``cuda_time`` calls ``torch.cuda.synchronize()``; on a host
without a GPU it is replaced by ``time.perf_counter`` (timing only).
"""

from __future__ import annotations

import argparse
import hashlib
import json
import os
import sys
import time
from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent
sys.path.insert(0, str(HERE.parents[1]))

from retree_b200 import synthetic  # noqa: E402

ENV_KEYS = (
    "DDTREE_TREE_STRATEGY", "DDTREE_NGRAM_MAX_N", "DDTREE_NGRAM_BETA", "DDTREE_NGRAM_RANK_CAP",
    "DDTREE_NGRAM_MIN_COUNT", "DDTREE_NGRAM_CONTEXT_WINDOW", "DDTREE_NGRAM_USE_LOG_COUNT",
    "DDTREE_NGRAM_LONGER_WEIGHT", "DDTREE_NGRAM_MAX_TOKEN_BONUS", "DDTREE_NGRAM_EXACT_BETA0",
)

# name, logits recipe, budget, strategy, context recipe, env overrides
TREE_CASES = [
    # config 1: vocab 151936, last 15 of 16 draft rows, rank-gated n-gram, budget 16, 513-token context
    ("cfg1_rank_gated_b16", dict(seed=0, rows=16, vocab=151936, slice_last=15), 16,
     "rank_gated_ngram", dict(seed=0, length=513, vocab=151936), {}),
    ("cfg1_heap_b16", dict(seed=0, rows=16, vocab=151936, slice_last=15), 16, "heap", None, {}),
    ("full_vocab_rank_gated_b64", dict(seed=1, rows=15, vocab=151936), 64,
     "rank_gated_ngram", dict(seed=1, length=2049, vocab=151936), {}),
    ("full_vocab_heap_b256", dict(seed=2, rows=15, vocab=151936), 256, "heap", None, {}),
    ("full_vocab_rank_gated_b256_repeats", dict(seed=3, rows=15, vocab=151936, amp=8.0), 256,
     "rank_gated_ngram", dict(seed=3, length=3000, vocab=151936, alphabet=40), {}),
]
# small-vocab cases where the context shares the draft's alphabet so n-grams fire
for i, (budget, strategy, env) in enumerate([
    (16, "rank_gated_ngram", {}),
    (64, "rank_gated_ngram", {}),
    (256, "rank_gated_ngram", {}),
    (64, "ngram", {}),
    (64, "continuity", {"DDTREE_NGRAM_BETA": "0.6"}),
    (64, "rank_gated_ngram", {"DDTREE_NGRAM_RANK_CAP": "2", "DDTREE_NGRAM_BETA": "1.0"}),
    (64, "rank_gated_ngram", {"DDTREE_NGRAM_MAX_N": "2"}),
    (64, "rank_gated_ngram", {"DDTREE_NGRAM_MAX_N": "6", "DDTREE_NGRAM_LONGER_WEIGHT": "2.0"}),
    (64, "ngram", {"DDTREE_NGRAM_USE_LOG_COUNT": "0", "DDTREE_NGRAM_MAX_TOKEN_BONUS": "0"}),
    (64, "ngram", {"DDTREE_NGRAM_MIN_COUNT": "3", "DDTREE_NGRAM_BETA": "0.4"}),
    (64, "ngram", {"DDTREE_NGRAM_CONTEXT_WINDOW": "64"}),
    (64, "ngram", {"DDTREE_NGRAM_BETA": "-0.3"}),
    (64, "rank_gated_ngram", {"DDTREE_NGRAM_BETA": "0.0"}),
    (64, "rank_gated_ngram", {"DDTREE_NGRAM_BETA": "0.0", "DDTREE_NGRAM_EXACT_BETA0": "0"}),
    (100, "heap", {}),
    (1, "rank_gated_ngram", {}),
    (2, "heap", {}),
    (0, "heap", {}),
    (0, "rank_gated_ngram", {}),
]):
    TREE_CASES.append((
        f"small_vocab_{i:02d}_{strategy}_b{budget}",
        dict(seed=100 + i, rows=15, vocab=48, amp=3.0, n_boost=12),
        budget, strategy, dict(seed=200 + i, length=600, vocab=48, alphabet=48), env))
TREE_CASES += [
    ("ctx_none_rank_gated", dict(seed=7, rows=15, vocab=48, amp=3.0, n_boost=12), 32,
     "rank_gated_ngram", None, {}),
    ("ctx_len1_ngram", dict(seed=8, rows=15, vocab=48, amp=3.0, n_boost=12), 32, "ngram",
     dict(seed=8, length=1, vocab=48, alphabet=48), {"DDTREE_NGRAM_MIN_COUNT": "0"}),
    ("ctx_len2_ngram", dict(seed=9, rows=15, vocab=48, amp=3.0, n_boost=12), 32, "ngram",
     dict(seed=9, length=2, vocab=48, alphabet=48), {}),
    ("rows1_heap", dict(seed=10, rows=1, vocab=48, amp=3.0, n_boost=12), 32, "heap", None, {}),
    ("rows1_ngram", dict(seed=11, rows=1, vocab=48, amp=3.0, n_boost=12), 32, "ngram",
     dict(seed=11, length=300, vocab=48, alphabet=20), {}),
    ("budget_gt_vocab", dict(seed=12, rows=4, vocab=10, amp=3.0, n_boost=5), 200, "ngram",
     dict(seed=12, length=300, vocab=10, alphabet=10), {}),
    # ties in the draft scores: only 4 distinct logit values per row
    ("tied_scores_heap", dict(seed=13, rows=6, vocab=40, quantize=4), 64, "heap", None, {}),
    ("tied_scores_ngram", dict(seed=14, rows=6, vocab=40, quantize=4), 64, "ngram",
     dict(seed=14, length=300, vocab=40, alphabet=40), {}),
]


def make_logits(spec: dict) -> np.ndarray:
    """Draft logits for a golden case (shared with the tests)."""
    x = synthetic.draft_logits(spec["seed"], spec["rows"], spec["vocab"],
                               amp=spec.get("amp", synthetic.DEFAULT_ZIPF_AMP),
                               n_boost=spec.get("n_boost", 32))
    if "quantize" in spec:
        x = np.round(np.clip(x, -1.5, 1.5) * (spec["quantize"] / 3.0)).astype(np.float32)
    if "slice_last" in spec:
        x = x[-spec["slice_last"]:]
    return np.ascontiguousarray(x)


def make_context(spec: dict | None):
    if spec is None:
        return None
    return synthetic.context_ids(spec["seed"], spec["length"], spec["vocab"], spec.get("alphabet"))


def _import_reference(path: str):
    sys.path.insert(0, path)
    import dflash  # type: ignore
    dflash.cuda_time = time.perf_counter
    import ddtree  # type: ignore
    import retree  # type: ignore
    ddtree.cuda_time = time.perf_counter
    retree.cuda_time = time.perf_counter
    from model import recovery  # type: ignore
    return ddtree, retree, recovery


def _with_env(env: dict):
    saved = {k: os.environ.get(k) for k in ENV_KEYS}
    for k in ENV_KEYS:
        os.environ.pop(k, None)
    os.environ.update(env)
    return saved


def _restore_env(saved: dict):
    for k, v in saved.items():
        if v is None:
            os.environ.pop(k, None)
        else:
            os.environ[k] = v


def _packed_rows(vis: np.ndarray) -> list[list[int]]:
    n = vis.shape[0]
    w = (n + 31) // 32
    out = np.zeros((n, w), dtype=np.uint64)
    for j in range(n):
        out[vis[:, j], j // 32] |= np.uint64(1 << (j % 32))
    return out.astype(np.int64).tolist()


def gen_trees(ddtree):
    cases = []
    for name, lspec, budget, strategy, cspec, env in TREE_CASES:
        logits = make_logits(lspec)
        ctx = make_context(cspec)
        saved = _with_env(dict(env, DDTREE_TREE_STRATEGY=strategy))
        try:
            tok, dep, parents, maps, vis, _ = ddtree.build_ddtree_tree(
                torch.from_numpy(logits), budget,
                context_ids=None if ctx is None else torch.from_numpy(ctx))
        finally:
            _restore_env(saved)
        k = min(max(budget, 1), logits.shape[1])
        x = torch.from_numpy(logits).float()
        tv, ti = torch.topk(x, k=k, dim=-1)
        ties = bool((tv[:, 1:] == tv[:, :-1]).any().item()) if k > 1 else False
        entry = dict(
            name=name, logits=lspec, budget=budget, strategy=strategy, context=cspec, env=env,
            tokens=tok.tolist(), depths=dep.tolist(), parents=[int(p) for p in parents],
            child_maps=[{str(t): int(c) for t, c in m.items()} for m in maps],
            visibility_bits=_packed_rows(vis.numpy()), topk_has_ties=ties,
        )
        if ties:
            # torch.topk orders equal values arbitrarily: keep the reference's own
            # top-k (ddtree.py:362-366) so the builder can be checked on it
            lz = torch.logsumexp(x, dim=-1, keepdim=True)
            entry["ref_top_ids"] = ti.tolist()
            entry["ref_top_logp"] = (tv - lz).tolist()
        cases.append(entry)
    return cases


def gen_topk():
    """Reference top-k / logsumexp of ddtree.py:362-365 on tie-free rows."""
    out = {}
    for name, spec, k in [("cfg1_k16", dict(seed=0, rows=16, vocab=151936, slice_last=15), 16),
                          ("full_k256", dict(seed=2, rows=15, vocab=151936), 256)]:
        x = torch.from_numpy(make_logits(spec))
        tl, ti = torch.topk(x.float(), k=k, dim=-1)
        lz = torch.logsumexp(x.float(), dim=-1, keepdim=True)
        out[name] = dict(spec=spec, k=k, ids=ti.numpy(), logp=(tl - lz).numpy(),
                         log_z=lz[:, 0].numpy(), ties=bool((tl[:, 1:] == tl[:, :-1]).any()))
    return out


def gen_compile(ddtree, trees):
    cases = []
    for case in trees:
        if not case["name"].startswith(("cfg1", "small_vocab_02", "small_vocab_14", "full_vocab_heap")):
            continue
        n = 1 + len(case["tokens"])
        for dtype in (torch.float32, torch.bfloat16):
            past, start, root = 37, 37, 4242
            maxlen = past + 2 * n + 8
            ids_buf = torch.zeros((1, n), dtype=torch.long)
            pos_buf = torch.zeros((1, n), dtype=torch.long)
            mask_buf = torch.zeros((1, 1, n, maxlen), dtype=dtype)
            vis_buf = torch.zeros((n, n), dtype=torch.bool)
            vis = torch.from_numpy(ddtree_visibility_from_bits(case["visibility_bits"], n))
            # a previous, smaller tree block at a different offset must be cleared
            mask_buf[0, 0, :3, 20:23] = torch.finfo(dtype).min
            ids, pos, mask, ps, pl = ddtree.compile_ddtree_tree(
                torch.tensor(root), start, torch.tensor(case["tokens"], dtype=torch.long),
                torch.tensor(case["depths"], dtype=torch.long), vis, past, dtype, torch.device("cpu"),
                ids_buf, pos_buf, mask_buf, vis_buf, 20, 3)
            m = mask[0, 0].float().numpy()
            visible = m == 0
            cases.append(dict(
                tree=case["name"], dtype=str(dtype), past=past, start=start, root=root,
                ids=ids[0].tolist(), pos=pos[0].tolist(),
                prefix_all_visible=bool(visible[:, :past].all()),
                masked_value=float(m[~visible][0]) if (~visible).any() else None,
                tree_bits=_packed_rows(visible[:, past:past + n]), prev=[ps, pl]))
    return cases


def ddtree_visibility_from_bits(bits, n):
    b = np.asarray(bits, dtype=np.int64)
    j = np.arange(n)
    return ((b[:n, j // 32] >> (j % 32)) & 1).astype(np.bool_)


def gen_follow(ddtree, trees):
    rng = np.random.default_rng(5)
    cases = []
    for case in trees:
        if case["budget"] < 2:
            continue
        n = 1 + len(case["tokens"])
        maps = [{int(t): c for t, c in m.items()} for m in case["child_maps"]]
        for trial in range(3):
            post = rng.integers(0, 10_000, size=n)
            # make the posterior follow a random root-to-leaf path for a while
            path = synthetic.accepted_path(int(rng.integers(1 << 30)), case["parents"])
            stop = int(rng.integers(1, len(path) + 1))
            for a, b in zip(path[:stop - 1], path[1:stop]):
                post[a] = case["tokens"][b - 1]
            acc, nxt = ddtree.follow_verified_tree(maps, torch.from_numpy(post)[None])
            cases.append(dict(tree=case["name"], posterior=post.tolist(), accepted=acc, next=int(nxt)))
    return cases


def gen_compact(ddtree):
    from transformers import DynamicCache
    rng = np.random.default_rng(11)
    cases = []
    specs = [
        (5, 7, [0, 2, 5]), (5, 7, [0]), (5, 7, []), (5, 7, list(range(7))),
        (0, 9, [0, 3, 4, 8]), (12, 17, [0, 1, 2, 9, 16]), (3, 4, [0, 1, 3]),
        (4, 6, [2, 0, 5]),  # not monotone: index_select semantics
        (6, 0, []), (6, 3, [0, 2]),
    ]
    for past, cur, keep in specs:
        layers = []
        cache = DynamicCache()
        for li in range(3):
            k = rng.standard_normal((1, 2, past + cur, 8)).astype(np.float32)
            v = rng.standard_normal((1, 2, past + cur, 8)).astype(np.float32)
            layers.append((k.copy(), v.copy()))
            cache.update(torch.from_numpy(k.copy()), torch.from_numpy(v.copy()), li)
        for use_cpp in (False, True):
            if use_cpp and os.environ.get("GOLDEN_SKIP_CPP"):
                continue
            c2 = DynamicCache()
            for li, (k, v) in enumerate(layers):
                c2.update(torch.from_numpy(k.copy()), torch.from_numpy(v.copy()), li)
            ddtree.maybe_enable_cpp_compact(use_cpp)
            ddtree.compact_dynamic_cache(c2, past, keep)
            res = [(l.keys.numpy().copy(), l.values.numpy().copy()) for l in c2.layers]
            cases.append(dict(past=past, cur=cur, keep=keep, cpp=use_cpp,
                              inputs=layers, outputs=res))
    ddtree.maybe_enable_cpp_compact(False)
    return cases


def gen_attention(ddtree, trees):
    """Config-1 tree-verify attention through the reference's SDPA path (fp32, CPU)."""
    from transformers.integrations.sdpa_attention import sdpa_attention_forward
    case = next(c for c in trees if c["name"] == "cfg1_rank_gated_b16")
    n = 1 + len(case["tokens"])
    past = 512
    g = torch.Generator().manual_seed(0)
    q = torch.randn((1, 32, n, 128), generator=g)
    k = torch.randn((1, 8, past + n, 128), generator=g)
    v = torch.randn((1, 8, past + n, 128), generator=g)
    vis = torch.from_numpy(ddtree_visibility_from_bits(case["visibility_bits"], n))
    ids_buf = torch.zeros((1, n), dtype=torch.long)
    pos_buf = torch.zeros((1, n), dtype=torch.long)
    mask_buf = torch.zeros((1, 1, n, past + n), dtype=torch.float32)
    vis_buf = torch.zeros((n, n), dtype=torch.bool)
    _, _, mask, _, _ = ddtree.compile_ddtree_tree(
        torch.tensor(1), past, torch.tensor(case["tokens"]), torch.tensor(case["depths"]), vis, past,
        torch.float32, torch.device("cpu"), ids_buf, pos_buf, mask_buf, vis_buf, 0, 0)

    class _Attn(torch.nn.Module):
        num_key_value_groups = 4
        is_causal = True

    out, _ = sdpa_attention_forward(_Attn(), q, k, v, mask, dropout=0.0, scaling=128 ** -0.5)
    return dict(tree=case["name"], past=past, n=n, out=out.numpy().astype(np.float32))


def gen_recovery(retree, recovery, trees):
    """Target-gated sibling recovery walks (retree.py:57-190) on small-vocab trees."""
    rng = np.random.default_rng(21)
    cases = []
    for case in trees:
        if not case["name"].startswith("small_vocab") or case["budget"] < 16:
            continue
        n = 1 + len(case["tokens"])
        maps = [{int(t): c for t, c in m.items()} for m in case["child_maps"]]
        vocab = case["logits"]["vocab"]
        for trial in range(2):
            logits = rng.standard_normal((n, vocab)).astype(np.float32) * 2.0
            post = logits.argmax(-1)
            # bias some steps towards children so exact accepts and rescues both occur
            path = synthetic.accepted_path(int(rng.integers(1 << 30)), case["parents"])
            stop_bias = int(rng.integers(0, len(path)))
            for a, b in list(zip(path[:-1], path[1:]))[:stop_bias]:
                logits[a, case["tokens"][b - 1]] += 8.0
            post = logits.argmax(-1)
            mem = recovery.RecoveryMemory(freq_threshold=int(rng.integers(1, 4)))
            prior = []
            tree_toks = np.asarray(case["tokens"])
            for _ in range(int(rng.integers(40, 120))):
                # mostly (tree token, target argmax) pairs, so that rescues happen
                if rng.random() < 0.7:
                    d, t = int(rng.choice(tree_toks)), int(rng.choice(post))
                else:
                    d, t = int(rng.integers(vocab)), int(rng.integers(vocab))
                c = int(rng.integers(1, 4))
                mem.record_prior(d, t, count=c)
                prior.append((d, t, c))
            # seed the prior with the pairs met at the exact walk's stopping point
            # (the children the target ranks highest), so that rescues happen
            cur, nxt0 = 0, int(post[0])
            while nxt0 in maps[cur]:
                cur = maps[cur][nxt0]
                nxt0 = int(post[cur])
            kids = list(maps[cur].keys())
            kids.sort(key=lambda tk: -float(logits[cur, tk]))
            for tk in kids[:3]:
                if rng.random() < 0.7:
                    c = int(rng.integers(1, 5))
                    mem.record_prior(tk, nxt0, count=c)
                    prior.append((tk, nxt0, c))
            stop = sorted({int(x) for x in rng.choice(vocab, size=2, replace=False)}) if trial else None
            acc, nxt, rescued = retree.follow_verified_tree_with_recovery(
                maps, torch.from_numpy(post)[None], torch.from_numpy(logits)[None], mem,
                gate_threshold=float([0.01, 0.2][trial]), online_update=True,
                record_top_k=int([8, 2][trial]), rescue_top_k=int([8, 3][trial]),
                disallow_rescue_target_ids=None if stop is None else set(stop))
            cases.append(dict(
                tree=case["name"], logits=logits, freq_threshold=mem.freq_threshold, prior=prior,
                gate_threshold=[0.01, 0.2][trial], record_top_k=[8, 2][trial],
                rescue_top_k=[8, 3][trial], stop=stop, accepted=acc, next=int(nxt),
                rescued=int(rescued),
                online=sorted([d, t, c] for (d, t), c in mem.online_counts().items())))
    return cases


def gen_bonus(ddtree):
    """Raw continuity bonus values (ddtree.py:113-186) as exact binary64 hex."""
    out = []
    rng = np.random.default_rng(31)
    for seed, length, alphabet, max_n, min_count, use_log, lw, cap in [
        (1, 600, 12, 4, 1, True, 1.5, 6.0), (2, 2048, 30, 4, 1, True, 1.5, 6.0),
        (3, 300, 8, 6, 2, True, 2.0, 0.0), (4, 300, 8, 3, 1, False, 1.5, 2.5),
    ]:
        ctx = synthetic.context_ids(seed, length, alphabet, alphabet).tolist()
        table = ddtree._build_ngram_next_table(ctx, max_n, 2048)
        for _ in range(40):
            tl = int(rng.integers(0, max_n))
            start = int(rng.integers(0, length - tl)) if tl else 0
            tail = tuple(ctx[start:start + tl]) if rng.random() < 0.8 else tuple(
                int(x) for x in rng.integers(0, alphabet, size=tl))
            tok = int(rng.integers(0, alphabet))
            b = ddtree._ngram_bonus_for_token(tail, tok, table, max_n, min_count, use_log, lw, cap)
            out.append(dict(ctx=dict(seed=seed, length=length, alphabet=alphabet), max_n=max_n,
                            min_count=min_count, use_log=use_log, longer_weight=lw, cap=cap,
                            tail=list(tail), token=tok, bonus_hex=float(b).hex()))
    return out


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", default=os.environ.get("RETREE_REFERENCE"),
                    help="checkout of the reference repository (or set RETREE_REFERENCE)")
    args = ap.parse_args()
    if not args.reference:
        ap.error("--reference (or RETREE_REFERENCE) must name the reference checkout")
    ddtree, retree, recovery = _import_reference(args.reference)
    torch.set_num_threads(max(1, os.cpu_count() or 1))

    trees = gen_trees(ddtree)
    meta = dict(
        reference_files={f: hashlib.sha256((Path(args.reference) / f).read_bytes()).hexdigest()
                         for f in ("ddtree.py", "retree.py", "model/recovery.py")},
        torch=torch.__version__, numpy=np.__version__,
    )
    import transformers
    meta["transformers"] = transformers.__version__
    (HERE / "trees.json").write_text(json.dumps(dict(meta=meta, cases=trees)))
    (HERE / "compile.json").write_text(json.dumps(gen_compile(ddtree, trees)))
    (HERE / "follow.json").write_text(json.dumps(gen_follow(ddtree, trees)))
    (HERE / "bonus.json").write_text(json.dumps(gen_bonus(ddtree)))

    topk = gen_topk()
    np.savez_compressed(HERE / "topk.npz", **{f"{n}__{k}": v for n, d in topk.items()
                                              for k, v in d.items() if isinstance(v, np.ndarray)})
    (HERE / "topk.json").write_text(json.dumps({n: dict(spec=d["spec"], k=d["k"], ties=d["ties"])
                                                for n, d in topk.items()}))

    compact = gen_compact(ddtree)
    arrays = {}
    meta_c = []
    for i, c in enumerate(compact):
        for li, (k, v) in enumerate(c["inputs"]):
            arrays[f"c{i}_in{li}_k"], arrays[f"c{i}_in{li}_v"] = k, v
        for li, (k, v) in enumerate(c["outputs"]):
            arrays[f"c{i}_out{li}_k"], arrays[f"c{i}_out{li}_v"] = k, v
        meta_c.append(dict(past=c["past"], cur=c["cur"], keep=c["keep"], cpp=c["cpp"],
                           layers=len(c["inputs"])))
    np.savez_compressed(HERE / "compact.npz", **arrays)
    (HERE / "compact.json").write_text(json.dumps(meta_c))

    att = gen_attention(ddtree, trees)
    np.savez_compressed(HERE / "attention_cfg1.npz", out=att["out"])
    (HERE / "attention_cfg1.json").write_text(json.dumps(dict(tree=att["tree"], past=att["past"], n=att["n"])))

    rec = gen_recovery(retree, recovery, trees)
    np.savez_compressed(HERE / "recovery.npz", **{f"r{i}_logits": c.pop("logits") for i, c in enumerate(rec)})
    (HERE / "recovery.json").write_text(json.dumps(rec))
    print(f"wrote {len(trees)} tree cases, {len(compact)} compaction cases, {len(rec)} recovery cases")


if __name__ == "__main__":
    main()
