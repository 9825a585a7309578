"""Kernel-level measurements of the verification path (one JSON line per case).

    python bench_kernels.py sweep  [--prefix 4096] [--budgets 16,32,64,128,256] [--layers 36]
    python bench_kernels.py single --budget 16 --prefix 2048 [--reps 3]
    python bench_kernels.py topk --budget 16 [--reps 3]
    python bench_kernels.py parts
    python bench_kernels.py linear [--m 17,65,257] [--shapes qkv,o,gate_up,down,lm_head]

``sweep`` is the tree-verify attention budget sweep (Qwen3-4B head geometry:
32 query / 8 KV heads, head_dim 128, bf16): random trees from seeded parent
arrays (depth <= 16, Geometric(0.5) branching), K/V ~ N(0,1), one KV cache per
layer so consecutive launches stream from HBM (36 x (L+n) x 4 KiB > L2), all
layers captured in one CUDA graph and timed with CUDA events.  Each line
reports the algorithmic bytes and FLOPs per launch, the achieved GB/s and
TFLOP/s, and both as fractions of the measured peaks (MEASURED_PEAKS.json).
``single`` runs a few launches of one shape (for ncu captures), ``topk`` a
few draft top-k calls on the bench workload's logits (the same); ``parts``
times the draft top-k, the tree build and the compaction kernels; ``linear``
times rt_linear against cuBLAS on the Qwen3-4B projection shapes (36 weight
copies per graph, so every launch streams its weights from HBM).
"""

from __future__ import annotations

import argparse
import json
import os
import sys

import numpy as np
import torch

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

from retree_b200 import kernels, synthetic  # noqa: E402
HQ, HKV, HD = 32, 8, 128


def peaks():
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(path):
        d = json.load(open(path))
        return float(d["hbm_gbs"]), float(d["bf16_tflops"]), "measured"
    return 6650.0, 1590.0, "fallback"


def attn_bytes(L, n):
    return (L + n) * 2 * HKV * HD * 2 + 2 * n * HQ * HD * 2 + n * ((n + 31) // 32) * 4


def attn_flops(L, n):
    return 4 * HQ * HD * n * (L + n)


def tree_bits(seed: int, n: int, device) -> torch.Tensor:
    parents = synthetic.random_tree_parents(seed, n - 1, max_depth=16, p=0.5)
    n = len(parents)
    vis = np.zeros((n, n), dtype=np.bool_)
    vis[0, 0] = True
    for i in range(1, n):
        vis[i, :i] = vis[parents[i], :i]
        vis[i, i] = True
    w = (n + 31) // 32
    padded = np.zeros((n, w * 32), dtype=np.bool_)
    padded[:, :n] = vis
    return torch.from_numpy(np.packbits(padded, axis=1, bitorder="little").view("<u4").view(np.int32)).to(device)


def graph_time_us(fn, reps: int = 20) -> float:
    fn()
    torch.cuda.synchronize()
    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=side, capture_error_mode="thread_local"):
        fn()
    for _ in range(3):
        g.replay()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(reps):
        g.replay()
    e1.record()
    torch.cuda.synchronize()
    return 1000.0 * e0.elapsed_time(e1) / reps


def attention_case(n: int, L: int, layers: int, dev, seed: int = 0, splits: int = 0) -> dict:
    bits = tree_bits(seed + n, n, dev)
    g = torch.Generator(device=dev).manual_seed(seed)
    caches = [torch.randn((2, HKV, L + n, HD), device=dev, generator=g).to(torch.bfloat16) for _ in range(layers)]
    q = torch.randn((1, HQ, n, HD), device=dev, generator=g).to(torch.bfloat16)
    out = torch.empty((n, HQ, HD), device=dev, dtype=torch.bfloat16)
    sp = splits or kernels.default_splits(n, HQ, HKV, L)

    def run():
        for c in caches:
            kernels.tree_attention(q, c[0], c[1], bits, L, out=out, num_splits=sp)

    us = graph_time_us(run) / layers
    kernels.check_device_status(dev)
    hbm, tf, kind = peaks()
    b, f = attn_bytes(L, n), attn_flops(L, n)
    gbs, tfs = b / us / 1e3, f / us / 1e6
    return dict(kernel="tree_attn", budget=n - 1, nodes=n, prefix=L, layers=layers, splits=sp, us_per_launch=us,
                bytes_per_launch=b, flops_per_launch=f, gbs=gbs, tflops=tfs, hbm_frac=gbs / hbm,
                tensor_frac=tfs / tf, bound="hbm" if b / hbm > f / (tf * 1e3) else "tensor", peak_kind=kind,
                path="tcgen05" if n * (HQ // HKV) >= 64 else "warp")


def parts(dev) -> list[dict]:
    from retree_b200.ddtree import NgramParams
    out = []
    logits = torch.from_numpy(synthetic.draft_logits(0, 16, 151936)[-15:]).to(dev).to(torch.bfloat16)
    ctx = torch.from_numpy(synthetic.context_ids(0, 2049, 151936)).to(dev)
    for budget in (16, 64, 256):
        us = graph_time_us(lambda: kernels.draft_topk(logits, budget))
        out.append(dict(kernel="draft_topk", budget=budget, rows=15, vocab=151936, us=us,
                        gbs=15 * 151936 * 2 / us / 1e3))
        lp, ids, _ = kernels.draft_topk(logits, budget)
        # the heap strategy has no n-gram table and no bonus lookups: the difference
        # bounds what the per-round table rebuild and the lookups cost
        for strategy in ("rank_gated_ngram", "heap"):
            buf = {}
            tree = kernels.tree_build(lp, ids, budget, strategy, NgramParams.from_env({}), ctx=ctx, out=None)
            buf.update(tree)
            us = graph_time_us(lambda: kernels.tree_build(lp, ids, budget, strategy, NgramParams.from_env({}),
                                                          ctx=ctx, out=buf))
            out.append(dict(kernel="tree_build", strategy=strategy, budget=budget, context=2049, us=us))
    slab = torch.randn((72, 8, 4096 + 17, 128), device=dev).to(torch.bfloat16)
    keep = torch.tensor([0, 1, 3, 7, 9, 12, 15], dtype=torch.long, device=dev)
    us = graph_time_us(lambda: kernels.kv_compact(slab, 4096, keep))
    moved = 72 * 8 * len(keep) * 256 * 2
    out.append(dict(kernel="kv_compact", layers=36, kept=len(keep), us=us, bytes_moved=moved, gbs=moved / us / 1e3))
    return out


LINEAR_SHAPES = {  # Qwen3-4B projections (n_out, k, epilogue)
    "qkv": (6144, 2560, 0), "o": (2560, 4096, 0), "gate_up": (19456, 2560, 1), "down": (2560, 9728, 0),
    "lm_head": (151936, 2560, 0)}


def linear_case(name: str, m: int, layers: int, dev) -> list[dict]:
    """rt_linear vs cuBLAS (torch.mm) on one projection shape, ``layers`` weight copies per graph."""
    n_out, k, epi = LINEAR_SHAPES[name]
    copies = 1 if name == "lm_head" else layers
    g = torch.Generator(device=dev).manual_seed(0)
    ws = [(torch.randn((n_out, k), device=dev, generator=g) * 0.02).to(torch.bfloat16) for _ in range(copies)]
    x = torch.randn((m, k), device=dev, generator=g).to(torch.bfloat16)
    width = n_out // 2 if epi == 1 else n_out
    out = torch.empty((m, width), dtype=torch.bfloat16, device=dev)
    full = torch.empty((m, n_out), dtype=torch.bfloat16, device=dev)
    hbm, tf, kind = peaks()
    rows = []
    for impl in ("rt_linear", "cublas"):
        def run():
            for w in ws:
                if impl == "rt_linear":
                    kernels.linear(x, w, out=out, epilogue=epi)
                elif epi == 1:
                    torch.mm(x, w.t(), out=full)
                    kernels.silu_mul(full, out)
                else:
                    torch.mm(x, w.t(), out=out)
        us = graph_time_us(run, reps=10) / copies
        kernels.check_device_status(dev)
        b = n_out * k * 2 + m * k * 2 + m * width * 2
        rows.append(dict(kernel="linear", shape=name, impl=impl, m=m, n_out=n_out, k=k, us=us, bytes=b,
                         gbs=b / us / 1e3, hbm_frac=b / us / 1e3 / hbm, peak_kind=kind,
                         plan=kernels.linear_plan(m, n_out, k, epi) if impl == "rt_linear" else None))
    del ws
    torch.cuda.empty_cache()
    return rows


def draft_case(dev, hidden: int = 4096, layers: int = 5, ctx: int = 5, prefix: int = 2048, block: int = 16,
               vocab: int = 151936) -> list[dict]:
    """One DFlash draft call on the fused stages (``FusedDraft``): a decode-sized call (``ctx`` new
    context rows) and the first call of a request (the whole ``prefix`` as context rows).

    Synthetic draft of the Qwen3-8B geometry (``layers`` draft layers; the draft checkpoints' layer
    counts are not part of the reference), target embedding and lm_head of that vocabulary.
    """
    from torch import nn

    from retree_b200.draft import FusedDraft, random_draft

    ids = [1, 9, 17, 25, 33][:layers]
    draft = random_draft(hidden, layers, 32, 8, 3 * hidden, block, ids, dev)

    class _Target(nn.Module):
        pass

    tgt = _Target()
    tgt.config = type("Cfg", (), {"hidden_size": hidden})()
    tgt.model = nn.Module()
    tgt.model.embed_tokens = nn.Embedding(vocab, hidden, device=dev, dtype=torch.bfloat16).requires_grad_(False)
    tgt.lm_head = nn.Linear(hidden, vocab, bias=False, device=dev, dtype=torch.bfloat16).requires_grad_(False)
    fd = FusedDraft(draft, tgt, capacity=prefix + 4 * block)
    g = torch.Generator(device=dev).manual_seed(0)
    block_ids = torch.randint(0, vocab, (block,), device=dev, generator=g)
    w_layer = sum(p.numel() * 2 for L in fd.layers for p in (L.qkv_w, L.o_w, L.gate_up_w, L.down_w))
    rows = []
    for c, start in ((ctx, prefix), (prefix, prefix)):
        th = torch.randn((c, len(ids) * hidden), device=dev, generator=g).to(torch.bfloat16)

        def call():
            fd.length = start - c
            fd.forward(block_ids, th, start)

        us = graph_time_us(call, reps=10)
        kernels.check_device_status(dev)
        w = w_layer + fd.fc_w.numel() * 2 + fd.lm_head.numel() * 2
        rows.append(dict(kernel="draft_forward", context_rows=c, start=start, block=block, draft_layers=layers,
                         us_per_call=us, weight_bytes=w, gbs_weights=w / us / 1e3, hbm_frac=w / us / 1e3 / peaks()[0]))
    return rows


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("mode", choices=("sweep", "single", "topk", "parts", "linear", "draft"))
    ap.add_argument("--m", default="17,65,257")
    ap.add_argument("--shapes", default="qkv,o,gate_up,down,lm_head")
    ap.add_argument("--prefix", type=int, default=4096)
    ap.add_argument("--budgets", default="16,32,64,128,256")
    ap.add_argument("--budget", type=int, default=16)
    ap.add_argument("--layers", type=int, default=36)
    ap.add_argument("--reps", type=int, default=3)
    ap.add_argument("--splits", type=int, default=0)
    a = ap.parse_args()
    dev = torch.device("cuda:0")
    torch.cuda.set_device(dev)
    if a.mode == "sweep":
        for b in (int(x) for x in a.budgets.split(",")):
            print(json.dumps(attention_case(b + 1, a.prefix, a.layers, dev, splits=a.splits)), flush=True)
    elif a.mode == "single":
        n = a.budget + 1
        bits = tree_bits(n, n, dev)
        c = torch.randn((2, HKV, a.prefix + n, HD), device=dev).to(torch.bfloat16)
        q = torch.randn((1, HQ, n, HD), device=dev).to(torch.bfloat16)
        for _ in range(a.reps):
            kernels.tree_attention(q, c[0], c[1], bits, a.prefix, num_splits=a.splits)
        torch.cuda.synchronize()
        kernels.check_device_status(dev)
        print(json.dumps(dict(ok=True, budget=a.budget, prefix=a.prefix)))
    elif a.mode == "topk":
        # a few calls of the draft top-k on the bench workload's logits (for ncu captures)
        logits = torch.from_numpy(synthetic.draft_logits(0, 16, 151936)[-15:]).to(dev).to(torch.bfloat16)
        for _ in range(a.reps):
            kernels.draft_topk(logits, a.budget)
        torch.cuda.synchronize()
        print(json.dumps(dict(ok=True, budget=a.budget, rows=15, vocab=151936)))
    elif a.mode == "draft":
        for row in draft_case(dev, prefix=a.prefix):
            print(json.dumps(row), flush=True)
    elif a.mode == "linear":
        for m in (int(x) for x in a.m.split(",")):
            for name in a.shapes.split(","):
                for row in linear_case(name, m, a.layers, dev):
                    print(json.dumps(row), flush=True)
    else:
        for row in parts(dev):
            print(json.dumps(row), flush=True)


if __name__ == "__main__":
    main()
