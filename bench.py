#!/usr/bin/env python
"""Verify-round throughput of the B200 tree-verification path.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

One step = one ReTree/DDTree verify round on every rank: draft top-k and
rank-gated n-gram tree build from that round's draft logits, the target
forward over the 1+budget tree nodes with tree-verify attention and in-place
cache append, argmax posterior, exact walk + commit, and KV compaction.
The draft model forward is not part of the round (the reference times it as a
separate stage); seeded synthetic draft logits (N(0,1) + Zipf boost, bf16 as
an lm_head emits them) stand in for it.  Default workload: random-init
Qwen3-4B (bf16, 36 layers), 2048-token uniform random prompt, draft block 16,
tree budget 16.  With N>1 ranks (torchrun) every rank verifies its own
request (data parallel, as the reference's benchmark shards requests) and the
ranks all-gather a fixed-shape recovery-memory delta after every step.

Prints ONE JSON line (rank 0).  ``value`` = verify rounds/s over all ranks with
inputs resident on the device; ``e2e`` = the same through the public API with
the draft logits copied from pinned host memory and the committed tokens read
back every round; ``roofline`` = the tree-verify attention kernel measured
live on the timed rounds; ``cpu_baseline`` = the reference's round on the host
cores (a bounded sample).  ``--impl reference`` times that CPU round alone.
"""

from __future__ import annotations

import argparse
import datetime
import json
import os
import statistics
import subprocess
import sys
import tempfile
import time

import numpy as np
import torch

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

WORKLOADS = {
    # name: model geometry, prompt length, tree budget, draft block
    "qwen3-4b-b16": dict(model="qwen3-4b", prompt=2048, budget=16, block=16),
    "qwen3-4b-b64": dict(model="qwen3-4b", prompt=2048, budget=64, block=16),
    # one request per GPU, request r's prompt length the r-th draw of U[1024, 8192] (seed 0)
    "qwen3-8b-b64": dict(model="qwen3-8b", prompt=(1024, 8192), budget=64, block=16),
    # one long request split by KV head over the ranks (random N(0,1) KV prefix, no prompt forward)
    "qwen3-8b-l32k-b256-split": dict(model="qwen3-8b", prompt=32768, budget=256, block=16, split=True),
}
DELTA_PAIRS = 4096  # recovery-memory delta exchanged per step at N>1 (int32 draft, target, count)
RECOVERY_PRIOR_PAIRS = 100_000  # --recovery: size of the seeded recovery-memory prior


def prompt_len(wl: dict, req: int) -> int:
    """Prompt length of request ``req``: fixed, or the req-th seeded draw of a uniform range."""
    p = wl["prompt"]
    if isinstance(p, int):
        return p
    lo, hi = p
    return int(np.random.default_rng(0).integers(lo, hi + 1, size=max(8, req + 1))[req])


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=24)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=("ours", "reference"), default="ours")
    ap.add_argument("--workload", choices=sorted(WORKLOADS), default="qwen3-4b-b16")
    ap.add_argument("--strategy", default="rank_gated_ngram")
    ap.add_argument("--cpu-sample-rounds", type=int, default=24,
                    help="rounds of the reference path on the host cores for cpu_baseline (N=1 only; ~10 s)")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--eager", action="store_true", help="launch every kernel from Python instead of graph replays")
    ap.add_argument("--gemm", choices=("auto", "tcgen05", "cublas"), default="auto",
                    help="projections of the fused verify forward")
    ap.add_argument("--hf-forward", action="store_true",
                    help="run the verify forward through the transformers modules instead of the fused stages")
    ap.add_argument("--fused-argmax", action="store_true",
                    help="the lm_head projection also returns the posterior (rt_linear_argmax), no argmax pass")
    ap.add_argument("--recovery", action="store_true",
                    help="walk with ReTree's target-gated sibling recovery on the device (rt_recovery_walk) over a "
                         "seeded recovery memory, instead of the exact walk")
    ap.add_argument("--dp-exchange", choices=("nccl", "p2p"), default="nccl",
                    help="request DP at N>1: the per-step recovery-delta all-gather over NCCL or over peer memory")
    ap.add_argument("--pdl", choices=("auto", "off"), default="auto",
                    help="programmatic dependent launch at N=1 (auto: on); always off at N>1, where NCCL runs "
                         "beside the kernels")
    ap.add_argument("--exchange", choices=("nccl", "p2p", "p2p_fused"), default="nccl",
                    help="split workloads: attention-output all-gather over NCCL or over peer memory")
    return ap.parse_args()


def draft_logits_np(seed: int, block: int, vocab: int) -> np.ndarray:
    from retree_b200 import synthetic
    return synthetic.draft_logits(seed, block, vocab)[-(block - 1):]


def measured_peaks():
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(path):
        with open(path) as f:
            d = json.load(f)
        return float(d["hbm_gbs"]), float(d["bf16_tflops"]), "measured"
    return 6650.0, 1590.0, "fallback"


# DRAM bytes (dram__bytes_read.sum + dram__bytes_write.sum) of one tree-attention launch, from an ncu capture
# of the current kernel at the workload's live shape: workload -> (bytes, prefix_len, tree_nodes, how taken).
# Scaled to the live prefix by the K/V bytes per key when the bench's prefix differs.
ATTN_TRAFFIC = {
    "qwen3-4b-b16": (8776704, 2075, 17, "ncu dram__bytes_read.sum + dram__bytes_write.sum of one tree_attn_tc_kernel "
                     "launch, cold L2 (bench_kernels.py single --budget 16 --prefix 2075)"),
}


def attn_traffic(workload: str, prefix_len: int, n_tree: int, hkv: int):
    """The ncu-measured DRAM traffic of one attention launch at this workload, or None when not captured."""
    rec = ATTN_TRAFFIC.get(workload)
    if rec is None or rec[2] != n_tree:
        return None
    byts, L, n, how = rec
    per_key = 2 * hkv * 128 * 2
    scaled = byts + (prefix_len - L) * per_key
    return {"bytes": scaled, "source": f"{how}; captured at prefix {L}, scaled to {prefix_len} at {per_key} B per key"
            if prefix_len != L else how}


CLOCK_QUERY = ("timestamp,index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
               "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
               "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")
REASONS = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]


def summarize_clocks(lines: list[str], t0: float, t1: float, interval_s: float) -> dict:
    """Median SM clock and active throttle reasons of the samples taken during [t0, t1].

    ``lines`` are nvidia-smi CSV rows of CLOCK_QUERY (timestamp first, local
    time); a sample within one interval of the region counts as taken during
    it.  With none there, the sample nearest the region stands in
    (``samples_in_region`` 0).
    """
    rows = []
    for line in lines:
        r = [x.strip() for x in line.split(",")]
        if len(r) < 10:
            continue
        try:
            sm, sm_max = float(r[2]), float(r[3])
        except ValueError:
            continue
        try:
            ts = datetime.datetime.strptime(r[0], "%Y/%m/%d %H:%M:%S.%f").timestamp()
        except ValueError:
            ts = None
        rows.append((ts, sm, sm_max, r[6:10]))
    if not rows:
        return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["no samples"], "samples": 0}
    timed_rows = [x for x in rows if x[0] is not None]
    if not timed_rows:  # unreadable timestamps: every sample counts, as before the region was marked
        inside, use = [], rows
    else:
        inside = [x for x in timed_rows if t0 - interval_s <= x[0] <= t1 + interval_s]
        use = inside or [min(timed_rows, key=lambda x: min(abs(x[0] - t0), abs(x[0] - t1)))]
    reasons = sorted({REASONS[i] for x in use for i in range(4) if x[3][i] == "Active"})
    return {"sm_mhz": statistics.median(x[1] for x in use), "sm_max_mhz": use[0][2], "reasons": reasons,
            "samples": len(rows), "samples_in_region": len(inside)}


class ClockSampler:
    """nvidia-smi clocks and throttle reasons, sampled every ``interval_ms`` from before the timed
    region (so that sampling is running when it starts) and summarised over the region."""

    def __init__(self, index: int, interval_ms: int = 20):
        vis = os.environ.get("CUDA_VISIBLE_DEVICES")
        if vis:
            ids = [x.strip() for x in vis.split(",") if x.strip()]
            if index < len(ids) and ids[index].isdigit():
                index = int(ids[index])
        self.interval_s = interval_ms / 1000.0
        self.t0 = self.t1 = None
        self.f = tempfile.NamedTemporaryFile("w+", suffix=".csv", delete=False)
        try:
            self.p = subprocess.Popen(["nvidia-smi", f"--id={index}", f"--query-gpu={CLOCK_QUERY}",
                                       "--format=csv,noheader,nounits", "-lms", str(interval_ms)],
                                      stdout=self.f, stderr=subprocess.DEVNULL)
        except FileNotFoundError:
            self.p = None

    def mark_start(self) -> None:
        self.t0 = time.time()

    def mark_end(self) -> None:
        self.t1 = time.time()

    def stop(self) -> dict:
        if self.p is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        time.sleep(2 * self.interval_s)  # a sample after the region's end
        self.p.terminate()
        self.p.wait()
        self.f.seek(0)
        lines = self.f.read().strip().splitlines()
        os.unlink(self.f.name)
        t1 = self.t1 if self.t1 is not None else time.time()
        t0 = self.t0 if self.t0 is not None else t1
        return summarize_clocks(lines, t0, t1, self.interval_s)


def cpu_round_sample(cfg, wl, rounds: int, strategy: str):
    """The reference's verify round on the host cores; returns (rounds/s, seconds, cores)."""
    from oracle.tree import NgramParams
    from oracle.verify_round import CpuVerifyRound

    cores = os.cpu_count() or 1
    torch.set_num_threads(cores)
    r = CpuVerifyRound(cfg, prompt_len(wl, 0), wl["budget"], strategy=strategy, params=NgramParams())
    drafts = [draft_logits_np(1000 + i, wl["block"], cfg.vocab_size) for i in range(rounds + 1)]
    r.round(drafts[0])  # warm-up
    t0 = time.perf_counter()
    for i in range(rounds):
        r.round(drafts[i + 1])
    dt = time.perf_counter() - t0
    return rounds / dt, dt, cores


def run_reference(args, wl, rank, world):
    if rank != 0:
        return
    from retree_b200.target import qwen3_config
    cfg = qwen3_config(wl["model"])
    from oracle.tree import NgramParams
    from oracle.verify_round import CpuVerifyRound

    cores = os.cpu_count() or 1
    torch.set_num_threads(cores)
    r = CpuVerifyRound(cfg, prompt_len(wl, 0), wl["budget"], strategy=args.strategy, params=NgramParams())
    drafts = [draft_logits_np(1000 + i, wl["block"], cfg.vocab_size) for i in range(args.warmup + args.steps)]
    for i in range(args.warmup):
        r.round(drafts[i])
    t0 = time.perf_counter()
    for i in range(args.steps):
        r.round(drafts[args.warmup + i])
    dt = time.perf_counter() - t0
    value = args.steps / dt
    sample = (f"{args.steps} verify rounds of the reference path on the host CPU (oracle restatement: tree build, "
              f"dense-mask compile, HF sdpa forward bf16, walk, index_select compaction) over a random-KV prefix of "
              f"{prompt_len(wl, 0)} tokens")
    print(json.dumps({
        "impl": "reference", "metric": "verify rounds/sec", "value": value, "unit": "rounds/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": 1000 * dt / args.steps, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
        "config": {"workload": args.workload, "model": wl["model"], "prompt": prompt_len(wl, 0), "budget": wl["budget"],
                   "draft_block": wl["block"], "strategy": args.strategy, "parallelism": "host CPU, rank 0 only"},
        "cpu_baseline": {"value": value, "unit": "rounds/s", "cores": cores, "kind": "port", "sample": sample},
        "e2e": {"value": value, "unit": "rounds/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }), flush=True)


def attn_bytes(L: int, n: int, hq: int, hkv: int, hd: int = 128) -> int:
    """Algorithmic HBM bytes of one tree-attention launch: K+V prefix and tree rows, q in, out, mask."""
    return (L + n) * 2 * hkv * hd * 2 + 2 * n * hq * hd * 2 + n * ((n + 31) // 32) * 4


def log(rank: int, msg: str) -> None:
    """Per-rank progress on stderr (the JSON line stays alone on stdout)."""
    print(f"[bench r{rank} {time.strftime('%H:%M:%S')}] {msg}", file=sys.stderr, flush=True)


def run_ours(args, wl, rank, world, local_rank):
    import torch.distributed as dist

    from retree_b200 import kernels
    from retree_b200.target import build_target, qwen3_config
    from retree_b200.verify import TreeVerifier

    os.environ["DDTREE_TREE_STRATEGY"] = args.strategy
    dev = torch.device("cuda", local_rank)
    torch.cuda.set_device(dev)
    cfg = qwen3_config(wl["model"])
    split = bool(wl.get("split")) and world > 1
    if split:
        from retree_b200 import headsplit
        headsplit.register()
        target = build_target(cfg, device=dev, seed=0, attn_implementation=headsplit.NAME)
        headsplit.shard_attention_heads(target, rank, world)
    else:
        target = build_target(cfg, device=dev, seed=0)
    log(rank, "target built")
    steps, warm = args.steps, args.warmup
    total_rounds = warm + steps
    req = 0 if wl.get("split") else rank  # a split request is the same request on every rank
    plen = prompt_len(wl, req)
    max_len = plen + total_rounds * (wl["block"] + 2) + 64
    # draft logits for every round: bf16 as the lm_head emits them; pinned host copies for the e2e leg
    host = [torch.from_numpy(draft_logits_np(1000 + 7919 * req + i, wl["block"], cfg.vocab_size)).to(torch.bfloat16)
            for i in range(total_rounds)]
    pinned = [h.pin_memory() for h in host]
    resident = [h.to(dev) for h in host]
    prompt = torch.from_numpy(np.random.default_rng(req).integers(0, cfg.vocab_size, size=plen))[None]

    def fresh():
        v = TreeVerifier(target, tree_budget=wl["budget"], max_length=max_len, draft_horizon=wl["block"] - 1,
                         fused=not args.hf_forward, gemm=args.gemm, exchange=args.exchange,
                         fused_argmax=args.fused_argmax)
        if wl.get("split"):
            v.prefill_random(plen, seed=req)
        else:
            v.prefill(prompt.to(dev))
        if args.recovery:
            from retree_b200.recovery import RecoveryMemory
            from retree_b200.recovery_device import DeviceRecoveryMemory
            # seeded prior: RECOVERY_PRIOR_PAIRS (draft, target) pairs with counts 1..10; a log large
            # enough for every round of the run between syncs
            mem = RecoveryMemory(freq_threshold=6)
            rng = np.random.default_rng(4242 + req)
            pairs = rng.integers(0, cfg.vocab_size, size=(RECOVERY_PRIOR_PAIRS, 2))
            counts = rng.integers(1, 11, size=RECOVERY_PRIOR_PAIRS)
            for (d, t), c in zip(pairs.tolist(), counts.tolist()):
                mem.record_prior(d, t, c)
            v.enable_recovery(DeviceRecoveryMemory(mem, dev, capacity=1 << 21, log_capacity=1 << 20),
                              gate_threshold=0.01,
                              rescue_top_k=8, record_top_k=8, online_update=True)
        return v

    # the step's recovery-memory delta: seeded random (draft, target) pairs and counts
    g = torch.Generator(device=dev).manual_seed(1234 + rank)
    delta_send = torch.stack([torch.randint(0, cfg.vocab_size, (DELTA_PAIRS,), device=dev, generator=g),
                              torch.randint(0, cfg.vocab_size, (DELTA_PAIRS,), device=dev, generator=g),
                              torch.randint(1, 5, (DELTA_PAIRS,), device=dev, generator=g)], dim=1).to(torch.int32)
    delta_recv = torch.zeros((world, DELTA_PAIRS, 3), dtype=torch.int32, device=dev) if world > 1 else None
    delta_peer = None
    if world > 1 and not wl.get("split") and args.dp_exchange == "p2p":
        from retree_b200.peer import PeerExchange
        # one row of DELTA_PAIRS * 3 int32 per rank, carried as bf16 columns; two slots by step parity
        delta_peer = PeerExchange(None, rank, world, 1, DELTA_PAIRS * 3 * 2, 2, dev)
    n_exchanges = [0]
    pending = [None]

    def exchange():
        if world <= 1 or wl.get("split"):
            return
        if delta_peer is None:
            # issued on NCCL's stream without a wait, so it overlaps the next round's
            # replay; the previous step's gather is waited for before its buffer is reused
            settle()
            pending[0] = dist.all_gather_into_tensor(delta_recv.view(world * DELTA_PAIRS, 3), delta_send,
                                                     async_op=True)
            return
        slot = n_exchanges[0] % 2
        if slot == 0:
            delta_peer.step()
        delta_peer.slot(slot, 1).view(torch.int32).copy_(delta_send.view(1, -1))
        delta_peer.signal(slot)
        delta_peer.gather(slot, 1, delta_recv.view(1, -1).view(torch.bfloat16))
        n_exchanges[0] += 1

    def settle():
        # the current stream waits for the last step's delta gather
        if pending[0] is not None:
            pending[0].wait()
            pending[0] = None

    def barrier():
        settle()
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()

    def timed(fn):
        barrier()
        t0 = time.perf_counter()
        fn()
        barrier()
        dt = torch.tensor([time.perf_counter() - t0], dtype=torch.float64, device=dev)
        if world > 1:
            dist.all_reduce(dt, op=dist.ReduceOp.MAX)
        return float(dt.item())

    log(rank, "inputs ready")
    # ---- device-resident rounds (value): every round is one CUDA-graph replay ----
    v = fresh()
    v.enable_graph(not args.eager)
    sampler = ClockSampler(dev.index) if rank == 0 else None  # running before the timed region starts
    for i in range(warm):
        v.round(resident[i])
        exchange()
    log(rank, "warm-up rounds done")
    kernels.LAUNCHES = 0
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    accepted = []

    def rounds_resident():
        torch.cuda.nvtx.range_push("timed_rounds")
        ev0.record()
        for i in range(steps):
            accepted.append(v.round(resident[warm + i]))
            exchange()
        settle()
        ev1.record()
        torch.cuda.nvtx.range_pop()

    if sampler:
        sampler.mark_start()
    wall = timed(rounds_resident)
    if sampler:
        sampler.mark_end()
    clocks = sampler.stop() if sampler else None
    launches = kernels.LAUNCHES
    torch.cuda.synchronize()
    dev_ms = torch.tensor([ev0.elapsed_time(ev1)], dtype=torch.float64, device=dev)
    if world > 1:
        dist.all_reduce(dev_ms, op=dist.ReduceOp.MAX)
    dev_s = float(dev_ms.item()) / 1000.0

    log(rank, "timed rounds done")
    projections = None if v.fused is None else {
        kd: ("rt_linear" if use else "cublas") for kd, use in v.fused.use_rt.items()}
    # ---- the tree-attention kernel on the live cache: all layers back to back, as in the round ----
    n_tree = 1 + wl["budget"]
    L_live = v.start
    cap = v.cache.capacity
    hq, hkv = cfg.num_attention_heads, cfg.num_key_value_heads
    if split:  # each rank attends over its own heads only
        hq, hkv = hq // world, hkv // world
    q_probe = torch.randn((1, hq, n_tree, 128), device=dev, dtype=torch.bfloat16)
    bits = v.tree["mask"][:n_tree].clone()
    live_len_dev = torch.tensor([L_live], dtype=torch.int64, device=dev)
    splits = kernels.default_splits(n_tree, hq, hkv, cap - n_tree)
    out_probe = torch.empty((n_tree, hq, 128), device=dev, dtype=torch.bfloat16)

    def attn_all_layers():
        for li in range(cfg.num_hidden_layers):
            kernels.tree_attention(q_probe, v.cache.slab[2 * li], v.cache.slab[2 * li + 1], bits, cap - n_tree,
                                   out=out_probe, prefix_len_dev=live_len_dev, kv_capacity=cap, num_splits=splits)

    attn_all_layers()
    side = torch.cuda.Stream(dev)
    side.wait_stream(torch.cuda.current_stream(dev))
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=side, capture_error_mode="thread_local"):
        attn_all_layers()
    for _ in range(3):
        g.replay()
    a0, a1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    reps = 20
    a0.record()
    for _ in range(reps):
        g.replay()
    a1.record()
    torch.cuda.synchronize()
    attn_us = 1000.0 * a0.elapsed_time(a1) / (reps * cfg.num_hidden_layers)
    byts = attn_bytes(L_live, n_tree, hq, hkv)
    del g

    log(rank, "attention probe done")
    # ---- end to end through the public API: host draft logits in, committed tokens out ----
    v2 = fresh()
    v2.enable_graph(not args.eager)
    out_host = torch.empty(wl["budget"] + 2, dtype=torch.int64).pin_memory()
    for i in range(warm):
        v2.round(pinned[i].to(dev, non_blocking=True))
        exchange()

    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)

    def rounds_e2e():
        e0.record()
        for i in range(steps):
            logits = pinned[warm + i].to(dev, non_blocking=True)
            s0 = v2.start
            acc = v2.round(logits)
            out_host[: acc + 1].copy_(v2.output_ids[s0: s0 + acc + 1])
            exchange()
        settle()
        e1.record()

    timed(rounds_e2e)
    log(rank, "e2e rounds done")
    e2e_ms = torch.tensor([e0.elapsed_time(e1)], dtype=torch.float64, device=dev)
    if world > 1:
        dist.all_reduce(e2e_ms, op=dist.ReduceOp.MAX)
    e2e_s = float(e2e_ms.item()) / 1000.0
    h2d = host[0].numel() * host[0].element_size()
    d2h = 8 * (wl["budget"] + 2) + 4  # committed tokens + accepted count

    # graphs that captured NCCL calls are released before the process group goes away
    v.graph = None
    v2.graph = None
    torch.cuda.synchronize()
    for vv in (v, v2):  # peer-memory exchanges unmap on every rank together
        if vv.fused is not None and vv.fused.peer is not None:
            vv.fused.peer.close()
    if delta_peer is not None:
        delta_peer.close()
    if rank != 0:
        return
    traffic = attn_traffic(args.workload, L_live, n_tree, hkv)
    cpu = None  # the host-core sample runs at N=1 only
    if not args.no_cpu_baseline and world == 1:
        del v, v2
        torch.cuda.empty_cache()
        rps, secs, cores = cpu_round_sample(cfg, wl, args.cpu_sample_rounds, args.strategy)
        cpu = {"value": rps, "unit": "rounds/s", "cores": cores, "kind": "port",
               "sample": (f"{args.cpu_sample_rounds} verify rounds ({secs:.1f} s) of the reference path on the host "
                          f"CPU: oracle tree build, dense-mask compile, HF sdpa forward (bf16), walk, compaction, "
                          f"random-KV prefix of {prompt_len(wl, 0)} tokens")}
    reqs = 1 if wl.get("split") else world  # a split request is one request over all ranks
    print(result_line(args, wl, world=world, reqs=reqs, steps=steps, warm=warm, dev_s=dev_s, e2e_s=e2e_s,
                      wall=wall, prompt=plen, projections=projections, pdl=kernels.pdl_enabled(),
                      accepted=accepted, attn_us=attn_us, byts=byts, prefix_len=L_live, n_tree=n_tree,
                      splits=splits, layers=cfg.num_hidden_layers, traffic=traffic, cpu=cpu, h2d=h2d, d2h=d2h,
                      launches=launches, clocks=clocks), flush=True)


def plain(x):
    """``x`` with tensors and numpy values turned into Python numbers and lists (JSON-serialisable)."""
    if isinstance(x, torch.Tensor):
        x = x.detach().cpu()
        return x.item() if x.numel() == 1 else x.tolist()
    if isinstance(x, np.ndarray):
        return x.tolist()
    if isinstance(x, np.generic):
        return x.item()
    if isinstance(x, dict):
        return {str(k): plain(v) for k, v in x.items()}
    if isinstance(x, (list, tuple)):
        return [plain(v) for v in x]
    return x


def result_line(args, wl, *, world, reqs, steps, warm, dev_s, e2e_s, wall, prompt, projections, pdl, accepted,
                attn_us, byts, prefix_len, n_tree, splits, layers, traffic, cpu, h2d, d2h, launches, clocks) -> str:
    """The bench's JSON line from the measured quantities (any of which may be a 1-element tensor)."""
    dev_s, e2e_s, attn_us, byts = (float(plain(x)) for x in (dev_s, e2e_s, attn_us, byts))
    hbm_peak, _, peak_kind = measured_peaks()
    achieved = byts / (attn_us * 1e-6) / 1e9
    split_exchange = dict(nccl="NCCL", p2p="peer memory", p2p_fused="peer memory, pulled by o_proj")[args.exchange]
    dp_exchange = "peer memory" if args.dp_exchange == "p2p" else "NCCL"
    accepted = [plain(a) for a in accepted]
    line = {
        "metric": "verify rounds/sec", "value": reqs * steps / dev_s, "unit": "rounds/s", "n_gpus": world,
        "steps": steps, "warmup": warm, "ms_per_step": 1000.0 * dev_s / steps, "higher_is_better": True,
        "scaling": "strong" if wl.get("split") else "weak",
        "vs_baseline": None, "dtype": "bf16", "data": "synthetic (seeded draft logits, uniform prompt, random-init "
                                                      "weights)",
        "config": {"workload": args.workload, "model": wl["model"] + " (random init)", "prompt": prompt,
                   "prompt_lengths": [prompt_len(wl, 0 if wl.get("split") else r) for r in range(world)],
                   "budget": wl["budget"], "draft_block": wl["block"], "strategy": args.strategy,
                   "verify_forward": "transformers modules" if args.hf_forward else f"fused stages ({args.gemm})",
                   "projections": projections,
                   "walk": "target-gated sibling recovery (device)" if args.recovery else "exact",
                   "posterior": "argmax fused into the lm_head projection" if args.fused_argmax else "torch.argmax",
                   "parallelism": (f"kv-head split over {world} GPUs (attention-output all-gather per layer, "
                                   f"{split_exchange})" if wl.get("split") else
                                   f"dp{world} (one request per GPU)" + (
                                       f", recovery-delta all-gather per step ({dp_exchange})" if world > 1 else "")),
                   "pdl": pdl,
                   "l2": "inputs > L2 (8 GB of weights and the KV cache stream every round)",
                   "mean_accepted": sum(accepted) / max(1, len(accepted)), "wall_s": wall},
        "roofline": {"kernel": "tree_attn (rt_tree_attn)", "bound": "hbm", "achieved": achieved,
                     "peak": hbm_peak, "unit": "GB/s", "frac": achieved / hbm_peak,
                     "traffic": None if traffic is None else traffic["bytes"],
                     "traffic_source": None if traffic is None else traffic["source"],
                     "peak_kind": peak_kind, "avg_launch_us": attn_us, "algorithmic_bytes_per_launch": byts,
                     "prefix_len": prefix_len, "tree_nodes": n_tree, "key_splits": splits,
                     "share_of_round": layers * attn_us * 1e-3 / (1000.0 * dev_s / steps)},
        "cpu_baseline": cpu,
        "e2e": {"value": reqs * steps / e2e_s, "unit": "rounds/s", "h2d_bytes_per_step": h2d,
                "d2h_bytes_per_step": d2h},
        "gpu_launches": launches,
        "clocks": clocks,
    }
    return json.dumps(plain(line))


def main():
    args = parse()
    wl = WORKLOADS[args.workload]
    rank = int(os.environ.get("RANK", 0))
    world = int(os.environ.get("WORLD_SIZE", 1))
    local_rank = int(os.environ.get("LOCAL_RANK", 0))
    if args.impl == "reference":
        run_reference(args, wl, rank, world)
        return
    if world > 1:
        import torch.distributed as dist
        # the per-step exchanges are tiny all-gathers: no NVLink multicast objects needed
        os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
        # no programmatic dependent launch in a process with NCCL collectives, from the first launch on
        os.environ["RETREE_B200_PDL"] = "0"

        torch.cuda.set_device(local_rank)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300),
                                device_id=torch.device("cuda", local_rank))
        from retree_b200 import kernels
        kernels.set_pdl(False)  # NCCL collectives run between the forward's kernels
        log(rank, "process group up")
    elif args.pdl == "off":
        from retree_b200 import kernels
        kernels.set_pdl(False)
    try:
        run_ours(args, wl, rank, world, local_rank)
    finally:
        if world > 1:
            import torch.distributed as dist
            dist.destroy_process_group()


if __name__ == "__main__":
    main()
