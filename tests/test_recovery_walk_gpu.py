"""rt_recovery_walk (GPU) against the reference walk: the golden walks and the seeded random trees of
tests/test_recovery_native_cpu.py, fp32 and bf16 logits; accepted nodes, next token, rescues, online
counts and the increment log must match exactly."""

import numpy as np
import pytest
import torch

from retree_b200 import kernels
from retree_b200.recovery import RecoveryMemory
from retree_b200.recovery_device import DeviceRecoveryMemory
from tests import golden_cases as gc
from tests.gpu_util import cuda
from tests.test_recovery_native_cpu import _clone, _random_case, run_reference

pytestmark = [pytest.mark.gpu, pytest.mark.late]


def run_device(parents, tokens, logits, mem, gate, rescue_k, record_k, online, stop):
    dev = cuda()
    dm = DeviceRecoveryMemory(mem, dev, capacity=1 << 12, log_capacity=4096, stop_ids=stop)
    n = len(parents)
    par = torch.tensor(parents, dtype=torch.int32, device=dev)
    tok = torch.tensor(tokens if tokens else [0], dtype=torch.int64, device=dev)
    lg = logits.to(dev).contiguous()
    post = lg.argmax(-1)
    out = kernels.recovery_walk(par, tok, post, lg, dm.table,
                                dict(gate_threshold=gate, freq_threshold=mem.freq_threshold, rescue_top_k=rescue_k,
                                     record_top_k=record_k, online_update=online),
                                count=n - 1, stop_ids=dm.stop_ids, log=dm.log())
    kernels.check_device_status(dev)
    acc = out["accepted"][: int(out["accepted_len"].item())].tolist()
    logged = dm.sync()
    return acc, int(out["next_token"].item()), int(out["rescued"].item()), mem.online_counts(), logged


def test_golden_recovery_walks_on_device():
    trees = {c["name"]: c for c in gc.tree_cases()}
    arr = gc.load_npz("recovery.npz")
    for i, c in enumerate(gc.load_json("recovery.json")):
        t = trees[c["tree"]]
        logits = torch.from_numpy(arr[f"r{i}_logits"])
        mem = RecoveryMemory(c["freq_threshold"])
        for d, g, k in c["prior"]:
            mem.record_prior(d, g, k)
        stop = None if c["stop"] is None else set(c["stop"])
        acc, nxt, resc, online, _ = run_device(t["parents"], t["tokens"], logits, mem, c["gate_threshold"],
                                               c["rescue_top_k"], c["record_top_k"], True, stop)
        assert (acc, nxt, resc) == (c["accepted"], c["next"], c["rescued"]), i
        assert sorted([d, g, k] for (d, g), k in online.items()) == c["online"], i


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_random_recovery_walks_on_device(dtype):
    for seed in range(60):
        parents, tokens, lg, mem, gate, rk, ck, online, stop = _random_case(seed)
        logits = torch.from_numpy(lg).to(dtype)
        got = run_device(parents, tokens, logits, _clone(mem), gate, rk, ck, online, stop)
        want = run_reference(parents, tokens, logits, _clone(mem), gate, rk, ck, online, stop)
        assert got[:4] == want, seed


@torch.inference_mode()
def test_retree_generate_device_recovery_equals_host_walk(monkeypatch):
    """retree_generate with the recovery walk on the GPU commits what the host walk commits.

    Both runs verify with the same forward, so they see the same logits; the
    recovery memory starts from the same priors, and its online counts after
    the request must agree too.  ``freq_threshold`` 0 lets every candidate
    through the frequency test, so rescues are decided by the logit gate.
    """
    from retree_b200 import synthetic
    from retree_b200.retree import retree_generate
    from retree_b200.target import build_target, qwen3_config

    monkeypatch.setenv("DDTREE_TREE_STRATEGY", "rank_gated_ngram")
    dev = cuda()
    vocab = 2000
    cfg = qwen3_config("small", hidden_size=512, intermediate_size=1024, num_hidden_layers=2, num_attention_heads=8,
                       num_key_value_heads=2, vocab_size=vocab, tie_word_embeddings=False)
    model = build_target(cfg, device=dev, seed=21)
    prompt = torch.from_numpy(synthetic.context_ids(3, 64, vocab, alphabet=30))[None].to(dev)

    def draft_fn(output_ids, start, r):
        return torch.randn((15, vocab), device=dev, generator=torch.Generator(device=dev).manual_seed(100 + r))

    def memory():
        m = RecoveryMemory(freq_threshold=0)
        rng = np.random.default_rng(0)
        for _ in range(500):
            m.record_prior(int(rng.integers(vocab)), int(rng.integers(vocab)), int(rng.integers(1, 4)))
        return m

    runs = []
    for device_walk in (False, True):
        mem = memory()
        res = retree_generate(None, model, prompt, mask_token_id=vocab - 1, max_new_tokens=48, block_size=16,
                              stop_token_ids=[7], tree_budget=24, recovery_memory=mem, gate_threshold=0.01,
                              draft_fn=draft_fn, device_recovery=device_walk)
        kernels.check_device_status(dev)
        runs.append((res.output_ids[0].tolist(), res.acceptance_lengths, res.total_rescued, mem.online_counts()))
    assert runs[0][2] > 0, "no rescue happened: the case does not exercise the recovery walk"
    assert runs[1] == runs[0]
