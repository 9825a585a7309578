"""The recovery walk of csrc/recovery_walk.cuh (the code the GPU kernel runs), built for the host,
against the reference's walk and RecoveryMemory (retree.py:57-190, model/recovery.py:35-298):
the golden walks, and seeded random trees with repeated sibling tokens, stop sets, both logit
dtypes and the knobs' ranges.  Accepted nodes, next token, rescue count and the online counts
must match exactly."""

import ctypes
import math
import shutil
import subprocess
from pathlib import Path

import numpy as np
import pytest
import torch

from oracle import tree as ot
from retree_b200 import synthetic
from retree_b200.recovery import RecoveryMemory
from retree_b200.recovery_device import RecoveryTable
from retree_b200.retree import follow_verified_tree_with_recovery
from tests import golden_cases as gc

HERE = Path(__file__).resolve().parent


@pytest.fixture(scope="module")
def walk_lib(tmp_path_factory):
    if shutil.which("g++") is None:
        pytest.skip("needs g++")
    out = tmp_path_factory.mktemp("native") / "librecovery_host.so"
    subprocess.run(["g++", "-O2", "-std=c++17", "-shared", "-fPIC", "-Wall", "-Werror",
                    str(HERE / "native" / "recovery_host.cpp"), "-o", str(out)], check=True)
    lib = ctypes.CDLL(str(out))
    P, I, I64, F = ctypes.c_void_p, ctypes.c_int, ctypes.c_int64, ctypes.c_float
    lib.host_recovery_walk.argtypes = [I, P, P, P, P, I64, I, I64, I, F, I64, I, I, I, P, I, P, P, P, I64, P, P, I,
                                       P, P, P, P]
    lib.host_recovery_walk.restype = I
    lib.host_round_to_bf16.argtypes = [F]
    lib.host_round_to_bf16.restype = F
    return lib


def _ptr(a):
    return None if a is None else a.ctypes.data


def run_native(lib, parents, tokens, logits: torch.Tensor, mem: RecoveryMemory, gate_threshold, rescue_k, record_k,
               online, stop):
    n = len(parents)
    par = np.asarray(parents, dtype=np.int32)
    tok = np.asarray(tokens if len(tokens) else [0], dtype=np.int64)
    post = logits.float().argmax(-1).numpy().astype(np.int64) if logits.dtype == torch.float32 else \
        logits.argmax(-1).numpy().astype(np.int64)
    if logits.dtype == torch.bfloat16:
        lg = logits.contiguous().view(torch.int16).numpy()
        dtype = 1
    else:
        lg = logits.contiguous().numpy()
        dtype = 0
    gate_on = 1 if gate_threshold > 0 else 0
    log_thr = math.log(gate_threshold) if gate_on else 0.0
    log_thr = lib.host_round_to_bf16(log_thr) if dtype == 1 else float(np.float32(log_thr))
    table = RecoveryTable.from_memory(mem, capacity=1 << 12, extra_pairs=0)
    stop_arr = None if stop is None else np.asarray(sorted(stop) if len(stop) else [0], dtype=np.int64)
    logp = np.zeros(2 * 4096, dtype=np.int32)
    logc = np.zeros(1, dtype=np.int32)
    acc = np.zeros(n, dtype=np.int64)
    alen = np.zeros(1, dtype=np.int32)
    nxt = np.zeros(1, dtype=np.int64)
    resc = np.zeros(1, dtype=np.int32)
    code = lib.host_recovery_walk(n, _ptr(par), _ptr(tok), _ptr(post), _ptr(lg), lg.shape[1], dtype, lg.shape[1],
                                  gate_on, log_thr, mem.freq_threshold, rescue_k, record_k, int(online),
                                  _ptr(stop_arr), 0 if stop is None else len(stop), _ptr(table.keys),
                                  _ptr(table.prior), _ptr(table.online), table.capacity, _ptr(logp), _ptr(logc), 4096,
                                  _ptr(acc), _ptr(alen), _ptr(nxt), _ptr(resc))
    assert code == 0
    log = [tuple(p) for p in logp[: 2 * int(logc[0])].reshape(-1, 2).tolist()]
    return acc[: int(alen[0])].tolist(), int(nxt[0]), int(resc[0]), table.online_counts(), log


def run_reference(parents, tokens, logits, mem, gate_threshold, rescue_k, record_k, online, stop):
    post = logits.argmax(-1)[None]
    acc, nxt, resc = follow_verified_tree_with_recovery(
        ot.child_maps(parents, list(tokens)), post, logits[None], mem, gate_threshold=gate_threshold,
        online_update=online, record_top_k=record_k, rescue_top_k=rescue_k, disallow_rescue_target_ids=stop)
    return acc, nxt, resc, mem.online_counts()


def test_golden_recovery_walks(walk_lib):
    trees = {c["name"]: c for c in gc.tree_cases()}
    arr = gc.load_npz("recovery.npz")
    for i, c in enumerate(gc.load_json("recovery.json")):
        t = trees[c["tree"]]
        logits = torch.from_numpy(arr[f"r{i}_logits"])
        mem = RecoveryMemory(c["freq_threshold"])
        for d, tt, cnt in c["prior"]:
            mem.record_prior(d, tt, cnt)
        stop = None if c["stop"] is None else set(c["stop"])
        acc, nxt, resc, online, _ = run_native(walk_lib, t["parents"], t["tokens"], logits, mem, c["gate_threshold"],
                                               c["rescue_top_k"], c["record_top_k"], True, stop)
        assert (acc, nxt, resc) == (c["accepted"], c["next"], c["rescued"]), i
        assert sorted([d, g, k] for (d, g), k in online.items()) == c["online"], i


def _random_case(seed):
    rng = np.random.default_rng(seed)
    budget = int(rng.choice([8, 16, 40, 96]))
    parents = synthetic.random_tree_parents(seed, budget, max_depth=int(rng.integers(3, 12))).tolist()
    n = len(parents)
    vocab = int(rng.integers(12, 40))
    tokens = rng.integers(0, vocab, size=n - 1)          # small vocab: siblings repeat tokens
    logits = rng.standard_normal((n, vocab)).astype(np.float32) * 2.0
    for a in range(n):                                    # boost some children so walks go deep
        kids = [b for b in range(1, n) if parents[b] == a]
        if kids and rng.random() < 0.7:
            logits[a, tokens[int(rng.choice(kids)) - 1]] += 6.0
    mem = RecoveryMemory(int(rng.integers(0, 5)))
    for _ in range(int(rng.integers(0, 60))):
        mem.record_prior(int(rng.integers(vocab)), int(rng.integers(vocab)), int(rng.integers(1, 6)))
    for _ in range(int(rng.integers(0, 10))):
        mem.record_online(int(rng.integers(vocab)), int(rng.integers(vocab)), int(rng.integers(1, 3)))
    gate = float(rng.choice([0.0, 0.01, 0.2, 0.9]))
    rescue_k, record_k = int(rng.integers(0, 9)), int(rng.integers(0, 9))
    online = bool(rng.random() < 0.8)
    stop = [None, set(), {int(x) for x in rng.choice(vocab, size=2, replace=False)}][int(rng.integers(3))]
    return parents, tokens.tolist(), logits, mem, gate, rescue_k, record_k, online, stop


def _clone(mem):
    m = RecoveryMemory(mem.freq_threshold)
    for (d, g), c in mem.prior_counts().items():
        m.record_prior(d, g, c)
    for (d, g), c in mem.online_counts().items():
        m.record_online(d, g, c)
    return m


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_random_recovery_walks_match_reference(walk_lib, dtype):
    rescues = 0
    for seed in range(160):
        parents, tokens, lg, mem, gate, rk, ck, online, stop = _random_case(seed)
        logits = torch.from_numpy(lg).to(dtype)
        before = mem.online_counts()
        got = run_native(walk_lib, parents, tokens, logits, _clone(mem), gate, rk, ck, online, stop)
        want = run_reference(parents, tokens, logits, _clone(mem), gate, rk, ck, online, stop)
        assert got[:4] == want, seed
        # the log holds exactly the online increments of this walk
        inc = {}
        for p in got[4]:
            inc[p] = inc.get(p, 0) + 1
        assert {p: c - before.get(p, 0) for p, c in got[3].items() if c - before.get(p, 0)} == inc, seed
        rescues += got[2]
    assert rescues > 20  # the cases exercise the recovery branch, not only exact walks


def test_bf16_rounding_matches_torch(walk_lib):
    rng = np.random.default_rng(0)
    x = np.concatenate([rng.standard_normal(20000).astype(np.float32) * 10, [0.0, -0.0, 1e-40, 3.3895e38, -7.5]])
    got = np.array([walk_lib.host_round_to_bf16(float(v)) for v in x], dtype=np.float32)
    want = torch.from_numpy(x.astype(np.float32)).to(torch.bfloat16).float().numpy()
    assert np.array_equal(got, want)


def test_device_table_layout_matches_host_lookup():
    mem = RecoveryMemory(3)
    for d, g, c in [(1, 2, 3), (5, 2, 1), (2 ** 31 - 1, 7, 2), (0, 0, 4)]:
        mem.record_prior(d, g, c)
    mem.record_online(1, 2, 2)
    t = RecoveryTable.from_memory(mem, capacity=16, extra_pairs=0)
    for (d, g) in [(1, 2), (5, 2), (2 ** 31 - 1, 7), (0, 0), (9, 9)]:
        assert t.frequency(d, g) == mem.get_frequency(d, g)
    assert t.online_counts() == {(1, 2): 2}


def test_device_memory_host_logic_on_cpu_tensors():
    """DeviceRecoveryMemory's host side: table build, log sync into the host memory, delta application."""
    from retree_b200.recovery_device import DeviceRecoveryMemory

    mem = RecoveryMemory(2)
    mem.record_prior(3, 4, 5)
    mem.record_online(3, 4, 1)
    dm = DeviceRecoveryMemory(mem, "cpu", capacity=64, log_capacity=8, stop_ids={7, 9})
    assert dm.stop_ids.tolist() == [7, 9] and dm.freq_threshold == 2
    keys, prior, online = dm.table
    host = RecoveryTable(64)
    host.keys[:] = keys.numpy().view(np.uint64)
    host.prior[:] = prior.numpy()
    host.online[:] = online.numpy()
    assert host.frequency(3, 4) == 6 and host.frequency(4, 3) == 0
    # the walk's log: two increments of (10, 11), one of (3, 4)
    dm.log_pairs[:3] = torch.tensor([[10, 11], [3, 4], [10, 11]], dtype=torch.int32)
    dm.log_count.fill_(3)
    assert dm.sync() == 3 and int(dm.log_count.item()) == 0
    assert mem.online_counts() == {(3, 4): 2, (10, 11): 2}
    # another rank's delta lands in both copies, in place
    keys_ptr = keys.data_ptr()
    dm.apply_online_delta({(20, 21): 4, (3, 4): 1})
    assert dm.table[0].data_ptr() == keys_ptr
    host.keys[:] = dm.table[0].numpy().view(np.uint64)
    host.prior[:] = dm.table[1].numpy()
    host.online[:] = dm.table[2].numpy()
    assert host.frequency(20, 21) == 4 and host.frequency(3, 4) == 5 + 1 + 1
    assert mem.online_counts() == {(3, 4): 3, (10, 11): 2, (20, 21): 4}
    assert DeviceRecoveryMemory(mem, "cpu", capacity=64, stop_ids=set()).stop_ids is None
