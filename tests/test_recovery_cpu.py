"""Recovery memory and the sibling-recovery walk of the drop-in API (CPU).

The RecoveryMemory cases restate the reference's own tests
(tests/test_recovery_memory.py:10-87); the walk is checked against the
reference's outputs (golden vectors).
"""

import json
import tempfile
from pathlib import Path

import torch

from oracle import tree as ot
from retree_b200.recovery import RecoveryMemory
from retree_b200.retree import follow_verified_tree_with_recovery
from tests import golden_cases as gc


def test_prior_and_online_counts_are_separate():
    m = RecoveryMemory(freq_threshold=3)
    m.record_prior(10, 20, count=2)
    m.record_online(10, 20)
    assert (m.get_prior_frequency(10, 20), m.get_online_frequency(10, 20), m.get_frequency(10, 20)) == (2, 1, 3)
    assert m.is_frequent(10, 20)


def test_ranked_recording_skips_exact_and_stop_tokens():
    m = RecoveryMemory()
    n = m.record_prior_divergences([20, 99, 10, 11, 12], target_token=20, top_k=2, stop_token_ids={99})
    assert n == 2
    assert (m.get_prior_frequency(10, 20), m.get_prior_frequency(11, 20), m.get_prior_frequency(12, 20)) == (1, 1, 0)


def test_prior_file_does_not_persist_online_delta():
    m = RecoveryMemory(freq_threshold=4)
    m.record_prior(10, 20, count=3)
    m.record_online(10, 20, count=2)
    with tempfile.TemporaryDirectory() as d:
        prior, runtime = Path(d) / "prior.json", Path(d) / "runtime.json"
        m.save_prior(str(prior))
        m.save_runtime_state(str(runtime))
        a = RecoveryMemory.from_file(str(prior))
        assert a.get_frequency(10, 20) == 3 and a.online_total_events() == 0
        b = RecoveryMemory.from_file(str(runtime))
        assert b.get_frequency(10, 20) == 3 and b.online_total_events() == 0
        c = RecoveryMemory.from_file(str(runtime), load_online=True)
        assert c.get_prior_frequency(10, 20) == 3 and c.get_online_frequency(10, 20) == 2
        payload = json.loads(runtime.read_text())
        assert payload["format"] == "retree-recovery-state-v1"
        assert "prior_counts" in payload and "online_counts" in payload


def test_online_delta_can_be_synchronized_without_copying_prior():
    a, b = RecoveryMemory(), RecoveryMemory()
    a.record_prior(10, 20, count=5)
    b.record_prior(10, 20, count=5)
    before = a.online_counts()
    a.record_online(10, 20, count=2)
    b.apply_online_delta(a.online_delta_since(before))
    assert b.get_prior_frequency(10, 20) == 5 and b.get_online_frequency(10, 20) == 2


def test_pre_update_snapshot_prevents_self_recovery():
    m = RecoveryMemory(freq_threshold=2)
    m.record_prior(10, 20)
    snap = m.snapshot_frequencies([(10, 20)])
    m.record_online(10, 20)
    assert snap[(10, 20)] < m.freq_threshold
    assert m.get_frequency(10, 20) == 2
    assert m.snapshot_frequencies([(10, 20)])[(10, 20)] >= m.freq_threshold


def test_legacy_rescue_pairs_layout_loads():
    with tempfile.TemporaryDirectory() as d:
        p = Path(d) / "legacy.json"
        p.write_text(json.dumps({"rescue_pairs": {"1,2": 3}}))
        assert RecoveryMemory.from_file(str(p)).get_prior_frequency(1, 2) == 3


def test_recovery_walk_matches_reference():
    trees = {c["name"]: c for c in gc.tree_cases()}
    arr = gc.load_npz("recovery.npz")
    for i, c in enumerate(gc.load_json("recovery.json")):
        t = trees[c["tree"]]
        logits = torch.from_numpy(arr[f"r{i}_logits"])
        mem = RecoveryMemory(c["freq_threshold"])
        for d, tt, cnt in c["prior"]:
            mem.record_prior(d, tt, cnt)
        post = logits.argmax(-1)[None]
        acc, nxt, resc = follow_verified_tree_with_recovery(
            ot.child_maps(t["parents"], t["tokens"]), post, logits[None], mem, gate_threshold=c["gate_threshold"],
            online_update=True, record_top_k=c["record_top_k"], rescue_top_k=c["rescue_top_k"],
            disallow_rescue_target_ids=None if c["stop"] is None else set(c["stop"]))
        assert (acc, nxt, resc) == (c["accepted"], c["next"], c["rescued"]), i
        assert sorted([d, tt, n] for (d, tt), n in mem.online_counts().items()) == c["online"]


def test_files_match_the_reference_writer_byte_for_byte(golden_dir):
    """save_prior / save_runtime_state write what the reference's RecoveryMemory wrote for the same records,
    and loading those files gives back the same tables (tests/golden/make_recovery_files.py)."""
    import importlib.util
    import tempfile

    spec = importlib.util.spec_from_file_location("make_recovery_files", f"{golden_dir}/make_recovery_files.py")
    gen = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(gen)
    mem = RecoveryMemory(freq_threshold=4)
    for kind, d, t, c in gen.records():
        (mem.record_prior if kind == "prior" else mem.record_online)(d, t, c)
    with tempfile.TemporaryDirectory() as td:
        for name, save in (("recovery_prior.json", mem.save_prior), ("recovery_state.json", mem.save_runtime_state)):
            save(str(Path(td) / name))
            assert (Path(td) / name).read_bytes() == (Path(golden_dir) / name).read_bytes(), name
    loaded = RecoveryMemory.from_file(f"{golden_dir}/recovery_state.json", freq_threshold=4, load_online=True)
    assert loaded.prior_counts() == mem.prior_counts() and loaded.online_counts() == mem.online_counts()
    flat = RecoveryMemory.from_file(f"{golden_dir}/recovery_prior.json")
    assert flat.prior_counts() == mem.prior_counts() and flat.online_counts() == {}


def test_pair_table_orders_and_totals():
    """Iteration and tie order follow when each pair became present in each table; totals count
    positive entries only; clearing the online counts leaves the prior untouched."""
    m = RecoveryMemory(freq_threshold=2)
    m.record_online(5, 6)          # online-only pair, first of all
    m.record_prior(1, 2, count=2)
    m.record_prior(3, 4, count=2)
    m.record_online(1, 2)
    m.record_prior(5, 6, count=1)  # now in both tables
    assert list(m.prior_counts()) == [(1, 2), (3, 4), (5, 6)]
    assert list(m.online_counts()) == [(5, 6), (1, 2)]
    # combined counts (1,2)=3, (3,4)=2, (5,6)=2: ties keep prior order
    assert m.top_k_pairs(3) == [((1, 2), 3), ((3, 4), 2), ((5, 6), 2)]
    assert (m.prior_total_pairs(), m.online_total_pairs(), m.total_pairs()) == (3, 2, 3)
    assert (m.prior_total_events(), m.online_total_events(), m.total_rejections()) == (5, 2, 7)
    m.get_frequency(9, 9)          # a lookup creates nothing
    assert m.total_pairs() == 3
    m.clear_online()
    assert m.online_counts() == {} and m.total_pairs() == 3 and m.get_frequency(1, 2) == 2
    m.record_online(3, 4)
    assert list(m.online_counts()) == [(3, 4)]
    assert [r for r in m.rows()] == [(5, 6, 1, 0), (1, 2, 2, 0), (3, 4, 2, 1)]


def test_divergence_recording_stops_at_top_k_without_reading_further():
    m = RecoveryMemory()
    seen = []

    def ranked():
        for t in (7, 20, 8, 9, 10):
            seen.append(t)
            yield t

    assert m.record_online_divergences(ranked(), target_token=20, top_k=2, stop_token_ids=None) == 2
    assert seen == [7, 20, 8] and m.online_counts() == {(7, 20): 1, (8, 20): 1}
