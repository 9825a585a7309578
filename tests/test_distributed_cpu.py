"""World-size-2 gloo tests of the multi-process plumbing (CPU, no GPU)."""

import os
import socket
import traceback

import pytest
import torch.multiprocessing as mp

from retree_b200 import distributed as rdist
from retree_b200.recovery import RecoveryMemory


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _worker(r, world, port, fn, q):
    os.environ.update(RANK=str(r), WORLD_SIZE=str(world), LOCAL_RANK=str(r), LOCAL_WORLD_SIZE=str(world),
                      MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    try:
        rdist.init(timeout_s=60, backend="gloo")
        q.put((r, fn(r, world)))
    except Exception:
        q.put((r, "ERROR " + traceback.format_exc()))
    finally:
        import torch.distributed as dist
        if dist.is_initialized():
            dist.destroy_process_group()


def _run(fn, world=2):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    ps = [ctx.Process(target=_worker, args=(r, world, port, fn, q)) for r in range(world)]
    for p in ps:
        p.start()
    out = dict(q.get(timeout=120) for _ in ps)
    for p in ps:
        p.join(timeout=60)
    for r, v in out.items():
        assert not (isinstance(v, str) and v.startswith("ERROR")), v
    return out


def _sync_memory(r, world):
    mem = RecoveryMemory(freq_threshold=2)
    mem.record_prior(1, 2, count=5)
    before = mem.online_counts()
    # each rank records its own events during "its request"
    mem.record_online(10 + r, 20, count=r + 1)
    mem.record_online(7, 8)
    rdist.synchronize_online_memory(mem, before, capacity=16)
    return sorted(mem.online_counts().items()), sorted(mem.prior_counts().items())


def test_delta_sync_matches_reference_semantics():
    out = _run(_sync_memory)
    # every rank ends with its own events plus the other ranks' deltas; priors untouched
    want = sorted({(10, 20): 1, (11, 20): 2, (7, 8): 2}.items())
    for r in range(2):
        online, prior = out[r]
        assert online == want
        assert prior == [((1, 2), 5)]


def _gather_objects(r, world):
    return rdist.all_gather({"rank": r}), rdist.gather(r * 10), rdist.is_main()


def test_object_collectives_like_reference():
    out = _run(_gather_objects)
    assert out[0][0] == [{"rank": 0}, {"rank": 1}] == out[1][0]
    assert out[0][1] == [0, 10] and out[1][1] is None
    assert out[0][2] and not out[1][2]


def _overflow(r, world):
    try:
        rdist.all_gather_recovery_delta({(i, i): 1 for i in range(20)}, capacity=8)
    except ValueError as e:
        return "refused" if "capacity" in str(e) else str(e)
    return "accepted"


def test_delta_over_capacity_is_refused_on_every_rank():
    out = _run(_overflow)
    assert out == {0: "refused", 1: "refused"}


def test_single_process_fallbacks():
    assert rdist.all_gather(5) == [5] and rdist.gather(5) == [5]
    assert rdist.all_gather_recovery_delta({(1, 2): 3}) == [{(1, 2): 3}]
    enc = rdist.encode_delta({(3, 4): 2, (1, 2): 1}, 4)
    assert rdist.decode_deltas(enc[None]) == [{(1, 2): 1, (3, 4): 2}]
    with pytest.raises(ValueError):
        rdist.encode_delta({(1, 2): 0}, 4)


def _headsplit_forward(r, world):
    import torch
    from oracle import tree as ot
    from retree_b200 import headsplit, synthetic
    from retree_b200.target import qwen3_config
    from oracle.verify_round import cpu_target

    headsplit.register()
    cfg = qwen3_config("small", hidden_size=256, intermediate_size=512, num_hidden_layers=2,
                       num_attention_heads=8, num_key_value_heads=2, vocab_size=500)
    full = cpu_target(cfg, dtype=torch.float32, seed=4)          # every rank builds the same weights
    shard = cpu_target(qwen3_config("small", hidden_size=256, intermediate_size=512, num_hidden_layers=2,
                                    num_attention_heads=8, num_key_value_heads=2, vocab_size=500),
                       dtype=torch.float32, seed=4)
    headsplit.shard_attention_heads(shard, r, world)
    shard.config._attn_implementation = headsplit.SDPA_NAME
    from transformers import DynamicCache
    ids = torch.randint(0, 500, (1, 40), generator=torch.Generator().manual_seed(0))
    pos = torch.arange(40)[None]
    c_full, c_shard = DynamicCache(), DynamicCache()
    a = full(ids, position_ids=pos, past_key_values=c_full, use_cache=True).logits
    b = shard(ids, position_ids=pos, past_key_values=c_shard, use_cache=True).logits
    # a tree verify step with the reference's dense mask on top of the prefix
    parents = synthetic.random_tree_parents(3, 12).tolist()
    n = len(parents)
    depths = synthetic.depths_from_parents(parents)
    tok = torch.randint(0, 500, (1, n), generator=torch.Generator().manual_seed(1))
    _, _, dense = ot.compile_tree(0, 40, tok[0, 1:].tolist(), depths[1:], parents, 40)
    mask = torch.from_numpy(dense)[None, None]
    tpos = torch.from_numpy(40 + depths)[None]
    a2 = full(tok, position_ids=tpos, attention_mask=mask, past_key_values=c_full, use_cache=True).logits
    b2 = shard(tok, position_ids=tpos, attention_mask=mask, past_key_values=c_shard, use_cache=True).logits
    kv_local = c_shard.layers[0].keys.shape[1]
    return (float((a - b).abs().max()), float((a2 - b2).abs().max()), kv_local)


def test_kv_head_split_forward_equals_unsplit():
    out = _run(_headsplit_forward)
    for r in range(2):
        prefill_err, tree_err, kv_local = out[r]
        assert prefill_err < 1e-4 and tree_err < 1e-4
        assert kv_local == 1  # 2 kv heads over 2 ranks
