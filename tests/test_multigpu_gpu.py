"""Two-GPU checks (skipped on a one-GPU machine): KV-head split of one request over NCCL."""

import os
import socket
import traceback

import pytest
import torch
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _split_worker(r, world, port, q):
    os.environ.update(RANK=str(r), WORLD_SIZE=str(world), LOCAL_RANK=str(r), LOCAL_WORLD_SIZE=str(world),
                      MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    try:
        from retree_b200 import distributed as rdist
        from retree_b200 import headsplit, synthetic
        from retree_b200.attention import attach
        from retree_b200.cache import TreeKVCache
        from retree_b200.target import build_target, qwen3_config
        from retree_b200.verify import TreeVerifier
        from oracle import tree as ot
        import numpy as np

        rdist.init(timeout_s=120, backend="nccl")
        dev = torch.device("cuda", r)
        headsplit.register()
        cfg = lambda: qwen3_config("small", hidden_size=512, intermediate_size=1024, num_hidden_layers=2,  # noqa: E731
                                   num_attention_heads=8, num_key_value_heads=2, vocab_size=1000)
        full = build_target(cfg(), device=dev, seed=5)
        shard = build_target(cfg(), device=dev, seed=5, attn_implementation=headsplit.NAME)
        headsplit.shard_attention_heads(shard, r, world)
        L = 200
        ids = torch.randint(0, 1000, (1, L), device=dev, generator=torch.Generator(device=dev).manual_seed(0))
        pos = torch.arange(L, device=dev)[None]
        c1 = TreeKVCache.for_model(full.config, 512, device=dev)
        c2 = TreeKVCache(2, 1, 128, 512, device=dev)
        with torch.inference_mode():
            a = full(ids, position_ids=pos, past_key_values=c1, use_cache=True).logits
            b = shard(ids, position_ids=pos, past_key_values=c2, use_cache=True).logits
            parents = synthetic.random_tree_parents(9, 32).tolist()
            n = len(parents)
            depths = synthetic.depths_from_parents(parents)
            tok = torch.randint(0, 1000, (1, n), device=dev, generator=torch.Generator(device=dev).manual_seed(2))
            bits = torch.from_numpy(ot.pack_bits(ot.visibility(parents)).view(np.int32)).to(dev)
            tpos = torch.from_numpy(L + depths).to(dev)[None]
            m = attach(bits.view(1, 1, n, -1), bits)
            a2 = full(tok, position_ids=tpos, attention_mask=m, past_key_values=c1, use_cache=True).logits
            b2 = shard(tok, position_ids=tpos, attention_mask=m, past_key_values=c2, use_cache=True).logits
            rel = lambda x, y: float((x.float() - y.float()).norm() / y.float().norm())  # noqa: E731
            # graph rounds of the split target run and agree across ranks
            v = TreeVerifier(shard, tree_budget=16, max_length=400, draft_horizon=15)
            v.prefill(ids)
            v.enable_graph(True)
            acc = [v.round(torch.from_numpy(synthetic.draft_logits(50 + i, 15, 1000)).to(dev)) for i in range(4)]
            toks = v.output_ids[: v.start + 1].cpu()
        q.put((r, (rel(b, a), rel(b2, a2), acc, toks.tolist(), v.cache.num_kv_heads)))
    except Exception:
        q.put((r, "ERROR " + traceback.format_exc()))
    finally:
        import torch.distributed as dist
        if dist.is_initialized():
            dist.destroy_process_group()


def test_kv_head_split_on_two_gpus():
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    ps = [ctx.Process(target=_split_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in ps:
        p.start()
    out = dict(q.get(timeout=600) for _ in ps)
    for p in ps:
        p.join(timeout=120)
        if p.is_alive():  # a rank stuck in teardown must not hold the test process open
            p.kill()
            p.join(timeout=30)
    for r in range(2):
        assert not isinstance(out[r], str), out[r]
        e1, e2, acc, toks, kv = out[r]
        assert e1 < 2e-2 and e2 < 2e-2
        assert kv == 1
    assert out[0][2] == out[1][2] and out[0][3] == out[1][3]
