"""The restated DFlash draft forward (oracle.dflash) against the reference module's golden outputs,
and the fused draft's model check, on the CPU."""

import json

import numpy as np
import torch

from oracle import dflash as od
from retree_b200 import draft


def test_restated_draft_forward_matches_reference_golden(golden_dir):
    meta = json.load(open(f"{golden_dir}/dflash.json"))
    spec = od.GOLDEN_CALLS
    assert meta["input_seeds"] == list(spec.input_seeds) and meta["ctx_rows"] == list(spec.ctx_rows)
    cfg = od.small_config()
    assert meta["config"]["target_layer_ids"] == cfg.dflash_config["target_layer_ids"]
    module = od.build_module(cfg, od.seeded_weights(cfg, spec.seed))
    calls = [od.seeded_inputs(cfg, s, c) for s, c in zip(spec.input_seeds, spec.ctx_rows)]
    outs = od.run_calls(module, calls)
    golden = np.load(f"{golden_dir}/dflash.npz")
    for j, out in enumerate(outs):
        want = torch.from_numpy(golden[f"call{j}"])
        assert out.shape == want.shape
        assert float((out - want).abs().max()) < 1e-5, j


def test_restated_forward_depends_on_the_cropped_cache():
    """Call 2 sees call 1's context rows but not its block rows: skipping the crop changes it."""
    cfg = od.small_config()
    module = od.build_module(cfg, od.seeded_weights(cfg, 0))
    a, b = od.seeded_inputs(cfg, 1, 6), od.seeded_inputs(cfg, 2, 3)
    cropped = od.run_calls(module, [a, b])[1]
    from transformers import DynamicCache
    cache = DynamicCache()
    with torch.no_grad():
        module(position_ids=torch.arange(0, 6 + cfg.block_size)[None], noise_embedding=a[1][None],
               target_hidden=a[0][None], past_key_values=cache, use_cache=True)
        # no crop: the first call's block rows stay cached (positions then run past them)
        past = cache.get_seq_length()
        kept = module(position_ids=torch.arange(past, past + 3 + cfg.block_size)[None], noise_embedding=b[1][None],
                      target_hidden=b[0][None], past_key_values=cache, use_cache=True)[0]
    assert float((kept - cropped).abs().max()) > 1e-3


def test_fused_draft_model_check():
    cfg = od.small_config()
    w = od.seeded_weights(cfg, 0)
    assert draft.supports(od.build_module(cfg, w, dtype=torch.bfloat16))
    assert not draft.supports(od.build_module(cfg, w, dtype=torch.float32))
    swa = od.small_config()
    swa.layer_types = ["sliding_attention"] * swa.num_hidden_layers
    assert not draft.supports(od.build_module(swa, w, dtype=torch.bfloat16))
    assert not draft.supports(torch.nn.Linear(4, 4))
