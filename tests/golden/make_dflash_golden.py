"""Golden vectors for the DFlash block-draft forward, written by the reference's own module.

Builds ``DFlashDraftModel`` (model/dflash.py:176-238, imported from a local
checkout of Adamlong3/ReTree) on ``oracle.dflash.small_config()`` with the
seeded weights of ``oracle.dflash.seeded_weights``, runs three consecutive
draft calls over one ``DynamicCache`` in fp32 on the CPU -- a first call over
the whole prompt's context rows, then two decode calls, each cropped back to
``start`` as ddtree.py:832-846 does -- and stores each call's ``[block,
hidden]`` output next to this script:

    python tests/golden/make_dflash_golden.py --reference /path/to/ReTree
"""

from __future__ import annotations

import argparse
import json
import os
import sys
from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent
sys.path.insert(0, str(HERE.parents[1]))

from oracle import dflash as od  # noqa: E402


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", default=os.environ.get("RETREE_REFERENCE"),
                    help="checkout of the reference repository (or set RETREE_REFERENCE)")
    args = ap.parse_args()
    if not args.reference:
        ap.error("--reference (or RETREE_REFERENCE) must name the reference checkout")
    sys.path.insert(0, args.reference)
    from model.dflash import DFlashDraftModel  # type: ignore
    from transformers import DynamicCache

    torch.manual_seed(0)
    cfg = od.small_config()
    spec = od.GOLDEN_CALLS
    model = DFlashDraftModel(cfg).float().eval()
    missing, unexpected = model.load_state_dict(od.seeded_weights(cfg, spec.seed), strict=False)
    assert not unexpected and all(k.endswith("inv_freq") for k in missing), (missing, unexpected)
    assert list(model.target_layer_ids) == cfg.dflash_config["target_layer_ids"]
    cache = DynamicCache()
    outs = {}
    with torch.no_grad():
        for j, (seed, c) in enumerate(zip(spec.input_seeds, spec.ctx_rows)):
            th, noise = od.seeded_inputs(cfg, seed, c)
            past = cache.get_seq_length()
            start = past + c
            pos = torch.arange(past, start + cfg.block_size).unsqueeze(0)
            out = model(position_ids=pos, noise_embedding=noise.unsqueeze(0), target_hidden=th.unsqueeze(0),
                        past_key_values=cache, use_cache=True, is_causal=False)
            cache.crop(start)
            outs[f"call{j}"] = out[0].numpy().astype(np.float32)
    np.savez_compressed(HERE / "dflash.npz", **outs)
    meta = dict(config=dict(hidden=cfg.hidden_size, layers=cfg.num_hidden_layers, heads=cfg.num_attention_heads,
                            kv_heads=cfg.num_key_value_heads, inter=cfg.intermediate_size,
                            block_size=cfg.block_size, target_layer_ids=cfg.dflash_config["target_layer_ids"]),
                weight_seed=spec.seed, input_seeds=list(spec.input_seeds), ctx_rows=list(spec.ctx_rows),
                torch=torch.__version__, source="model/dflash.py DFlashDraftModel.forward, fp32, CPU")
    (HERE / "dflash.json").write_text(json.dumps(meta, indent=1) + "\n")
    print({k: v.shape for k, v in outs.items()})


if __name__ == "__main__":
    main()
