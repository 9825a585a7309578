"""bench.py's JSON line: assembled from measured values that may still be tensors, it must serialise."""

import json
import sys

import torch

import bench


def _args(argv=()):
    old = sys.argv
    sys.argv = ["bench.py", *argv]
    try:
        return bench.parse()
    finally:
        sys.argv = old


def test_result_line_serialises_tensor_and_plain_inputs():
    args = _args()
    wl = bench.WORKLOADS[args.workload]
    line = bench.result_line(
        args, wl, world=1, reqs=1, steps=20, warm=5, dev_s=torch.tensor([0.066], dtype=torch.float64),
        e2e_s=0.07, wall=0.08, prompt=2048, projections={"qkv": "rt_linear"}, pdl=True,
        accepted=[torch.tensor(1), 2, 1], attn_us=torch.tensor(4.5), byts=8_853_572, prefix_len=torch.tensor([2075]),
        n_tree=17, splits=8, layers=36, traffic={"bytes": 8.9e6, "source": "ncu"}, cpu=None, h2d=4_558_080, d2h=148,
        launches=4000, clocks={"sm_mhz": 1965.0, "sm_max_mhz": 1965.0, "reasons": []})
    d = json.loads(line)
    assert d["metric"] == "verify rounds/sec" and d["unit"] == "rounds/s"
    assert abs(d["value"] - 20 / 0.066) < 1e-6
    assert d["config"]["prompt"] == 2048 and d["roofline"]["prefix_len"] == 2075
    assert d["roofline"]["traffic"] == 8.9e6 and d["roofline"]["bound"] == "hbm"
    assert 0 < d["roofline"]["frac"] < 10
    assert d["e2e"]["h2d_bytes_per_step"] == 4_558_080
    assert d["config"]["mean_accepted"] == 4 / 3


def test_pdl_cannot_be_forced_on():
    """The bench has no switch that turns programmatic dependent launch on (it is on by default at N=1 only)."""
    assert _args(["--pdl", "off"]).pdl == "off"
    try:
        _args(["--pdl", "on"])
    except SystemExit:
        pass
    else:
        raise AssertionError("--pdl on must not parse")


def test_attn_traffic_scales_with_the_live_prefix():
    old = dict(bench.ATTN_TRAFFIC)
    try:
        bench.ATTN_TRAFFIC["w"] = (1_000_000, 2000, 17, "ncu capture")
        assert bench.attn_traffic("w", 2000, 17, 8)["bytes"] == 1_000_000
        assert bench.attn_traffic("w", 2010, 17, 8)["bytes"] == 1_000_000 + 10 * 4096
        assert bench.attn_traffic("w", 2010, 65, 8) is None
        assert bench.attn_traffic("other", 2010, 17, 8) is None
    finally:
        bench.ATTN_TRAFFIC.clear()
        bench.ATTN_TRAFFIC.update(old)
