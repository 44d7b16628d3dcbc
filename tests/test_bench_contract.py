"""bench.py's reference arm on the CPU: the JSON line carries the contract's
keys, the same metric and `config` as the GPU arm's model line (so the two
arms compare the same workload), and an e2e with no host<->device bytes."""
import os
import sys
import types

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def test_reference_model_line_contract():
    sys.path.insert(0, ROOT)
    import bench
    from spikestack_lite_b200.dist import RankGroup

    cfg = dict(bench.WORKLOADS["model_full"])
    args = types.SimpleNamespace(steps=1, warmup=0)
    res = bench.run_reference_model(args, RankGroup("gloo"), cfg)
    for key in ("metric", "value", "unit", "n_gpus", "steps", "warmup", "ms_per_step", "higher_is_better", "scaling",
                "vs_baseline", "dtype", "data", "config", "impl", "cpu_baseline", "e2e"):
        assert key in res, key
    assert res["impl"] == "reference" and res["unit"] == "tokens/s" and res["value"] > 0
    assert res["metric"] == bench.METRIC
    assert res["config"] == bench.model_config(cfg, 1)
    assert res["e2e"]["h2d_bytes_per_step"] == 0 and res["e2e"]["d2h_bytes_per_step"] == 0
    assert res["cpu_baseline"]["kind"] == "port" and res["cpu_baseline"]["cores"] >= 1
