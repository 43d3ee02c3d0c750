"""bench.py host-side pieces that need no GPU: the per-launch DRAM traffic reported beside the
roofline comes from the committed ncu summary and follows the rank's share of the cache rows."""

import json
import os
import sys

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, REPO)

import bench  # noqa: E402


def test_traffic_from_summary_scaled_by_share():
    with open(os.path.join(REPO, "profiles", "traffic.json")) as f:
        summary = json.load(f)
    keys = [k for k in summary if not k.startswith("_")]
    assert keys
    for w in keys:
        assert bench.ncu_traffic(w) == summary[w]
    assert bench.ncu_traffic(keys[0], 0.5) == round(summary[keys[0]] * 0.5)
    assert bench.ncu_traffic("no-such-workload") is None


def test_workload_shapes_match_baseline_configs():
    assert bench.workload_spec("cfg1")["lens"] == [8192]
    assert bench.workload_spec("cfg3")["lens"] == [131072]
    spec4 = bench.workload_spec("cfg4")
    assert spec4["lens"] == [4096] * 256 and spec4["sharding"] == "batch"
    lens2 = bench.workload_spec("cfg2")["lens"]
    assert len(lens2) == 64 and min(lens2) >= 1024 and max(lens2) <= 16384


def test_reference_and_main_arm_print_the_same_config():
    for w in ("cfg1", "cfg2", "cfg3", "cfg4"):
        spec = bench.workload_spec(w)
        a = bench.config_of(spec, 1)
        assert a["workload"] == spec["desc"] and a["seq_len"] == max(spec["lens"])


def test_args_defaults():
    a = bench.parse_args([])
    assert a.gpus == 1 and a.rope == "otf" and a.workload == "cfg1" and not a.no_extra and a.warmup >= 3


def test_cpu_model_string():
    assert isinstance(bench.cpu_model(), str) and bench.cpu_model()
