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
    for w in ("cfg1", "cfg2", "cfg3", "cfg4"):
        assert bench.ncu_traffic(w) == summary[w]
    assert bench.ncu_traffic("cfg3", 0.5) == round(summary["cfg3"] * 0.5)
    assert bench.ncu_traffic("no-such-workload") is None


def test_workload_shapes_match_baseline_configs():
    assert bench.workload_spec("cfg1")["lens"] == [8192]
    assert bench.workload_spec("cfg3")["lens"] == [131072]
    spec4 = bench.workload_spec("cfg4")
    assert spec4["lens"] == [4096] * 256 and spec4["sharding"] == "batch"
    lens2 = bench.workload_spec("cfg2")["lens"]
    assert len(lens2) == 64 and min(lens2) >= 1024 and max(lens2) <= 16384
