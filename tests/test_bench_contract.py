"""CPU: the parts of bench.py the driver relies on, without a GPU: the default workload is BASELINE
config 4, both arms describe the workload with the same config object, the reference arm prints
one JSON line with the contract's keys, and the head-aligned shards of config 4's fused input
linear cover its rows exactly once at 1, 2, 4 and 8 ranks."""
import json
import os
import subprocess
import sys

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)

import bench  # noqa: E402
from invision_b200.nsplit import segment_rows  # noqa: E402


class _Args:
    def __init__(self, config, only=None):
        self.config = config
        self.only = only


def test_default_workload_is_config4():
    desc, items = bench.WORKLOADS["c4"]
    assert [it["name"] for it in items] == ["fused_in", "out"]
    assert (items[0]["M"], items[0]["K"], items[0]["N"]) == (18432, 4096, 36864)
    assert (items[1]["M"], items[1]["K"], items[1]["N"]) == (18432, 16384, 4096)
    assert sum(bench.item_flops(it) for it in items) == 2.0 * 18432 * (4096 * 36864 + 16384 * 4096)


def test_config_object_is_arm_independent():
    for cfg in ("c4", "c2", "c3_m16"):
        desc, items = bench.WORKLOADS[cfg]
        a = bench.workload_config(_Args(cfg), desc, items)
        b = bench.workload_config(_Args(cfg), desc, items)
        assert a == b and a["config"] == cfg and a["flops_per_step"] > 0 and "L2" in a["l2"]


def test_head_aligned_shards_of_config4():
    segs = bench.WORKLOADS["c4"][1][0]["segments"]
    assert sum(segs) == 36864
    for world in (1, 2, 4, 8):
        rows = np.concatenate([segment_rows(segs, world, r, 128) for r in range(world)])
        assert np.array_equal(np.sort(rows), np.arange(36864))
        for r in range(world):
            mine = segment_rows(segs, world, r, 128)
            q = mine[mine < 4096]
            assert len(q) % 128 == 0 and (len(q) == 0 or q[0] % 128 == 0)  # whole heads of Q


def test_reference_arm_line(tmp_path):
    r = subprocess.run([sys.executable, "bench.py", "--impl", "reference", "--config", "c1", "--steps", "1",
                        "--warmup", "0"], cwd=ROOT, capture_output=True, text=True, timeout=600)
    assert r.returncode == 0, r.stderr[-2000:]
    lines = [l for l in r.stdout.splitlines() if l.strip()]
    assert len(lines) == 1
    d = json.loads(lines[0])
    for k in ("metric", "value", "unit", "n_gpus", "steps", "warmup", "ms_per_step", "higher_is_better", "config",
              "cpu_baseline", "e2e", "impl"):
        assert k in d, k
    assert d["impl"] == "reference" and d["cpu_baseline"]["kind"] in ("reference", "port")
    desc, items = bench.WORKLOADS["c1"]
    assert d["config"] == bench.workload_config(_Args("c1"), desc, items)
    assert d["e2e"]["h2d_bytes_per_step"] == 0 and d["value"] > 0
