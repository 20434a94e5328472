"""Host-side pieces of bench.py (no GPU): the kernel-launch count it claims,
the DRAM traffic it quotes from the committed ncu summary, and the reference
arm's JSON line."""
from __future__ import annotations

import os
import sys

from conftest import ROOT

sys.path.insert(0, ROOT)


def test_block_launches_follow_the_dispatch():
    import bench
    # at most four tokens: the whole block in one cooperative launch
    assert [bench.block_launches(T) for T in (1, 2, 3, 4)] == [1] * 4
    # router (sort inside while T*k <= 1024), x records, gate/up, h records, down, combine
    assert [bench.block_launches(T) for T in (5, 16, 64, 102)] == [6] * 4
    assert bench.block_launches(103) == 7            # separate one-CTA permutation
    assert bench.block_launches(205) == 6            # T*k >= 4E: x gather and two GEMMs
    assert bench.block_launches(300) == 8            # tiled router: logits, top-k, shared gate
    assert bench.block_launches(1638) == 8           # 16,380 routes: one permutation CTA
    assert bench.block_launches(2048) == 10          # sliced permutation: count, scan, scatter


def test_traffic_only_for_the_captured_workload():
    import json
    import bench
    d = json.load(open(os.path.join(ROOT, "profiles", "ncu_traffic.json")))
    for kernel, e in d.items():
        assert bench.traffic_for(kernel, e["tokens"]) == e["dram_bytes_per_launch"]
        assert bench.traffic_for(kernel, e["tokens"] + 1) is None
    assert bench.traffic_for("no_such_kernel", 64) is None


def test_reference_arm_prints_the_contract_line():
    """`bench.py --impl reference` (the driver's reference arm) times the C
    restatement of the block on the host cores and prints one JSON line with
    the main arm's metric, unit and config, its own CPU baseline and an
    end-to-end figure without device copies."""
    import json
    import subprocess

    import bench

    proc = subprocess.run([sys.executable, os.path.join(ROOT, "bench.py"), "--impl", "reference",
                           "--steps", "1", "--warmup", "1"],
                          capture_output=True, text=True, timeout=600, cwd=ROOT)
    assert proc.returncode == 0, proc.stderr[-2000:]
    line = json.loads([ln for ln in proc.stdout.splitlines() if ln.startswith("{")][-1])
    assert line["impl"] == "reference" and line["metric"] == bench.METRIC
    assert line["unit"] == "tokens/s" and line["higher_is_better"] is True
    assert (line["n_gpus"], line["steps"], line["warmup"]) == (1, 1, 1)
    assert line["value"] > 0 and line["config"]["workload"].startswith("BASELINE config 2")
    cpu = line["cpu_baseline"]
    assert cpu["kind"] == "port" and cpu["cores"] >= 1 and cpu["value"] == line["value"]
    assert line["e2e"] == {"value": line["value"], "unit": "tokens/s", "h2d_bytes_per_step": 0,
                           "d2h_bytes_per_step": 0}
