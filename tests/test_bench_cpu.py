"""Host-side pieces of bench.py (no GPU): the kernel-launch count it claims
and the DRAM traffic it quotes from the committed ncu summary."""
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
