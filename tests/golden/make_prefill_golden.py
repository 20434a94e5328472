"""Golden chunk plans from the reference's own planner.

Run in a checkout where the Veystrix-Core reference tree is available:

    python tests/golden/make_prefill_golden.py --reference <path-to-Veystrix-Core>

It imports models/flashnext/prefill.py (the planner of :109-207 and the
budgeted policy's estimate in prefill_budget.py:115-135) and layer_major.py
(the window planner of :155-186).  Those modules also import MLX and two
runtime modules at the top, which the planning functions never call; they are
replaced by empty stand-ins for the import.  The plans are written to
prefill_plans.json beside this script; nothing at test time touches the
reference tree.
"""
from __future__ import annotations

import argparse
import json
import os
import sys
import types

CASES = [
    # (total, chunk, boundaries, offset, policy, anchors, budget_mb)
    (5000, 2048, [], 0, "grid", None, None),
    (4130, 2048, [4100], 0, "grid", None, None),
    (9000, 2048, [700, 5100], 2048, "grid", None, None),
    (9000, 2048, [700, 5100], 0, "balanced", None, None),
    (6300, 2048, [700, 5100], 2700, "balanced", [700, 5100], None),
    (10001, 2048, [], 0, "balanced", None, None),
    (20000, 0, [], 0, "budgeted", None, 1000),
    (20000, 1024, [3000], 0, "budgeted", None, 1000),
    (30000, 0, [700, 12000], 0, "budgeted", None, 600),
    (25000, 0, [700, 12000], 5000, "budgeted", [700, 12000], 600),
    (50000, 0, [], 0, "budgeted", None, 250),
    (3000, 0, [], 0, "budgeted", None, 100),
]

WINDOWS = [
    # (total, chunk, offset, window, required, anchors)
    (9000, 2048, 0, 4096, [], []),
    (9000, 2048, 0, 8192, [4096], []),
    (9000, 2048, 0, 8192, [], [6144]),
    (12000, 1024, 3000, 6000, [7000], [10000, 12500]),
    (20000, 512, 0, 3000, [], [1536, 2560, 9000]),
    (6000, 5000, 0, 4096, [], []),
]


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", required=True)
    args = ap.parse_args()
    sys.path.insert(0, os.path.abspath(args.reference))
    mlx = types.ModuleType("mlx")
    mlx.core = types.ModuleType("mlx.core")
    sys.modules["mlx"], sys.modules["mlx.core"] = mlx, mlx.core
    sys.modules["models.flashnext.memory_controller"] = types.ModuleType("memory_controller")
    qsa = types.ModuleType("qsa_chunk")
    qsa.QSA_CHUNK_THRESHOLD = 2048
    sys.modules["models.flashnext.qsa_chunk"] = qsa
    from models.flashnext import layer_major, prefill, prefill_budget

    out = {"estimate": {"per_token": prefill_budget.PER_TOKEN_TRANSIENT,
                        "pair_bytes": prefill_budget.SDPA_PAIR_BYTES,
                        "query_cap": prefill_budget.QSA_QUERY_CHUNK,
                        "kv_per_token": prefill_budget.KV_BYTES_PER_TOKEN_TOTAL},
           "candidates": list(prefill.CANDIDATE_CHUNKS), "cases": []}
    for total, chunk, bounds, offset, policy, anchors, mb in CASES:
        if mb is not None:
            os.environ[prefill.FLAG_CHUNK_BUDGET_MB] = str(mb)
        spans = prefill.plan_chunks(total, chunk, bounds, offset, policy=policy, anchors=anchors)
        out["cases"].append({"total": total, "chunk": chunk, "boundaries": bounds, "offset": offset,
                             "policy": policy, "anchors": anchors,
                             "budget": None if mb is None else prefill.chunk_budget_bytes(),
                             "spans": [list(s) for s in spans]})
    out["windows"] = []
    for total, chunk, offset, window, required, anchors in WINDOWS:
        spans = prefill.plan_chunks(total, chunk, [], offset, policy="grid")
        groups = layer_major.plan_windows(spans, offset, window, required, anchors)
        out["windows"].append({"spans": [list(x) for x in spans], "offset": offset, "window": window,
                               "required": required, "anchors": anchors,
                               "groups": [[list(x) for x in g] for g in groups]})
    path = os.path.join(os.path.dirname(os.path.abspath(__file__)), "prefill_plans.json")
    with open(path, "w") as f:
        json.dump(out, f, indent=1)
    print(f"wrote {len(out['cases'])} plans and {len(out['windows'])} window plans to {path}")


if __name__ == "__main__":
    main()
