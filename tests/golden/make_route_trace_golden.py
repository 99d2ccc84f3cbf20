"""Golden route-trace lines and routing counters from the reference itself.

    python tests/golden/make_route_trace_golden.py  --reference <checkout of the reference> (or $REFERENCE_DIR)

Runs the reference's ``ExpertCacheManager.record_routing``
(spark_runtime/lazy_official_runtime.py:550-603, the call LazyMoE.forward
makes at :985-987) with ``DEEPSEEK_SPARK_EXPERT_ROUTE_TRACE_JSONL`` set, on the
fixed calls of ``CALLS``, and writes what it produced:

* route_trace_ref.jsonl: its JSONL lines with "timestamp" set to 0;
* route_trace_ref_stats.json: its routing counters after the calls.
"""

from __future__ import annotations

import argparse
import json
import os
import sys
import tempfile
from pathlib import Path

import torch

HERE = Path(__file__).resolve().parent

# (layer_id, input_ids, expert_indices): a [1, 4] prompt of a top-4 layer with
# a repeated token, and a one-token decode step of a top-6 layer
CALLS = [
    (3, [[11, 2, 7, 2]], [[3, 1, 0, 9], [1, 4, 3, 12], [15, 3, 1, 0], [1, 4, 3, 12]]),
    (0, [5], [[201, 7, 64, 3, 255, 130]]),
]


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", default=os.environ.get("REFERENCE_DIR"), required="REFERENCE_DIR" not in os.environ)
    args = ap.parse_args()
    sys.path.insert(0, str(Path(args.reference)))
    with tempfile.TemporaryDirectory() as tmp:
        trace = Path(tmp) / "trace.jsonl"
        os.environ["DEEPSEEK_SPARK_EXPERT_ROUTE_TRACE_JSONL"] = str(trace)
        import spark_runtime.lazy_official_runtime as lor

        cache = lor.ExpertCacheManager(0)
        for layer_id, ids, idx in CALLS:
            cache.record_routing(layer_id=layer_id, input_ids=torch.tensor(ids, dtype=torch.int64),
                                 expert_indices=torch.tensor(idx, dtype=torch.int64))
        lines = []
        for line in trace.read_text().splitlines():
            d = json.loads(line)
            d["timestamp"] = 0
            lines.append(json.dumps(d, sort_keys=True, separators=(",", ":")))
        (HERE / "route_trace_ref.jsonl").write_text("\n".join(lines) + "\n")
        st = cache.stats.as_dict()
        keep = {k: st[k] for k in ("routed_calls", "routed_tokens", "routed_activations")}
        (HERE / "route_trace_ref_stats.json").write_text(
            json.dumps({"counters": keep, "stats_keys": sorted(st)}, indent=1, sort_keys=True) + "\n")
    print("wrote route_trace_ref.jsonl, route_trace_ref_stats.json")


if __name__ == "__main__":
    main()
