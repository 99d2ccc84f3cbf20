"""Route-trace telemetry against the reference's own output
(tests/golden/route_trace_ref.jsonl, written by make_route_trace_golden.py from
ExpertCacheManager.record_routing): the same JSONL lines and counters."""

import json
import sys

import torch

from conftest import REPO

GOLDEN = REPO / "tests" / "golden"
sys.path.insert(0, str(GOLDEN))


def _calls():
    from make_route_trace_golden import CALLS

    return CALLS


def test_route_trace_lines_match_the_reference(tmp_path):
    from spark_b200.telemetry import ExpertTelemetry

    t = ExpertTelemetry(tmp_path / "trace" / "routes.jsonl")
    for layer_id, ids, idx in _calls():
        t.record_routing(layer_id=layer_id, input_ids=torch.tensor(ids, dtype=torch.int64),
                         expert_indices=torch.tensor(idx, dtype=torch.int64))
    got = []
    for line in (tmp_path / "trace" / "routes.jsonl").read_text().splitlines():
        d = json.loads(line)
        assert d["timestamp"] > 0
        d["timestamp"] = 0
        got.append(json.dumps(d, sort_keys=True, separators=(",", ":")))
    assert got == (GOLDEN / "route_trace_ref.jsonl").read_text().splitlines()


def test_counters_and_snapshot_keys_match_the_reference():
    from spark_b200.telemetry import ExpertTelemetry

    ref = json.loads((GOLDEN / "route_trace_ref_stats.json").read_text())
    t = ExpertTelemetry(None)  # counting only: no host copy, no file
    for layer_id, ids, idx in _calls():
        t.record_routing(layer_id=layer_id, input_ids=torch.tensor(ids), expert_indices=torch.tensor(idx))
    snap = t.snapshot()
    assert sorted(snap) == ref["stats_keys"]
    assert {k: snap[k] for k in ref["counters"]} == ref["counters"]
    assert snap["hits"] == snap["routed_activations"] and snap["misses"] == 0


def test_resident_arena_and_reads_are_counted(monkeypatch, tmp_path):
    from spark_b200 import telemetry as tm

    monkeypatch.setenv(tm.TRACE_ENV, str(tmp_path / "r.jsonl"))
    tm.set_expert_telemetry(None)
    try:
        t = tm.expert_telemetry()
        assert t.route_trace_path == tmp_path / "r.jsonl"
        t.register_resident(256, 1000)
        t.record_materialize(13369344)
        t.record_packed_read(2, 4096, 0.5)
        s = t.snapshot()
        assert s["entries"] == 256 and s["resident_bytes"] == 1000 and s["copied_bytes"] == 13369344
        assert s["packed_loads"] == 2 and s["packed_read_bytes"] == 4096 and s["arena_allocations"] == 1
    finally:
        tm.set_expert_telemetry(None)
