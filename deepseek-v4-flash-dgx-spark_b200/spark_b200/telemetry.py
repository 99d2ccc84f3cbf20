"""Expert routing telemetry with the reference's observability contract.

The reference's expert cache counts every routed call and, when
``DEEPSEEK_SPARK_EXPERT_ROUTE_TRACE_JSONL`` names a file, appends one JSON line
per MoE call with the layer, the token ids, each token's expert indices and the
expert histogram (``ExpertCacheManager.record_routing`` /
``_write_route_trace``, spark_runtime/lazy_official_runtime.py:550-603, called
from LazyMoE.forward at :985-987; counters ``ExpertCacheStats`` :405-452).
``ExpertTelemetry`` keeps the same counters, the same snapshot keys and writes
the same lines, so the reference's trace readers work unchanged.

On B200 every expert of a layer is resident in its arena, so the cache fields
describe that: ``policy`` is "resident", ``entries`` / ``max_entries`` /
``inserts`` count the resident experts, every routed activation is a hit and
there are no misses or evictions.  Tracing needs the routing on the host (one
device-to-host copy per call), so it is off unless the variable is set; the
counters cost nothing.
"""

from __future__ import annotations

import json
import os
import threading
import time
from pathlib import Path
from typing import Any

import torch

TRACE_ENV = "DEEPSEEK_SPARK_EXPERT_ROUTE_TRACE_JSONL"


class ExpertTelemetry:
    def __init__(self, route_trace_path: str | Path | None = None):
        self.route_trace_path = Path(route_trace_path) if route_trace_path else None
        if self.route_trace_path is not None:
            self.route_trace_path.parent.mkdir(parents=True, exist_ok=True)
        self._lock = threading.Lock()
        self.resident_experts = 0
        self.resident_bytes = 0
        self.routed_calls = 0
        self.routed_tokens = 0
        self.routed_activations = 0
        self.copied_bytes = 0
        self.arena_allocations = 0
        self.packed_loads = 0
        self.packed_read_bytes = 0
        self.packed_read_seconds = 0.0

    @classmethod
    def from_env(cls) -> "ExpertTelemetry":
        return cls(os.getenv(TRACE_ENV) or None)

    # -- recording ---------------------------------------------------------
    def register_resident(self, experts: int, nbytes: int) -> None:
        """An arena holding ``experts`` experts in ``nbytes`` was created."""
        with self._lock:
            self.resident_experts += int(experts)
            self.resident_bytes += int(nbytes)
            self.arena_allocations += 1

    def record_materialize(self, copied_bytes: int) -> None:
        with self._lock:
            self.copied_bytes += int(copied_bytes)

    def record_packed_read(self, experts: int, nbytes: int, seconds: float) -> None:
        with self._lock:
            self.packed_loads += int(experts)
            self.packed_read_bytes += int(nbytes)
            self.packed_read_seconds += float(seconds)

    def count_routing(self, tokens: int, activations: int) -> None:
        """The counters of one routed call, without the routing itself."""
        with self._lock:
            self.routed_calls += 1
            self.routed_tokens += int(tokens)
            self.routed_activations += int(activations)

    def record_routing(self, *, layer_id: int, input_ids: torch.Tensor,
                       expert_indices: torch.Tensor, tokens: int | None = None) -> None:
        """Counters plus, when tracing, the reference's ``expert_route`` line.

        ``tokens`` is the number of routed tokens when ``input_ids`` does not
        hold one id per token (a caller without token ids passes an empty
        tensor); by default it is ``input_ids.numel()``, the reference's count.
        The line's ``token_ids`` / ``token_count`` always describe
        ``input_ids`` as given."""
        flat = expert_indices.flatten()
        self.count_routing(input_ids.numel() if tokens is None else tokens, flat.numel())
        if self.route_trace_path is None:
            return
        ids = flat.detach().cpu().tolist()
        histogram: dict[int, int] = {}
        for e in ids:
            histogram[int(e)] = histogram.get(int(e), 0) + 1
        nested = expert_indices.detach().cpu().tolist()
        if nested and not isinstance(nested[0], list):
            nested = [nested]
        payload = {
            "timestamp": time.time(),
            "event": "expert_route",
            "layer_id": int(layer_id),
            "token_ids": [int(v) for v in input_ids.flatten().detach().cpu().tolist()],
            "token_count": int(input_ids.numel()),
            "activation_count": int(flat.numel()),
            "expert_indices": [[int(v) for v in row] for row in nested],
            "expert_histogram": {str(k): v for k, v in sorted(histogram.items())},
        }
        line = json.dumps(payload, sort_keys=True, separators=(",", ":"))
        with self._lock:
            with self.route_trace_path.open("a", encoding="utf-8") as fh:
                fh.write(line + "\n")

    # -- reading -----------------------------------------------------------
    def snapshot(self) -> dict[str, Any]:
        """The reference's ``ExpertCacheStats.as_dict()`` keys."""
        with self._lock:
            return {
                "enabled": True,
                "max_entries": self.resident_experts,
                "policy": "resident",
                "layer_quota": 0,
                "entries": self.resident_experts,
                "resident_bytes": self.resident_bytes,
                "hits": self.routed_activations,
                "misses": 0,
                "inserts": self.resident_experts,
                "evictions": 0,
                "materialize_seconds": 0.0,
                "copied_bytes": self.copied_bytes,
                "routed_calls": self.routed_calls,
                "routed_tokens": self.routed_tokens,
                "routed_activations": self.routed_activations,
                "packed_loads": self.packed_loads,
                "packed_misses": 0,
                "packed_read_seconds": self.packed_read_seconds,
                "packed_read_bytes": self.packed_read_bytes,
                "arena_reuses": 0,
                "arena_allocations": self.arena_allocations,
            }


_telemetry: ExpertTelemetry | None = None
_telemetry_lock = threading.Lock()


def expert_telemetry() -> ExpertTelemetry:
    """The process-wide telemetry (from the environment on first use)."""
    global _telemetry
    with _telemetry_lock:
        if _telemetry is None:
            _telemetry = ExpertTelemetry.from_env()
        return _telemetry


def set_expert_telemetry(t: ExpertTelemetry | None) -> None:
    """Replace the process-wide telemetry (None: re-read the environment on next use)."""
    global _telemetry
    with _telemetry_lock:
        _telemetry = t
