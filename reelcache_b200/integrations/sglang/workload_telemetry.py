"""Per-request workload telemetry (the counterpart of reference
reelcache/integrations/sglang/workload_telemetry.py:1-40): host-clock marks of each request (restore
issue, first chunk, end), the restore route and bytes, and the archive frontiers, kept in a bounded
ring and summarized as percentiles."""

from __future__ import annotations

import threading
import time
from collections import deque
from typing import Any

import numpy as np

SCHEMA = "reelcache.workload_telemetry.v1"


class _Span:
    def __init__(self, session: str, action: str):
        self.session = session
        self.action = action
        self.start_ns = time.perf_counter_ns()
        self.marks: dict[str, float] = {}

    def mark(self, name: str) -> None:
        self.marks[name] = (time.perf_counter_ns() - self.start_ns) / 1e6


class _NullSpan:
    def mark(self, name: str) -> None:
        pass


class WorkloadTelemetry:
    def __init__(self, *, enabled: bool = True, capacity: int = 4096):
        self.enabled = enabled
        self._records: deque = deque(maxlen=capacity)
        self._lock = threading.Lock()

    def begin(self, session: str, action: str):
        return _Span(session, action) if self.enabled else _NullSpan()

    def end(self, span, report: dict[str, Any]) -> None:
        if not self.enabled or isinstance(span, _NullSpan):
            return
        record = {"session": span.session, "action": span.action, "marks_ms": dict(span.marks),
                  "ttfc_ms": report.get("ttfc_ms"), "ttfc_gpu_ms": report.get("ttfc_gpu_ms"),
                  "route": report.get("route"), "chunks": report.get("chunks"), "wall_ms": report.get("wall_ms"),
                  "restore": {k: v for k, v in (report.get("restore") or {}).items()
                              if isinstance(v, (int, float, str))}}
        with self._lock:
            self._records.append(record)

    def records(self) -> list[dict]:
        with self._lock:
            return list(self._records)

    def summary(self) -> dict[str, Any]:
        rows = self.records()
        out: dict[str, Any] = {"schema": SCHEMA, "requests": len(rows), "actions": {}}
        for action in sorted({r["action"] for r in rows}):
            values = [r["ttfc_ms"] for r in rows if r["action"] == action and r["ttfc_ms"] is not None]
            if values:
                out["actions"][action] = {"count": len(values), "p50_ttfc_ms": float(np.percentile(values, 50)),
                                          "p90_ttfc_ms": float(np.percentile(values, 90)),
                                          "p99_ttfc_ms": float(np.percentile(values, 99))}
        return out
