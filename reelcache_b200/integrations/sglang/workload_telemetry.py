"""Workload telemetry (the counterpart of reference reelcache/integrations/sglang/workload_telemetry.py:1-40,
144-470, 555-620): :class:`WorkloadTelemetry` keeps every request's host-clock marks (restore issue, first chunk,
end), route and TTFC in a bounded ring summarized as percentiles; :class:`RequestTelemetry` is the opt-in detailed
record of one request -- spans with GPU times, the exposed stall of every readiness wait, the hidden restore work,
tier segments of a synchronous restore, and bytes."""

from __future__ import annotations

import contextlib
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


# ---------------------------------------------------------------------------------------------------------
# Per-request record (opt-in: ``workload_telemetry``)
# ---------------------------------------------------------------------------------------------------------

#: Span names a request record may hold.
SPAN_NAMES = ("request_begin", "restore_sync", "restore_sync.gpu_raw", "restore_sync.host_raw", "restore_sync.store",
              "replay", "recache", "first_forward", "chunk_commit", "drain", "session_open", "decode")
_ACTIVE = threading.local()


class _Event:
    """A CUDA timing event on a stream, or None off CUDA."""

    @staticmethod
    def record(stream: Any) -> Any:
        import torch
        if stream is None:
            return None
        event = torch.cuda.Event(enable_timing=True)
        event.record(stream)
        return event


def _elapsed_ms(start: Any, end: Any) -> float | None:
    if start is None or end is None:
        return None
    end.synchronize()
    return float(start.elapsed_time(end))


def _union_ms(windows: list[tuple[float, float]]) -> float:
    """Length of the union of ``[start, end)`` windows (milliseconds)."""
    total, reach = 0.0, None
    for start, end in sorted(windows):
        if reach is None or start > reach:
            total += end - start
            reach = end
        elif end > reach:
            total += end - reach
            reach = end
    return total


class RequestTelemetry:
    """The record of one session request: host spans (``time.monotonic_ns``) with GPU times from event pairs on
    the request's stream, the GPU idle time each readiness wait of an overlapped restore exposed (an event right
    before the wait and one right after the stream's device waits were queued: their elapsed time is the stall),
    the phase (``prep`` until the first forward of the first new chunk, then ``generation``), the restore's tiers
    and bytes, and the hidden restore work (restore windows not covered by stalls). Creating no events off CUDA,
    it records host times only."""

    def __init__(self, device: Any):
        import torch
        self.device = torch.device(device)
        self.cuda = self.device.type == "cuda"
        self.phase = "prep"
        self.spans: list[dict] = []
        self.stalls: list[dict] = []
        self.windows: list[tuple[float, float]] = []
        self.restore: dict[str, Any] = {}
        self.bytes: dict[str, int] = {}
        self._origin_ns = time.monotonic_ns()
        self._origin_event = self._record()
        self._open: list[list] = []

    def _record(self, stream: Any = None) -> Any:
        import torch
        if not self.cuda:
            return None
        return _Event.record(stream or torch.cuda.current_stream(self.device))

    def mark_generation(self) -> None:
        self.phase = "generation"

    def begin(self, name: str, *, stream: Any = None, gpu: bool = True) -> list:
        if name not in SPAN_NAMES:
            raise ValueError(f"unknown span {name!r}")
        token = [name, self.phase, time.monotonic_ns(), self._record(stream) if gpu else None, stream]
        self._open.append(token)
        return token

    def end(self, token: list | None) -> None:
        if token is None or token not in self._open:
            return
        self._open.remove(token)
        name, phase, start_ns, start_event, stream = token
        end_event = self._record(stream) if start_event is not None else None
        self.spans.append({"name": name, "phase": phase, "host_start_ns": start_ns - self._origin_ns,
                           "host_end_ns": time.monotonic_ns() - self._origin_ns, "_events": (start_event, end_event),
                           "stream": "compute" if stream is None else "restore"})

    @contextlib.contextmanager
    def span(self, name: str, *, stream: Any = None, gpu: bool = True):
        token = self.begin(name, stream=stream, gpu=gpu)
        try:
            yield token
        finally:
            self.end(token)

    def wrap_wait(self, wait):
        """A readiness wait ``wait(layer[, stream])`` that records the stall it exposes on the consuming stream."""
        def timed(layer, stream=None):
            import torch
            host = time.monotonic_ns()
            consumer = stream if stream is not None else (torch.cuda.current_stream(self.device) if self.cuda
                                                          else None)
            before = self._record(consumer)
            wait(layer, stream) if stream is not None else wait(layer)
            after = self._record(consumer)
            self.stalls.append({"layer": layer, "phase": self.phase, "host_ms": (time.monotonic_ns() - host) / 1e6,
                                "_events": (before, after)})
        return timed

    def restore_window(self, start_ms: float, end_ms: float) -> None:
        """A restore stream's active window, in milliseconds after the record's origin."""
        self.windows.append((start_ms, end_ms))

    def set_restore(self, report: dict | None, *, per_token: int = 0, tokens: int = 0) -> None:
        self.restore = {k: v for k, v in (report or {}).items() if isinstance(v, (int, float, str, bool))}
        if per_token and tokens:
            self.bytes = {"restored_native_bytes": per_token * tokens}

    def resolve(self) -> dict[str, Any]:
        """The plain-data record (resolves the CUDA events: call once the request's work is done)."""
        for token in list(self._open):
            self.end(token)
        spans = []
        for item in self.spans:
            start, end = item.pop("_events")
            spans.append({**item, "gpu_ms": _elapsed_ms(start, end)})
        stalls = []
        for item in self.stalls:
            before, after = item.pop("_events")
            gpu = _elapsed_ms(before, after)
            stalls.append({**item, "gpu_ms": gpu, "clock": "host" if gpu is None else "device"})
        exposed = sum((s["gpu_ms"] if s["gpu_ms"] is not None else s["host_ms"]) for s in stalls)
        hidden = max(0.0, _union_ms(self.windows) - exposed) if self.windows else None
        self.spans, self.stalls = spans, stalls
        return {"schema": SCHEMA, "spans": spans, "exposed_stalls": stalls, "exposed_stall_ms": exposed,
                "hidden_rebuild_gpu_ms": hidden, "restore": self.restore, "bytes": self.bytes,
                "kv_rebuild_exposed_ms": sum((s["gpu_ms"] or 0.0) for s in spans
                                             if s["name"].startswith("restore_sync")) + exposed}


@contextlib.contextmanager
def request_scope(telemetry: "RequestTelemetry | None"):
    """Make ``telemetry`` this thread's active request record for the body (None: no record)."""
    previous = getattr(_ACTIVE, "telemetry", None)
    _ACTIVE.telemetry = telemetry
    try:
        yield telemetry
    finally:
        _ACTIVE.telemetry = previous


def active_telemetry() -> "RequestTelemetry | None":
    return getattr(_ACTIVE, "telemetry", None)


@contextlib.contextmanager
def tier_segment(tier: str):
    """A synchronous restore's work from one tier (``gpu_raw``, ``host_raw``, ``store``) in the active record."""
    record = active_telemetry()
    if record is None:
        yield None
        return
    with record.span(f"restore_sync.{tier}") as token:
        yield token


@contextlib.contextmanager
def drain_span():
    record = active_telemetry()
    if record is None:
        yield None
        return
    with record.span("drain", gpu=False) as token:
        yield token


def bytes_per_token(*, num_layers: int, num_heads: int, head_dim: int, capture_dtypes: dict | None = None,
                    native_bytes: int = 2) -> int:
    """Native K + V bytes of one token over every layer."""
    sizes = {"float32": 4, "bfloat16": 2, "float16": 2}
    k = sizes.get((capture_dtypes or {}).get("K", ""), native_bytes)
    v = sizes.get((capture_dtypes or {}).get("V", ""), native_bytes)
    return num_layers * num_heads * head_dim * (k + v)
