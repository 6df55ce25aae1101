"""Opt-in runtime telemetry: inclusive CPU-wall spans per named stage, optional CUDA-event spans
(the counterpart of reference reelcache/telemetry.py:26-124).

A :class:`RuntimeTelemetry` collector is active in a context (``with collector.capture():``);
``span(stage, nbytes=...)`` and ``cuda_span(stage, device)`` are no-ops without one. Spans nest and
overlap freely, so their durations are attributions, not additive totals. The bounded executor
carries the submitting context's collector into its worker.
"""

from __future__ import annotations

import threading
import time
from contextlib import contextmanager, nullcontext
from contextvars import ContextVar

from .errors import ConfigurationError

_ACTIVE: ContextVar = ContextVar("reelcache_b200_telemetry", default=None)

# Stage names shared with the reference's telemetry snapshots.
STAGES = (
    "store.read", "store.hash", "store.commit",
    "decode.validate", "decode.basis", "decode.coefficients",
    "decode.hevc", "decode.dequantize", "decode.reconstruct",
    "history.restore", "history.copy", "transport.collective",
    "native.h2d", "native.rope", "native.insert",
    "decode.checksum_readback", "prefetch.wait", "prefetch.restore",
    "quality.append",
    "nvdec.demux", "nvdec.decode", "nvdec.unpack", "decode.transfer",
    "history.packet", "sp.packets", "sp.decode", "sp.exchange", "seal.stream_add",
    "seal.prefit", "seal.encode", "seal.wait", "seal.persist", "seal.publish",
)


class RuntimeTelemetry:
    def __init__(self, *, cuda_timing: bool = False):
        if type(cuda_timing) is not bool:
            raise ConfigurationError("cuda_timing must be boolean")
        self.cuda_timing = cuda_timing
        self._lock = threading.Lock()
        self._rows = {name: {"calls": 0, "completed": 0, "failed": 0, "inflight": 0, "wall_seconds": 0.0,
                             "attempted_bytes": 0, "completed_bytes": 0} for name in STAGES}
        self._cuda = {name: {"calls": 0, "seconds": 0.0} for name in STAGES}

    @contextmanager
    def capture(self):
        token = _ACTIVE.set(self)
        try:
            yield self
        finally:
            _ACTIVE.reset(token)

    @contextmanager
    def _span(self, stage: str, nbytes: int):
        if stage not in self._rows or type(nbytes) is not int or nbytes < 0:
            raise ConfigurationError("telemetry requires a known stage and nonnegative integer bytes")
        row = self._rows[stage]
        with self._lock:
            row["calls"] += 1
            row["inflight"] += 1
            row["attempted_bytes"] += nbytes
        started = time.perf_counter()
        ok = False
        try:
            yield
            ok = True
        finally:
            elapsed = time.perf_counter() - started
            with self._lock:
                row["inflight"] -= 1
                row["wall_seconds"] += elapsed
                row["completed" if ok else "failed"] += 1
                if ok:
                    row["completed_bytes"] += nbytes

    @contextmanager
    def _cuda_span(self, stage: str, device):
        import torch
        if stage not in self._cuda:
            raise ConfigurationError("unknown CUDA telemetry stage")
        with torch.cuda.device(device):
            start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            start.record()
            try:
                yield
            finally:
                end.record()
                end.synchronize()
                with self._lock:
                    self._cuda[stage]["calls"] += 1
                    self._cuda[stage]["seconds"] += start.elapsed_time(end) / 1e3

    def snapshot(self) -> dict:
        with self._lock:
            return {"schema": "reelcache.runtime_telemetry.v1",
                    "timing": "inclusive CPU wall; nested/concurrent spans are not additive",
                    "bytes": "stage-specific attempted/completed application bytes, not unique storage",
                    "cuda_synchronized": any(row["calls"] for row in self._cuda.values()),
                    "cuda_timing_enabled": self.cuda_timing,
                    "cuda_stages": {k: dict(v) for k, v in self._cuda.items()},
                    "physical_memory_measured": False,
                    "stages": {k: dict(v) for k, v in self._rows.items()}}


def current_telemetry() -> RuntimeTelemetry | None:
    return _ACTIVE.get()


def span(stage: str, *, nbytes: int = 0):
    collector = _ACTIVE.get()
    return nullcontext() if collector is None else collector._span(stage, nbytes)


def cuda_span(stage: str, device):
    collector = _ACTIVE.get()
    if collector is None or not collector.cuda_timing or str(device).split(":")[0] != "cuda":
        return nullcontext()
    return collector._cuda_span(stage, device)
