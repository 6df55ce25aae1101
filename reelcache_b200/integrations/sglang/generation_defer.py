"""Generation-first archival, the bridge side (the counterpart of reference
reelcache/integrations/sglang/generation_defer.py:1-40, ``_BridgeHolds`` :57; config
``defer_archival_during_generation``, default off).

A request's generation -- from the return of its restore to the exit of its VAE-decode seam -- is a
**generation hold** of the archive pipeline (:meth:`ArchivePipeline.open_generation`): no new GPU archival
work starts inside it. With ``archival_defer_inflight="wait"`` a node already on the GPU finishes first and the
wait is the request's ``archival_defer_wait``; ``"overlap"`` opens at once and records the overlap. The restore
itself is never held (its publish waits need archival). The pipeline's starvation guard (oldest-hold age,
backlog, a caller waiting in ``drain``) bounds every hold.

Hold boundaries in the bridge: opened after the restore returns (:meth:`GenerationDefer.after_restore`), closed
at the exit of a decode seam (:meth:`GenerationDefer.decode_seam`, driven by ``memory_critical_section("...decode")``),
else at the request's end; a request that starts closes holds left open by earlier ones. Off, nothing here acts.
"""

from __future__ import annotations

import contextlib
import threading
import time
from typing import Any


def decode_reason(reason: Any) -> bool:
    """The seams that end a request's generation: the VAE decode (``"decode"`` or ``"*_decode"``)."""
    return isinstance(reason, str) and (reason == "decode" or reason.endswith("_decode"))


class _BridgeHolds:
    """A bridge's open holds (request key -> hold record) and the finished records."""

    def __init__(self):
        self.open: dict[Any, dict[str, Any]] = {}
        self.records: dict[Any, dict[str, Any]] = {}
        self.decode_depth: dict[Any, int] = {}


class GenerationDefer:
    """Opens and closes a bridge's generation holds on its archive pipeline."""

    def __init__(self, pipeline, *, inflight: str = "wait", max_age_seconds: float = 30.0,
                 backlog_fraction: float = 0.5):
        self.pipeline = pipeline
        self.inflight = inflight
        self.holds = _BridgeHolds()
        self._lock = threading.Lock()
        pipeline.hold_max_age = float(max_age_seconds)
        pipeline.hold_max_backlog = max(1, int(backlog_fraction * pipeline.max_unpublished))

    @classmethod
    def from_config(cls, config, pipeline) -> "GenerationDefer | None":
        if not getattr(config, "defer_archival_during_generation", False) or pipeline is None:
            return None
        return cls(pipeline, inflight=config.archival_defer_inflight,
                   max_age_seconds=config.archival_defer_max_age_seconds,
                   backlog_fraction=config.archival_defer_backlog_fraction)

    def begin(self, key: Any) -> None:
        """A new request: holds left open by earlier requests (no decode seam came) close here."""
        with self._lock:
            stale = [k for k in self.holds.open if k != key]
        for other in stale:
            self._close(other, "next_request")

    def after_restore(self, key: Any) -> dict[str, Any]:
        """The restore returned: the request's generation starts."""
        started = time.perf_counter()
        record = self.pipeline.open_generation(key, inflight=self.inflight)
        with self._lock:
            self.holds.open[key] = {"record": record, "opened": started}
        return record

    def _close(self, key: Any, why: str) -> dict[str, Any] | None:
        with self._lock:
            hold = self.holds.open.pop(key, None)
        if hold is None:
            return None
        record = dict(self.pipeline.close_generation(key) or hold["record"])
        record["closed_by"] = why
        with self._lock:
            self.holds.records[key] = record
        return record

    @contextlib.contextmanager
    def decode_seam(self, key: Any, reason: Any):
        """A memory-critical section of the request; a decode seam closes the hold at its (outermost) exit."""
        decode = decode_reason(reason)
        if decode:
            with self._lock:
                self.holds.decode_depth[key] = self.holds.decode_depth.get(key, 0) + 1
        try:
            yield
        finally:
            if decode:
                with self._lock:
                    depth = self.holds.decode_depth.get(key, 1) - 1
                    if depth:
                        self.holds.decode_depth[key] = depth
                    else:
                        self.holds.decode_depth.pop(key, None)
                if not depth:
                    self._close(key, "decode_seam")

    def finish(self, key: Any) -> dict[str, Any] | None:
        """The request's record (closing a hold that is still open)."""
        self._close(key, "finish")
        with self._lock:
            return self.holds.records.pop(key, None)

    def close(self) -> None:
        with self._lock:
            keys = list(self.holds.open)
        for key in keys:
            self._close(key, "close")


__all__ = ["GenerationDefer", "decode_reason"]
