"""Layer-overlapped history restore for LingBot's first forward (reference:
integrations/lingbot/reelcache_lingbot/lb_overlap.py:1-186).

The archive starts the restore on its own stream (and, when asked, its own host thread) and returns at once with
an :class:`OverlapSession`. The session puts a forward pre-hook on the self-attention module of every block: before
block ``l`` attends, the hook blocks the host until the restore has issued layer ``l`` and makes the generation
stream wait on that layer's event -- never a device-wide synchronize. After the last layer's wait the hooks are
removed, so the remaining forwards of the chunk read the installed cache in stream order. :meth:`OverlapSession.join`
collects the restore's outcome (a failed restore raises here, typed) before anything derived from the restored
history leaves the model; :meth:`OverlapSession.abort` cancels a restore whose request was abandoned.

:class:`StallEvents` measures what the overlap costs: an event pair on the consuming stream around every layer
wait (the GPU idle time the wait caused) and the restore stream's active window, both relative to an anchor
event recorded before the restore started.
"""

from __future__ import annotations

import time
from typing import Any, Callable, Mapping, Sequence

import torch

from ...errors import StateError
from ...overlapped_restore import RestoreFailure


class StallEvents:
    """CUDA-event telemetry of one overlapped restore (no-ops off CUDA except the counts)."""

    def __init__(self, device: Any, anchor: Any = None):
        self.device = torch.device(device)
        self.cuda = self.device.type == "cuda"
        self.anchor = anchor
        self._pairs: list[tuple[int, Any, Any, bool]] = []
        self._windows: dict[str, tuple[Any, Any]] = {}

    def _record(self, stream=None):
        if not self.cuda:
            return None
        event = torch.cuda.Event(enable_timing=True)
        event.record(stream if stream is not None else torch.cuda.current_stream(self.device))
        return event

    def stall_begin(self, layer: int, ready: bool, stream=None):
        return (layer, self._record(stream), ready, stream)

    def stall_end(self, token) -> None:
        layer, begin, ready, stream = token
        self._pairs.append((layer, begin, self._record(stream), ready))

    def window_begin(self, source: str, stream=None):
        return (source, self._record(stream), stream)

    def window_end(self, token) -> None:
        source, begin, stream = token
        self._windows[source] = (begin, self._record(stream))

    def summary(self) -> dict[str, Any]:
        """Per-layer GPU stall (ms) and the restore windows (ms from the anchor); call after a synchronize."""
        out: dict[str, Any] = {"layers_waited": len(self._pairs),
                               "ready_at_wait": sum(1 for pair in self._pairs if pair[3])}
        if not self.cuda:
            return out
        layers = 1 + max((pair[0] for pair in self._pairs), default=-1)
        stall = [0.0] * layers
        for layer, begin, end, _ in self._pairs:
            stall[layer] += begin.elapsed_time(end)
        out["stall_ms"] = stall
        out["stall_ms_total"] = float(sum(stall))
        if self.anchor is not None:
            for source, (begin, end) in self._windows.items():
                out[f"{source}_window_ms"] = [self.anchor.elapsed_time(begin), self.anchor.elapsed_time(end)]
        return out


class OverlapSession:
    """One pending overlapped restore: its readiness, the per-layer waits of the first forward and the record.

    ``restore`` is the restorer's result (``wait(layer, stream)``, ``join()``, ``readiness``); ``layers`` the model's
    blocks; ``tiles`` readiness layers per block (a restore that marks channel tiles separately: readiness layer
    ``l * tiles + t``). ``finish(info)`` adds entries to the record after a successful join."""

    def __init__(self, restore: Any, *, layers: int, tiles: int = 1, record: dict | None = None,
                 recorder: StallEvents | None = None, stream=None,
                 finish: Callable[[Mapping[str, Any]], Mapping[str, Any]] | None = None):
        if type(layers) is not int or layers < 1 or type(tiles) is not int or tiles < 1:
            raise StateError(f"an overlap session needs positive layer and tile counts, got {layers} x {tiles}")
        self.restore = restore
        self.layers, self.tiles = layers, tiles
        self.record = {} if record is None else record
        self.recorder = recorder
        self.stream = stream
        self.finish = finish
        self.started = time.perf_counter()
        self._handles: list = []
        self.waited = 0
        self.host_wait_seconds = 0.0
        self.first_wait: float | None = None
        self.last_wait: float | None = None
        self.state = "pending"

    # -- the consumer: the first forward ---------------------------------------------------------------------------

    def attach(self, attention_modules: Sequence[torch.nn.Module]) -> None:
        """Pre-hooks on ``attention_modules[l]`` (block ``l``'s self-attention) that wait for layer ``l``."""
        if len(attention_modules) != self.layers:
            raise StateError(f"{len(attention_modules)} attention modules for a restore of {self.layers} layers")
        if self._handles:
            raise StateError("this overlapped restore is already attached to a model")
        for layer, module in enumerate(attention_modules):
            self._handles.append(module.register_forward_pre_hook(self._pre_hook(layer)))

    def _pre_hook(self, layer: int):
        def hook(_module, _inputs):
            self.wait(layer)
        return hook

    def wait(self, layer: int) -> None:
        """Host wait until every tile of ``layer`` was issued, then the consuming stream waits on its events."""
        now = time.perf_counter()
        if self.first_wait is None:
            self.first_wait = now
        readiness = self.restore.readiness
        for tile in range(self.tiles):
            index = layer * self.tiles + tile
            token = None
            if self.recorder is not None:
                token = self.recorder.stall_begin(layer, readiness.ready(index), self.stream)
            self.restore.wait(index, self.stream)
            if token is not None:
                self.recorder.stall_end(token)
        done = time.perf_counter()
        self.host_wait_seconds += done - now
        self.last_wait = done
        self.waited += 1
        if layer == self.layers - 1:
            self.detach()

    def detach(self) -> None:
        handles, self._handles = self._handles, []
        for handle in handles:
            handle.remove()

    @property
    def attached(self) -> bool:
        return bool(self._handles)

    # -- completion -----------------------------------------------------------------------------------------------

    def join(self) -> dict:
        """The restore's outcome (raises :class:`RestoreFailure` if it failed) merged into the record."""
        self.detach()
        if self.state == "joined":
            return self.record
        if self.state == "aborted":
            raise RestoreFailure("the overlapped restore was aborted")
        try:
            info = self.restore.join()
        except BaseException:
            self.state = "aborted"
            self.restore.readiness.cancel()
            raise
        self.state = "joined"
        joined = time.perf_counter()
        self.record.update({
            "overlapped": True,
            "seconds": joined - self.started,
            "layers_waited": self.waited,
            "host_wait_seconds": self.host_wait_seconds,
            "first_wait_seconds": None if self.first_wait is None else self.first_wait - self.started,
            "last_wait_seconds": None if self.last_wait is None else self.last_wait - self.started,
            "restore": dict(info or {}),
        })
        if self.finish is not None:
            self.record.update(dict(self.finish(info or {}) or {}))
        return self.record

    def abort(self) -> bool:
        """An abandoned request: hooks removed and the restore cancelled; True if it had already completed."""
        self.detach()
        if self.state != "pending":
            return self.state == "joined"
        self.state = "aborted"
        self.restore.readiness.cancel()
        completed = False
        try:
            self.restore.join()
            completed = all(self.restore.readiness.ready(i) for i in range(self.layers * self.tiles))
        except BaseException:  # noqa: BLE001 - an abandoned restore's failure is reported, not raised
            completed = False
        self.record.update({"aborted": True, "restore_completed": completed})
        return completed

    def gpu_summary(self) -> dict[str, Any] | None:
        return None if self.recorder is None else self.recorder.summary()
