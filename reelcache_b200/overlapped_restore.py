"""Layer-overlapped restore readiness (reference: reelcache/overlapped_restore.py:70-536).

:class:`LayerReadiness` is the contract between a restore running on a side stream (or thread) and the
first forward of the next chunk: the restore marks layer ``L`` ready with the CUDA event recorded
after its last write; attention of layer ``L`` calls :meth:`LayerReadiness.wait` which blocks the host
until layer ``L`` was *issued* (bounded by a timeout) and then makes the consumer stream wait on its
event, so each layer waits only for its own KV. Failures are typed and delivered to every later wait
and to :meth:`join`. Sources: ``restore`` (archive reconstruction) and ``raw`` (raw-tier installs);
a layer is ready when every registered source marked it.
"""

from __future__ import annotations

import threading
import time
from typing import Any, Callable, Iterable, Sequence

import torch

from .errors import ReelCacheError, StateError

SOURCES = ("restore", "raw")
DEFAULT_TIMEOUT = 60.0


class RestoreFailure(StateError):
    """The overlapped restore failed; the history of the affected layers is not valid."""


class LayerReadiness:
    """Per-layer readiness of restored history for one request."""

    def __init__(self, layers: int, *, sources: Sequence[str] = ("restore",), timeout: float = DEFAULT_TIMEOUT):
        if any(source not in SOURCES for source in sources):
            raise StateError(f"readiness sources must be in {SOURCES}")
        self.layers = layers
        self.sources = tuple(sources)
        self.timeout = timeout
        self._cond = threading.Condition()
        self._events: dict[str, list[Any]] = {s: [None] * layers for s in self.sources}
        self._marked: dict[str, list[bool]] = {s: [False] * layers for s in self.sources}
        self._next: dict[str, int] = {s: 0 for s in self.sources}
        self._error: BaseException | None = None
        self._cancelled = False
        self.stall_seconds = [0.0] * layers

    def mark(self, layer: int, event=None, *, source: str = "restore") -> None:
        """Layer ``layer`` of ``source`` is issued; ``event`` completes after its last write. Layers of
        one source must be marked in order (an out-of-order mark is a bug and raises)."""
        with self._cond:
            if layer != self._next[source]:
                raise StateError(f"{source} marked layer {layer} out of order (expected {self._next[source]})")
            self._events[source][layer] = event
            self._marked[source][layer] = True
            self._next[source] = layer + 1
            self._cond.notify_all()

    def mark_all(self, event=None, *, source: str = "restore") -> None:
        for layer in range(self._next[source], self.layers):
            self.mark(layer, event, source=source)

    def fail(self, error: BaseException) -> None:
        with self._cond:
            if self._error is None:
                self._error = error
            self._cond.notify_all()

    def cancel(self) -> None:
        with self._cond:
            self._cancelled = True
            self._cond.notify_all()

    def ready(self, layer: int) -> bool:
        with self._cond:
            return all(self._marked[s][layer] for s in self.sources)

    def wait(self, layer: int, stream=None) -> None:
        """Block until ``layer`` is issued by every source, then order ``stream`` after its events."""
        started = time.perf_counter()
        deadline = started + self.timeout
        with self._cond:
            while True:
                if self._error is not None:
                    raise RestoreFailure(f"overlapped restore failed before layer {layer}: {self._error}") \
                        from self._error
                if self._cancelled:
                    raise RestoreFailure("overlapped restore was cancelled")
                if all(self._marked[s][layer] for s in self.sources):
                    events = [self._events[s][layer] for s in self.sources]
                    break
                remaining = deadline - time.perf_counter()
                if remaining <= 0:
                    raise StateError(f"timed out after {self.timeout} s waiting for restored layer {layer}")
                self._cond.wait(remaining)
        for event in events:
            if event is not None:
                (torch.cuda.current_stream() if stream is None else stream).wait_event(event)
        self.stall_seconds[layer] += time.perf_counter() - started

    def layer(self, layer: int):
        readiness = self

        class _Layer:
            def wait(self, stream=None):
                readiness.wait(layer, stream)

        return _Layer()

    @property
    def error(self) -> BaseException | None:
        return self._error


class OverlappedRestore:
    """A restore issuing layer by layer on a worker thread and side stream."""

    def __init__(self, readiness: LayerReadiness, thread: threading.Thread | None):
        self.readiness = readiness
        self._thread = thread
        self.result: Any = None

    def join(self, timeout: float | None = None) -> Any:
        if self._thread is not None:
            self._thread.join(timeout)
            if self._thread.is_alive():
                raise StateError("overlapped restore did not finish in time")
        if self.readiness.error is not None:
            raise RestoreFailure(str(self.readiness.error)) from self.readiness.error
        return self.result

    def cancel(self) -> None:
        self.readiness.cancel()


def start_overlapped_restore(issue: Callable[[int], Any], layers: int, *, stream=None, thread: bool = True,
                             readiness: LayerReadiness | None = None, after: OverlappedRestore | None = None,
                             finish: Callable[[], Any] | None = None) -> OverlappedRestore:
    """Issue ``issue(layer)`` for every layer in order on ``stream`` (side stream), marking each layer
    with an event. ``after`` chains behind another restore (its layer ``L`` before ours)."""
    readiness = readiness or LayerReadiness(layers)
    device_stream = stream

    def run():
        try:
            ctx = torch.cuda.stream(device_stream) if device_stream is not None else _Null()
            with ctx:
                for layer in range(layers):
                    if readiness._cancelled:
                        raise RestoreFailure("cancelled")
                    if after is not None:
                        after.readiness.wait(layer, device_stream)
                    issue(layer)
                    event = None
                    if device_stream is not None:
                        event = torch.cuda.Event()
                        event.record(device_stream)
                    readiness.mark(layer, event)
                if finish is not None:
                    handle.result = finish()
        except BaseException as error:  # noqa: BLE001 - delivered to every waiter
            readiness.fail(error)

    handle = OverlappedRestore(readiness, None)
    if thread:
        worker = threading.Thread(target=run, name="reelcache-restore", daemon=True)
        handle._thread = worker
        worker.start()
    else:
        run()
    return handle


def start_overlapped_install(install: Callable[[int], Any], layers: int, *, stream=None, thread: bool = True,
                             readiness: LayerReadiness | None = None, after: OverlappedRestore | None = None,
                             finish: Callable[[], Any] | None = None) -> OverlappedRestore:
    """A RAW (dense) install alone, layer-overlapped: ``install(layer)`` writes that layer's exact captured rows
    (the dense RoPE-and-store kernel), each layer marked as a ``raw`` source so a forward that also waits for a
    compressed restore (``sources=("restore", "raw")``) sees both."""
    readiness = readiness or LayerReadiness(layers, sources=("raw",))
    if "raw" not in readiness.sources:
        raise StateError("an overlapped RAW install marks the 'raw' source of its readiness")

    def issue(layer):
        install(layer)

    handle = start_overlapped_restore(issue, layers, stream=stream, thread=thread, readiness=_SourceView(readiness,
                                                                                                          "raw"),
                                      after=after, finish=finish)
    handle.readiness = readiness
    return handle


class _SourceView:
    """A readiness seen through one of its sources: ``mark`` marks that source."""

    def __init__(self, readiness: LayerReadiness, source: str):
        self._readiness, self._source = readiness, source

    def mark(self, layer: int, event=None) -> None:
        self._readiness.mark(layer, event, source=self._source)

    def __getattr__(self, name):
        return getattr(self._readiness, name)


class _Null:
    def __enter__(self):
        return self

    def __exit__(self, *args):
        return False
