"""Bounded CPU job executor: admission by job count and declared staging bytes, cancellation and
failure observation (the counterpart of reference reelcache/execution.py:65-293).

A job's ``staging_bytes`` are the input bytes it keeps alive until it finishes; the executor admits a
job only while running + queued jobs stay within ``max_pending`` and their staging bytes within
``max_staging_bytes``. ``submit(block=True, timeout=...)`` waits for room; otherwise a full executor
raises :class:`CapacityError`. A job that failed and whose result nobody read makes the next
``submit``/``check_errors`` raise, so background failures are never silent.
"""

from __future__ import annotations

import threading
import time
from collections import deque
from concurrent.futures import CancelledError, Future, ThreadPoolExecutor
from dataclasses import dataclass, field
from typing import Any, Callable, Generic, TypeVar

from .errors import CapacityError, ConfigurationError, StateError
from .telemetry import current_telemetry

T = TypeVar("T")


def _check_timeout(value):
    if value is not None and (isinstance(value, bool) or not isinstance(value, (int, float)) or value < 0):
        raise ConfigurationError(f"timeout={value!r}: expected None or a number of seconds >= 0")


@dataclass
class _JobState:
    job_id: int
    label: str
    staging_bytes: int
    submitted: float
    function: Any = None
    args: tuple = ()
    kwargs: dict = field(default_factory=dict)
    started: float | None = None
    finished: float | None = None
    status: str = "queued"
    error: str | None = None
    observed: bool = False
    telemetry: Any = None

    def summary(self) -> dict:
        queued = (self.started if self.started is not None else (self.finished or time.monotonic())) - self.submitted
        running = None
        if self.started is not None:
            running = (self.finished or time.monotonic()) - self.started
        return {"job_id": self.job_id, "label": self.label, "status": self.status, "staging_bytes": self.staging_bytes,
                "queue_seconds": queued, "run_seconds": running, "error": self.error}


class Job(Generic[T]):
    """Handle of one submitted job."""

    def __init__(self, executor: "BoundedExecutor", state: _JobState, future: Future):
        self._executor = executor
        self._state = state
        self._future = future

    @property
    def job_id(self) -> int:
        return self._state.job_id

    def done(self) -> bool:
        return self._future.done()

    def cancel(self) -> bool:
        return self._future.cancel()

    def add_done_callback(self, callback: Callable[["Job[T]"], None]) -> None:
        self._future.add_done_callback(lambda _future: callback(self))

    def result(self, timeout: float | None = None) -> T:
        _check_timeout(timeout)
        try:
            return self._future.result(timeout)
        finally:
            if self._future.done():
                self._executor._observe(self._state)

    def metrics(self) -> dict:
        return self._state.summary()


class BoundedExecutor:
    """Thread-pool executor bounded by pending jobs and retained staging bytes."""

    def __init__(self, *, max_workers: int = 1, max_pending: int = 2, max_staging_bytes: int = 1 << 30,
                 history_size: int = 128) -> None:
        sizes = {"max_workers": max_workers, "max_pending": max_pending, "max_staging_bytes": max_staging_bytes,
                 "history_size": history_size}
        bad = {name: value for name, value in sizes.items() if not (type(value) is int and value > 0)}
        if bad:
            raise ConfigurationError(f"BoundedExecutor sizes must be ints >= 1: {bad}")
        self.max_workers = max_workers
        self.max_pending = max_pending
        self.max_staging_bytes = max_staging_bytes
        self._cv = threading.Condition()
        self._pool = ThreadPoolExecutor(max_workers=max_workers, thread_name_prefix="reelcache-job")
        self._closed = False
        self._next = 1
        self._pending: dict[int, _JobState] = {}
        self._failed_unread: dict[int, str] = {}
        self._history: deque = deque(maxlen=history_size)
        self._staging = 0
        self._peak_staging = 0
        self._peak_pending = 0
        self._counts = {"submitted": 0, "succeeded": 0, "failed": 0, "cancelled": 0}

    def submit(self, function: Callable[..., T], *args, staging_bytes: int = 0, label: str | None = None,
               block: bool = False, timeout: float | None = None, **kwargs) -> Job[T]:
        if not callable(function):
            raise ConfigurationError(f"submit() needs a callable, got {type(function).__name__}")
        if type(block) is not bool or (label is not None and (not isinstance(label, str) or not label.strip())):
            raise ConfigurationError(f"block={block!r} must be True/False and label={label!r} a non-blank string or None")
        if type(staging_bytes) is not int or staging_bytes < 0:
            raise ConfigurationError(f"staging_bytes={staging_bytes!r}: expected an int >= 0")
        _check_timeout(timeout)
        if timeout is not None and not block:
            raise ConfigurationError("timeout bounds the wait for admission, so it needs block=True")
        if staging_bytes > self.max_staging_bytes:
            raise CapacityError(f"a job staging {staging_bytes} bytes can never fit max_staging_bytes={self.max_staging_bytes}")
        deadline = None if timeout is None else time.monotonic() + timeout
        with self._cv:
            while True:
                if self._closed:
                    raise StateError("BoundedExecutor was closed")
                self._raise_unread()
                if len(self._pending) < self.max_pending and self._staging + staging_bytes <= self.max_staging_bytes:
                    break
                if not block:
                    raise CapacityError(f"executor full: {len(self._pending)}/{self.max_pending} jobs, "
                                        f"{self._staging}/{self.max_staging_bytes} staging bytes")
                left = None if deadline is None else deadline - time.monotonic()
                if left is not None and left <= 0:
                    raise CapacityError(f"no executor capacity freed up within {timeout} s")
                self._cv.wait(left)
            state = _JobState(self._next, label or getattr(function, "__name__", type(function).__name__),
                              staging_bytes, time.monotonic(), function, args, kwargs,
                              telemetry=current_telemetry())
            self._next += 1
            self._pending[state.job_id] = state
            self._staging += staging_bytes
            self._peak_pending = max(self._peak_pending, len(self._pending))
            self._peak_staging = max(self._peak_staging, self._staging)
            try:
                future = self._pool.submit(self._run, state)
            except RuntimeError:
                del self._pending[state.job_id]
                self._staging -= staging_bytes
                self._cv.notify_all()
                raise
            self._counts["submitted"] += 1
        future.add_done_callback(lambda done: self._finish(state, done))
        return Job(self, state, future)

    def _run(self, state: _JobState):
        with self._cv:
            state.started = time.monotonic()
            state.status = "running"
            function, args, kwargs = state.function, state.args, state.kwargs
            state.function, state.args, state.kwargs = None, (), {}
        if state.telemetry is None:
            return function(*args, **kwargs)
        with state.telemetry.capture():  # the submitter's collector follows the job into the worker
            return function(*args, **kwargs)

    def _finish(self, state: _JobState, future: Future) -> None:
        with self._cv:
            state.finished = time.monotonic()
            if future.cancelled():
                state.status = "cancelled"
                self._counts["cancelled"] += 1
            else:
                error = future.exception()
                if error is None:
                    state.status = "succeeded"
                    self._counts["succeeded"] += 1
                else:
                    state.status = "failed"
                    state.error = f"{type(error).__name__}: {error}"
                    self._counts["failed"] += 1
                    if not state.observed:
                        self._failed_unread[state.job_id] = state.error
            state.function, state.args, state.kwargs = None, (), {}
            self._pending.pop(state.job_id, None)
            self._staging -= state.staging_bytes
            self._history.append(state.summary())
            self._cv.notify_all()

    def _observe(self, state: _JobState) -> None:
        with self._cv:
            state.observed = True
            self._failed_unread.pop(state.job_id, None)

    def _raise_unread(self) -> None:
        if self._failed_unread:
            job_id, error = next(iter(self._failed_unread.items()))
            del self._failed_unread[job_id]
            raise StateError(f"background job {job_id} failed and its result was never read: {error}")

    def check_errors(self) -> None:
        with self._cv:
            self._raise_unread()

    def stats(self) -> dict:
        with self._cv:
            return {**self._counts, "pending": len(self._pending), "staging_bytes": self._staging,
                    "peak_staging_bytes": self._peak_staging, "peak_pending": self._peak_pending,
                    "max_workers": self.max_workers, "max_pending": self.max_pending,
                    "max_staging_bytes": self.max_staging_bytes, "history": list(self._history)}

    def close(self, *, wait: bool = True, cancel_pending: bool = False) -> None:
        with self._cv:
            self._closed = True
        self._pool.shutdown(wait=wait, cancel_futures=cancel_pending)

    def __enter__(self) -> "BoundedExecutor":
        return self

    def __exit__(self, exc_type, exc, traceback) -> None:
        self.close(cancel_pending=exc_type is not None)
        if exc_type is None:
            self.check_errors()


__all__ = ["BoundedExecutor", "Job", "CancelledError"]
