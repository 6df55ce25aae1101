"""Ordered asynchronous archival of complete clean chunks (the counterpart of reference
reelcache/archive_pipeline.py; behaviour from its module docstring, lines 1-61).

Generation keeps going while archival runs behind it with two frontiers per lineage: the
**generated** frontier (the newest submitted chunk) and the **published** frontier (the lineage head
in the store). A submitted chunk is a checkpoint only once it is published.

* One **fitter thread** plans each chunk on the GPU (rank method, basis reuse/extension) against its
  lineage's published head and finalizes its coefficients; chunks of one lineage are planned in
  submission order, each after its predecessor is published (its parent state).
* **Encode workers** (a :class:`BoundedExecutor`) build and store the node packs.
* The **publisher** publishes stored chunks strictly in order per lineage with a compare-and-swap of
  the head, then trains the predictor registry.
* Bounded: at most ``max_unpublished`` submitted-but-unpublished chunks per pipeline; ``submit`` waits
  up to ``submit_timeout`` for room, then raises :class:`CapacityError`. With a raw tier the tier holds
  the sources (``admit``) and its own budgets apply.
* A failure of chunk ``n`` fails every later chunk of its lineage and is raised by ``submit``,
  ``drain`` and the tickets until :meth:`reset` acknowledges it. :meth:`cancel` retires a lineage's
  unpublished work; :meth:`close` drains (or cancels) everything.
* :meth:`defer_gpu_work` (a context manager) holds new planning while a memory-critical section runs
  (e.g. a VAE decode next to archival); restores in flight can be yielded to the same way.
"""

from __future__ import annotations

import os
import threading
import time
from collections import deque
from contextlib import contextmanager
from dataclasses import dataclass, field
from typing import Any, Callable, Mapping

import torch

from .errors import CapacityError, ConfigurationError, StateError
from .execution import BoundedExecutor
from .lineage import LineageRuntime
from .lineage_commit import ArchiveOptions
from .rank_method import RankMethodConfig

#: Seconds a pause waits by default for the planning node to reach a step boundary.
PAUSE_ACK_TIMEOUT = 0.5
#: Seconds after which open pauses expire and the fitter resumes (a pause never starves archival).
PAUSE_MAX_SECONDS = 30.0


@dataclass
class ArchiveTicket:
    lineage: str
    chunk_id: str
    index: int
    matrices: Any = None
    contexts: Any = None
    execution_state: Any = None
    raw_token: int | None = None
    state: str = "queued"          # queued | planning | encoding | stored | published | failed | cancelled
    node_ref: str | None = None
    error: BaseException | None = None
    plan: dict | None = None
    timings: dict = field(default_factory=dict)
    submitted: float = field(default_factory=time.monotonic)
    _done: threading.Event = field(default_factory=threading.Event)
    _job: Any = None

    def done(self) -> bool:
        return self._done.is_set()

    def result(self, timeout: float | None = None) -> str:
        if not self._done.wait(timeout):
            raise TimeoutError(f"archival of {self.lineage}/{self.chunk_id} is still running")
        if self.state != "published":
            raise StateError(f"archival of {self.lineage}/{self.chunk_id} {self.state}: {self.error}")
        return self.node_ref


class ArchivePipeline:
    def __init__(self, runtime: LineageRuntime, *, method: RankMethodConfig, device: Any = "cuda",
                 options: ArchiveOptions | None = None, raw_tier=None, max_unpublished: int = 4,
                 submit_timeout: float | None = None, encode_workers: int = 1, registry=None,
                 max_source_chunks: int | None = None, stream_priority: int | None = None,
                 dedicated_stream: bool = True, encode_cpus: set[int] | None = None,
                 on_publish: Callable[[str, str], None] | None = None):
        """``max_source_chunks``: captured chunks that may wait for planning (submit blocks beyond it; default:
        unbounded apart from ``max_unpublished``). ``stream_priority`` / ``dedicated_stream``: the fitter's
        CUDA stream (a dedicated stream of that priority -- default -1, above the engine's -- or the device's
        current stream). ``encode_cpus``: CPUs the encode worker threads run on. ``on_publish(lineage,
        node_ref)`` runs after every publication (the session archive prepares new packs for restores)."""
        if type(max_unpublished) is not int or max_unpublished < 1:
            raise ConfigurationError("max_unpublished must be a positive integer")
        if max_source_chunks is not None and (type(max_source_chunks) is not int or max_source_chunks < 1):
            raise ConfigurationError("max_source_chunks must be a positive integer or None")
        self.max_source_chunks = max_source_chunks
        self.encode_cpus = None if encode_cpus is None else set(encode_cpus)
        self.on_publish = on_publish
        self._affinity_set = threading.local()
        self.runtime = runtime
        self.method = method
        self.device = torch.device(device)
        self.options = options or ArchiveOptions()
        self.raw_tier = raw_tier
        self.registry = registry
        self.max_unpublished = max_unpublished
        self.submit_timeout = submit_timeout
        self.cv = threading.Condition()
        self._queue: deque[ArchiveTicket] = deque()
        self._tickets: dict[str, list[ArchiveTicket]] = {}
        self._failed: dict[str, BaseException] = {}
        self._generated: dict[str, int] = {}
        self._defer = 0
        # generation holds (generation-first archival): key -> {"opened": t, "record": {...}}
        self._holds: dict[Any, dict] = {}
        self._planning = False          # a node is on the GPU (planning / finalization)
        self._drain_waiters = 0
        self.hold_max_age = 30.0
        self.hold_max_backlog = max(1, max_unpublished // 2)
        self._defer_counts = {"holds_opened": 0, "held_seconds": 0.0, "inflight_waits": 0,
                              "inflight_wait_seconds": 0.0, "inflight_overlaps": 0, "starvation_overrides": 0}
        self._closed = False
        self._counts = {"submitted": 0, "published": 0, "failed": 0, "cancelled": 0, "backpressure_waits": 0,
                        "backpressure_seconds": 0.0}
        # pauses of the node on the GPU (pause_gpu_work): open pauses, whether the fitter sits at a boundary
        self._pauses = 0
        self._pause_opened = 0.0
        self._fitter_paused = False
        self._pause_counts = {"requests": 0, "acked": 0, "ack_timeouts": 0, "paused_seconds": 0.0, "expired": 0}
        self._detaching: set[str] = set()
        self._prewarm: list[dict] = []
        self._stream = None
        if self.device.type == "cuda" and dedicated_stream:
            self._stream = torch.cuda.Stream(self.device, priority=-1 if stream_priority is None else stream_priority)
        self._encoders = BoundedExecutor(max_workers=encode_workers, max_pending=max(2, 2 * encode_workers))
        self._fitter = threading.Thread(target=self._fitter_loop, name="reelcache-fitter", daemon=True)
        self._fitter.start()

    # -- producer side ------------------------------------------------------------------------------------------

    def _unpublished(self) -> int:
        return sum(1 for tickets in self._tickets.values() for t in tickets if not t.done())

    def submit(self, lineage: str, chunk_id: str, matrices: Mapping[Any, torch.Tensor], contexts, *,
               execution_state=None, capture_event=None, holder: Any = None) -> ArchiveTicket:
        """Queue one clean chunk. The tensors are owned by the pipeline (or its raw tier) from here on;
        ``capture_event`` orders planning after the producer's capture writes."""
        deadline = None if self.submit_timeout is None else time.monotonic() + self.submit_timeout
        with self.cv:
            if self._closed:
                raise StateError("archive pipeline is closed")
            if lineage in self._failed:
                raise StateError(f"lineage {lineage} has a failed archival: {self._failed[lineage]}")
            waited = None
            while self._unpublished() >= self.max_unpublished or (
                    self.max_source_chunks is not None and len(self._queue) >= self.max_source_chunks):
                if waited is None:
                    waited = time.monotonic()
                    self._counts["backpressure_waits"] += 1
                left = None if deadline is None else deadline - time.monotonic()
                if left is not None and left <= 0:
                    raise CapacityError("archival backlog is full (max_unpublished)")
                self.cv.wait(0.05 if left is None else min(left, 0.05))
                if lineage in self._failed:
                    raise StateError(f"lineage {lineage} has a failed archival: {self._failed[lineage]}")
            if waited is not None:
                self._counts["backpressure_seconds"] += time.monotonic() - waited
            index = self._generated.get(lineage, 0)
            self._generated[lineage] = index + 1
            ticket = ArchiveTicket(lineage, chunk_id, index, matrices, contexts, execution_state)
            ticket.timings["capture_event"] = capture_event
            self._tickets.setdefault(lineage, []).append(ticket)
            self._counts["submitted"] += 1
        if self.raw_tier is not None:
            ticket.raw_token = self.raw_tier.admit(matrices, chunk_id, holder)
            ticket.matrices = None  # the tier owns the sources now
        with self.cv:
            self._queue.append(ticket)
            self.cv.notify_all()
        return ticket

    # -- fitter / encoders / publisher ----------------------------------------------------------------------------

    def _next(self) -> ArchiveTicket | None:
        with self.cv:
            while True:
                if self._closed and not self._queue:
                    return None
                for ticket in list(self._queue):
                    if ticket.lineage in self._detaching:
                        continue
                    earlier = [t for t in self._tickets[ticket.lineage] if t.index < ticket.index]
                    if any(not t.done() for t in earlier):
                        continue  # planned after its predecessor is published
                    if self._defer or self._held():
                        break
                    self._queue.remove(ticket)
                    self._planning = True
                    return ticket
                self.cv.wait(0.05)

    def _step_boundary(self) -> None:
        """Runs on the fitter thread between lockstep rounds of a node's planning: while a pause is open the node
        waits here (no device read pending, no lock held), until the last pause closes, a caller drains, the
        pipeline closes, or the pause outlives ``PAUSE_MAX_SECONDS``."""
        with self.cv:
            if not self._pauses:
                return
            self._fitter_paused = True
            self.cv.notify_all()
            started = time.monotonic()
            while self._pauses and not self._closed and not self._drain_waiters:
                if time.monotonic() - self._pause_opened > PAUSE_MAX_SECONDS:
                    self._pauses = 0
                    self._pause_counts["expired"] += 1
                    break
                self.cv.wait(0.01)
            self._fitter_paused = False
            self._pause_counts["paused_seconds"] += time.monotonic() - started
            self.cv.notify_all()

    def _fitter_loop(self) -> None:
        from .deferred_reads import set_step_hook
        set_step_hook(lambda: self._step_boundary())
        while True:
            ticket = self._next()
            if ticket is None:
                return
            if ticket.state == "cancelled":
                continue
            try:
                self._plan(ticket)
            except BaseException as error:  # noqa: BLE001 - delivered to the ticket and its lineage
                self._fail(ticket, error)
            finally:
                with self.cv:
                    self._planning = False
                    self.cv.notify_all()

    def _plan(self, ticket: ArchiveTicket) -> None:
        started = time.perf_counter()
        ticket.state = "planning"
        event = ticket.timings.pop("capture_event", None)
        ctx = torch.cuda.stream(self._stream) if self._stream is not None else _Null()
        with ctx:
            if event is not None and self._stream is not None:
                self._stream.wait_event(event)
            matrices = ticket.matrices if ticket.raw_token is None else self.raw_tier.source(ticket.raw_token)
            job = self.runtime.prepare_commit("chunk", ticket.lineage, ticket.chunk_id,
                                              [(ticket.chunk_id, matrices, ticket.contexts)], method=self.method,
                                              registry=self.registry, execution_state=ticket.execution_state,
                                              device=self.device, options=self.options)
            job.plan().finalize()
            if self._stream is not None:
                self._stream.synchronize()
            elif self.device.type == "cuda":
                torch.cuda.current_stream(self.device).synchronize()
        ticket._job = job
        ticket.matrices = None
        ticket.timings["plan_seconds"] = time.perf_counter() - started
        ticket.state = "encoding"
        self._encoders.submit(self._encode_and_publish, ticket, block=True)

    def _encode_and_publish(self, ticket: ArchiveTicket) -> None:
        if self.encode_cpus and not getattr(self._affinity_set, "done", False):
            try:
                os.sched_setaffinity(0, self.encode_cpus)  # this worker thread only
            except (AttributeError, OSError):
                pass
            self._affinity_set.done = True
        try:
            started = time.perf_counter()
            job = ticket._job
            job.encode().store()
            ticket.timings["encode_seconds"] = time.perf_counter() - started
            ticket.state = "stored"
            with self.cv:
                if ticket.state == "cancelled" or ticket.lineage in self._failed:
                    raise StateError("cancelled")
            commit = self.runtime.publish_job(job, job.expected_head, registry=self.registry)
            ticket.node_ref = commit.node_ref
            ticket.plan = commit.plan
            job.release()
            ticket._job = None
            if ticket.raw_token is not None:
                self.raw_tier.published(ticket.raw_token, commit.node_ref)
            with self.cv:
                ticket.state = "published"
                self._counts["published"] += 1
                ticket._done.set()
                self.cv.notify_all()
        except BaseException as error:  # noqa: BLE001
            self._fail(ticket, error)
            return
        if self.on_publish is not None:
            try:
                self.on_publish(ticket.lineage, ticket.node_ref)
            except Exception:  # noqa: BLE001 - preparation for later restores is best effort
                self._counts["publish_hook_errors"] = self._counts.get("publish_hook_errors", 0) + 1

    def _fail(self, ticket: ArchiveTicket, error: BaseException) -> None:
        with self.cv:
            cancelled = ticket.state == "cancelled"
            if not cancelled:
                self._failed.setdefault(ticket.lineage, error)
            for t in self._tickets.get(ticket.lineage, []):
                if t.index >= ticket.index and not t.done():
                    t.state = "cancelled" if cancelled else "failed"
                    t.error = error
                    self._counts["cancelled" if cancelled else "failed"] += 1
                    if t in self._queue:
                        self._queue.remove(t)
                    if t._job is not None:
                        t._job.release()
                        t._job = None
                    if t.raw_token is not None and self.raw_tier is not None:
                        self.raw_tier.failed(t.raw_token)
                    t._done.set()
            self.cv.notify_all()

    # -- control --------------------------------------------------------------------------------------------------

    def commit_recache(self, lineage: str, recache_id: str, ranges, *, epoch_id: str, details=None,
                       execution_state=None, holder: Any = None) -> str:
        """Publish a ``kv_recache`` epoch after every submitted chunk of the lineage (exact RAW ranges, or none
        for a latents-only archive); the tier keeps each range's KV under :func:`range_holder`."""
        self.drain(lineage)
        commit = self.runtime.commit_raw_recache(lineage, recache_id, ranges, epoch_id=epoch_id, details=details,
                                                 execution_state=execution_state, kv_objects=self.kv_objects)
        admit_ranges(self.raw_tier, commit.node_ref, ranges, holder)
        return commit.node_ref

    def commit_recache(self, lineage: str, recache_id: str, ranges, *, epoch_id: str, details=None,
                       execution_state=None, holder: Any = None) -> str:
        """Publish a ``kv_recache`` epoch (the re-materialized chunk ranges of a prompt switch) after every
        submitted chunk of the lineage, planned and encoded like a chunk; the raw tier keeps each range's source
        under :func:`range_holder` until evicted."""
        self.drain(lineage)
        with self.cv:
            self._defer += 1   # the fitter takes no other work while the recache plans on the GPU
        try:
            commit = self.runtime.commit_recache(lineage, recache_id, ranges, method=self.method,
                                                 registry=self.registry, epoch_id=epoch_id, details=details,
                                                 execution_state=execution_state, device=self.device,
                                                 options=self.options)
        finally:
            with self.cv:
                self._defer -= 1
                self.cv.notify_all()
        admit_ranges(self.raw_tier, commit.node_ref, ranges, holder)
        return commit.node_ref

    def frontiers(self, lineage: str) -> dict:
        with self.cv:
            tickets = self._tickets.get(lineage, [])
            published = [t for t in tickets if t.state == "published"]
            return {"generated": self._generated.get(lineage, 0),
                    "published": published[-1].node_ref if published else self.runtime.lineage_head(lineage),
                    "unpublished": sum(1 for t in tickets if not t.done()),
                    "failed": None if lineage not in self._failed else str(self._failed[lineage])}

    def drain(self, lineage: str | None = None, timeout: float | None = None) -> float:
        """Wait until every submitted chunk (of ``lineage``) is published; returns the seconds waited."""
        started = time.monotonic()
        deadline = None if timeout is None else started + timeout
        with self.cv:
            self._drain_waiters += 1  # a waiting caller overrides generation holds
            self.cv.notify_all()
            try:
                while True:
                    lineages = [lineage] if lineage is not None else list(self._tickets)
                    failed = [name for name in lineages if name in self._failed]
                    if failed:
                        raise StateError(f"lineage {failed[0]} has a failed archival: {self._failed[failed[0]]}")
                    if all(t.done() for name in lineages for t in self._tickets.get(name, [])):
                        return time.monotonic() - started
                    left = None if deadline is None else deadline - time.monotonic()
                    if left is not None and left <= 0:
                        raise TimeoutError("archival drain timed out")
                    self.cv.wait(0.05 if left is None else min(0.05, left))
            finally:
                self._drain_waiters -= 1

    def cancel(self, lineage: str) -> int:
        """Retire the lineage's unpublished work (queued or not yet stored); returns the count."""
        with self.cv:
            pending = [t for t in self._tickets.get(lineage, []) if not t.done() and t.state in ("queued", "encoding")]
            for t in pending:
                t.state = "cancelled"
        for t in pending:
            self._fail(t, StateError("cancelled"))
        return len(pending)

    def forget(self, lineage: str, timeout: float | None = 60.0) -> None:
        """Cancel the lineage's unpublished work, wait for what is already publishing, and drop every
        record of it (a deleted session)."""
        self.cancel(lineage)
        deadline = None if timeout is None else time.monotonic() + timeout
        with self.cv:
            while any(not t.done() for t in self._tickets.get(lineage, [])):
                left = None if deadline is None else deadline - time.monotonic()
                if left is not None and left <= 0:
                    raise TimeoutError(f"archival of {lineage} did not settle")
                self.cv.wait(0.05 if left is None else min(0.05, left))
            self._tickets.pop(lineage, None)
            self._failed.pop(lineage, None)
            self._generated.pop(lineage, None)

    def reset(self, lineage: str) -> BaseException | None:
        """Acknowledge a lineage's failure so new chunks may be submitted again."""
        with self.cv:
            self._tickets[lineage] = [t for t in self._tickets.get(lineage, []) if t.state == "published"]
            self._generated[lineage] = len(self._tickets[lineage])
            return self._failed.pop(lineage, None)

    @contextmanager
    def defer_gpu_work(self):
        """Hold new planning on the GPU while the body runs (memory-critical sections)."""
        with self.cv:
            self._defer += 1
        try:
            yield
        finally:
            with self.cv:
                self._defer -= 1
                self.cv.notify_all()

    @contextmanager
    def pause_gpu_work(self, *, ack_timeout: float | None = None):
        """Pause archival GPU work for the caller's section (a decode or another memory-critical section): queued
        nodes are held like :meth:`defer_gpu_work`, and a node already planning stops at its next step boundary (a
        round of its lockstep planner). Waits at most ``ack_timeout`` seconds (default ``PAUSE_ACK_TIMEOUT``) for
        that boundary and yields ``{"acked", "ack_seconds", "inflight", "landed"}`` (``landed``: ``"idle"`` when no
        node was on the GPU, ``"boundary"`` otherwise). The node resumes when the last pause exits, a caller
        drains, or the pause outlives ``PAUSE_MAX_SECONDS``."""
        timeout = PAUSE_ACK_TIMEOUT if ack_timeout is None else ack_timeout
        if isinstance(timeout, bool) or not isinstance(timeout, (int, float)) or timeout < 0:
            raise ConfigurationError("ack_timeout must be a nonnegative number of seconds")
        started = time.monotonic()
        with self.cv:
            self._defer += 1
            if not self._pauses:
                self._pause_opened = started
            self._pauses += 1
            self._pause_counts["requests"] += 1
            inflight = self._planning
            while self._planning and not self._fitter_paused and time.monotonic() - started < timeout:
                self.cv.wait(0.002)
            acked = not self._planning or self._fitter_paused
            self._pause_counts["acked" if acked else "ack_timeouts"] += 1
            record = {"acked": acked, "ack_seconds": time.monotonic() - started, "inflight": inflight,
                      "landed": "idle" if not inflight else ("boundary" if acked else None)}
        try:
            yield record
        finally:
            with self.cv:
                self._defer -= 1
                self._pauses = max(0, self._pauses - 1)
                self.cv.notify_all()

    def detach(self, lineage: str, new_lineage: str) -> dict:
        """Hand ``lineage``'s unpublished chunks to a new lineage ``new_lineage`` that starts at its published head
        (the cut): they keep publishing in order there and never move ``lineage``'s head (which the caller may then
        rewind). Waits for the node in flight, if any, to publish first. Returns ``{"branch", "moved", "cut"}``."""
        with self.cv:
            if new_lineage in self._tickets and self._tickets[new_lineage]:
                raise StateError(f"lineage {new_lineage} is already in the pipeline")
            self._detaching.add(lineage)
            try:
                while any(t.state in ("planning", "encoding", "stored") for t in self._tickets.get(lineage, [])):
                    self.cv.wait(0.01)
                if lineage in self._failed:
                    raise StateError(f"lineage {lineage} has a failed archival: {self._failed[lineage]}")
                cut = self.runtime.lineage_head(lineage)
                moved = [t for t in self._tickets.get(lineage, []) if not t.done()]
                if not moved:
                    return {"branch": new_lineage, "moved": [], "cut": cut}
                self.runtime.fork_lineage(cut, new_lineage)
                kept = [t for t in self._tickets[lineage] if t.done()]
                self._tickets[lineage] = kept
                self._generated[lineage] = len(kept)
                for index, ticket in enumerate(moved):
                    ticket.lineage, ticket.index = new_lineage, index
                self._tickets[new_lineage] = list(moved)
                self._generated[new_lineage] = len(moved)
                return {"branch": new_lineage, "moved": [t.chunk_id for t in moved], "cut": cut}
            finally:
                self._detaching.discard(lineage)
                self.cv.notify_all()

    def prewarm(self, contexts: Mapping[Any, Any], *, seed: int = 0, max_frames: int | None = None) -> dict:
        """Pay the archive path's cold start before the first chunk: :func:`~reelcache_b200.lineage_commit.
        warm_commit_path` (plan and finalize two synthetic chunks of ``contexts``' geometry, fresh then against
        the first one's rows; nothing stored or learned) on the fitter's stream, so kernels, library handles and
        allocator pools exist. Returns per-phase seconds (also in ``stats()["prewarm"]``)."""
        from .lineage_commit import warm_commit_path
        ctx = torch.cuda.stream(self._stream) if self._stream is not None else _Null()
        with ctx:
            report = warm_commit_path(self.method, contexts, options=self.options, device=self.device,
                                      max_frames=max_frames, seed=seed)
            if self._stream is not None:
                self._stream.synchronize()
        with self.cv:
            self._prewarm.append(dict(report))
        return report

    # -- generation holds ---------------------------------------------------------------------------------------

    def _held(self) -> bool:
        """Whether an open generation hold keeps new GPU archival work from starting (called under ``cv``).
        The starvation guard lets work through when the oldest hold is older than ``hold_max_age``, the
        queued backlog reaches ``hold_max_backlog`` or a caller waits in :meth:`drain`."""
        if not self._holds:
            return False
        oldest = min(h["opened"] for h in self._holds.values())
        if (time.monotonic() - oldest > self.hold_max_age or len(self._queue) >= self.hold_max_backlog
                or self._drain_waiters):
            self._defer_counts["starvation_overrides"] += 1
            return False
        return True

    def open_generation(self, key: Any, *, inflight: str = "wait", timeout: float | None = 60.0) -> dict:
        """Open a generation hold: no new GPU archival work starts until :meth:`close_generation`. With
        ``inflight="wait"`` a node already on the GPU finishes first (the wait is returned as
        ``archival_defer_wait``); ``"overlap"`` opens at once and records the overlap."""
        if inflight not in ("wait", "overlap"):
            raise ConfigurationError("inflight must be 'wait' or 'overlap'")
        record = {"archival_defer_wait": 0.0, "inflight_overlaps": 0}
        with self.cv:
            if key in self._holds:
                return self._holds[key]["record"]
            self._holds[key] = {"opened": time.monotonic(), "record": record}
            self._defer_counts["holds_opened"] += 1
            if self._planning:
                if inflight == "overlap":
                    record["inflight_overlaps"] = 1
                    self._defer_counts["inflight_overlaps"] += 1
                else:
                    started = time.monotonic()
                    deadline = None if timeout is None else started + timeout
                    while self._planning and (deadline is None or time.monotonic() < deadline):
                        self.cv.wait(0.01)
                    waited = time.monotonic() - started
                    record["archival_defer_wait"] = waited
                    self._defer_counts["inflight_waits"] += 1
                    self._defer_counts["inflight_wait_seconds"] += waited
        return record

    def close_generation(self, key: Any) -> dict | None:
        with self.cv:
            hold = self._holds.pop(key, None)
            if hold is None:
                return None
            held = time.monotonic() - hold["opened"]
            hold["record"]["held_seconds"] = held
            self._defer_counts["held_seconds"] += held
            self.cv.notify_all()
            return hold["record"]

    @contextmanager
    def generation(self, key: Any, *, inflight: str = "wait"):
        record = self.open_generation(key, inflight=inflight)
        try:
            yield record
        finally:
            self.close_generation(key)

    def stats(self) -> dict:
        with self.cv:
            return {**self._counts, "unpublished": self._unpublished(), "lineages": len(self._tickets),
                    "failed_lineages": sorted(self._failed), "encoders": self._encoders.stats(),
                    "generation_defer": {**self._defer_counts, "open_holds": len(self._holds)},
                    "fitter_pause": dict(self._pause_counts), "prewarm": list(self._prewarm)}

    def close(self, *, drain: bool = True, timeout: float | None = None) -> None:
        if drain:
            try:
                self.drain(timeout=timeout)
            except (StateError, TimeoutError):
                pass
        with self.cv:
            for lineage in list(self._tickets):
                for t in self._tickets[lineage]:
                    if not t.done():
                        t.state = "cancelled"
            self._closed = True
            self.cv.notify_all()
        self._fitter.join(timeout=30)
        self._encoders.close(cancel_pending=True)


def range_holder(node_ref: str, range_id: str) -> str:
    """The raw-tier key of one epoch range (a chunk node's own range is keyed by its node ref)."""
    return f"{node_ref}#{range_id}"


def admit_ranges(raw_tier, node_ref: str, ranges, holder: Any) -> None:
    """Keep each published epoch range's exact source in the raw tier (published at once)."""
    if raw_tier is None:
        return
    for range_id, matrices, _contexts in ranges:
        token = raw_tier.admit({entry: tensor.clone() for entry, tensor in matrices.items()}, range_id, holder)
        raw_tier.published(token, range_holder(node_ref, range_id))


class _Null:
    def __enter__(self):
        return self

    def __exit__(self, *args):
        return False


class RawArchive:
    """Exact RAW archival of clean chunks with the producer interface of :class:`ArchivePipeline` (the
    counterpart of reference reelcache/archive_pipeline.py:2685 ``RawArchive`` and the write-behind RAW
    session archive of reelcache/integrations/sglang/archive.py).

    Synchronous (default): ``submit`` commits the chunk's captured pre-RoPE K/V bit for bit
    (:meth:`LineageRuntime.commit_raw_node`) before it returns, so tickets are already published.
    ``write_behind=True`` (``representation="raw_offload"``): the captured tensors are adopted by the raw tier and
    one ordered background writer commits them; the tier entry becomes evictable only after its node is
    published, and ``submit`` waits only while the writer's queue is full. RAW is the identity reference of the
    capture / restore / install path, not a compression path."""

    def __init__(self, runtime: LineageRuntime, *, raw_tier=None, write_behind: bool = False, max_unwritten: int = 4,
                 kv_objects: bool = True):
        if type(max_unwritten) is not int or max_unwritten < 1:
            raise ConfigurationError("max_unwritten must be a positive integer")
        if write_behind and raw_tier is None:
            raise ConfigurationError("write-behind RAW archival needs a raw tier")
        if write_behind and not kv_objects:
            raise ConfigurationError("a latents-only archive writes no KV behind the tier")
        self.runtime, self.raw_tier, self.write_behind = runtime, raw_tier, write_behind
        self.kv_objects = kv_objects
        self.max_unpublished = max_unwritten
        self.cv = threading.Condition()
        self._queue: deque[ArchiveTicket] = deque()
        self._tickets: dict[str, list[ArchiveTicket]] = {}
        self._failed: dict[str, BaseException] = {}
        self._closed = False
        self._counts = {"submitted": 0, "published": 0, "failed": 0, "payload_bytes": 0, "commit_seconds": 0.0,
                        "writer_waits": 0}
        self._writer = None
        if write_behind:
            self._writer = threading.Thread(target=self._writer_loop, name="reelcache-raw-writer", daemon=True)
            self._writer.start()

    def _commit(self, ticket: ArchiveTicket, matrices) -> None:
        started = time.perf_counter()
        commit = self.runtime.commit_raw_node(ticket.lineage, ticket.chunk_id, matrices, ticket.contexts,
                                              execution_state=ticket.execution_state, kv_objects=self.kv_objects)
        ticket.node_ref = commit.node_ref
        ticket.state = "published"
        with self.cv:
            self._counts["published"] += 1
            self._counts["commit_seconds"] += time.perf_counter() - started
            self._counts["payload_bytes"] += sum(m.numel() * m.element_size() for m in matrices.values())
        if ticket.raw_token is not None:
            self.raw_tier.published(ticket.raw_token, commit.node_ref)
        ticket._done.set()

    def submit(self, lineage: str, chunk_id: str, matrices: Mapping[Any, torch.Tensor], contexts, *,
               execution_state=None, capture_event=None, holder: Any = None) -> ArchiveTicket:
        if self._closed:
            raise StateError("the RAW archive is closed")
        if lineage in self._failed:
            raise StateError(f"lineage {lineage} has a failed archival: {self._failed[lineage]}")
        if capture_event is not None:
            capture_event.synchronize()
        with self.cv:
            index = len(self._tickets.setdefault(lineage, []))
            ticket = ArchiveTicket(lineage, chunk_id, index, None, contexts, execution_state)
            self._tickets[lineage].append(ticket)
            self._counts["submitted"] += 1
        if not self.write_behind:
            if not self.kv_objects and self.raw_tier is not None:
                # the tier keeps the only KV copy of a latents-only node (a miss replays the path)
                ticket.raw_token = self.raw_tier.admit(matrices, chunk_id, holder)
            try:
                self._commit(ticket, matrices)
            except BaseException as error:  # noqa: BLE001 - delivered to the ticket and raised
                self._fail(ticket, error)
                raise
            return ticket
        with self.cv:
            while sum(1 for t in self._queue if not t.done()) >= self.max_unpublished and not self._closed:
                self._counts["writer_waits"] += 1
                self.cv.wait(0.05)
        ticket.raw_token = self.raw_tier.admit(matrices, chunk_id, holder)
        with self.cv:
            self._queue.append(ticket)
            self.cv.notify_all()
        return ticket

    def _writer_loop(self) -> None:
        while True:
            with self.cv:
                while not self._queue and not self._closed:
                    self.cv.wait(0.05)
                if not self._queue:
                    return
                ticket = self._queue[0]
            try:
                if ticket.lineage in self._failed:
                    raise StateError("an earlier chunk of the lineage failed")
                self._commit(ticket, self.raw_tier.source(ticket.raw_token))
            except BaseException as error:  # noqa: BLE001 - delivered to the ticket and its lineage
                self._fail(ticket, error)
            with self.cv:
                self._queue.popleft()
                self.cv.notify_all()

    def _fail(self, ticket: ArchiveTicket, error: BaseException) -> None:
        ticket.state, ticket.error = "failed", error
        with self.cv:
            self._failed.setdefault(ticket.lineage, error)
            self._counts["failed"] += 1
        if ticket.raw_token is not None:
            self.raw_tier.failed(ticket.raw_token)
        ticket._done.set()

    def commit_recache(self, lineage: str, recache_id: str, ranges, *, epoch_id: str, details=None,
                       execution_state=None, holder: Any = None) -> str:
        """Publish a ``kv_recache`` epoch after every submitted chunk of the lineage (exact RAW ranges, or none
        for a latents-only archive); the tier keeps each range's KV under :func:`range_holder`."""
        self.drain(lineage)
        commit = self.runtime.commit_raw_recache(lineage, recache_id, ranges, epoch_id=epoch_id, details=details,
                                                 execution_state=execution_state, kv_objects=self.kv_objects)
        admit_ranges(self.raw_tier, commit.node_ref, ranges, holder)
        return commit.node_ref

    def frontiers(self, lineage: str) -> dict:
        with self.cv:
            tickets = self._tickets.get(lineage, [])
            published = [t for t in tickets if t.state == "published"]
            return {"generated": len(tickets), "published": len(published),
                    "published_ref": published[-1].node_ref if published else None,
                    "error": None if lineage not in self._failed else repr(self._failed[lineage])}

    def drain(self, lineage: str | None = None, timeout: float | None = None) -> float:
        started = time.monotonic()
        with self.cv:
            tickets = [t for name, ts in self._tickets.items() if lineage in (None, name) for t in ts]
        for ticket in tickets:
            left = None if timeout is None else max(0.0, timeout - (time.monotonic() - started))
            if not ticket._done.wait(left):
                raise TimeoutError("RAW write-behind drain timed out")
        if lineage is not None and lineage in self._failed:
            raise StateError(f"lineage {lineage} has a failed archival: {self._failed[lineage]}")
        return time.monotonic() - started

    def cancel(self, lineage: str) -> int:
        return 0  # every submitted chunk is (or will be) written in order

    def forget(self, lineage: str, timeout: float | None = 60.0) -> None:
        self.drain(lineage, timeout)
        with self.cv:
            self._tickets.pop(lineage, None)

    def reset(self, lineage: str) -> BaseException | None:
        with self.cv:
            self._tickets[lineage] = [t for t in self._tickets.get(lineage, []) if t.state == "published"]
            return self._failed.pop(lineage, None)

    @contextmanager
    def defer_gpu_work(self):
        yield

    def open_generation(self, key: Any, **_) -> dict:
        return {"archival_defer_wait": 0.0, "inflight_overlaps": 0}

    def close_generation(self, key: Any) -> dict | None:
        return None

    def stats(self) -> dict:
        with self.cv:
            return {**self._counts, "representation": "raw_offload" if self.write_behind else "raw",
                    "unwritten": len(self._queue), "failed_lineages": sorted(self._failed)}

    def close(self, *, drain: bool = True, timeout: float | None = None) -> None:
        if drain:
            try:
                self.drain(timeout=timeout)
            except (StateError, TimeoutError):
                pass
        with self.cv:
            self._closed = True
            self.cv.notify_all()
        if self._writer is not None:
            self._writer.join(timeout=30)
