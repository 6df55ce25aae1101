"""The serving bridge: the engine seam between a chunked causal video engine and the archive (the counterpart of
reference reelcache/integrations/sglang/bridge.py:554-3173).

The engine drives a request through the seam (:mod:`.seam`): ``begin_request`` resolves the session action
(create / resume / rewind / fork) and returns a run; ``run.restore`` puts the attended history into the cache the
engine generates into; the clean forward of each chunk hands every layer's pre-RoPE K / V to a capture scope;
``run.end_chunk`` submits the sealed chunk to the asynchronous archive; a prompt switch re-runs the recache window
between ``begin_recache`` and ``end_recache`` (a ``kv_recache`` cache epoch); ``run.finish`` returns the request's
summary. :meth:`CausalWanKVBridge.request` is that loop over the bridge's own engine.

Restore routes, in order of preference:

1. **resident** -- the session's cache from its previous request still holds the target path
   (:class:`ResidentKV`; a rewind onto a prefix of it is free unless a recache rewrote that prefix since).
2. **archive** -- the attended history (:func:`.visibility.build_visibility_plan`, cut at KV-version boundaries
   and cached per head in a :class:`PlanCache`) is installed from the raw tier where it still holds the exact
   capture and otherwise decoded by the fused sm_100a restore, layer by layer, overlapped with the first forward
   (``overlap_restore``); the archival pipeline's GPU work is held meanwhile (``archival_pump_pause``).
3. **recompute** (``restore_mode="recompute"``) -- the raw tier when it holds every attended range, else the
   engine replays the path's recorded steps (each chunk's clean forward from its stored latents, each recache under
   its recorded prompt) between ``begin_replay`` and ``end_replay``.

A memory-critical section of the engine (its VAE decode) runs inside :meth:`CausalWanKVBridge.memory_critical_section`:
the decode guard frees device caches when free memory is below the section's reserve plus the working-set floor,
and new archival GPU work waits until the section ends. Every request leaves a summary (``request_summary``).
"""

from __future__ import annotations

import contextlib
import hashlib
import threading
import time
from collections import OrderedDict
from dataclasses import dataclass, field
from typing import Any

import torch

from ...errors import ConfigurationError, IntegrityError, PendingError, StateError, UnsupportedError
from .capture import CleanChunkBuilder
from .config import LATENTS_ONLY, ReelCacheRuntimeConfig
from .controls import session_control
from .generation_defer import GenerationDefer
from .lineage_archive import LineageSessionArchive
from .nodes import chunk_nodes, path_nodes
from .profiles import ModelProfile
from .restore import (GC_PAUSES, configured_verification_mode, decoder_pool_record, decoder_pool_snapshot,
                      gc_pause_record, install_gc_pauses, resident_lease_record, tier_record)
from .seam import (CLEAN_COMMIT, KV_RECACHE, CaptureScope, CausalKVRequest, ChunkSlot, KVRecache, RecachePlan,
                   ReplayStep, RestoreTarget, check_capture, drive_request, plan_recache)
from .session import SGLangSessionController, SGLangSessionState, prompt_tensor
from .visibility import VisibilityPlan, build_visibility_plan, resolve_plan
from .workload_telemetry import RequestTelemetry, WorkloadTelemetry, bytes_per_token, drain_span, request_scope

ACTIONS = ("create", "resume", "rewind", "fork")
#: Recent request summaries kept for ``request_summary`` (oldest dropped first).
MAX_REQUEST_SUMMARIES = 64
#: Memory-critical section records that ran outside any request (oldest dropped first).
MAX_UNATTRIBUTED_SECTIONS = 64
#: Visibility plans kept per bridge (a plan is a pure function of the head and the next chunk).
PLAN_CACHE_ENTRIES = 32
LATENTS_KEY = "latents"


def latents_digest(tensor: torch.Tensor) -> str:
    return hashlib.sha256(tensor.detach().float().cpu().contiguous().numpy().tobytes()).hexdigest()[:16]


@dataclass
class ResidentKV:
    """A session's native cache kept across requests: the chunks it holds, the latents of each (for recache
    windows) and the request that left it."""

    session_id: str
    request_id: Any
    cache: Any
    chunks: int
    nbytes: int
    latents: dict = field(default_factory=dict)

    def describe(self) -> dict[str, Any]:
        return {"session": self.session_id, "request": self.request_id, "chunks": self.chunks, "bytes": self.nbytes}


class PlanCache:
    """LRU of resolved visibility plans keyed by ``(head_ref, next_chunk)``; a head never changes its history, so
    an entry is valid for as long as the head exists."""

    def __init__(self, capacity: int = PLAN_CACHE_ENTRIES):
        if type(capacity) is not int or capacity < 0:
            raise ConfigurationError("plan cache capacity is a nonnegative integer")
        self.capacity = capacity
        self._plans: OrderedDict[tuple, VisibilityPlan] = OrderedDict()
        self.hits = self.misses = 0

    def get(self, key: tuple) -> VisibilityPlan | None:
        plan = self._plans.get(key)
        if plan is None:
            self.misses += 1
            return None
        self._plans.move_to_end(key)
        self.hits += 1
        return plan

    def put(self, key: tuple, plan: VisibilityPlan) -> None:
        if self.capacity == 0:
            return
        self._plans[key] = plan
        self._plans.move_to_end(key)
        while len(self._plans) > self.capacity:
            self._plans.popitem(last=False)

    def describe(self) -> dict[str, Any]:
        return {"entries": len(self._plans), "capacity": self.capacity, "hits": self.hits, "misses": self.misses}

    def clear(self) -> None:
        self._plans.clear()


class _PathLatents(dict):
    """Chunk index -> clean latents: this request's and the resident cache's first, else the chunk node's
    stored execution state (loaded on first use)."""

    def __init__(self, runtime, nodes, known: dict | None = None):
        super().__init__(known or {})
        self.runtime = runtime
        self._nodes = nodes      # chunk node refs, or a callable returning them (asked on the first miss)

    def __missing__(self, index: int) -> torch.Tensor:
        if callable(self._nodes):
            self._nodes = self._nodes()
        if not 0 <= index < len(self._nodes):
            raise KeyError(index)
        state = self.runtime.execution_state(self._nodes[index])
        if LATENTS_KEY not in state:
            raise IntegrityError(f"chunk {index} stored no latents (nothing to replay or recache it from)")
        self[index] = state[LATENTS_KEY]
        return self[index]


class CausalWanKVBridge:
    """One engine worker's archive backend: sessions, the resident cache, the request seam and its reports."""

    def __init__(self, config: ReelCacheRuntimeConfig, engine, profile: ModelProfile, *, cache_chunks: int = 16):
        self.config = config
        self.engine = engine
        self.profile = profile
        self.device = torch.device(engine.device)
        if config.cuda_memory_limit_bytes is not None and self.device.type == "cuda":
            total = torch.cuda.get_device_properties(self.device).total_memory
            torch.cuda.set_per_process_memory_fraction(min(1.0, config.cuda_memory_limit_bytes / total), self.device)
        self.archive = LineageSessionArchive(config, engine.identity, profile, self.device)
        self.sessions = SGLangSessionController(self.archive, retention=config.tree_retention,
                                                tree_switch=config.tree_switch)
        self.cache_chunks = cache_chunks
        self.telemetry = WorkloadTelemetry(enabled=config.workload_telemetry)
        self.defer = GenerationDefer.from_config(config, getattr(self.archive, "pipeline", None))
        self.plans = PlanCache()
        self._requests = 0
        self._uses = 0
        self.resident_evictions = 0
        self._active = None
        self._closed = False
        self._lock = threading.RLock()
        self._summaries: OrderedDict[Any, dict] = OrderedDict()
        self._by_session: dict[str, list] = {}
        self._unattributed: list[dict] = []
        self._boundary_hook = None
        self._inflight: list[tuple[str, dict]] = []
        install_gc_pauses()
        from ...device_pressure import register_device_trim
        self._trims = [register_device_trim("raw_tier", self._trim_raw_tier, order=5, device=self.device),
                       register_device_trim("restorer", self._trim_restorer, device=self.device),
                       register_device_trim("bridge_resident", self._trim_resident, device=self.device)]

    # -- the seam ---------------------------------------------------------------------------------------------------

    def begin_request(self, request: CausalKVRequest) -> "_BridgeRun | _ObserverRun | None":
        """Resolve the request's session action and return its run (one run at a time per bridge). A request
        without a session returns None, or an observer when ``observe_plain_requests`` is on."""
        with self._lock:
            if self._closed:
                raise StateError("the bridge is closed")
            if self._active is not None:
                raise PendingError("one causal KV request runs at a time per bridge")
            self._requests += 1
            if request.session_id is None:
                if not self.config.observe_plain_requests:
                    return None
                run = _ObserverRun(self, request)
                self._active = run
                return run
            started = time.perf_counter()
            sessions = self.sessions
            action, sid = request.action, request.session_id
            workload = RequestTelemetry(self.device) if self.config.workload_telemetry else None
            with request_scope(workload), (workload.span("request_begin", gpu=False) if workload is not None
                                           else contextlib.nullcontext()):
                if action == "create":
                    state = sessions.create(sid)
                elif action == "fork":
                    with drain_span():
                        state = sessions.fork(request.source, sid, checkpoint=request.checkpoint)
                elif action == "rewind":
                    with drain_span():
                        state = sessions.rewind(sid, request.checkpoint)
                else:
                    state = sessions.get(sid, required=False) or sessions.create(sid)
            sessions.check_ready(state)
            if state.status == "running":
                raise PendingError(f"session {sid!r} is already running")
            if (request.prompt is not None and request.prompt != state.prompt and state.generated
                    and self.profile.recache != "kv_recache"):
                raise UnsupportedError(f"profile {self.profile.name} has no KV recache: a session keeps the prompt "
                                       "it was generated under")
            state.status = "running"
            state.pause_requested = False
            state.log("request", action=action, request_id=request.request_id)
            run = _BridgeRun(self, request, state, started, workload=workload)
            self._active = run
            return run

    def request(self, session_id: str | None, *, chunks: int = 1, action: str = "resume", checkpoint: Any = None,
                source: str | None = None, seed: int = 0, prompt: str | None = None, request_id: Any = None,
                overlap_restore: bool | None = None, pause_after_chunks: int | None = None) -> dict:
        """One request through the seam on the bridge's own engine; returns its summary."""
        request = CausalKVRequest(request_id if request_id is not None else f"request-{self._requests + 1}",
                                  session_id, action, chunks, checkpoint, source, seed, prompt, overlap_restore,
                                  pause_after_chunks)
        return drive_request(self, self.engine, request)

    def _release(self, run) -> None:
        with self._lock:
            if self._active is run:
                self._active = None

    @property
    def active_request(self) -> bool:
        return self._active is not None

    # -- resident caches --------------------------------------------------------------------------------------------

    def _chunk_bytes(self) -> int:
        """Bytes of one chunk of native K/V history (16-bit cache)."""
        p = self.profile
        return 2 * p.num_layers * p.chunk_tokens * p.num_heads * p.head_dim * 2 * max(1, len(p.cfg_streams or ()))

    @staticmethod
    def _cache_bytes(cache) -> int:
        tensors = (list(cache["k"]) + list(cache["v"])) if isinstance(cache, dict) else (list(cache.k) + list(cache.v))
        return sum(t.numel() * t.element_size() for t in tensors)

    def _capacity(self, cache) -> int:
        """Chunks of history a cache can hold."""
        rows = cache["k"][0].shape[0] if isinstance(cache, dict) else cache.k[0].shape[1]
        return rows // self.profile.chunk_tokens

    def _make_resident_room(self, nbytes: int, *, keep) -> None:
        """Drop the least recently used sessions' resident caches (never ``keep``'s) until ``nbytes`` more fit
        under ``max_resident_bytes``; a dropped session restores from the raw tier or the archive next time."""
        budget = self.config.max_resident_bytes
        holders = sorted((s for s in self.sessions.resident_states() if s is not keep), key=lambda s: s.resident_used)
        total = sum(s.resident.nbytes for s in holders)
        for victim in holders:
            if total + nbytes <= budget:
                break
            total -= victim.resident.nbytes
            self._drop(victim)
            self.resident_evictions += 1

    @staticmethod
    def _drop(state: SGLangSessionState) -> None:
        state.resident = None
        state.resident_chunks = 0
        state.recaches = []

    def resident(self, session_id: str) -> dict[str, Any] | None:
        state = self.sessions.get(session_id, required=False)
        return None if state is None or state.resident is None else state.resident.describe()

    def drop_resident(self, session_id: str | None = None) -> int:
        """Forget one session's resident cache (every session's with no argument); returns how many were dropped."""
        states = self.sessions.resident_states() if session_id is None else [self.sessions.get(session_id)]
        dropped = 0
        for state in states:
            if state.resident is not None:
                dropped += 1
            self._drop(state)
        return dropped

    def _take_resident(self, state: SGLangSessionState, need: int) -> ResidentKV | None:
        """The session's resident cache when it holds the generated path and room for ``need`` chunks."""
        claim = state.resident
        if (not self.config.resident_reuse or claim is None or state.resident_chunks < state.generated
                or need > self._capacity(claim.cache)):
            return None
        return claim

    # -- sessions and controls ----------------------------------------------------------------------------------

    def open_session(self, session_id: str) -> dict[str, Any]:
        """Open a persisted session; with ``prewarm`` its attended history's packs are prepared for a restore."""
        info = self.sessions.open(session_id)
        if self.config.prewarm and hasattr(self.archive.restorer, "prewarm"):
            started = time.perf_counter()
            head = self.sessions.head(session_id)
            info["prewarmed"] = self.archive.restorer.prewarm(head) if chunk_nodes(self.archive.runtime, head) else 0
            info["prewarm_seconds"] = time.perf_counter() - started
        return info

    def pause(self, session_id: str, timeout: float | None = None) -> dict:
        """Pause a session: when it is the running request's, the request stops at its next chunk boundary."""
        state = self.sessions.get(session_id)
        if state.status == "running":
            state.pause_requested = True
            return {"session": session_id, "pause_requested": True}
        return self.sessions.pause(session_id, timeout=timeout)

    def checkpoint(self, session_id: str, name: str | None = None, timeout: float | None = None) -> dict:
        return self.sessions.checkpoint(session_id, name, timeout=timeout)

    def close(self, session_id: str, *, delete: bool = False) -> dict:
        return self.sessions.close(session_id, delete=delete)

    def drain_all(self, *, timeout: float | None = None) -> dict[str, float]:
        """Wait until every session's submitted chunks are published."""
        started = time.perf_counter()
        waited = self.archive.drain(None, timeout)
        return {"waited_seconds": waited, "seconds": time.perf_counter() - started}

    def commit_reports(self, request_id: Any, *, wait: bool = True, timeout: float | None = None) -> list[dict]:
        """The archive outcome of every chunk a request submitted (optionally after waiting for them)."""
        summary = self._summaries.get(request_id)
        if summary is None:
            raise StateError(f"no summary of request {request_id!r}")
        tickets = summary.get("_tickets", [])
        if wait:
            deadline = None if timeout is None else time.monotonic() + timeout
            for ticket in tickets:
                left = None if deadline is None else max(0.0, deadline - time.monotonic())
                ticket.result(left) if hasattr(ticket, "result") else ticket._done.wait(left)
        return [{"chunk": t.chunk_id, "state": t.state, "node": t.node_ref,
                 "error": None if t.error is None else str(t.error)} for t in tickets]

    def control(self, op: str, args: dict | None = None) -> dict[str, Any]:
        """A session control (``controls.OPS``); while a request runs, controls of its session are queued to its
        next chunk boundary (``inflight_control``)."""
        return session_control(self, op, args)

    def inflight_control(self, op: str, args: dict | None = None) -> dict[str, Any] | None:
        """Queue a control to run at the active request's next chunk boundary (None when no request runs)."""
        with self._lock:
            if self._active is None:
                return None
            self._inflight.append((op, dict(args or {})))
            return {"queued": op, "position": len(self._inflight)}

    def set_boundary_hook(self, hook) -> None:
        """``hook(run)`` runs at every chunk boundary of every request (after queued controls)."""
        self._boundary_hook = hook

    def _at_boundary(self, run, *, final: bool = False) -> list[dict]:
        """Run the queued controls (a pause of the running session marks it to stop here); ``final``: the request
        has ended, so every queued control runs as a plain control and the hook is skipped."""
        with self._lock:
            queued, self._inflight = self._inflight, []
        results = []
        for op, args in queued:
            if not final and op == "pause" and args.get("session") == getattr(run, "session_id", None):
                run.state.pause_requested = True
                results.append({"op": op, "pause_requested": True})
                continue
            try:
                results.append({"op": op, "result": self.control(op, args)})
            except Exception as error:  # noqa: BLE001 - reported in the request summary
                results.append({"op": op, "error": str(error)})
        if self._boundary_hook is not None and not final:
            self._boundary_hook(run)
        return results

    # -- reports ------------------------------------------------------------------------------------------------

    def _remember(self, request_id: Any, session_id: str | None, summary: dict) -> None:
        with self._lock:
            self._summaries[request_id] = summary
            while len(self._summaries) > MAX_REQUEST_SUMMARIES:
                old, entry = self._summaries.popitem(last=False)
                ids = self._by_session.get(entry.get("session"))
                if ids and old in ids:
                    ids.remove(old)
            if session_id is not None:
                self._by_session.setdefault(session_id, []).append(request_id)

    def request_summary(self, request_id: Any) -> dict[str, Any] | None:
        summary = self._summaries.get(request_id)
        return None if summary is None else {k: v for k, v in summary.items() if not k.startswith("_")}

    def session_requests(self, session_id: str) -> list[dict[str, Any]]:
        return [self.request_summary(r) for r in self._by_session.get(session_id, []) if r in self._summaries]

    def workload_record(self, request_id: Any) -> dict[str, Any] | None:
        summary = self._summaries.get(request_id)
        return None if summary is None else summary.get("workload")

    # -- memory-critical sections -------------------------------------------------------------------------------

    def _trim_raw_tier(self, reason: str) -> int:
        tier = self.archive.raw_tier
        return 0 if tier is None else int(tier.trim_device_cache(reason) or 0)

    def _trim_restorer(self, reason: str) -> int:
        trim = getattr(self.archive.restorer, "trim", None)
        return 0 if trim is None else int(trim() or 0)

    def _trim_resident(self, reason: str) -> int:
        """Drop idle sessions' resident caches (never the running request's)."""
        keep = getattr(self._active, "state", None)
        freed = 0
        for state in self.sessions.resident_states():
            if state is not keep:
                freed += state.resident.nbytes
                self._drop(state)
                self.resident_evictions += 1
        return freed

    def _relieve(self, reason: str, need: int) -> dict[str, Any]:
        """Free registered device caches, in trim order (raw-tier device copies, the restorer's caches, then idle
        resident caches), until ``need`` bytes are free; returns the trim record."""
        from ...device_pressure import trim_device_caches
        headroom = lambda: torch.cuda.mem_get_info(self.device)[0]  # noqa: E731
        if headroom() >= need:
            return {"trims": [], "bytes": 0}
        record = trim_device_caches(reason, device=self.device, needed_bytes=need, headroom=headroom)
        record["free_after"] = headroom()
        return record

    @contextlib.contextmanager
    def memory_critical_section(self, reason: str = "decode", *, request_id: Any = None, key: Any = None):
        """A memory-critical section of the engine (its VAE decode). The decode guard (``decode_entry_guard``)
        first frees device caches when free memory is below ``decode_reserve_prior_bytes`` (the section's need)
        plus ``decode_working_set_floor_bytes``; new archival GPU work waits for the section
        (``defer_archival_during_decode``) and a decode seam closes the request's generation hold. The record goes
        to the request's summary (or the unattributed list)."""
        run = self._active
        record: dict[str, Any] = {"reason": reason, "started": time.time()}
        clock = time.perf_counter()
        if self.config.decode_entry_guard and self.device.type == "cuda":
            need = (self.config.decode_reserve_prior_bytes or 0) + (self.config.decode_working_set_floor_bytes or 0)
            record["guard"] = {"need_bytes": need, "free_bytes": torch.cuda.mem_get_info(self.device)[0],
                               **self._relieve(reason, need)}
        pipeline = getattr(self.archive, "pipeline", None)
        key = key if key is not None else (None if run is None else run.key)
        with contextlib.ExitStack() as stack:
            if self.config.defer_archival_during_decode and pipeline is not None:
                if self.config.decode_entry_guard and hasattr(pipeline, "pause_gpu_work"):
                    record["archival_pause"] = stack.enter_context(pipeline.pause_gpu_work())
                else:
                    stack.enter_context(pipeline.defer_gpu_work())
            if self.defer is not None and key is not None:
                stack.enter_context(self.defer.decode_seam(key, reason))
            try:
                yield record
            finally:
                record["seconds"] = time.perf_counter() - clock
                target = run if run is not None and (request_id is None or request_id == run.request.request_id) \
                    else None
                if target is not None:
                    target.sections.append(record)
                else:
                    self._unattributed.append({**record, "request": request_id})
                    del self._unattributed[:-MAX_UNATTRIBUTED_SECTIONS]

    # -- lifecycle ----------------------------------------------------------------------------------------------

    def collect_garbage(self) -> dict[str, Any]:
        self.plans.clear()
        return self.sessions.gc()

    def describe(self) -> dict[str, Any]:
        return {"profile": self.profile.name, "device": str(self.device), "representation": self.config.representation,
                "requests": self._requests, "active": self._active is not None,
                "resident": [s.resident.describe() for s in self.sessions.resident_states()],
                "resident_evictions": self.resident_evictions, "plans": self.plans.describe(),
                "unattributed_sections": len(self._unattributed), "archive": self.archive.stats()}

    def shutdown(self) -> None:
        with self._lock:
            self._closed = True
        for handle in self._trims:
            handle.unregister()
        if self.defer is not None:
            self.defer.close()
        self.archive.close()


class _BridgeRun:
    """One session request in flight (returned by :meth:`CausalWanKVBridge.begin_request`)."""

    def __init__(self, bridge: CausalWanKVBridge, request: CausalKVRequest, state: SGLangSessionState, started: float,
                 *, workload: RequestTelemetry | None = None):
        self.bridge, self.request, self.state = bridge, request, state
        self.workload = workload
        self.session_id = state.session_id
        self.key = (state.session_id, request.request_id)
        self.started = started
        self.span = bridge.telemetry.begin(state.session_id, request.action)
        self.prompt = request.prompt if request.prompt is not None else state.prompt
        self.first_new = state.generated
        self._switch = request.prompt is not None and request.prompt != state.prompt and state.generated > 0
        self.route = "none"
        self.restore_report: dict[str, Any] = {}
        self.tickets: list = []
        self.chunk_marks: list[dict] = []
        self.recaches: list[dict] = []
        self.sections: list[dict] = []
        self.boundary_controls: list[dict] = []
        self.target: RestoreTarget | None = None
        self.install = None
        self._deferral = None
        self._restored = False
        self._joined = False
        self._replaying = False
        self._replay_started = None
        self.ttfc_ms = None
        self.ttfc_gpu_ms = None
        self._start_event = None
        self.paused = False
        self.last_latents = None
        self._last_capture = None
        if bridge.defer is not None:
            bridge.defer.begin(self.key)

    # -- restore --------------------------------------------------------------------------------------------------

    def _plan(self, head: str, done: int) -> VisibilityPlan:
        bridge = self.bridge
        key = (head, done)
        plan = bridge.plans.get(key)
        if plan is None:
            runtime = bridge.archive.runtime
            plan = resolve_plan(runtime, head, build_visibility_plan(bridge.profile, chunk_nodes(runtime, head), done))
            bridge.plans.put(key, plan)
        return plan

    def restore(self, target: RestoreTarget) -> int:
        """Put the session's attended history into ``target.cache``; returns the chunks already generated."""
        if self._restored:
            raise StateError("restore runs once per request")
        self._restored = True
        bridge, state = self.bridge, self.state
        self.target = target
        done = state.generated
        need = done + self.request.chunks
        clock = time.perf_counter()
        if bridge.device.type == "cuda":
            self._start_event = torch.cuda.Event(enable_timing=True)
            self._start_event.record()
        claim = bridge._take_resident(state, need)
        runtime = bridge.archive.runtime
        self._gc_before = GC_PAUSES.snapshot()
        self._pool_before = decoder_pool_snapshot(getattr(bridge.archive, "decoder_pool", None))
        verification = configured_verification_mode(bridge.config)
        if claim is not None:
            target.cache = claim.cache
            self.route = "resident"
            known = {i: t for i, t in claim.latents.items() if i < done}

            def published_nodes():
                bridge.archive.drain(state.session_id)
                return chunk_nodes(runtime, bridge.sessions.head(state.session_id))
            target.latents = _PathLatents(runtime, published_nodes, known)
            self.restore_report = {"mode": "resident", "chunks": done, "from_request": claim.request_id,
                                   "lease": resident_lease_record(range(done), verification_mode=verification)}
        else:
            bridge._drop(state)
            capacity = max(need, bridge.cache_chunks)
            bridge._make_resident_room(capacity * bridge._chunk_bytes(), keep=state)
            target.cache = bridge.engine.new_cache(capacity) if target.engine is bridge.engine else \
                target.engine.new_cache(capacity)
            if done == 0:
                target.latents = _PathLatents(runtime, [])
                self.restore_report = {"mode": "none", "chunks": 0}
            else:
                if any(not t.done() for t in state.pending) or len(bridge.sessions.chunks(state.session_id)) < done:
                    bridge.archive.drain(state.session_id)  # the history to restore must be published
                head = bridge.sessions.head(state.session_id)
                nodes = chunk_nodes(runtime, head)
                target.latents = _PathLatents(runtime, nodes)
                plan = self._plan(head, done)
                self.span.mark("restore_issue")
                with (self.workload.span("restore_sync") if self.workload is not None
                      else contextlib.nullcontext()), request_scope(self.workload):
                    if bridge.config.restore_mode == "recompute":
                        self._recompute(target, head, plan, done)
                    else:
                        tier = bridge.archive.raw_tier
                        held = set()
                        if tier is not None and bridge.config.raw_restore == "prefer":
                            for holder in {span.node_ref for span in plan.spans}:
                                lease = tier.lookup(holder)
                                if lease is not None:
                                    held.add(holder)
                                    lease.release()
                        self._archive_install(target, head, plan)
                        self.restore_report["lease"] = tier_record(plan, held, verification_mode=verification)
                if self.workload is not None:
                    p = bridge.profile
                    self.workload.set_restore(self.restore_report, tokens=plan.attended_tokens,
                                              per_token=bytes_per_token(num_layers=p.num_layers, num_heads=p.num_heads,
                                                                        head_dim=p.head_dim,
                                                                        capture_dtypes=p.capture_dtypes))
        if self.workload is not None and target.layer_wait is not None:
            target.layer_wait = self.workload.wrap_wait(target.layer_wait)
        self.restore_report["seconds"] = time.perf_counter() - clock
        return done

    def _archive_install(self, target: RestoreTarget, head: str, plan: VisibilityPlan) -> None:
        bridge = self.bridge
        overlapped = bridge.config.overlap_restore if self.request.overlap_restore is None \
            else self.request.overlap_restore
        pipeline = bridge.archive.pipeline
        paused = None
        if bridge.config.archival_pump_pause and hasattr(pipeline, "defer_gpu_work"):
            # released when the install is joined; a node already planning pauses at its next step boundary
            self._deferral = pipeline.pause_gpu_work() if hasattr(pipeline, "pause_gpu_work") else \
                pipeline.defer_gpu_work()
            paused = self._deferral.__enter__()
        self.install = target.engine.install(target.cache, bridge.archive, head, plan, overlapped=overlapped)
        target.layer_wait = self.install.wait
        self.route = "archive"
        self.restore_report = {"mode": "archive", "head": head, "attended_tokens": plan.attended_tokens,
                               "spans": len(plan.spans), "overlapped": bool(overlapped)}
        if self._deferral is not None and isinstance(paused, dict):
            self.restore_report["archival_pause"] = paused

    def _tier_holds(self, plan: VisibilityPlan) -> bool:
        tier = self.bridge.archive.raw_tier
        if tier is None or self.bridge.config.raw_restore == "off":
            return False
        for holder in {span.node_ref for span in plan.spans}:
            lease = tier.lookup(holder)
            if lease is None:
                return False
            lease.release()
        return True

    def _recompute(self, target: RestoreTarget, head: str, plan: VisibilityPlan, done: int) -> None:
        """The raw tier when it holds every attended range, else the replay steps of the head's path."""
        if self._tier_holds(plan):
            self.install = target.engine.install(target.cache, self.bridge.archive, head, plan, overlapped=False)
            self.route = "raw_tier"
            self.restore_report = {"mode": "raw_tier", "head": head, "attended_tokens": plan.attended_tokens}
            return
        runtime = self.bridge.archive.runtime
        profile = self.bridge.profile
        steps, chunk = [], 0
        for node in path_nodes(runtime, head)[1:]:
            state = runtime.execution_state(node.node_ref)
            prompt = None if "prompt" not in state else bytes(state["prompt"].tolist()).decode()
            if node.kind == "chunk":
                if LATENTS_KEY not in state:
                    raise IntegrityError(f"chunk {chunk} stored no latents: it cannot be replayed")
                target.latents[chunk] = state[LATENTS_KEY]
                steps.append(ReplayStep("chunk", ChunkSlot.of(profile, chunk), prompt, state[LATENTS_KEY]))
                chunk += 1
            elif node.kind == "recache":
                details = runtime.load_epoch(runtime.load_node(node.node_ref).epoch_ref).details
                plan_record = details.get("plan")
                if plan_record is None:
                    raise IntegrityError("a recache node recorded no plan: it cannot be replayed")
                steps.append(ReplayStep("recache", None, prompt, plan=RecachePlan(**plan_record)))
        target.replay = steps
        self.route = "recompute"
        self.restore_report = {"mode": "recompute", "head": head, "steps": len(steps), "chunks": done}

    def begin_replay(self) -> dict[str, Any]:
        if self.route != "recompute" or self._replaying:
            raise StateError("no replay is pending for this request")
        self._replaying = True
        self._replay_started = time.perf_counter()
        self._replay_span = None if self.workload is None else self.workload.begin("replay")
        return {"steps": len(self.target.replay)}

    def end_replay(self) -> dict[str, Any]:
        if not self._replaying:
            raise StateError("end_replay without begin_replay")
        self._replaying = False
        if self.workload is not None:
            self.workload.end(self._replay_span)
        seconds = time.perf_counter() - self._replay_started
        self.restore_report["replay_seconds"] = seconds
        return {"steps": len(self.target.replay), "seconds": seconds}

    def _join_install(self, *, error: BaseException | None = None) -> None:
        """Wait for the restore (once); generation proper starts here (the generation hold opens)."""
        if self._joined:
            return
        self._joined = True
        install, self.install = self.install, None
        try:
            if install is not None:
                stats = install.join()
                self.restore_report["stats"] = stats if stats is not None else install.stats
        finally:
            if getattr(self, "_gc_before", None) is not None:
                self.restore_report["gc"] = gc_pause_record(self._gc_before, GC_PAUSES.snapshot())
                self.restore_report["decoder_pool"] = decoder_pool_record(
                    self._pool_before, decoder_pool_snapshot(getattr(self.bridge.archive, "decoder_pool", None)))
            self._release_deferral()
            if self.bridge.defer is not None and error is None:
                self.bridge.defer.after_restore(self.key)

    def _release_deferral(self) -> None:
        if self._deferral is not None:
            deferral, self._deferral = self._deferral, None
            deferral.__exit__(None, None, None)

    # -- recache --------------------------------------------------------------------------------------------------

    def needs_recache(self, index: int) -> bool:
        """Whether a prompt switch re-runs the recache window before chunk ``index`` (the request's first)."""
        return self._switch and index == self.first_new and not self.recaches

    def begin_recache(self, index: int) -> KVRecache:
        bridge, profile = self.bridge, self.bridge.profile
        if not self.needs_recache(index):
            raise StateError(f"no recache is due before chunk {index}")
        self._join_install()
        window = profile.window_frames if profile.visibility == "sink_window" else -1
        plan = plan_recache(generated_frames=index * profile.chunk_frames, window_frames=window,
                            sink_frames=profile.sink_frames, frame_tokens=profile.tokens_per_frame,
                            chunk_frames=profile.chunk_frames, global_sink=True)
        written_start, written_end = plan.written_tokens
        frames = (written_end - written_start) // profile.tokens_per_frame
        h, w = profile.grid
        builder = None
        if frames:
            builder = CleanChunkBuilder(bridge.engine.identity, index, written_start, frames, h, w,
                                        profile.cfg_streams)
        epoch = f"recache-{index}-{hashlib.sha256(self.prompt.encode()).hexdigest()[:12]}"
        self._recache_span = None if self.workload is None else self.workload.begin("recache")
        return KVRecache(plan, epoch, self.prompt, CaptureScope(KV_RECACHE, ChunkSlot.of(profile, index), builder))

    def end_recache(self, recache: KVRecache) -> dict[str, Any]:
        """Commit what the recache wrote back as a ``kv_recache`` epoch: one range per re-materialized chunk,
        never the sink; a latents-only archive records the ranges without KV."""
        bridge, profile, state = self.bridge, self.bridge.profile, self.state
        scope = recache.capture
        scope.ended = True
        if not scope.complete:
            raise IntegrityError("recache ended without a complete clean capture")
        plan = recache.plan
        record = {"epoch": recache.epoch_id, "plan": plan.to_dict(), "written": recache.written}
        node_ref = None
        if scope.builder is not None:
            matrices, _ = scope.builder.seal()
            per_chunk = profile.chunk_tokens
            ranges = []
            h, w = profile.grid
            for index in range(plan.write_start_frame // profile.chunk_frames, plan.end_frame // profile.chunk_frames):
                offset = index * per_chunk - plan.written_tokens[0]
                piece = CleanChunkBuilder(bridge.engine.identity, index, index * per_chunk, profile.chunk_frames, h, w,
                                          profile.cfg_streams)
                piece.matrices = {entry: tensor[offset:offset + per_chunk] for entry, tensor in matrices.items()}
                chunk_matrices, contexts = piece.seal()
                ranges.append((f"chunk-{index}", chunk_matrices, contexts))
            plan_fields = {"before_chunk": plan.before_chunk, "window_start_frame": plan.window_start_frame,
                           "end_frame": plan.end_frame, "write_start_frame": plan.write_start_frame,
                           "frame_tokens": plan.frame_tokens, "sink_frames": plan.sink_frames}
            details = {"cause": recache.cause, "plan": plan_fields, "written": [list(r) for r in recache.written]}
            node_ref = bridge.archive.commit_recache(state.session_id, f"recache-{recache.epoch_id}", ranges,
                                                     epoch_id=recache.epoch_id, details=details,
                                                     execution_state=prompt_tensor(recache.prompt))
            record["ranges"] = [r[0] for r in ranges]
        record["node"] = node_ref
        if self.workload is not None:
            self.workload.end(getattr(self, "_recache_span", None))
        state.prompt = recache.prompt
        state.recaches.append(plan.before_chunk)
        state.log("recache", epoch=recache.epoch_id, node=node_ref)
        self.recaches.append(record)
        return record

    # -- capture and commit ---------------------------------------------------------------------------------------

    def begin_clean_forward(self, slot: ChunkSlot) -> CaptureScope:
        if self.target is None:
            raise StateError("restore runs before the first clean forward")
        profile = self.bridge.profile
        h, w = profile.grid
        builder = CleanChunkBuilder(self.bridge.engine.identity, slot.index, slot.token_start, slot.num_frames, h, w,
                                    profile.cfg_streams)
        if self.workload is not None and slot.index == self.first_new:
            self.workload.mark_generation()
            self._first_span = self.workload.begin("first_forward")
        return CaptureScope(CLEAN_COMMIT, slot, builder)

    @staticmethod
    def capture_layer(capture: CaptureScope, layer: int, key: torch.Tensor, value: torch.Tensor,
                      stream: str = "cond") -> None:
        capture.capture_layer(layer, key, value, stream)

    def end_clean_forward(self, capture: CaptureScope) -> None:
        capture.ended = True
        capture.forwards += 1
        self._last_capture = capture
        if self.bridge.config.verify_capture_rope and capture.builder is not None and self.target is not None:
            check = getattr(self.target.engine, "rope_check", None)
            if check is not None:
                entry = capture.builder.entry(0, "K", capture.builder.streams[0])
                error = check(self.target.cache, 0, capture.slot.token_start, capture.builder.matrices[entry])
                if error is not None and error > 0.0625:
                    raise IntegrityError(f"captured K of chunk {capture.slot.index} is not the pre-RoPE K the cache "
                                         f"holds (max error {error:.3g})")

    def end_chunk(self, slot: ChunkSlot, latents: torch.Tensor) -> bool:
        """Submit the chunk to the archive; returns True when the request stops here (a pause at this boundary)."""
        bridge, state = self.bridge, self.state
        capture, self._last_capture = self._last_capture, None
        if slot.index != state.generated:
            raise IntegrityError(f"chunk {slot.index} is not the session's next chunk ({state.generated})")
        if slot.index == self.first_new:
            self._join_install()
            cuda = bridge.device.type == "cuda"
            if cuda:
                first = torch.cuda.Event(enable_timing=True)
                first.record()
                first.synchronize()
                if self._start_event is not None:
                    self.ttfc_gpu_ms = self._start_event.elapsed_time(first)
            self.ttfc_ms = (time.perf_counter() - self.started) * 1e3
            self.span.mark("first_chunk")
            if self.workload is not None:
                self.workload.end(getattr(self, "_first_span", None))
        if self.workload is None:
            return self._commit(slot, latents, capture)
        with self.workload.span("chunk_commit", gpu=False):
            return self._commit(slot, latents, capture)

    def _commit(self, slot: ChunkSlot, latents: torch.Tensor, capture: CaptureScope | None) -> bool:
        bridge, state = self.bridge, self.state
        if capture is None:
            raise IntegrityError(f"chunk {slot.index} ended without a clean capture")
        check_capture(capture, CLEAN_COMMIT, slot)
        matrices, contexts = capture.builder.seal()
        capture_event = None
        if bridge.device.type == "cuda":
            capture_event = torch.cuda.Event()
            capture_event.record()
        stored = latents.detach().to("cpu", copy=True)
        execution_state = {LATENTS_KEY: stored, **prompt_tensor(self.prompt)}
        ticket = bridge.archive.commit_chunk(state.session_id, f"chunk-{slot.index}", matrices, contexts,
                                             execution_state=execution_state, capture_event=capture_event)
        self.tickets.append(ticket)
        state.pending.append(ticket)
        state.generated = slot.index + 1
        state.prompt = self.prompt
        self.target.latents[slot.index] = stored
        self.last_latents = latents
        self.chunk_marks.append({"chunk": slot.index, "latents": latents_digest(stored),
                                 "submitted_seconds": time.perf_counter() - self.started})
        if bridge.config.durability == "always":
            bridge.archive.drain(state.session_id)
        self.boundary_controls.extend(bridge._at_boundary(self))
        done = state.generated - self.first_new
        pause = state.pause_requested or (self.request.pause_after_chunks is not None
                                          and done >= self.request.pause_after_chunks)
        if pause and done < self.request.chunks:
            self.paused = True
            return True
        return False

    # -- finish ---------------------------------------------------------------------------------------------------

    def finish(self, *, error: BaseException | None) -> dict[str, Any]:
        """End the request (always called): keep the cache resident on success, then file the summary."""
        bridge, state = self.bridge, self.state
        try:
            try:
                self._join_install(error=error)
            except BaseException as join_error:  # noqa: BLE001 - the stage's own error wins
                if error is None:
                    error = join_error
            if error is None and self.target is not None and self.target.cache is not None:
                if bridge.config.resident_reuse:
                    bridge._uses += 1
                    latents = {i: t for i, t in self.target.latents.items() if isinstance(i, int)}
                    state.resident = ResidentKV(state.session_id, self.request.request_id, self.target.cache,
                                                state.generated, bridge._cache_bytes(self.target.cache), latents)
                    state.resident_chunks = state.generated
                    state.resident_used = bridge._uses
                else:
                    bridge._drop(state)
            elif error is not None:
                bridge._drop(state)  # the cache may hold a partial chunk
            bridge.sessions.reconcile(state)
            if state.failure is None:
                state.status = "paused" if (self.paused and state.pause_requested) else "idle"
            if state.pause_requested and error is None:
                state.pause_requested = False
            if state.status == "running":
                state.status = "idle"
            self.boundary_controls.extend(bridge._at_boundary(self, final=True))
            deferral = bridge.defer.finish(self.key) if bridge.defer is not None else None
            summary = {
                "request": self.request.request_id, "session": state.session_id, "action": self.request.action,
                "start_chunk": self.first_new, "chunks": state.generated - self.first_new,
                "requested_chunks": self.request.chunks, "generated": state.generated, "route": self.route,
                "restore": self.restore_report, "ttfc_ms": self.ttfc_ms, "prompt": self.prompt,
                "recaches": self.recaches, "paused": self.paused, "tickets": [t.chunk_id for t in self.tickets],
                "frontiers": bridge.archive.pipeline.frontiers(state.session_id), "chunk_marks": self.chunk_marks,
                "sections": self.sections, "boundary_controls": self.boundary_controls,
                "wall_ms": (time.perf_counter() - self.started) * 1e3,
                "error": None if error is None else f"{type(error).__name__}: {error}",
                "latents": self.last_latents, "_tickets": list(self.tickets),
            }
            if self.ttfc_gpu_ms is not None:
                summary["ttfc_gpu_ms"] = self.ttfc_gpu_ms
            if self.workload is not None:
                summary["workload"] = self.workload.resolve()
            if deferral is not None:
                summary["archival_defer"] = deferral
            bridge.telemetry.end(self.span, summary)
            bridge._remember(self.request.request_id, state.session_id, summary)
            return {k: v for k, v in summary.items() if not k.startswith("_")}
        finally:
            if state.status == "running":
                state.status = "idle"
            bridge._release(self)


class _ObserverRun:
    """A plain request (no session) the bridge observes: timings only, nothing archived or restored."""

    def __init__(self, bridge: CausalWanKVBridge, request: CausalKVRequest):
        self.bridge, self.request = bridge, request
        self.key = (None, request.request_id)
        self.session_id = None
        self.started = time.perf_counter()
        self.target = None
        self.chunks = 0
        self.ttfc_ms = None
        self.sections: list[dict] = []
        self.prompt = request.prompt

    def restore(self, target: RestoreTarget) -> int:
        self.target = target
        target.cache = target.engine.new_cache(max(self.request.chunks, self.bridge.cache_chunks))
        target.latents = {}
        return 0

    def needs_recache(self, index: int) -> bool:
        return False

    def begin_clean_forward(self, slot: ChunkSlot) -> CaptureScope:
        return CaptureScope(CLEAN_COMMIT, slot, None)

    @staticmethod
    def capture_layer(capture: CaptureScope, layer: int, key: torch.Tensor, value: torch.Tensor,
                      stream: str = "cond") -> None:
        return None

    def end_clean_forward(self, capture: CaptureScope) -> None:
        capture.ended = True

    def end_chunk(self, slot: ChunkSlot, latents: torch.Tensor) -> bool:
        self.chunks += 1
        if self.ttfc_ms is None:
            self.ttfc_ms = (time.perf_counter() - self.started) * 1e3
        return False

    def begin_replay(self):
        raise StateError("a plain request has no history to replay")

    end_replay = begin_replay

    def finish(self, *, error: BaseException | None) -> dict[str, Any]:
        summary = {"request": self.request.request_id, "session": None, "observed": True, "chunks": self.chunks,
                   "ttfc_ms": self.ttfc_ms, "wall_ms": (time.perf_counter() - self.started) * 1e3,
                   "sections": self.sections, "error": None if error is None else f"{type(error).__name__}: {error}"}
        self.bridge._remember(self.request.request_id, None, summary)
        self.bridge._release(self)
        return summary
