"""The serving bridge: the engine seam between a chunked video-generation engine and the archive
(the counterpart of reference reelcache/integrations/sglang/bridge.py:875-3173).

A request (``request``) runs one action on a session -- create / resume / rewind / fork -- and then
generates chunks:

1. **Restore**: the session's resident cache is reused when it already holds the target path
   (``resident_reuse``; a rewind onto a prefix of the resident path is free); otherwise the attended
   history (:func:`build_visibility_plan`) is installed from the raw tier or the archive, overlapped
   layer by layer with the first denoising forward (``overlap_restore``).
2. **Generate**: per chunk, the engine's clean forward hands every layer's pre-RoPE K / V to a
   :class:`CleanChunkBuilder`.
3. **Commit**: the sealed chunk goes to the asynchronous archive (``durability="always"`` drains
   after every chunk; ``"pause"`` makes ``pause``/``checkpoint`` the durability points).

``request`` returns a report: time to first chunk (``ttfc_ms``, host wall clock and, on CUDA, device
events), the restore's route and statistics, the archive tickets and frontiers.
"""

from __future__ import annotations

import contextlib
import threading
import time
from typing import Any

import torch

from ...errors import ConfigurationError, StateError
from .capture import CleanChunkBuilder
from .config import ReelCacheRuntimeConfig
from .generation_defer import GenerationDefer
from .lineage_archive import LineageSessionArchive
from .nodes import chunk_nodes
from .profiles import ModelProfile
from .session import SGLangSessionController
from .visibility import build_visibility_plan
from .workload_telemetry import WorkloadTelemetry

ACTIONS = ("create", "resume", "rewind", "fork")


class CausalWanKVBridge:
    def __init__(self, config: ReelCacheRuntimeConfig, engine, profile: ModelProfile, *, cache_chunks: int = 16):
        self.config = config
        self.engine = engine
        self.profile = profile
        self.device = torch.device(engine.device)
        self.archive = LineageSessionArchive(config, engine.identity, profile, self.device)
        self.sessions = SGLangSessionController(self.archive)
        self.cache_chunks = cache_chunks
        self.telemetry = WorkloadTelemetry(enabled=config.workload_telemetry)
        self.defer = GenerationDefer.from_config(config, getattr(self.archive, "pipeline", None))
        self._requests = 0
        self._uses = 0
        self.resident_evictions = 0
        self._current = None
        self._lock = threading.RLock()

    # -- requests -------------------------------------------------------------------------------------------------

    def request(self, session_id: str, *, chunks: int = 1, action: str = "resume", checkpoint: Any = None,
                source: str | None = None, seed: int = 0) -> dict:
        if action not in ACTIONS:
            raise ConfigurationError(f"action must be one of {ACTIONS}")
        if type(chunks) is not int or chunks < 0:
            raise ConfigurationError("chunks must be a nonnegative integer")
        started = time.perf_counter()
        span = self.telemetry.begin(session_id, action)
        self._requests += 1
        key = (session_id, self._requests)
        self._current = key
        if self.defer is not None:
            self.defer.begin(key)
        with self._lock:
            if action == "create":
                state = self.sessions.create(session_id)
            elif action == "fork":
                if source is None:
                    raise ConfigurationError("fork needs a source session")
                state = self.sessions.fork(source, session_id, checkpoint=checkpoint)
            elif action == "rewind":
                state = self.sessions.rewind(session_id, checkpoint)
            else:
                state = self.sessions.get(session_id, required=False) or self.sessions.create(session_id)
            self.sessions.check_ready(state)
            state.status = "running"
        try:
            report = self._run(state, chunks, seed, started, span, key)
        except BaseException:
            state.status = "failed" if state.failure is not None else "idle"
            if self.defer is not None:
                self.defer.finish(key)
            raise
        state.status = "idle"
        if self.defer is not None:
            report["archival_defer"] = self.defer.finish(key)
        report["action"] = action
        report["wall_ms"] = (time.perf_counter() - started) * 1e3
        self.telemetry.end(span, report)
        return report

    def _run(self, state, chunks: int, seed: int, started: float, span, key=None) -> dict:
        start_chunk = state.generated
        need = start_chunk + chunks
        cache = state.resident
        route = "resident"
        install = None
        restore_stats: dict = {}
        if not (self.config.resident_reuse and cache is not None and state.resident_chunks >= start_chunk
                and need <= self._capacity(cache)):
            capacity = max(need, self.cache_chunks)
            state.resident = None  # replaced below; its memory may be reused
            self._make_resident_room(capacity * self._chunk_bytes(), keep=state)
            cache = self.engine.new_cache(capacity)
            route = "none"
            if start_chunk > 0:
                published = len(self.sessions.chunks(state.session_id))
                if published < start_chunk:
                    self.archive.drain(state.session_id)  # the history to restore must be published
                head = self.sessions.head(state.session_id)
                plan = build_visibility_plan(self.profile, chunk_nodes(self.archive.runtime, head), start_chunk)
                span.mark("restore_issue")
                install = self.engine.install(cache, self.archive, head, plan, overlapped=self.config.overlap_restore)
                route = "archive"
        cuda = self.device.type == "cuda"
        first_event = None
        if cuda:
            start_event = torch.cuda.Event(enable_timing=True)
            start_event.record()
        latents = None
        tickets = []
        ttfc_ms = None
        for i in range(chunks):
            index = start_chunk + i
            frames, (h, w) = self.profile.chunk_frames, self.profile.grid
            builder = CleanChunkBuilder(self.engine.identity, index, index * self.profile.chunk_tokens, frames, h, w,
                                        self.profile.cfg_streams)
            wait = install.wait if (install is not None and i == 0) else None
            latents = self.engine.generate_chunk(cache, index, builder, request_seed=seed, layer_wait=wait)
            if i == 0:
                if install is not None:
                    restore_stats = install.join() or install.stats
                if self.defer is not None:
                    self.defer.after_restore(key)  # generation starts once the restore has returned
                if cuda:
                    first_event = torch.cuda.Event(enable_timing=True)
                    first_event.record()
                    first_event.synchronize()
                ttfc_ms = (time.perf_counter() - started) * 1e3
                span.mark("first_chunk")
            matrices, contexts = builder.seal()
            capture_event = None
            if cuda:
                capture_event = torch.cuda.Event()
                capture_event.record()
            ticket = self.archive.commit_chunk(state.session_id, f"chunk-{index}", matrices, contexts,
                                               capture_event=capture_event)
            tickets.append(ticket)
            state.pending.append(ticket)
            state.generated = index + 1
            if self.config.durability == "always":
                self.archive.drain(state.session_id)
        state.resident = cache
        state.resident_chunks = state.generated
        self._uses += 1
        state.resident_used = self._uses
        self.sessions.reconcile(state)
        report = {"session": state.session_id, "start_chunk": start_chunk, "chunks": chunks, "route": route,
                  "ttfc_ms": ttfc_ms, "restore": restore_stats, "generated": state.generated,
                  "tickets": [t.chunk_id for t in tickets], "frontiers": self.archive.pipeline.frontiers(state.session_id),
                  "latents": latents}
        if cuda and first_event is not None:
            report["ttfc_gpu_ms"] = start_event.elapsed_time(first_event)
        return report

    def _chunk_bytes(self) -> int:
        """Bytes of one chunk of native K/V history (16-bit cache)."""
        p = self.profile
        return 2 * p.num_layers * p.chunk_tokens * p.num_heads * p.head_dim * 2 * max(1, len(p.cfg_streams or ()))

    @staticmethod
    def _cache_bytes(cache) -> int:
        tensors = (list(cache["k"]) + list(cache["v"])) if isinstance(cache, dict) else (list(cache.k) + list(cache.v))
        return sum(t.numel() * t.element_size() for t in tensors)

    def _make_resident_room(self, nbytes: int, *, keep) -> None:
        """Drop the least recently used sessions' resident caches (never ``keep``'s) until ``nbytes`` more fit
        under ``max_resident_bytes``; a dropped session restores from the raw tier or the archive next time."""
        budget = self.config.max_resident_bytes
        holders = sorted((s for s in self.sessions.resident_states() if s is not keep), key=lambda s: s.resident_used)
        total = sum(self._cache_bytes(s.resident) for s in holders)
        for victim in holders:
            if total + nbytes <= budget:
                break
            total -= self._cache_bytes(victim.resident)
            victim.resident = None
            victim.resident_chunks = 0
            self.resident_evictions += 1

    def _capacity(self, cache) -> int:
        """Chunks of history a cache can hold."""
        rows = cache["k"][0].shape[0] if isinstance(cache, dict) else cache.k[0].shape[1]
        return rows // self.profile.chunk_tokens

    @contextlib.contextmanager
    def memory_critical_section(self, reason: str = "decode", key=None):
        """A memory-critical section of the current request (the engine's VAE decode): new GPU archival work
        is deferred inside it (``defer_archival_during_decode``), and a decode seam closes the request's
        generation hold at its exit."""
        key = key if key is not None else self._current
        defer_gpu = (self.config.defer_archival_during_decode and getattr(self.archive, "pipeline", None)
                     is not None)
        with contextlib.ExitStack() as stack:
            if defer_gpu:
                stack.enter_context(self.archive.pipeline.defer_gpu_work())
            if self.defer is not None and key is not None:
                stack.enter_context(self.defer.decode_seam(key, reason))
            yield

    # -- controls -----------------------------------------------------------------------------------------------

    def pause(self, session_id: str, timeout: float | None = None) -> dict:
        return self.sessions.pause(session_id, timeout=timeout)

    def checkpoint(self, session_id: str, name: str | None = None, timeout: float | None = None) -> dict:
        return self.sessions.checkpoint(session_id, name, timeout=timeout)

    def close(self, session_id: str, *, delete: bool = False) -> dict:
        return self.sessions.close(session_id, delete=delete)

    def drop_resident(self, session_id: str) -> None:
        state = self.sessions.get(session_id)
        state.resident = None
        state.resident_chunks = 0

    def shutdown(self) -> None:
        if self.defer is not None:
            self.defer.close()
        self.archive.close()
