"""LongCat-Video sessions: per-epoch raw tiers, the group-level planning gate and the segment session provider (the
counterpart of reference reelcache_sglang_models/longcat_video/raw_tiers.py:236-692, planning_gate.py:51-317,
session_provider.py:275-1909, session_archive.py:92 and segment_resume.py).

* :class:`EpochRawTiers` keeps a segment epoch's conditioning cache (48 x pre-RoPE K/V) in front of the archive:
  ``gpu_raw`` (the built cache left on the device, within a byte budget), ``host_raw`` (a pinned host copy, the
  archive's source until the epoch's node is published, then an LRU entry) and ``compressed`` (the published
  node). Entries are keyed by the epoch's *content key* (model fingerprint, conditioning-latent digest, token grid),
  so regenerated or rewound epochs with other content never share an entry. Invariant: until an entry is
  published at least one complete copy exists (its GPU copy is dropped only after the host copy is complete, and
  an unpublished host copy is never evicted; :class:`HostFull` when every slot holds an unpublished epoch).
  RoPE is applied inside attention, so every raw copy is bitwise the native build.
* :class:`PlanningGate` gates the GPU part of archival one planner unit (matrix) at a time: a unit starts only
  while no memory-critical section (denoising, VAE decode) is open or waiting; a section waits only for the unit
  in progress. :func:`gated_plan_chunk` plans exactly like :func:`reelcache_b200.rank_method.plan_chunk`, one
  matrix per unit, with the sources on the host between units.
* :class:`LongCatSessionProvider` makes segment boundaries the session units: each segment's conditioning cache
  is restored from the best tier (or built), captured into the tiers and archived as a segment node; the
  session's boundaries are recorded in the store (``longcat/sessions/<id>``), so :meth:`resume` continues a
  session from any recorded boundary.
"""

from __future__ import annotations

import contextlib
import hashlib
import threading
import time
from collections import OrderedDict
from dataclasses import dataclass, field
from typing import Any, Mapping

import torch

from ..errors import CapacityError, ConfigurationError, StateError
from .longcat import ConditioningCacheEpoch, LongCatConditioningCache

SESSION_PREFIX = "longcat/sessions/"
SESSION_SCHEMA = "reelcache.longcat_session.v1"
RECORD_TIERS = ("resident", "gpu_raw", "host_raw", "compressed_prepared", "compressed_cold", "built")


class HostFull(CapacityError):
    """Every host slot holds an unpublished epoch: wait for the oldest to publish."""


def content_key(model_fingerprint: str, cond_latents: torch.Tensor, grid: tuple[int, int]) -> str:
    digest = hashlib.sha256(cond_latents.detach().contiguous().cpu().view(torch.uint8).numpy().tobytes()).hexdigest()
    return hashlib.sha256(f"{model_fingerprint}:{digest}:{tuple(grid)}:{tuple(cond_latents.shape)}".encode()
                          ).hexdigest()


@dataclass(eq=False)
class EpochEntry:
    key: str
    epoch: ConditioningCacheEpoch
    gpu: LongCatConditioningCache | None
    host: LongCatConditioningCache | None
    nbytes: int
    node_ref: str | None = None
    last_used: float = field(default_factory=time.monotonic)

    @property
    def published(self) -> bool:
        return self.node_ref is not None


def _copy_cache(cache: LongCatConditioningCache, device, *, pin: bool = False) -> LongCatConditioningCache:
    def move(t):
        if pin and torch.device(device).type == "cpu" and torch.cuda.is_available():
            # one copy straight into page-locked memory (not a pageable copy followed by a pinned one)
            out = torch.empty(t.shape, dtype=t.dtype, device="cpu", pin_memory=True)
            return out.copy_(t.detach())
        return t.detach().to(device, copy=True)
    return LongCatConditioningCache(cache.epoch, [move(k) for k in cache.k], [move(v) for v in cache.v])


class EpochRawTiers:
    """Per-epoch raw tiers (module docstring)."""

    def __init__(self, *, gpu_raw_budget_bytes: int = 0, host_raw_budget_bytes: int = 32 << 30,
                 host_slots: int | None = None, pin_memory: bool = True):
        self.gpu_budget, self.host_budget = gpu_raw_budget_bytes, host_raw_budget_bytes
        self.host_slots = host_slots
        self.pin_memory = pin_memory
        self.entries: OrderedDict[str, EpochEntry] = OrderedDict()
        self.records = {"captures": 0, "hits": {t: 0 for t in RECORD_TIERS}, "evictions": 0}
        self._lock = threading.Lock()

    def capture(self, key: str, cache: LongCatConditioningCache) -> EpochEntry:
        """Adopt a freshly built cache: host copy first (complete before any GPU copy can be dropped)."""
        with self._lock:
            if key in self.entries:
                return self.entries[key]
            unpublished = [e for e in self.entries.values() if not e.published]
            if self.host_slots is not None and len(unpublished) >= self.host_slots:
                raise HostFull("every host slot holds an unpublished epoch")
        host = _copy_cache(cache, "cpu", pin=self.pin_memory)
        gpu = cache if cache.k[0].is_cuda and self.gpu_budget >= cache.nbytes else None
        entry = EpochEntry(key, cache.epoch, gpu, host, cache.nbytes)
        with self._lock:
            self.entries[key] = entry
            self.records["captures"] += 1
            self._evict()
        return entry

    def published(self, key: str, node_ref: str) -> None:
        with self._lock:
            entry = self.entries.get(key)
            if entry is not None:
                entry.node_ref = node_ref
                self._evict()

    def lookup(self, key: str, device) -> tuple[str, LongCatConditioningCache] | None:
        with self._lock:
            entry = self.entries.get(key)
            if entry is None:
                return None
            entry.last_used = time.monotonic()
            self.entries.move_to_end(key)
            gpu, host = entry.gpu, entry.host
        if gpu is not None:
            self.records["hits"]["gpu_raw"] += 1
            return "gpu_raw", gpu
        if host is not None:
            self.records["hits"]["host_raw"] += 1
            return "host_raw", _copy_cache(host, device)
        return None

    def node_of(self, key: str) -> str | None:
        entry = self.entries.get(key)
        return None if entry is None else entry.node_ref

    def _evict(self) -> None:
        """Drop GPU copies over the GPU budget (host copy complete), then published host copies over the host
        budget, least recently used first. Called under the lock."""
        gpu_total = sum(e.nbytes for e in self.entries.values() if e.gpu is not None)
        for entry in sorted(self.entries.values(), key=lambda e: e.last_used):
            if gpu_total <= self.gpu_budget:
                break
            if entry.gpu is not None and entry.host is not None:
                entry.gpu = None
                gpu_total -= entry.nbytes
        host_total = sum(e.nbytes for e in self.entries.values() if e.host is not None)
        for entry in sorted(self.entries.values(), key=lambda e: e.last_used):
            if host_total <= self.host_budget:
                break
            if entry.published and entry.host is not None and entry.gpu is None:
                entry.host = None
                host_total -= entry.nbytes
                self.records["evictions"] += 1
        for key in [k for k, e in self.entries.items() if e.gpu is None and e.host is None]:
            del self.entries[key]

    def stats(self) -> dict[str, Any]:
        with self._lock:
            return {"entries": len(self.entries),
                    "gpu_bytes": sum(e.nbytes for e in self.entries.values() if e.gpu is not None),
                    "host_bytes": sum(e.nbytes for e in self.entries.values() if e.host is not None),
                    "unpublished": sum(1 for e in self.entries.values() if not e.published), **self.records}


class PlanningGate:
    """Sections (memory-critical GPU work of the served model) have priority over planner units: a unit starts
    only while no section is open or waiting; a section waits only for the unit in progress."""

    def __init__(self, *, unit_timeout: float = 600.0):
        self._cv = threading.Condition()
        self._sections = 0
        self._waiting_sections = 0
        self._unit_active = False
        self.unit_timeout = unit_timeout
        self.records = {"units": 0, "unit_wait_seconds": 0.0, "sections": 0, "section_wait_seconds": 0.0}

    @contextlib.contextmanager
    def unit(self):
        started = time.monotonic()
        with self._cv:
            while self._sections or self._waiting_sections:
                if time.monotonic() - started > self.unit_timeout:
                    raise StateError("a planner unit waited too long for memory-critical sections")
                self._cv.wait(0.01)
            self._unit_active = True
            self.records["units"] += 1
            self.records["unit_wait_seconds"] += time.monotonic() - started
        try:
            yield
        finally:
            with self._cv:
                self._unit_active = False
                self._cv.notify_all()

    @contextlib.contextmanager
    def section(self, release_memory: bool = True):
        started = time.monotonic()
        with self._cv:
            self._waiting_sections += 1
            try:
                while self._unit_active:
                    self._cv.wait(0.01)
            finally:
                self._waiting_sections -= 1
            self._sections += 1
            self.records["sections"] += 1
            self.records["section_wait_seconds"] += time.monotonic() - started
        if release_memory and torch.cuda.is_available():
            torch.cuda.empty_cache()  # the planner's cached blocks go back before the section runs
        try:
            yield
        finally:
            with self._cv:
                self._sections -= 1
                self._cv.notify_all()


def gated_plan_chunk(gate: PlanningGate, matrices, contexts, cfg, view, bindings, inherited, *, chunk_id: str = "chunk",
                     device: Any = None) -> dict:
    """:func:`reelcache_b200.rank_method.plan_chunk` with one gated unit per matrix: the matrix (and its inherited
    rows) moves to ``device`` when its unit starts and its device working set is gone when the unit ends."""
    from ..rank_method import plan_chunk
    plans = {}
    for entry in sorted(contexts, key=lambda e: (e.layer, e.target)):
        with gate.unit():
            inherited_one = {entry: inherited[entry]} if entry in inherited else {}
            plan = plan_chunk({entry: matrices[entry]}, {entry: contexts[entry]}, cfg, view,
                              {entry: bindings[entry]} if entry in bindings else {}, inherited_one,
                              chunk_id=chunk_id, device=device)[entry]
            if plan.coefficients is not None and device is not None:
                plan.coefficients = plan.coefficients.cpu()
            plans[entry] = plan
    return plans


@dataclass
class SegmentReport:
    session: str
    segment_index: int
    epoch_id: str
    tier: str
    node_ref: str | None
    seconds: float


class LongCatSessionProvider:
    """Segment boundaries as session units over a conditioning-cache backend and its raw tiers."""

    def __init__(self, model, backend, tiers: EpochRawTiers | None = None, *, gate: PlanningGate | None = None):
        self.model = model
        self.backend = backend
        self.tiers = tiers or EpochRawTiers()
        self.gate = gate or PlanningGate()
        self.store = backend.runtime.store
        self.reports: list[SegmentReport] = []
        self.nodes: dict[str, str] = {}      # content key -> archived segment node (built here or read from records)

    def _ref(self, session_id: str) -> str:
        return f"{SESSION_PREFIX}{session_id}"

    def boundaries(self, session_id: str) -> list[dict]:
        ref = self.store.get_ref(self._ref(session_id))
        return [] if ref is None else list(self.store.get_manifest(ref)["boundaries"])

    def _record(self, session_id: str, boundary: dict, *, base: list[dict] | None = None) -> None:
        boundaries = (self.boundaries(session_id) if base is None else base) + [boundary]
        manifest = self.store.put_manifest({"schema": SESSION_SCHEMA, "session": session_id,
                                            "boundaries": boundaries},
                                           references=[b["node_ref"] for b in boundaries if b.get("node_ref")])
        self.store.set_ref(self._ref(session_id), manifest)

    def segment_cache(self, session_id: str, segment_index: int, cond_latents: torch.Tensor, text: torch.Tensor, *,
                      first_frame: int, base: list[dict] | None = None) -> tuple[LongCatConditioningCache, str]:
        """The conditioning cache of one segment: raw tier, else the archive, else built (then captured and
        archived); the boundary is recorded in the session."""
        started = time.perf_counter()
        cfg = self.model.cfg
        key = content_key(getattr(self.backend.runtime.model, "fingerprint", "model"), cond_latents, cfg.grid)
        epoch = ConditioningCacheEpoch(f"{session_id}:{segment_index}:{key[:16]}", segment_index, first_frame,
                                       int(cond_latents.shape[1]))
        device = self.backend.device
        hit = self.tiers.lookup(key, device)
        node_ref = self.tiers.node_of(key) or self.nodes.get(key)
        if hit is not None:
            tier, cache = hit
            cache = LongCatConditioningCache(epoch, cache.k, cache.v)
        else:
            # the archived node of the same content restores under this session's epoch id (forks and resumed
            # sessions reach another session's segment node through the content key)
            cache = self.backend.restore(epoch, node_ref=node_ref)
            tier = "compressed_cold" if cache is not None else "built"
            if cache is None:
                with self.gate.section():
                    cache = self.model.build_conditioning_cache(cond_latents, epoch)
                self.tiers.capture(key, cache)
                node_ref = self.backend.on_cache_built(cache)
                self.tiers.published(key, node_ref)
            else:
                node_ref = node_ref or self.backend.segments.get(epoch.epoch_id)
        if node_ref is not None:
            self.nodes[key] = node_ref
        if tier in ("built", "compressed_cold"):
            self.tiers.records["hits"][tier] += 1
        self._record(session_id, {"segment": segment_index, "epoch": epoch.epoch_id, "first_frame": first_frame,
                                  "content_key": key, "node_ref": node_ref}, base=base)
        self.reports.append(SegmentReport(session_id, segment_index, epoch.epoch_id, tier, node_ref,
                                          time.perf_counter() - started))
        return cache, tier

    def resume(self, session_id: str, boundary: int, new_session: str | None = None) -> list[dict]:
        """Continue ``session_id`` from its ``boundary``-th segment (a fork when ``new_session`` is given): the
        session record is cut after that boundary; its segments' caches restore from their tiers or nodes."""
        boundaries = self.boundaries(session_id)
        if not 0 <= boundary < len(boundaries):
            raise ConfigurationError(f"session {session_id} has no boundary {boundary}")
        kept = boundaries[:boundary + 1]
        for b in kept:
            if b.get("node_ref") and b.get("content_key"):
                self.nodes.setdefault(b["content_key"], b["node_ref"])
        target = new_session or session_id
        head, last = kept[:-1], kept[-1]
        self._record(target, last, base=head)
        return kept
