"""Restore install: archived or raw-tier history -> engine RoPE -> native KV slots (the counterpart of reference
reelcache/integrations/sglang/restore.py: ``AttentionKVLease`` :41, ``RopeTableCache`` :181, ``DenseInstall``
:303, ``restore_dense`` :624, ``LineageInstall`` :693, ``kernel_warmup_shapes`` :753).

Only the attended context of the next chunk is installed (a :class:`~.visibility.VisibilityPlan`). Every K/V
write goes through :mod:`reelcache_b200.restore_kernels`:

* dense ranges (RAW archive, raw tier): the exact captured pre-RoPE rows (``DenseSource``), K rotated with the
  engine's RoPE table at the recorded position -- on CUDA by the dense RoPE-and-store kernel, one launch per
  layer for all spans (:class:`DenseInstall`);
* compressed ranges: the lineage restorer (fused tcgen05 reconstruction with RoPE straight into the slots);
  :class:`LineageInstall` hands it the destination and RoPE callbacks of the plan.

:class:`AttentionKVLease` owns what a restore borrowed (staging tensors, reconstruction handles, finalizers)
until ``close``, which waits for every reconstruction before releasing its inputs.
"""

from __future__ import annotations

import threading
import time
from collections import OrderedDict
from typing import Any, Callable, Mapping, Sequence

import torch

from ... import restore_kernels as rk
from ...errors import ConfigurationError, StateError, UnsupportedError
from ...types import MatrixKey

ROPE_TABLE_CACHE_BYTES = 64 << 20


class AttentionKVLease:
    """What one restore borrowed, released on :meth:`close` after its reconstructions completed."""

    def __init__(self, *, store_lease: Any = None, plans: Mapping[str, Any] | None = None,
                 description: Mapping[str, Any] | None = None):
        self.store_lease = store_lease
        self.plans = dict(plans or {})
        self.description = dict(description or {})
        self._handles: list = []
        self._staging: list = []
        self._finalizers: list[Callable[[], None]] = []
        self._closed = False
        self._lock = threading.Lock()

    def track(self, *, handle=None, staging=None, finalizer: Callable[[], None] | None = None) -> None:
        with self._lock:
            if self._closed:
                raise StateError("the KV lease is closed")
            if handle is not None:
                self._handles.append(handle)
            if staging is not None:
                self._staging.append(staging)
            if finalizer is not None:
                self._finalizers.append(finalizer)

    @property
    def open_handles(self) -> int:
        return sum(1 for h in self._handles if not _done(h))

    def complete(self) -> "AttentionKVLease":
        """Block until every tracked reconstruction has finished."""
        for handle in list(self._handles):
            _synchronize(handle)
        return self

    def wait(self, stream: Any = None) -> None:
        """Order ``stream`` (default: the current stream) after every tracked reconstruction."""
        for handle in list(self._handles):
            if hasattr(handle, "wait"):
                try:
                    handle.wait(stream)
                except TypeError:
                    handle.wait()

    def close(self) -> None:
        with self._lock:
            if self._closed:
                return
            self._closed = True
        errors = []
        try:
            self.complete()
        except BaseException as error:  # noqa: BLE001 - inputs are released regardless
            errors.append(error)
        for finalizer in reversed(self._finalizers):
            try:
                finalizer()
            except BaseException as error:  # noqa: BLE001
                errors.append(error)
        self._staging.clear()
        self._handles.clear()
        if self.store_lease is not None:
            self.store_lease.release()
        if errors:
            raise errors[0]

    def __enter__(self) -> "AttentionKVLease":
        return self

    def __exit__(self, *_: Any) -> None:
        self.close()


def _done(handle) -> bool:
    query = getattr(handle, "query", None)
    return bool(query()) if callable(query) else True


def _synchronize(handle) -> None:
    for name in ("synchronize", "join"):
        method = getattr(handle, name, None)
        if callable(method):
            method()
            return


class RopeTableCache:
    """LRU cache of RoPE tables per (start frame, frames, grid, device), bounded in bytes."""

    def __init__(self, max_bytes: int = ROPE_TABLE_CACHE_BYTES):
        if type(max_bytes) is not int or max_bytes <= 0:
            raise ConfigurationError("RoPE table cache bytes must be a positive integer")
        self.max_bytes = max_bytes
        self._tables: OrderedDict = OrderedDict()
        self._bytes = 0
        self.hits = self.misses = 0
        self._lock = threading.Lock()

    @staticmethod
    def key(start_frame: int, frames: int, grid: Sequence[int], device: Any) -> tuple:
        return (int(start_frame), int(frames), tuple(int(g) for g in grid), str(torch.device(device)))

    def get(self, key: tuple):
        with self._lock:
            hit = self._tables.get(key)
            if hit is None:
                self.misses += 1
                return None
            self.hits += 1
            self._tables.move_to_end(key)
            return hit

    def put(self, key: tuple, tables) -> None:
        size = sum(t.numel() * t.element_size() for t in tables)
        with self._lock:
            if key in self._tables:
                return
            self._tables[key] = tables
            self._bytes += size
            while self._bytes > self.max_bytes and len(self._tables) > 1:
                _, old = self._tables.popitem(last=False)
                self._bytes -= sum(t.numel() * t.element_size() for t in old)

    def bind(self, compute: Callable[[int, int], tuple], *, grid: Sequence[int], device: Any) -> "BoundRopeTables":
        return BoundRopeTables(self, compute, tuple(grid), device)

    def stats(self) -> dict[str, Any]:
        return {"tables": len(self._tables), "bytes": self._bytes, "hits": self.hits, "misses": self.misses}

    def __len__(self) -> int:
        return len(self._tables)


class BoundRopeTables:
    """``(start_frame, frames) -> (cos, sin)`` of one engine's RoPE, memoized in a :class:`RopeTableCache`."""

    def __init__(self, cache: RopeTableCache, compute: Callable[[int, int], tuple], grid: tuple, device: Any):
        self.cache, self.compute, self.grid, self.device = cache, compute, grid, device
        self.computed = 0

    def __call__(self, start_frame: int, frames: int):
        key = self.cache.key(start_frame, frames, self.grid, self.device)
        hit = self.cache.get(key)
        if hit is None:
            hit = tuple(self.compute(start_frame, frames))
            self.computed += 1
            self.cache.put(key, hit)
        return hit

    def report(self) -> dict[str, Any]:
        return {"computed": self.computed, **self.cache.stats()}


class DenseLayer:
    """One layer of a dense install in flight: the reconstruction handle and its staged inputs."""

    def __init__(self, handle: Any, staged: list, jobs: int):
        self.handle, self.staged, self.jobs = handle, staged, jobs

    def release(self) -> None:
        if self.handle is not None:
            _synchronize(self.handle)
        self.staged.clear()


class DenseInstall:
    """Dense pre-RoPE rows of a plan's spans into native BTHD slots: per layer one batched reconstruction
    (K rotated with the engine's RoPE at the recorded positions, V copied), through the dense RoPE-and-store
    kernel on CUDA. ``rows_of(span, key)`` returns the span's ``[length, C]`` rows (host or device);
    ``rope(span)`` the (table, (t_row, h_row, w_row)) of the span's node-relative first frame."""

    def __init__(self, *, plan, destination: Callable[[int, str], torch.Tensor],
                 rope: Callable[[Any], tuple], rows_of: Callable[[Any, MatrixKey], torch.Tensor],
                 grid: tuple[int, int], key_space: str = "pre_rope", device: Any = None, stream: Any = None):
        self.plan = plan
        self.destination = destination
        self.rope = rope
        self.rows_of = rows_of
        self.height, self.width = grid
        self.key_space = key_space
        self.device = torch.device(device) if device is not None else None
        self.stream = stream
        self.stats_ = {"layers": 0, "jobs": 0, "h2d_bytes": 0, "seconds": 0.0}

    def _jobs(self, layer: int, staged: list) -> list:
        plane = self.height * self.width
        jobs = []
        for span in self.plan.spans:
            if span.node_offset % plane or span.length % plane:
                raise ConfigurationError("dense installs take whole latent frames")
            for target in ("K", "V"):
                cache = self.destination(layer, target)
                rows = self.rows_of(span, MatrixKey(layer, target))
                if rows.device != cache.device:
                    rows = rows.to(cache.device, non_blocking=True)
                    self.stats_["h2d_bytes"] += rows.numel() * rows.element_size()
                staged.append(rows)
                positions = None
                if target == "K" and self.key_space == "pre_rope":
                    table, first = self.rope(span)
                    offset = span.node_offset // plane
                    positions = rk.RopePositions(table, (first[0] + offset, first[1], first[2]))
                jobs.append(rk.ReconstructionJob(rk.DenseSource(rows), rk.NativeView(cache, "BTHD", span.slot_start),
                                                 (span.length // plane, self.height, self.width), rope=positions))
        return jobs

    def layer(self, layer: int) -> DenseLayer:
        started = time.perf_counter()
        staged: list = []
        jobs = self._jobs(layer, staged)
        handle = rk.reconstruct(jobs, stream=self.stream) if jobs else None
        self.stats_["layers"] += 1
        self.stats_["jobs"] += len(jobs)
        self.stats_["seconds"] += time.perf_counter() - started
        return DenseLayer(handle, staged, len(jobs))

    def stats(self) -> dict[str, Any]:
        return dict(self.stats_)


def restore_dense(lease: AttentionKVLease, *, plan, destination, rope, rows_of, grid, layers: int,
                  key_space: str = "pre_rope", stream: Any = None, readiness=None) -> dict[str, Any]:
    """Install every layer of a plan's dense spans; each layer's handle is tracked by ``lease`` and marked on
    ``readiness`` (when given) as it is issued."""
    install = DenseInstall(plan=plan, destination=destination, rope=rope, rows_of=rows_of, grid=grid,
                           key_space=key_space, stream=stream)
    for layer in range(layers):
        handle = install.layer(layer)
        lease.track(handle=handle.handle, staging=handle.staged)
        if readiness is not None:
            event = None
            if stream is not None and torch.cuda.is_available():
                event = torch.cuda.Event()
                event.record(stream)
            readiness.mark(layer, event, source="raw")
    return install.stats()


class LineageInstall:
    """The callbacks a lineage restorer needs to install a plan's compressed spans: destination caches, the
    engine RoPE of each piece and the cache row of each piece (sink + window plans place spans below their
    global positions)."""

    def __init__(self, *, plan, destination: Callable[[int, str], torch.Tensor],
                 rope_rows: Callable[[int], tuple], table: Any, tokens_per_frame: int):
        self.plan = plan
        self._destination = destination
        self._rope_rows = rope_rows
        self.table = table
        self.tokens_per_frame = tokens_per_frame
        self._slots = {span.token_start: span for span in plan.spans}

    def ranges(self) -> list[tuple[int, int]]:
        return self.plan.ranges()

    def destination(self, layer: int, target: str) -> torch.Tensor:
        return self._destination(layer, target)

    def _span(self, piece):
        span = self._slots.get(piece.token_start)
        if span is None:
            raise StateError(f"restored piece at token {piece.token_start} is not in the visibility plan")
        return span

    def slot_of(self, piece) -> int:
        return self._span(piece).slot_start

    def rope(self, piece) -> tuple:
        """(table, rows) of the piece's node (the restorer adds the piece's frame offset inside the node)."""
        span = self._span(piece)
        return self.table, self._rope_rows(span.chunk_index)

    def restore(self, restorer, head_ref: str, **kwargs):
        return restorer.restore(head_ref, self.destination, self.rope, ranges=self.ranges(), slot_of=self.slot_of,
                                **kwargs)


def kernel_warmup_shapes(profile: Any, *, paths: Sequence[str] = ("pictures", "dense"),
                         cache_dtype: torch.dtype = torch.bfloat16, max_rank: int = 256) -> list:
    """Restore-kernel warm-up shapes of a profile: its head geometry and cache dtype for each restore path
    (``pictures``/``uint8`` compressed sources, ``float`` factor packs, ``dense`` RAW and raw-tier ranges)."""
    return [rk.WarmupShape(heads=profile.num_heads, head_dim=profile.head_dim, dtype=cache_dtype, source=path,
                           max_rank=max_rank) for path in paths]


# -- per-restore records (records only: a restore never waits for, changes or frees anything for them) ------------

class GcPauses:
    """Python's garbage collections and the seconds spent in them, per generation, counted by one ``gc.callbacks``
    hook per process; a restore reports the change over its window. It never freezes, disables or runs a
    collection."""

    def __init__(self) -> None:
        self.collections = [0, 0, 0]
        self.seconds = [0.0, 0.0, 0.0]
        self._open: float | None = None

    def __call__(self, phase: str, info: Mapping[str, Any]) -> None:
        if phase == "start":
            self._open = time.perf_counter()
        elif phase == "stop" and self._open is not None:
            generation = max(0, min(2, int(info.get("generation", 2))))
            self.collections[generation] += 1
            self.seconds[generation] += time.perf_counter() - self._open
            self._open = None

    def snapshot(self) -> tuple[tuple[int, ...], tuple[float, ...]]:
        return tuple(self.collections), tuple(self.seconds)


GC_PAUSES = GcPauses()
_GC_LOCK = threading.Lock()


def install_gc_pauses() -> GcPauses:
    """Install the process's collection counter once, however many bridges ask."""
    import gc
    with _GC_LOCK:
        if all(callback is not GC_PAUSES for callback in gc.callbacks):
            gc.callbacks.append(GC_PAUSES)
    return GC_PAUSES


def gc_pause_record(before, after) -> dict[str, Any]:
    """The collections (per generation) and their seconds between two snapshots."""
    if before is None or after is None:
        return {"available": False}
    collections = [b - a for a, b in zip(before[0], after[0])]
    seconds = [b - a for a, b in zip(before[1], after[1])]
    return {"available": True, "collections": collections, "seconds": seconds, "total_seconds": sum(seconds)}


#: The tier of a resume that continues on the session's resident engine cache.
RESIDENT_TIER = "resident"


def configured_verification_mode(config: Any) -> str:
    """How a restore verifies the payloads it reads: ``sync`` (hash every read, ``verify_reads``) or ``off``."""
    return "sync" if getattr(config, "verify_reads", False) else "off"


def resident_lease_record(chunks: Sequence[int], *, verification_mode: str) -> dict[str, Any]:
    """A resident resume in the archive restore's record shape: every chunk ``resident``, nothing read or
    verified."""
    per_chunk = [{"chunk": index, "node": None, "tier": RESIDENT_TIER} for index in chunks]
    return {"tiers": {"per_chunk": per_chunk, "chunks": {RESIDENT_TIER: len(per_chunk)} if per_chunk else {},
                      "bytes": {}},
            "verification": {"mode": verification_mode, "payload_wait_seconds": 0.0, "verified_payloads": 0}}


def tier_record(plan, raw_holders: set, *, verification_mode: str) -> dict[str, Any]:
    """An archive restore's per-span tiers: ``gpu_raw`` where the raw tier held the exact capture, else
    ``compressed``."""
    per_chunk, counts = [], {}
    for span in plan.spans:
        tier = "gpu_raw" if span.node_ref in raw_holders else "compressed"
        per_chunk.append({"chunk": span.chunk_index, "node": span.node_ref, "tier": tier,
                          "token_start": span.token_start, "tokens": span.length})
        counts[tier] = counts.get(tier, 0) + 1
    return {"tiers": {"per_chunk": per_chunk, "chunks": counts},
            "verification": {"mode": verification_mode}}


def check_restorable(plan, *, rope: bool = True) -> None:
    """The fused restore installs whole latent frames when it applies RoPE: a span that cuts a frame is refused
    before anything is issued (a RoPE-free install takes any rows)."""
    if not rope:
        return
    for span in plan.spans:
        frame = getattr(span, "frame_tokens", None)
        if frame and (span.node_offset % frame or span.length % frame):
            raise UnsupportedError(f"span of chunk {span.chunk_index} (offset {span.node_offset}, length {span.length})"
                                   " cuts a latent frame")


def decoder_pool_snapshot(pool: Any) -> dict[str, Any] | None:
    """The decoder pool's counters now (None without a pool or readable stats: a record never fails a restore)."""
    stats = getattr(pool, "stats", None)
    if not callable(stats):
        return None
    try:
        return dict(stats())
    except Exception:  # noqa: BLE001 - records only
        return None


def decoder_pool_record(before: Mapping[str, Any] | None, after: Mapping[str, Any] | None) -> dict[str, Any]:
    """The pool's numeric counters' change over one restore."""
    if before is None or after is None:
        return {"available": False}
    delta = {k: after[k] - before[k] for k in after if isinstance(after.get(k), (int, float))
             and isinstance(before.get(k), (int, float))}
    return {"available": True, "delta": delta}


__all__ = ["GC_PAUSES", "GcPauses", "RESIDENT_TIER", "check_restorable", "configured_verification_mode",
           "decoder_pool_record", "decoder_pool_snapshot", "gc_pause_record", "install_gc_pauses",
           "resident_lease_record", "tier_record", "AttentionKVLease", "BoundRopeTables", "DenseInstall", "DenseLayer", "LineageInstall", "RopeTableCache",
           "kernel_warmup_shapes", "restore_dense"]
