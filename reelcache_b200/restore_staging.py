"""Cold-pack staging engine: parallel, GIL-free positioned reads of archived payloads into a pinned host
ring, hash checks, and the host->device copies that follow (the counterpart of reference
reelcache/restore_staging.py:122-946).

* :class:`PinnedRing` -- one pinned host allocation carved into variable-size slots, recycled in
  order once the copies that read a slot completed (CUDA events).
* :class:`StagingEngine` -- ``stage(object_ids)`` reads every payload file with the native
  ``pread_many`` (C++, threads, GIL released) straight into ring slots, verifies SHA-256 against the
  content address when the store verifies reads, and returns a :class:`StagedHistory` of host views;
  ``to_device`` issues one ``cudaMemcpyAsync`` per payload on the engine's copy stream.
"""

from __future__ import annotations

import hashlib
import threading
import time
from typing import Iterable

import torch

from .errors import CapacityError, ConfigurationError, IntegrityError


class PinnedRing:
    def __init__(self, nbytes: int, *, pinned: bool = True):
        if type(nbytes) is not int or nbytes <= 0:
            raise ConfigurationError("ring size must be a positive byte count")
        self.nbytes = nbytes
        self.buffer = torch.empty(nbytes, dtype=torch.uint8, pin_memory=pinned and torch.cuda.is_available())
        self._lock = threading.Lock()
        self._head = 0
        self._live: list[tuple[int, int, object]] = []   # (start, end, release event or None)

    def _reclaim(self) -> None:
        while self._live:
            start, end, event = self._live[0]
            if event is not None and not event.query():
                break
            if event is None:
                break
            self._live.pop(0)

    def allocate(self, size: int) -> tuple[int, torch.Tensor]:
        size = (size + 255) // 256 * 256
        if size > self.nbytes:
            raise CapacityError("payload larger than the staging ring")
        with self._lock:
            self._reclaim()
            start = self._head if self._head + size <= self.nbytes else 0
            end = start + size
            for s, e, _ in self._live:
                if s < end and start < e:
                    raise CapacityError("staging ring is full (copies still in flight)")
            self._head = end
            self._live.append((start, end, None))
            return start, self.buffer[start:end]

    def release(self, start: int, event=None) -> None:
        """The slot at ``start`` may be reused once ``event`` completed (now, without one)."""
        with self._lock:
            for i, (s, e, _) in enumerate(self._live):
                if s == start:
                    if event is None:
                        self._live.pop(i)
                    else:
                        self._live[i] = (s, e, event)
                    break
            self._reclaim()


class StagedHistory:
    """Host views of staged payloads (object id -> uint8 tensor) and their ring slots."""

    def __init__(self, engine: "StagingEngine", views: dict, slots: list, stats: dict):
        self.engine = engine
        self.views = views
        self.slots = slots
        self.stats = stats

    def bytes(self, object_id: str) -> bytes:
        return self.views[object_id].numpy().tobytes()

    def to_device(self, device, stream=None) -> dict:
        """One async copy per payload on the copy stream; the ring slots recycle after the copies."""
        device = torch.device(device)
        stream = stream or self.engine.copy_stream(device)
        out = {}
        with torch.cuda.stream(stream):
            for object_id, view in self.views.items():
                out[object_id] = view.to(device, non_blocking=True)
            event = torch.cuda.Event()
            event.record(stream)
        for start in self.slots:
            self.engine.ring.release(start, event)
        self.slots = []
        return out

    def release(self) -> None:
        for start in self.slots:
            self.engine.ring.release(start)
        self.slots = []


class StagingEngine:
    def __init__(self, store, *, pinned_bytes: int = 512 << 20, threads: int = 8, verify: bool | None = None):
        self.store = store
        self.ring = PinnedRing(pinned_bytes)
        self.threads = threads
        self.verify = store.verify_reads if verify is None else verify
        self._streams: dict = {}
        self.stats_ = {"staged": 0, "bytes": 0, "read_seconds": 0.0, "hash_seconds": 0.0}

    def copy_stream(self, device) -> torch.cuda.Stream:
        device = torch.device(device)
        if device not in self._streams:
            self._streams[device] = torch.cuda.Stream(device)
        return self._streams[device]

    def stage(self, object_ids: Iterable[str]) -> StagedHistory:
        from .ops._ext import ext

        ids = list(dict.fromkeys(object_ids))
        sizes = self.store.object_sizes(ids)
        missing = [i for i in ids if i not in sizes]
        if missing:
            raise IntegrityError(f"missing immutable objects: {missing[:3]}")
        views, slots = {}, []
        paths, offsets, lengths, dest = [], [], [], []
        try:
            for object_id in ids:
                start, slot = self.ring.allocate(sizes[object_id])
                slots.append(start)
                view = slot[:sizes[object_id]]
                views[object_id] = view
                paths.append(str(self.store.path_for(object_id)))
                offsets.append(0)
                lengths.append(sizes[object_id])
                dest.append(view.data_ptr())
            started = time.perf_counter()
            ext().pread_many(paths, offsets, lengths, dest, self.threads)
            self.stats_["read_seconds"] += time.perf_counter() - started
            if self.verify:
                started = time.perf_counter()
                for object_id, view in views.items():
                    if hashlib.sha256(view.numpy()).hexdigest() != object_id.split(":", 1)[1]:
                        raise IntegrityError(f"staged object fails its content hash: {object_id}")
                self.stats_["hash_seconds"] += time.perf_counter() - started
        except BaseException:
            for start in slots:
                self.ring.release(start)
            raise
        self.stats_["staged"] += len(ids)
        self.stats_["bytes"] += sum(lengths)
        return StagedHistory(self, views, slots, {"objects": len(ids), "bytes": sum(lengths)})

    def stats(self) -> dict:
        return dict(self.stats_)
