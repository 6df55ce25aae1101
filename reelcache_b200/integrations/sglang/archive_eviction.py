"""LRU eviction of a compressed archive's node payloads under ``archive_budget_bytes`` (the counterpart of
reference reelcache/integrations/sglang/archive_eviction.py:57-545; semantics from its docstring).

* Whole nodes go, all or nothing: every payload object (coefficient pack blobs, basis row blocks) a
  node's restore reads is evicted with :meth:`ObjectStore.evict`; manifests, records and execution
  state stay (the unevictable sidecar). A node with a protected object (leased, or reachable from a
  pending commit) is skipped and the next least recently used one is tried.
* ``live_bytes`` counts each payload object of the non-evicted nodes once (shared objects go with their
  last holder). Every payload write is admitted first (:meth:`reserve`): ``live + reserved`` never
  exceeds the budget; a reservation nothing can make room for fails at once (:class:`CapacityError`),
  one that only finds pinned nodes waits for the pins (bounded).
* Access order: publication, and every restore that reads a node (:meth:`touch`). Restores pin what
  they read (:meth:`pin`).
"""

from __future__ import annotations

import contextlib
import threading
import time
from collections import Counter, OrderedDict
from typing import Callable, Iterable

from ...errors import CapacityError, ConfigurationError

RESERVE_WAIT_SECONDS = 300.0


class ArchiveEviction:
    def __init__(self, store, budget_bytes: int, *, on_evict: Callable[[str, frozenset], None] | None = None,
                 wait_seconds: float = RESERVE_WAIT_SECONDS):
        if type(budget_bytes) is not int or budget_bytes <= 0:
            raise ConfigurationError("archive_budget_bytes must be a positive byte count")
        self.store = store
        self.budget = budget_bytes
        self.on_evict = on_evict
        self.wait_seconds = wait_seconds
        self.cv = threading.Condition()
        self._nodes: "OrderedDict[str, frozenset]" = OrderedDict()   # LRU: oldest first
        self._holders: Counter = Counter()                           # object -> live nodes holding it
        self._sizes: dict[str, int] = {}
        self._pins: Counter = Counter()
        self._evicted: set[str] = set()
        self.live_bytes = 0
        self.reserved_bytes = 0
        self.stats = {"evicted_nodes": 0, "evicted_bytes": 0, "skipped_protected": 0, "reserve_waits": 0}

    def _size(self, object_id: str) -> int:
        size = self._sizes.get(object_id)
        if size is None:
            size = self.store.object_size(object_id)
            self._sizes[object_id] = size
        return size

    # -- admission ----------------------------------------------------------------------------------------------

    def reserve(self, nbytes: int) -> None:
        """Admit ``nbytes`` of payload writes (evicting least recently used nodes as needed)."""
        deadline = time.monotonic() + self.wait_seconds
        with self.cv:
            while self.live_bytes + self.reserved_bytes + nbytes > self.budget:
                if self._evict_one():
                    continue
                if not any(self._pins[n] for n in self._nodes):
                    raise CapacityError(f"archive budget {self.budget} cannot admit {nbytes} more bytes")
                self.stats["reserve_waits"] += 1
                left = deadline - time.monotonic()
                if left <= 0:
                    raise CapacityError("archive budget: pinned nodes were not released in time")
                self.cv.wait(min(left, 0.1))
            self.reserved_bytes += nbytes

    def published(self, node_ref: str, objects: Iterable[str], reserved: int = 0) -> None:
        """A node is durable: its payload objects become live (its reservation is released)."""
        objects = frozenset(objects)
        with self.cv:
            self.reserved_bytes = max(0, self.reserved_bytes - reserved)
            self._nodes[node_ref] = objects
            for obj in objects:
                if self._holders[obj] == 0:
                    self.live_bytes += self._size(obj)
                self._holders[obj] += 1
            self.cv.notify_all()

    def release_reservation(self, nbytes: int) -> None:
        with self.cv:
            self.reserved_bytes = max(0, self.reserved_bytes - nbytes)
            self.cv.notify_all()

    # -- access ---------------------------------------------------------------------------------------------------

    def touch(self, node_refs: Iterable[str]) -> None:
        with self.cv:
            for ref in node_refs:
                if ref in self._nodes:
                    self._nodes.move_to_end(ref)

    @contextlib.contextmanager
    def pin(self, node_refs: Iterable[str]):
        refs = [r for r in node_refs]
        with self.cv:
            missing = [r for r in refs if r in self._evicted]
            for ref in refs:
                self._pins[ref] += 1
        try:
            yield missing
        finally:
            with self.cv:
                for ref in refs:
                    self._pins[ref] -= 1
                self.cv.notify_all()

    def evicted(self, node_ref: str) -> bool:
        with self.cv:
            return node_ref in self._evicted

    # -- eviction -------------------------------------------------------------------------------------------------

    def _evict_one(self) -> bool:
        for ref, objects in list(self._nodes.items()):
            if self._pins[ref]:
                continue
            last = [obj for obj in objects if self._holders[obj] == 1]
            result = self.store.evict(last) if last else {"leased": []}
            if result.get("leased"):
                self.stats["skipped_protected"] += 1
                continue
            del self._nodes[ref]
            for obj in objects:
                self._holders[obj] -= 1
                if self._holders[obj] == 0:
                    self.live_bytes -= self._size(obj)
                    self.stats["evicted_bytes"] += self._size(obj)
                    del self._holders[obj]
            self._evicted.add(ref)
            self.stats["evicted_nodes"] += 1
            if self.on_evict is not None:
                self.on_evict(ref, objects)
            return True
        return False

    def snapshot(self) -> dict:
        with self.cv:
            return {"budget_bytes": self.budget, "live_bytes": self.live_bytes, "reserved_bytes": self.reserved_bytes,
                    "nodes": len(self._nodes), "evicted": len(self._evicted), **self.stats}
