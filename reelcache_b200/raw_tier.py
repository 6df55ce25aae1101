"""Raw-chunk tier: the captured clean K/V of submitted chunks, kept on the capture device ("GPU raw")
or in host memory ("host raw") until their compressed nodes are published, and afterwards as an
evictable cache that serves lossless restores (the counterpart of reference reelcache/raw_tier.py;
invariants from its module docstring, lines 1-51).

* **I1** an unpublished entry keeps at least one complete copy; a device copy is dropped only after
  a complete host copy exists (demotion copies device -> host first).
* **I2** ``admit`` waits only when device and host budgets are both full of unpublished entries
  (backpressure, recorded with its cause); otherwise it returns at once.
* **I3** a published entry is evictable: device copies are demoted to host, host copies dropped, least
  recently used first; with ``retain="lru"`` published entries without holders stay as unheld cache
  entries and are evicted before held ones, otherwise they are dropped when their last holder leaves.
* ``source(token)`` re-stages a spilled entry on its capture device, so planning never depends on
  where the raw copy lives.

Device -> host copies run on a dedicated side stream into pinned host memory (``host_pinned``) and
are ordered by events, so they overlap the generation stream.
"""

from __future__ import annotations

import itertools
import threading
import time
from collections import OrderedDict
from dataclasses import dataclass, field
from typing import Any, Iterable, Mapping

import torch

from .device_pressure import register_device_trim
from .errors import CapacityError, ConfigurationError, StateError

TIER_NAMES = ("gpu", "host")


# -- budgets from the machine ------------------------------------------------------------------------------------

def cgroup_memory_limit(root: str = "/sys/fs/cgroup") -> int | None:
    """The memory limit of this process's cgroup (v2 ``memory.max`` or v1 ``memory.limit_in_bytes``), or
    None when unlimited or unknown."""
    import os
    candidates = []
    try:
        with open("/proc/self/cgroup") as handle:
            for line in handle:
                parts = line.strip().split(":", 2)
                if len(parts) == 3 and (parts[1] == "" or "memory" in parts[1].split(",")):
                    candidates.append((parts[1], parts[2]))
    except OSError:
        pass
    paths = []
    for controllers, rel in candidates:
        rel = rel.lstrip("/")
        if controllers == "":                               # v2 unified hierarchy
            paths.append(os.path.join(root, rel, "memory.max"))
        else:
            paths.append(os.path.join(root, "memory", rel, "memory.limit_in_bytes"))
    paths += [os.path.join(root, "memory.max"), os.path.join(root, "memory", "memory.limit_in_bytes")]
    for path in paths:
        try:
            with open(path) as handle:
                text = handle.read().strip()
        except OSError:
            continue
        if text == "max":
            return None
        try:
            value = int(text)
        except ValueError:
            continue
        return None if value >= (1 << 60) else value   # v1 reports "unlimited" as a huge number
    return None


def meminfo_available(path: str = "/proc/meminfo") -> int | None:
    """``MemAvailable`` of the host in bytes (None when unknown)."""
    try:
        with open(path) as handle:
            for line in handle:
                if line.startswith("MemAvailable:"):
                    return int(line.split()[1]) * 1024
    except (OSError, ValueError, IndexError):
        pass
    return None


def auto_host_budget(*, fraction: float = 0.5, workers: int | None = None, cgroup_root: str = "/sys/fs/cgroup",
                     meminfo: str = "/proc/meminfo") -> int:
    """A host raw-tier budget for one worker: ``fraction`` of the smaller of the cgroup limit and the host's
    available memory, shared by the node's workers (``LOCAL_WORLD_SIZE`` by default)."""
    import os
    if not 0 < fraction <= 1:
        raise ConfigurationError("fraction must lie in (0, 1]")
    if workers is None:
        workers = int(os.environ.get("LOCAL_WORLD_SIZE", "1") or 1)
    limits = [v for v in (cgroup_memory_limit(cgroup_root), meminfo_available(meminfo)) if v is not None]
    if not limits:
        return 8 << 30
    return max(0, int(min(limits) * fraction) // max(1, workers))


def device_headroom(device, reserve_bytes: int = 0) -> int | None:
    """Free device memory beyond ``reserve_bytes`` (negative when the reserve is already eaten into); None
    off CUDA."""
    device = torch.device(device)
    if device.type != "cuda" or not torch.cuda.is_available():
        return None
    free, _ = torch.cuda.mem_get_info(device)
    return int(free) - int(reserve_bytes)


class HostPool:
    """Pinned host blocks recycled by power-of-two size class: registering pinned memory is slow, so a
    demoted chunk reuses the blocks a dropped one gave back. At most ``cached_bytes`` stay cached."""

    def __init__(self, *, pinned: bool, cached_bytes: int = 4 << 30, min_block: int = 1 << 20):
        self.pinned = pinned
        self.cached_limit = cached_bytes
        self.min_block = min_block
        self._free: dict[int, list[torch.Tensor]] = {}
        self.cached = 0
        self.stats = {"allocated": 0, "reused": 0, "released": 0}
        self._lock = threading.Lock()

    def _class(self, nbytes: int) -> int:
        size = self.min_block
        while size < nbytes:
            size <<= 1
        return size

    def take(self, nbytes: int) -> torch.Tensor:
        size = self._class(max(1, nbytes))
        with self._lock:
            blocks = self._free.get(size)
            if blocks:
                self.cached -= size
                self.stats["reused"] += 1
                return blocks.pop()
        self.stats["allocated"] += 1
        return torch.empty(size, dtype=torch.uint8, pin_memory=self.pinned)

    def give(self, block: torch.Tensor) -> None:
        size = block.numel()
        with self._lock:
            if self.cached + size <= self.cached_limit:
                self._free.setdefault(size, []).append(block)
                self.cached += size
            else:
                self.stats["released"] += 1

    def view(self, block: torch.Tensor, shape, dtype) -> torch.Tensor:
        count = 1
        for dim in shape:
            count *= int(dim)
        nbytes = count * torch.empty((), dtype=dtype).element_size()
        return block[:nbytes].view(dtype).view(tuple(shape))


@dataclass
class RawEntry:
    token: int
    chunk_id: Any
    nbytes: int
    device: torch.device
    gpu: dict | None = None          # entry key -> tensor on the capture device
    host: dict | None = None         # entry key -> host tensor
    host_ready: Any = None           # event after which the host copy is complete
    host_blocks: list = field(default_factory=list)   # pooled pinned blocks behind the host copy
    node_ref: str | None = None      # set at publication
    holders: set = field(default_factory=set)
    last_used: float = field(default_factory=time.monotonic)
    failed: bool = False

    @property
    def published(self) -> bool:
        return self.node_ref is not None


class RawLease:
    """Device tensors of one entry for a restore (the entry is pinned against eviction until release)."""

    def __init__(self, tier: "RawChunkTier", entry: RawEntry, tensors: dict, retained: bool):
        self._tier = tier
        self.entry = entry
        self.tensors = tensors
        self.retained = retained
        self._active = True

    def release(self):
        if self._active:
            self._active = False
            self._tier._unpin(self.entry)

    def __enter__(self):
        return self

    def __exit__(self, *args):
        self.release()


class RawChunkTier:
    def __init__(self, device, *, gpu_budget_bytes: int, host_budget_bytes: int | None, host_pinned: bool = True,
                 retain: str = "drop", promote: str = "off", gpu_only: bool = False,
                 backpressure_timeout: float | None = 60.0, reserve_bytes: int | None = None,
                 pool_cached_bytes: int | None = None):
        """``host_budget_bytes=None``: :func:`auto_host_budget`. ``reserve_bytes``: device memory the tier keeps
        free -- published device copies are demoted while :func:`device_headroom` is below it.
        ``promote="host"``: a restore that finds an entry only in host memory copies it back to the device
        and keeps it there (budget and reserve permitting); :meth:`promote_host` does so ahead of time."""
        if host_budget_bytes is None:
            host_budget_bytes = auto_host_budget()
        if reserve_bytes is not None and (type(reserve_bytes) is not int or reserve_bytes < 0):
            raise ConfigurationError("reserve_bytes must be a nonnegative byte count or None")
        self.reserve = reserve_bytes
        if retain not in ("drop", "lru") or promote not in ("off", "host"):
            raise ConfigurationError("retain must be drop|lru and promote off|host")
        for name, value in (("gpu_budget_bytes", gpu_budget_bytes), ("host_budget_bytes", host_budget_bytes)):
            if type(value) is not int or value < 0:
                raise ConfigurationError(f"{name} must be a nonnegative byte count")
        self.device = torch.device(device)
        self.gpu_budget = gpu_budget_bytes
        self.host_budget = 0 if gpu_only else host_budget_bytes
        self.host_pinned = host_pinned and self.device.type == "cuda"
        self.retain = retain
        self.promote = promote
        self.gpu_only = gpu_only
        self.backpressure_timeout = backpressure_timeout
        self.cv = threading.Condition()
        self._tokens = itertools.count(1)
        self._entries: "OrderedDict[int, RawEntry]" = OrderedDict()
        self._by_node: dict[str, int] = {}
        self._pins: dict[int, int] = {}
        self.gpu_bytes = 0
        self.host_bytes = 0
        self._stream = torch.cuda.Stream(self.device) if self.device.type == "cuda" else None
        self.records = {"admitted": 0, "published": 0, "dropped": 0, "demoted": 0, "evicted": 0, "hits": 0,
                        "misses": 0, "retained_hits": 0, "backpressure_waits": 0, "backpressure_seconds": 0.0,
                        "restaged": 0, "trimmed_bytes": 0}
        self._closed = False
        self.pool = HostPool(pinned=self.host_pinned,
                             cached_bytes=min(self.host_budget, 4 << 30) if pool_cached_bytes is None
                             else pool_cached_bytes)
        self.records.update(promoted=0, reserve_demotions=0)
        self._trim = register_device_trim("raw_tier", self.trim_device_cache, device=self.device)

    # -- admission ------------------------------------------------------------------------------------------------

    def admit(self, tensors: Mapping[Any, torch.Tensor], chunk_id: Any, holder: Any = None,
              timeout: float | None = None) -> int:
        """Take ownership of a submitted chunk's captured tensors (no copy); returns its tier token."""
        nbytes = sum(t.numel() * t.element_size() for t in tensors.values())
        deadline = time.monotonic() + (self.backpressure_timeout if timeout is None else timeout)
        with self.cv:
            waited = None
            while True:
                if self._closed:
                    raise StateError("raw tier is closed")
                self._make_room(nbytes)
                unpublished = sum(e.nbytes for e in self._entries.values() if not e.published and not e.failed)
                if unpublished + nbytes <= self.gpu_budget + self.host_budget or not self._entries:
                    break
                if waited is None:
                    waited = time.monotonic()
                    self.records["backpressure_waits"] += 1
                left = deadline - time.monotonic()
                if left <= 0:
                    raise CapacityError("raw tier budgets are full of unpublished chunks (archival lags)")
                self.cv.wait(min(left, 0.05))
            if waited is not None:
                self.records["backpressure_seconds"] += time.monotonic() - waited
            token = next(self._tokens)
            entry = RawEntry(token, chunk_id, nbytes, self.device, gpu=dict(tensors))
            if holder is not None:
                entry.holders.add(holder)
            self._entries[token] = entry
            self.gpu_bytes += nbytes
            self.records["admitted"] += 1
            self._enforce()
            return token

    def _make_room(self, nbytes: int) -> None:
        """Evict published entries (unheld first, LRU) until ``nbytes`` more fit on the device or in host."""
        self._enforce(extra=nbytes)

    # -- budgets ------------------------------------------------------------------------------------------------

    def _order(self):
        """Eviction order: unheld published, then held published, then unpublished; LRU within each."""
        def rank(e: RawEntry):
            return (0 if e.published and not e.holders else 1 if e.published else 2, e.last_used)
        return sorted((e for e in self._entries.values() if self._pins.get(e.token, 0) == 0), key=rank)

    def _short_of_reserve(self) -> bool:
        if self.reserve is None:
            return False
        headroom = device_headroom(self.device, self.reserve)
        return headroom is not None and headroom < 0

    def _enforce(self, extra: int = 0) -> None:
        # device over budget (or eating into the reserve): demote to host (I1: the host copy exists before
        # the device copy goes)
        for entry in self._order():
            over_budget = self.gpu_bytes + extra > self.gpu_budget
            reserve_short = entry.published and entry.gpu is not None and self._short_of_reserve()
            if not over_budget and not reserve_short:
                break
            if not over_budget:
                self.records["reserve_demotions"] += 1
            if entry.gpu is None:
                continue
            if entry.published and (self.gpu_only or self.host_budget == 0):
                self._drop(entry)
                continue
            if entry.host is None and self.host_bytes + entry.nbytes > self.host_budget:
                self._evict_host(entry.nbytes, protect=entry)
                if self.host_bytes + entry.nbytes > self.host_budget:
                    continue
            self._demote(entry)
        # host over budget: drop published host copies (never the only copy of an unpublished entry)
        self._evict_host(0)

    def _evict_host(self, extra: int, protect: RawEntry | None = None) -> None:
        for entry in self._order():
            if self.host_bytes + extra <= self.host_budget:
                break
            if entry is protect or entry.host is None or not entry.published:
                continue
            if entry.gpu is None and self.retain == "drop" and entry.holders:
                pass  # held published entry: still evictable by I3
            self._drop_host(entry)
            if entry.gpu is None and entry.host is None:
                self._forget(entry)

    def _demote(self, entry: RawEntry) -> None:
        if entry.host is None:
            host = {}
            if self._stream is not None:
                self._stream.wait_stream(torch.cuda.current_stream(self.device))
                with torch.cuda.stream(self._stream):
                    for key, t in entry.gpu.items():
                        block = self.pool.take(t.numel() * t.element_size())
                        entry.host_blocks.append(block)
                        h = self.pool.view(block, t.shape, t.dtype)
                        h.copy_(t, non_blocking=True)
                        host[key] = h
                    event = torch.cuda.Event()
                    event.record(self._stream)
                entry.host_ready = event
                for t in entry.gpu.values():
                    t.record_stream(self._stream)
            else:
                host = {key: t.detach().clone() for key, t in entry.gpu.items()}
            entry.host = host
            self.host_bytes += entry.nbytes
        entry.gpu = None
        self.gpu_bytes -= entry.nbytes
        self.records["demoted"] += 1

    def _drop_host(self, entry: RawEntry) -> None:
        if entry.host is not None:
            if entry.host_ready is not None:
                entry.host_ready.synchronize()
            entry.host = None
            entry.host_ready = None
            for block in entry.host_blocks:
                self.pool.give(block)
            entry.host_blocks = []
            self.host_bytes -= entry.nbytes
            self.records["evicted"] += 1

    def _drop(self, entry: RawEntry) -> None:
        if entry.gpu is not None:
            entry.gpu = None
            self.gpu_bytes -= entry.nbytes
        self._drop_host(entry)
        self._forget(entry)

    def _forget(self, entry: RawEntry) -> None:
        if entry.gpu is None and entry.host is None and entry.token in self._entries:
            del self._entries[entry.token]
            if entry.node_ref is not None and self._by_node.get(entry.node_ref) == entry.token:
                del self._by_node[entry.node_ref]
            self.records["dropped"] += 1
            self.cv.notify_all()

    # -- lifecycle ------------------------------------------------------------------------------------------------

    def published(self, token: int, node_ref: str) -> None:
        with self.cv:
            entry = self._entries.get(token)
            if entry is None:
                return
            entry.node_ref = node_ref
            self._by_node[node_ref] = token
            self.records["published"] += 1
            if not entry.holders and self.retain == "drop":
                self._drop(entry)
            self._enforce()
            self.cv.notify_all()

    def failed(self, token: int) -> None:
        """A failed or cancelled commit: its raw entry goes (nothing will publish it)."""
        with self.cv:
            entry = self._entries.get(token)
            if entry is not None:
                entry.failed = True
                self._drop(entry)
            self.cv.notify_all()

    def hold(self, holder: Any, node_refs: Iterable[str]) -> int:
        with self.cv:
            count = 0
            for ref in node_refs:
                token = self._by_node.get(ref)
                if token is not None:
                    self._entries[token].holders.add(holder)
                    count += 1
            return count

    def release_holder(self, holder: Any, *, drop: bool = False) -> int:
        with self.cv:
            released = 0
            for entry in list(self._entries.values()):
                if holder in entry.holders:
                    entry.holders.discard(holder)
                    released += 1
                    if entry.published and not entry.holders and (drop or self.retain == "drop"):
                        if self._pins.get(entry.token, 0) == 0:
                            self._drop(entry)
            self.cv.notify_all()
            return released

    def lookup(self, node_ref: str) -> RawLease | None:
        """Device tensors of a published node's raw copy (re-staged from host when spilled), or None."""
        with self.cv:
            token = self._by_node.get(node_ref)
            if token is None:
                self.records["misses"] += 1
                return None
            entry = self._entries[token]
            retained = not entry.holders
            entry.last_used = time.monotonic()
            self._pins[token] = self._pins.get(token, 0) + 1
            self.records["hits"] += 1
            if retained:
                self.records["retained_hits"] += 1
            tensors = self._device_copy(entry)
        return RawLease(self, entry, tensors, retained)

    def source(self, token: int) -> dict:
        """The entry's tensors on its capture device (for the planner), re-staged if spilled."""
        with self.cv:
            entry = self._entries.get(token)
            if entry is None:
                raise StateError("raw entry is gone")
            return self._device_copy(entry)

    def _device_copy(self, entry: RawEntry, *, keep: bool | None = None) -> dict:
        if entry.gpu is not None:
            return dict(entry.gpu)
        self.records["restaged"] += 1
        if entry.host_ready is not None:
            torch.cuda.current_stream(self.device).wait_event(entry.host_ready)
        copy = {key: t.to(self.device, non_blocking=True) for key, t in entry.host.items()}
        keep = (self.promote == "host") if keep is None else keep
        if keep and self.device.type == "cuda" and self.gpu_bytes + entry.nbytes <= self.gpu_budget \
                and not self._short_of_reserve():
            entry.gpu = copy               # promoted: the device copy stays (the host copy too, until evicted)
            self.gpu_bytes += entry.nbytes
            self.records["promoted"] += 1
        return dict(copy)

    def promote_host(self, node_refs: Iterable[str]) -> int:
        """Copy the host-only entries of ``node_refs`` back to the device ahead of a restore (within the device
        budget and reserve); returns how many were promoted."""
        promoted = 0
        with self.cv:
            for ref in node_refs:
                token = self._by_node.get(ref)
                entry = None if token is None else self._entries.get(token)
                if entry is None or entry.gpu is not None or entry.host is None:
                    continue
                before = self.records["promoted"]
                self._device_copy(entry, keep=True)
                promoted += self.records["promoted"] - before
        return promoted

    def _unpin(self, entry: RawEntry) -> None:
        with self.cv:
            count = self._pins.get(entry.token, 0) - 1
            if count <= 0:
                self._pins.pop(entry.token, None)
            else:
                self._pins[entry.token] = count
            self._enforce()
            self.cv.notify_all()

    def trim_device_cache(self, reason: str) -> int:
        """Device-pressure response: demote every published device copy (I1 keeps unpublished ones)."""
        with self.cv:
            before = self.gpu_bytes
            for entry in self._order():
                if entry.published and entry.gpu is not None:
                    if self.gpu_only or self.host_budget == 0:
                        self._drop(entry)
                    else:
                        self._demote(entry)
            freed = before - self.gpu_bytes
            self.records["trimmed_bytes"] += freed
            return freed

    def stats(self) -> dict:
        with self.cv:
            return {"entries": len(self._entries), "gpu_bytes": self.gpu_bytes, "host_bytes": self.host_bytes,
                    "gpu_budget_bytes": self.gpu_budget, "host_budget_bytes": self.host_budget,
                    "reserve_bytes": self.reserve, "host_pool": dict(self.pool.stats, cached_bytes=self.pool.cached),
                    "unpublished": sum(1 for e in self._entries.values() if not e.published),
                    **self.records}

    def close(self) -> None:
        with self.cv:
            self._closed = True
            for entry in list(self._entries.values()):
                self._drop(entry)
            self.cv.notify_all()
        self._trim.unregister()
