"""Process-wide registry of trimmable device caches, run on GPU memory pressure (the counterpart of
reference reelcache/device_pressure.py:36-150).

Components register ``trim(reason) -> bytes_freed`` under a name; ``trim_device_caches(reason, ...)``
calls them in a fixed order (decoder pool, then restorer caches, then bridge-resident state, then
everything else), optionally stopping once a ``headroom()`` probe covers ``needed_bytes``, and then
empties the allocator cache. Bound methods are held weakly: a collected component drops out. A trim
that raises is recorded, never propagated.
"""

from __future__ import annotations

import itertools
import threading
import time
import weakref
from typing import Any, Callable

TRIM_ORDER = {"decoder_pool": 10, "restorer": 20, "bridge_resident": 30}
DEFAULT_ORDER = 50
REASONS = ("decode", "request_start", "oom")


def _device_index(device: Any) -> int | None:
    if device is None:
        return None
    index = getattr(device, "index", device)
    return None if index is None else int(index)


class TrimHandle:
    def __init__(self, registry: "DeviceTrimRegistry", key: int):
        self._registry = registry
        self.key = key

    def unregister(self) -> None:
        self._registry._remove(self.key)


class DeviceTrimRegistry:
    def __init__(self):
        self._lock = threading.Lock()
        self._entries: dict[int, dict] = {}
        self._ids = itertools.count()

    def register(self, name: str, trim: Callable[[str], int], *, order: int | None = None,
                 device: Any = None) -> TrimHandle:
        if not isinstance(name, str) or not name:
            raise ValueError("a trim needs a nonempty name")
        if not callable(trim):
            raise ValueError("trim must be callable")
        rank = TRIM_ORDER.get(name.split(":", 1)[0], DEFAULT_ORDER) if order is None else int(order)
        try:
            ref = weakref.WeakMethod(trim)
        except TypeError:
            ref = (lambda fn=trim: fn)
        key = next(self._ids)
        with self._lock:
            self._entries[key] = {"name": name, "order": rank, "device": _device_index(device), "trim": ref}
        return TrimHandle(self, key)

    def _remove(self, key: int) -> None:
        with self._lock:
            self._entries.pop(key, None)

    def _ordered(self):
        with self._lock:
            return sorted(self._entries.items(), key=lambda kv: (kv[1]["order"], kv[0]))

    def registered(self) -> list[dict]:
        return [{"name": e["name"], "order": e["order"], "device": e["device"]}
                for _, e in self._ordered() if e["trim"]() is not None]

    def trim(self, reason: str, *, device: Any = None, needed_bytes: int | None = None,
             headroom: Callable[[], int] | None = None, empty_cache: Callable[[], Any] | None = None) -> dict:
        started = time.perf_counter()
        wanted = _device_index(device)
        records, total = [], 0
        for key, entry in self._ordered():
            if wanted is not None and entry["device"] is not None and entry["device"] != wanted:
                continue
            if needed_bytes is not None and headroom is not None:
                try:
                    if headroom() >= needed_bytes:
                        break
                except Exception:  # noqa: BLE001 - no measurement: keep trimming
                    pass
            fn = entry["trim"]()
            if fn is None:
                self._remove(key)
                continue
            clock = time.perf_counter()
            record = {"name": entry["name"], "bytes": 0}
            try:
                freed = max(0, int(fn(reason) or 0))
                record["bytes"] = freed
                total += freed
            except Exception as error:  # noqa: BLE001 - recorded, never raised
                record["error"] = f"{type(error).__name__}: {error}"
            record["seconds"] = time.perf_counter() - clock
            records.append(record)
        clock = time.perf_counter()
        if empty_cache is None:
            import torch
            if torch.cuda.is_available():
                torch.cuda.empty_cache()
        else:
            empty_cache()
        return {"reason": reason, "trims": records, "bytes": total,
                "empty_cache_seconds": time.perf_counter() - clock, "seconds": time.perf_counter() - started}


REGISTRY = DeviceTrimRegistry()


def register_device_trim(name: str, trim: Callable[[str], int], *, order: int | None = None,
                         device: Any = None) -> TrimHandle:
    return REGISTRY.register(name, trim, order=order, device=device)


def trim_device_caches(reason: str, **kwargs) -> dict:
    return REGISTRY.trim(reason, **kwargs)


__all__ = ["DEFAULT_ORDER", "DeviceTrimRegistry", "REASONS", "REGISTRY", "TRIM_ORDER", "TrimHandle",
           "register_device_trim", "trim_device_caches"]
