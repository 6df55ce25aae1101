"""Byte-bounded decoded-history leases (the counterpart of reference reelcache/residency.py:14-180).

``ResidencyPool.acquire(nbytes, loader, scratch_bytes=0)`` admits a lease only while leased bytes plus
reserved decode workspace stay within ``max_bytes`` (else :class:`CapacityError`, before any decode
work), runs ``loader()`` and checks that the tensor it returned is exactly the admitted size. The
lease's tensor is readable only while the lease is active; release (explicit, ``with`` exit or
garbage collection) returns the bytes.
"""

from __future__ import annotations

import threading
from typing import Any, Callable

import torch

from .errors import CapacityError, ConfigurationError, IntegrityError, StateError


class HistoryLease:
    def __init__(self, pool: "ResidencyPool", tensor: torch.Tensor, nbytes: int, metadata: dict | None = None):
        self._pool = pool
        self._tensor = tensor
        self._nbytes = nbytes
        self.metadata = dict(metadata or {})
        self._active = True
        self._lock = threading.Lock()

    @property
    def active(self) -> bool:
        return self._active

    @property
    def nbytes(self) -> int:
        return self._nbytes

    @property
    def tensor(self) -> torch.Tensor:
        if not self._active:
            raise StateError("this history lease was released; its tensor is gone")
        return self._tensor

    def release(self) -> None:
        with self._lock:
            if not self._active:
                return
            self._active = False
            self._tensor = None
        self._pool._release(self._nbytes)

    def __enter__(self) -> "HistoryLease":
        if not self._active:
            raise StateError("history lease has been released")
        return self

    def __exit__(self, *args: Any) -> None:
        self.release()

    def __del__(self) -> None:
        try:
            self.release()
        except Exception:  # noqa: BLE001 - interpreter teardown
            pass


class ResidencyPool:
    def __init__(self, max_bytes: int) -> None:
        if type(max_bytes) is not int or max_bytes < 0:
            raise ConfigurationError(f"ResidencyPool budget {max_bytes!r}: expected an int >= 0")
        self.max_bytes = max_bytes
        self._lock = threading.Lock()
        self._resident = 0
        self._reserved = 0
        self._peak = 0
        self._leases = 0
        self._closed = False
        self._counts = {"acquired": 0, "rejected": 0}

    @property
    def resident_bytes(self) -> int:
        with self._lock:
            return self._resident

    @property
    def reserved_bytes(self) -> int:
        with self._lock:
            return self._resident + self._reserved

    @property
    def peak_reserved_bytes(self) -> int:
        with self._lock:
            return self._peak

    @property
    def active_leases(self) -> int:
        with self._lock:
            return self._leases

    def acquire(self, nbytes: int, loader: Callable[[], torch.Tensor], *, scratch_bytes: int = 0,
                metadata: dict | None = None) -> HistoryLease:
        if type(nbytes) is not int or nbytes < 0:
            raise ConfigurationError(f"lease of {nbytes!r} bytes: expected an int >= 0")
        if type(scratch_bytes) is not int or scratch_bytes < 0:
            raise ConfigurationError(f"scratch of {scratch_bytes!r} bytes: expected an int >= 0")
        if not callable(loader):
            raise ConfigurationError(f"the lease loader is a {type(loader).__name__}, not a callable")
        with self._lock:
            if self._closed:
                raise StateError("the residency pool was closed")
            if self._resident + self._reserved + nbytes + scratch_bytes > self.max_bytes:
                self._counts["rejected"] += 1
                raise CapacityError(f"history of {nbytes} bytes (+{scratch_bytes} scratch) exceeds the residency "
                                    f"budget ({self._resident + self._reserved} of {self.max_bytes} in use)")
            self._reserved += nbytes + scratch_bytes
            self._peak = max(self._peak, self._resident + self._reserved)
        try:
            tensor = loader()
            if not isinstance(tensor, torch.Tensor):
                raise IntegrityError(f"the history loader returned {type(tensor).__name__}, not a tensor")
            if tensor.numel() * tensor.element_size() != nbytes:
                raise IntegrityError(f"the history loader returned {tensor.numel() * tensor.element_size()} bytes; the lease "
                                     f"reserved {nbytes}")
        except BaseException:
            with self._lock:
                self._reserved -= nbytes + scratch_bytes
            raise
        with self._lock:
            self._reserved -= nbytes + scratch_bytes
            if self._closed:
                raise StateError("the residency pool was closed while this history was loading")
            self._resident += nbytes
            self._leases += 1
            self._counts["acquired"] += 1
        return HistoryLease(self, tensor, nbytes, metadata)

    def _release(self, nbytes: int) -> None:
        with self._lock:
            self._resident -= nbytes
            self._leases -= 1

    def stats(self) -> dict[str, int]:
        with self._lock:
            return {"max_bytes": self.max_bytes, "resident_bytes": self._resident, "reserved_bytes": self._reserved,
                    "peak_reserved_bytes": self._peak, "active_leases": self._leases, **self._counts}

    def close(self) -> None:
        with self._lock:
            self._closed = True

    def __enter__(self) -> "ResidencyPool":
        if self._closed:
            raise StateError("the residency pool was closed")
        return self

    def __exit__(self, *args: Any) -> None:
        self.close()
