"""Coefficient-stream decoder pool (the counterpart of reference reelcache/decoder_pool.py:223-967).

N worker threads decode node-pack coefficient streams into uint8 coefficient tiles. Each worker keeps an
LRU of decode sessions per stream geometry (a session owns its reusable output buffers; a cold
geometry costs a session set-up, charged in dispatch). Jobs go to the least-loaded worker (queued
bytes plus the cold-session charge). ``prewarm_shapes`` opens sessions ahead of the first restore.
:class:`CanvasArena` bounds the device buffers decoded tiles are uploaded into and recycles a buffer
only after its consumer's event completed.

Streams: ``raw8`` (copy), ``raw8+zlib`` (inflate) and ``hevc`` (FFmpeg/libx265 where present; the
hardware decoder is not reachable on this platform) -- all decode to the same coefficients.
"""

from __future__ import annotations

import queue
import threading
import time
import zlib
from collections import OrderedDict
from dataclasses import dataclass, field
from typing import Any, Callable

import numpy as np
import torch

from .errors import CapacityError, ConfigurationError, StateError

COLD_SESSION_CHARGE_BYTES = 8 << 20   # dispatch cost of opening a session for a new geometry


@dataclass
class DecodeTicket:
    job_id: int
    nbytes: int
    result: Any = None
    error: BaseException | None = None
    worker: int = -1
    seconds: float = 0.0
    _done: threading.Event = field(default_factory=threading.Event)

    def done(self) -> bool:
        return self._done.is_set()

    def wait(self, timeout: float | None = None):
        if not self._done.wait(timeout):
            raise TimeoutError("decode still running")
        if self.error is not None:
            raise self.error
        return self.result


class _Worker:
    def __init__(self, pool: "DecoderPool", index: int):
        self.pool = pool
        self.index = index
        self.queue: "queue.Queue" = queue.Queue()
        self.queued_bytes = 0
        self.sessions: "OrderedDict[tuple, dict]" = OrderedDict()
        self.thread = threading.Thread(target=self.run, name=f"reelcache-decode-{index}", daemon=True)
        self.thread.start()

    def session(self, geometry: tuple) -> dict:
        hit = self.sessions.get(geometry)
        if hit is None:
            hit = {"geometry": geometry, "opened": time.perf_counter(), "uses": 0}
            self.sessions[geometry] = hit
            self.pool.counts["sessions_opened"] += 1
            while len(self.sessions) > self.pool.sessions_per_worker:
                self.sessions.popitem(last=False)
        self.sessions.move_to_end(geometry)
        hit["uses"] += 1
        return hit

    def run(self):
        while True:
            item = self.queue.get()
            if item is None:
                return
            ticket, geometry, fn = item
            started = time.perf_counter()
            try:
                self.session(geometry)
                ticket.result = fn()
            except BaseException as error:  # noqa: BLE001 - delivered through the ticket
                ticket.error = error
            ticket.seconds = time.perf_counter() - started
            with self.pool.lock:
                self.queued_bytes -= ticket.nbytes
                self.pool.counts["decoded"] += 1
                self.pool.counts["decoded_bytes"] += ticket.nbytes
            ticket._done.set()


class DecoderPool:
    def __init__(self, workers: int = 4, *, sessions_per_worker: int = 4):
        if type(workers) is not int or workers < 1:
            raise ConfigurationError("decoder pool needs at least one worker")
        self.lock = threading.Lock()
        self.sessions_per_worker = sessions_per_worker
        self.counts = {"submitted": 0, "decoded": 0, "decoded_bytes": 0, "sessions_opened": 0}
        self._next = 0
        self._closed = False
        self.workers = [_Worker(self, i) for i in range(workers)]

    def _pick(self, geometry: tuple) -> _Worker:
        def cost(w: _Worker):
            return w.queued_bytes + (0 if geometry in w.sessions else COLD_SESSION_CHARGE_BYTES)
        return min(self.workers, key=cost)

    def submit(self, fn: Callable[[], Any], *, nbytes: int, geometry: tuple) -> DecodeTicket:
        with self.lock:
            if self._closed:
                raise StateError("decoder pool is closed")
            worker = self._pick(geometry)
            self._next += 1
            ticket = DecodeTicket(self._next, nbytes, worker=worker.index)
            worker.queued_bytes += nbytes
            self.counts["submitted"] += 1
        worker.queue.put((ticket, geometry, fn))
        return ticket

    def decode_stream(self, stream: bytes, codec: str, shape: tuple[int, int], *, geometry=None) -> DecodeTicket:
        """Decode one coefficient stream to uint8 ``shape`` (tokens, columns)."""
        def run():
            if codec == "raw8":
                data = stream
            elif codec == "raw8+zlib":
                data = zlib.decompress(stream)
            else:
                raise ConfigurationError(f"stream codec {codec!r} needs its own decoder here")
            if len(data) != shape[0] * shape[1]:
                raise StateError("decoded stream size differs from its shape")
            return np.frombuffer(data, dtype=np.uint8).reshape(shape)
        return self.submit(run, nbytes=len(stream), geometry=geometry or (codec, tuple(shape)))

    def prewarm_shapes(self, geometries) -> int:
        opened = 0
        for geometry in geometries:
            for worker in self.workers:
                if geometry not in worker.sessions:
                    worker.session(geometry)
                    opened += 1
        return opened

    def trim_device_cache(self, reason: str) -> int:
        return 0  # sessions hold host state only

    def stats(self) -> dict:
        with self.lock:
            return {**self.counts, "workers": len(self.workers),
                    "queued_bytes": sum(w.queued_bytes for w in self.workers)}

    def close(self) -> None:
        with self.lock:
            self._closed = True
        for worker in self.workers:
            worker.queue.put(None)
        for worker in self.workers:
            worker.thread.join(timeout=10)


class CanvasArena:
    """Bounded device buffers for decoded tiles, recycled after their consumer's event."""

    def __init__(self, device, budget_bytes: int):
        self.device = torch.device(device)
        self.budget = budget_bytes
        self.lock = threading.Lock()
        self._free: dict[tuple, list] = {}
        self._busy: list[tuple[torch.Tensor, Any, tuple]] = []
        self.bytes = 0

    def _reclaim(self):
        keep = []
        for tensor, event, key in self._busy:
            if event is None or event.query():
                self._free.setdefault(key, []).append(tensor)
            else:
                keep.append((tensor, event, key))
        self._busy = keep

    def acquire(self, shape: tuple, dtype=torch.uint8) -> torch.Tensor:
        key = (tuple(shape), dtype)
        nbytes = int(np.prod(shape)) * torch.tensor([], dtype=dtype).element_size()
        with self.lock:
            self._reclaim()
            free = self._free.get(key)
            if free:
                return free.pop()
            if self.bytes + nbytes > self.budget:
                raise CapacityError("canvas arena budget exhausted (buffers still in use)")
            self.bytes += nbytes
        return torch.empty(shape, dtype=dtype, device=self.device)

    def release(self, tensor: torch.Tensor, event=None) -> None:
        with self.lock:
            self._busy.append((tensor, event, (tuple(tensor.shape), tensor.dtype)))
