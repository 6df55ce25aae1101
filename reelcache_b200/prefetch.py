"""One-layer-ahead restoration and paired K/V decoding -- the older per-matrix restore paths (the counterpart of
reference reelcache/prefetch.py:26 ``LayerPrefetcher``, :258 ``PackedLayerPrefetcher`` and
reelcache/paired_decode.py:17 ``PairedDecoder``).

* :class:`LayerPrefetcher` restores the dense history of layer ``L + 1`` on a worker thread (and its own CUDA
  stream) while the consumer attends over layer ``L``. Outputs are charged against ``max_bytes``; a layer's
  output is retired after the consumer's event for it completes (``release``), so at most the acquired layer and
  the one in flight are alive.
* :class:`PackedLayerPrefetcher` drives a :class:`~reelcache_b200.packed_decode.PackedRestorer`: the decodes of
  the next ``depth`` layers are submitted ahead while the current layer reconstructs.
* :class:`PairedDecoder` decodes a matrix's K and V coefficient streams on two decoder workers at once (each with
  its own session) under an output byte bound.
"""

from __future__ import annotations

import threading
import time
from concurrent.futures import Future, ThreadPoolExecutor
from dataclasses import dataclass, field
from typing import Any, Callable, Sequence

import torch

from .errors import CapacityError, ConfigurationError, StateError
from .types import MatrixKey


@dataclass
class _Layer:
    future: Future
    nbytes: int
    started: float
    retire_event: Any = None
    tensors: dict = field(default_factory=dict)


class LayerPrefetcher:
    """Dense per-layer history one layer ahead of the consumer."""

    def __init__(self, runtime, *, device, layers: int, channels: int, native_dtype=torch.bfloat16,
                 max_bytes: int = 1 << 30, streams: Sequence[str | None] = (None,)):
        if type(max_bytes) is not int or max_bytes <= 0:
            raise ConfigurationError("prefetch needs a positive output byte budget")
        self.runtime, self.device = runtime, torch.device(device)
        self.layers, self.channels, self.native_dtype = layers, channels, native_dtype
        self.max_bytes = max_bytes
        self.streams = tuple(streams)
        self._pool = ThreadPoolExecutor(max_workers=1, thread_name_prefix="reelcache-layer-prefetch")
        self._cuda_stream = torch.cuda.Stream(self.device) if self.device.type == "cuda" else None
        self._active: dict[int, _Layer] = {}
        self._node = None
        self._ranges = None
        self._lock = threading.Lock()
        self.stats_ = {"layers": 0, "bytes": 0, "wait_seconds": 0.0, "restore_seconds": 0.0}

    def _charged(self) -> int:
        return sum(layer.nbytes for layer in self._active.values())

    def begin(self, node_ref: str, *, ranges=None) -> None:
        if self._node is not None:
            raise StateError("a prefetch is already active; call end() first")
        self._node, self._ranges = node_ref, ranges
        self._schedule(0)

    def _layer_bytes(self) -> int:
        pieces = self.runtime.resolve_history(self._node, self._ranges)
        tokens = sum(p.token_end - p.token_start for p in pieces)
        return 2 * len(self.streams) * tokens * self.channels * torch.empty((), dtype=self.native_dtype).element_size()

    def _schedule(self, layer: int) -> None:
        if layer >= self.layers or layer in self._active:
            return
        nbytes = self._layer_bytes()
        with self._lock:
            if self._charged() + nbytes > self.max_bytes:
                if self._active:
                    return  # scheduled again when a layer is released
                raise CapacityError("one prefetched layer exceeds the prefetch budget")
            started = time.perf_counter()

            def restore():
                out = {}
                ctx = torch.cuda.stream(self._cuda_stream) if self._cuda_stream is not None else _Null()
                with ctx:
                    for stream in self.streams:
                        for target in ("K", "V"):
                            out[(target, stream)] = self.runtime.acquire_node_history(
                                self._node, MatrixKey(layer, target), ranges=self._ranges, stream=stream,
                                device=self.device, dtype=self.native_dtype)
                    if self._cuda_stream is not None:
                        event = torch.cuda.Event()
                        event.record(self._cuda_stream)
                        out["_event"] = event
                return out

            self._active[layer] = _Layer(self._pool.submit(restore), nbytes, started)

    def acquire(self, layer: int) -> dict:
        """Block until ``layer`` is restored (and schedule ``layer + 1``); returns ``{(target, stream): tensor}``.
        On CUDA the current stream is ordered after the restore."""
        if self._node is None:
            raise StateError("no active prefetch")
        self._schedule(layer)
        entry = self._active.get(layer)
        if entry is None:
            raise StateError(f"layer {layer} is not scheduled (released or over budget)")
        waited = time.perf_counter()
        tensors = dict(entry.future.result())
        self.stats_["wait_seconds"] += time.perf_counter() - waited
        event = tensors.pop("_event", None)
        if event is not None:
            torch.cuda.current_stream(self.device).wait_event(event)
        entry.tensors = tensors
        self.stats_["layers"] += 1
        self.stats_["bytes"] += entry.nbytes
        self.stats_["restore_seconds"] += time.perf_counter() - entry.started
        self._schedule(layer + 1)
        return tensors

    def tensor(self, layer: int, key: str, stream: str | None = None) -> torch.Tensor:
        return self._active[layer].tensors[(key, stream)]

    def release(self, layer: int, *, consumer_event=None) -> None:
        """Retire ``layer`` (after ``consumer_event`` completes on CUDA) and schedule the next unscheduled layer."""
        with self._lock:
            entry = self._active.pop(layer, None)
        if entry is not None and consumer_event is not None:
            consumer_event.synchronize()
        nxt = max(self._active, default=layer) + 1
        self._schedule(nxt)

    def end(self) -> None:
        for entry in list(self._active.values()):
            entry.future.result()
        self._active.clear()
        self._node = None

    def stats(self) -> dict:
        return dict(self.stats_)

    def close(self) -> None:
        self.end()
        self._pool.shutdown(wait=True)


class _Null:
    def __enter__(self):
        return self

    def __exit__(self, *args):
        return False


class PackedLayerPrefetcher:
    """Decode-ahead for the packed restorer: the next ``depth`` layers' decodes are in flight while a layer
    reconstructs."""

    def __init__(self, restorer, *, depth: int = 8):
        if type(depth) is not int or depth < 1:
            raise ConfigurationError("depth must be a positive integer")
        self.restorer, self.depth = restorer, depth
        self._pieces = None
        self._batch = None
        self._layers = 0
        self.stats_ = {"layers": 0, "submitted_through": -1}

    def begin(self, node_ref: str, *, layers: int, ranges=None) -> None:
        self._pieces = self.restorer.plan(node_ref, ranges)
        self._layers = layers
        self._batch = self.restorer.submit(self._pieces, layers)
        self._advance(0)

    @property
    def layers(self) -> int:
        return self._layers

    def _advance(self, layer: int) -> None:
        through = min(self._layers - 1, layer + self.depth)
        for next_layer in range(self.stats_["submitted_through"] + 1, through + 1):
            self.restorer.submit_through(self._batch, next_layer)
        self.stats_["submitted_through"] = max(self.stats_["submitted_through"], through)

    def restore(self, layer: int, destination: Callable, rope: Callable, *, stream=None):
        if self._batch is None:
            raise StateError("no active packed prefetch")
        self._advance(layer)
        handle = self.restorer.reconstruct(self._batch, self._pieces, layer, destination, rope, stream=stream)
        self.stats_["layers"] += 1
        return handle

    def end(self) -> None:
        if self._batch is not None:
            self.restorer.release(self._batch)
        self._batch = self._pieces = None

    def stats(self) -> dict:
        return dict(self.stats_)


class PairedDecoder:
    """K and V coefficient streams of one matrix pair decoded concurrently on two decoder workers."""

    def __init__(self, pool, *, max_output_bytes: int, max_pairs: int = 1):
        if type(max_output_bytes) is not int or max_output_bytes <= 0:
            raise ConfigurationError("the paired output budget must be positive")
        if max_pairs not in (1, 2):
            raise ConfigurationError("the paired decoder holds one pair or active-plus-next pairs")
        self.pool = pool
        self.max_output_bytes, self.max_pairs = max_output_bytes, max_pairs
        self._active = 0
        self._bytes = 0
        self._lock = threading.Lock()
        self.stats_ = {"pairs": 0, "bytes": 0}

    def decode_pair(self, k_stream: tuple, v_stream: tuple) -> tuple[Any, Any]:
        """``(stream bytes, stream codec, raw shape)`` of K and of V -> their decoded coefficient arrays."""
        nbytes = int(torch.Size(k_stream[2]).numel() + torch.Size(v_stream[2]).numel())
        with self._lock:
            if self._active >= self.max_pairs or self._bytes + nbytes > self.max_output_bytes:
                raise CapacityError("the paired decoder is at its pair or output bound")
            self._active += 1
            self._bytes += nbytes
        try:
            k_ticket = self.pool.decode_stream(*k_stream)
            v_ticket = self.pool.decode_stream(*v_stream)
            out = (k_ticket.wait(), v_ticket.wait())
            self.stats_["pairs"] += 1
            self.stats_["bytes"] += nbytes
            return out
        finally:
            with self._lock:
                self._active -= 1
                self._bytes -= nbytes

    def stats(self) -> dict:
        return dict(self.stats_)


__all__ = ["LayerPrefetcher", "PackedLayerPrefetcher", "PairedDecoder"]
