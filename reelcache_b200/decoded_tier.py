"""Decoded-coefficient tier (the counterpart of reference reelcache/decoded_tier.py:196-602; routing rule
from its docstring, lines 1-30).

Pinned host memory holding the decoder's output -- the uint8 coefficient tiles of hot node packs --
keyed by the SHA-256 of the pack's coefficient stream (the content that determines the tiles, so a
routed restore is bitwise the same as a decoded one). :meth:`route` decides per restore which packs
skip the decoder and arrive by host->device copy instead:

* ``"deficit"`` routes the oldest cached history packs until the predicted decode time per layer
  (stream bytes / ``decode_gbps``) is at most ``target`` x the per-layer compute of the forward that
  consumes them, ``c(h) = a + b * min(h, window)`` ms for ``h`` history nodes;
* ``"all"`` routes every cached pack.

Routed entries are leased until released; eviction (LRU under ``budget_bytes``) skips leased entries.
"""

from __future__ import annotations

import threading
from collections import OrderedDict
from typing import Any, Mapping, Sequence

import numpy as np
import torch

from .errors import ConfigurationError

ROUTES = ("deficit", "all")
# Per-layer compute c(h) = a + b * min(h, window) [ms] of the first denoising forward, per model profile
# (measured by the reference on RTX PRO 6000; the B200 values are lower, which routes fewer packs).
LAYER_COMPUTE_MS = {"causvid": (2.58, 0.486, None), "raven": (3.23, 0.524, None), "longlive1": (4.04, 0.0, 3),
                    "longlive2": (10.91, 0.0, 3), "lingbot": (18.43, 1.188, None)}
DECODE_GBPS = 0.9
TARGET = 0.85


class DecodedTier:
    def __init__(self, budget_bytes: int, *, route: str = "deficit", decode_gbps: float = DECODE_GBPS,
                 layer_ms: tuple | None = None, model: str = "causvid", target: float = TARGET,
                 pinned: bool = True):
        if type(budget_bytes) is not int or budget_bytes < 0:
            raise ConfigurationError("decoded tier budget must be a nonnegative byte count")
        if route not in ROUTES:
            raise ConfigurationError(f"route must be one of {ROUTES}")
        self.budget = budget_bytes
        self.route_mode = route
        self.decode_gbps = decode_gbps
        self.layer_ms = layer_ms or LAYER_COMPUTE_MS.get(model, LAYER_COMPUTE_MS["causvid"])
        self.target = target
        self.pinned = pinned and torch.cuda.is_available()
        self.lock = threading.Lock()
        self._entries: "OrderedDict[str, dict]" = OrderedDict()   # digest -> {tiles, nbytes, leases}
        self._bindings: dict[str, str] = {}                        # packet ref -> digest
        self.bytes = 0
        self.counts = {"offered": 0, "stored": 0, "skipped": 0, "evicted": 0, "routed": 0, "hits": 0}

    def offer(self, digest: str, tiles: Sequence[np.ndarray]) -> bool:
        """Cache a pack's decoded tiles (copied into pinned memory); False when it cannot fit."""
        nbytes = sum(t.nbytes for t in tiles)
        with self.lock:
            self.counts["offered"] += 1
            if digest in self._entries:
                self._entries.move_to_end(digest)
                return True
            if nbytes > self.budget:
                self.counts["skipped"] += 1
                return False
            self._evict(nbytes)
            if self.bytes + nbytes > self.budget:
                self.counts["skipped"] += 1
                return False
        host = []
        for t in tiles:
            h = torch.from_numpy(np.array(t, copy=True))
            host.append(h.pin_memory() if self.pinned else h.clone())
        with self.lock:
            self._entries[digest] = {"tiles": host, "nbytes": nbytes, "leases": 0}
            self.bytes += nbytes
            self.counts["stored"] += 1
        return True

    def _evict(self, needed: int) -> None:
        for digest in list(self._entries):
            if self.bytes + needed <= self.budget:
                return
            entry = self._entries[digest]
            if entry["leases"]:
                continue
            del self._entries[digest]
            self.bytes -= entry["nbytes"]
            self.counts["evicted"] += 1

    def bind(self, packet_ref: str, digest: str) -> None:
        with self.lock:
            self._bindings[packet_ref] = digest

    def layer_compute_ms(self, history_nodes: int) -> float:
        a, b, window = self.layer_ms
        h = history_nodes if window is None else min(history_nodes, window)
        return a + b * h

    def route(self, packs: Sequence[tuple[str, int]], layers: int) -> list[str]:
        """``packs``: ``(packet ref, stream bytes)`` oldest first. Returns the packet refs to serve from
        the tier (leased until :meth:`release`)."""
        with self.lock:
            cached = [(ref, n) for ref, n in packs if self._bindings.get(ref) in self._entries]
            if self.route_mode == "all":
                chosen = [ref for ref, _ in cached]
            else:
                budget_ms = self.target * self.layer_compute_ms(len(packs))
                decode_ms = sum(n for _, n in packs) / layers / (self.decode_gbps * 1e6)
                chosen = []
                for ref, n in cached:
                    if decode_ms <= budget_ms:
                        break
                    chosen.append(ref)
                    decode_ms -= n / layers / (self.decode_gbps * 1e6)
            for ref in chosen:
                entry = self._entries[self._bindings[ref]]
                entry["leases"] += 1
                self._entries.move_to_end(self._bindings[ref])
            self.counts["routed"] += len(chosen)
            return chosen

    def tiles(self, packet_ref: str) -> list[torch.Tensor]:
        with self.lock:
            self.counts["hits"] += 1
            return self._entries[self._bindings[packet_ref]]["tiles"]

    def release(self, packet_refs: Sequence[str]) -> None:
        with self.lock:
            for ref in packet_refs:
                digest = self._bindings.get(ref)
                if digest in self._entries:
                    self._entries[digest]["leases"] = max(0, self._entries[digest]["leases"] - 1)

    def forget_packets(self, packet_refs: Sequence[str]) -> int:
        with self.lock:
            dropped = 0
            for ref in packet_refs:
                digest = self._bindings.pop(ref, None)
                if digest in self._entries and not self._entries[digest]["leases"]:
                    self.bytes -= self._entries.pop(digest)["nbytes"]
                    dropped += 1
            return dropped

    def stats(self) -> dict[str, Any]:
        with self.lock:
            return {"bytes": self.bytes, "budget_bytes": self.budget, "entries": len(self._entries), **self.counts}
