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

_TIERS: "list[DecodedTier]" = []
_TIERS_LOCK = threading.Lock()


def layer_compute_model(model_name: str | None, layer_ms: Any = None) -> tuple[float, float, int | None, str]:
    """``(a, b, window, source)`` of the per-layer compute model ``c(h) = a + b * min(h, window)`` [ms]:
    ``layer_ms`` (``[a, b]``, the ``decoded_tier_layer_ms`` setting) wins; otherwise the longest profile name of
    :data:`LAYER_COMPUTE_MS` contained in ``model_name`` (case-insensitive); otherwise the CausVid profile."""
    if layer_ms is not None:
        values = [float(v) for v in layer_ms]
        if len(values) != 2 or not all(np.isfinite(values)) or min(values) < 0:
            raise ConfigurationError(f"layer_ms {layer_ms!r}: expected two finite non-negative numbers [a, b]")
        return values[0], values[1], None, "configured"
    lowered = (model_name or "").lower()
    matches = [name for name in LAYER_COMPUTE_MS if name in lowered]
    if matches:
        best = max(matches, key=len)
        return (*LAYER_COMPUTE_MS[best], f"default:{best}")
    return (*LAYER_COMPUTE_MS["causvid"], "default:causvid(unknown model)")


def open_tiers() -> "list[DecodedTier]":
    """Every decoded tier of this process that is still open (decoders offer their output to each)."""
    with _TIERS_LOCK:
        return [tier for tier in _TIERS if not tier.closed]


def offer_decoded(digest: str, tiles: Sequence[np.ndarray]) -> int:
    """Offer one pack's decoded tiles to every open tier; returns how many kept them."""
    return sum(bool(tier.offer(digest, tiles)) for tier in open_tiers())


class DecodedTier:
    def __init__(self, budget_bytes: int, *, route: str = "deficit", decode_gbps: float = DECODE_GBPS,
                 layer_ms: Any = None, model: str = "causvid", target: float = TARGET,
                 pinned: bool = True, register: bool = False):
        """``model``: the engine's model name, matched against :data:`LAYER_COMPUTE_MS` by
        :func:`layer_compute_model`; ``layer_ms`` overrides it with ``[a, b]``. ``register``: list the tier in
        :func:`open_tiers` so decoders offer their output to it (:func:`offer_decoded`)."""
        if type(budget_bytes) is not int or budget_bytes < 0:
            raise ConfigurationError(f"decoded tier budget {budget_bytes!r}: expected a byte count >= 0")
        if route not in ROUTES:
            raise ConfigurationError(f"route {route!r}: expected one of {ROUTES}")
        self.budget = budget_bytes
        self.route_mode = route
        self.decode_gbps = decode_gbps
        if isinstance(layer_ms, tuple) and len(layer_ms) == 3:       # (a, b, window) given directly
            self.layer_model = (float(layer_ms[0]), float(layer_ms[1]), layer_ms[2], "configured")
        else:
            self.layer_model = layer_compute_model(model, layer_ms)
        self.layer_ms = self.layer_model[:3]
        self.last_route: dict[str, Any] | None = None
        self.closed = False
        self.target = target
        self.pinned = pinned and torch.cuda.is_available()
        self.lock = threading.Lock()
        self._entries: "OrderedDict[str, dict]" = OrderedDict()   # digest -> {tiles, nbytes, leases}
        self._bindings: dict[str, str] = {}                        # packet ref -> digest
        self.bytes = 0
        self.counts = {"offered": 0, "stored": 0, "skipped": 0, "evicted": 0, "routed": 0, "hits": 0,
                       "restores": 0, "misses": 0}
        if register:
            with _TIERS_LOCK:
                _TIERS.append(self)

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
        """``packs``: ``(packet ref, stream bytes)`` oldest first. Returns the packet refs to serve from the tier
        (leased until :meth:`release`); :attr:`last_route` records the decision: the predicted decode time per
        layer before and after routing, ``c(h)`` and its source, hits (cached packs taken) and misses."""
        layers = max(1, int(layers))
        ms_per_byte = 1.0 / (self.decode_gbps * 1e6)
        c_ms = self.layer_compute_ms(len(packs))
        before = sum(n for _, n in packs) * ms_per_byte / layers
        with self.lock:
            cached = [(ref, n) for ref, n in packs if self._bindings.get(ref) in self._entries]
            chosen, remaining = [], before
            for ref, n in cached:
                if self.route_mode == "deficit" and remaining <= self.target * c_ms:
                    break
                chosen.append(ref)
                remaining -= n * ms_per_byte / layers
            for ref in chosen:
                entry = self._entries[self._bindings[ref]]
                entry["leases"] += 1
                self._entries.move_to_end(self._bindings[ref])
            self.counts["routed"] += len(chosen)
            self.counts["restores"] += 1
            self.counts["misses"] += len(packs) - len(cached)
        self.last_route = {"route": self.route_mode, "history": len(packs), "layers": layers, "c_ms": c_ms,
                           "c_model": self.layer_model[3], "target": self.target, "decode_gbps": self.decode_gbps,
                           "predicted_decode_ms_per_layer": before, "predicted_decode_ms_per_layer_after": remaining,
                           "routed": len(chosen), "hits": len(chosen), "misses": len(packs) - len(cached),
                           "routed_bitstream_bytes": sum(n for ref, n in cached if ref in chosen)}
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
            return {"bytes": self.bytes, "budget_bytes": self.budget, "entries": len(self._entries),
                    "layer_model": list(self.layer_model), **self.counts}

    def close(self) -> None:
        """Drop every entry and leave the process registry."""
        with self.lock:
            self._entries.clear()
            self._bindings.clear()
            self.bytes = 0
            self.closed = True
        with _TIERS_LOCK:
            if self in _TIERS:
                _TIERS.remove(self)
