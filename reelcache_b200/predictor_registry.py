"""Model-scoped online rank learners (reference: reelcache/predictor_registry.py:45-335).

One :class:`~reelcache_b200.types.OnlineRidgeState` per :class:`~reelcache_b200.types.PredictorKey`
(model/source, layer, K|V, geometry, solver/detector, regime) learns ``ln r = a + b x`` with
``x = ln((1 - E_m) / (1 - E_t))``. Planners pin an immutable :class:`RegistryView` (optionally with
observations of not-yet-published nodes applied), so a plan never depends on publication timing;
verified observations are applied idempotently by observation id.
"""

from __future__ import annotations

import math
import threading
from dataclasses import dataclass
from types import MappingProxyType
from typing import Any, Iterable, Mapping

from .errors import ConfigurationError, IntegrityError
from .types import RANK_BUCKET, FitObservation, OnlineRidgeState, PredictorKey, canonical_digest

REGISTRY_SCHEMA = "reelcache.predictor_registry.v1"


def observation_origin(lineage: str, kind: str, node_id: str, view: "RegistryView") -> str:
    """Run context of an observation (never content): lineage, commit kind, node and pinned view."""
    return canonical_digest({"lineage": lineage, "kind": kind, "node": node_id, "view": view.digest})


@dataclass(frozen=True)
class PredictorUse:
    """A prediction made from a pinned learner state."""

    key: PredictorKey
    x: float
    predicted_rank: float
    revision: int
    state_digest: str

    @property
    def revision_ref(self) -> str:
        return f"{self.key.digest}@{self.revision}"

    def to_dict(self) -> dict[str, Any]:
        return {"key": self.key.to_dict(), "x": self.x,
                "predicted_rank": self.predicted_rank if math.isfinite(self.predicted_rank) else None,
                "revision": self.revision, "state": self.state_digest}


class RegistryView:
    """An immutable snapshot of every learner (missing keys read as the prior)."""

    def __init__(self, registry_id: str, sequence: int, states: Mapping[PredictorKey, OnlineRidgeState],
                 anchor_rank: int = RANK_BUCKET, prior_strength: float = 2.0):
        self.registry_id = registry_id
        self.sequence = sequence
        self._states = MappingProxyType(dict(states))
        self.anchor_rank = anchor_rank
        self.prior_strength = prior_strength

    @property
    def states(self) -> Mapping[PredictorKey, OnlineRidgeState]:
        return self._states

    def state(self, key: PredictorKey) -> OnlineRidgeState:
        state = self._states.get(key)
        return state if state is not None else OnlineRidgeState.initial(self.anchor_rank, self.prior_strength)

    def predict(self, key: PredictorKey, x: float) -> PredictorUse:
        state = self.state(key)
        return PredictorUse(key, float(x), state.predict(x), state.revision, state.digest)

    @property
    def digest(self) -> str:
        return canonical_digest({"registry": self.registry_id, "sequence": self.sequence,
                                 "states": sorted((k.digest, s.digest) for k, s in self._states.items())})


class RankPredictorRegistry:
    """Mutable owner of the learners; ``pin`` hands planners immutable views."""

    def __init__(self, registry_id: str, *, anchor_rank: int = RANK_BUCKET, prior_strength: float = 2.0,
                 mode: str = "shared"):
        if not isinstance(registry_id, str) or not registry_id:
            raise ConfigurationError("registry id must be a nonempty string")
        if mode not in ("shared", "frozen"):
            raise ConfigurationError("registry mode must be shared or frozen")
        self.registry_id = registry_id
        self.anchor_rank = anchor_rank
        self.prior_strength = float(prior_strength)
        self.mode = mode
        self._lock = threading.Lock()
        self._states: dict[PredictorKey, OnlineRidgeState] = {}
        self._applied: dict[str, tuple[str, str | None]] = {}
        self._sequence = 0
        self._log: list[str] = []

    @property
    def sequence(self) -> int:
        return self._sequence

    @property
    def log(self) -> tuple[str, ...]:
        return tuple(self._log)

    def pin(self) -> RegistryView:
        with self._lock:
            return RegistryView(self.registry_id, self._sequence, self._states, self.anchor_rank, self.prior_strength)

    def state(self, key: PredictorKey) -> OnlineRidgeState:
        return self.pin().state(key)

    def pin_with(self, pending: Iterable[FitObservation]) -> RegistryView:
        """A view with ``pending`` (observations of unpublished ancestors) applied on top, in order."""
        with self._lock:
            states = dict(self._states)
            applied = dict(self._applied)
            sequence = self._sequence
        for item in pending:
            ident = item.observation_id
            if ident in applied:
                continue
            applied[ident] = (item.payload_digest, item.origin)
            base = states.get(item.key) or OnlineRidgeState.initial(self.anchor_rank, self.prior_strength)
            states[item.key] = base.updated(item.x, item.observed_rank)
            sequence += 1
        return RegistryView(self.registry_id, sequence, states, self.anchor_rank, self.prior_strength)

    def observe(self, observations: Iterable[FitObservation]) -> tuple[bool, ...]:
        """Apply verified observations; returns which were applied (repeats are skipped, conflicting
        repeats from the same origin raise IntegrityError)."""
        results = []
        with self._lock:
            for item in observations:
                if not isinstance(item, FitObservation):
                    raise ConfigurationError("observe takes FitObservation values")
                ident = item.observation_id
                known = self._applied.get(ident)
                if known is not None:
                    payload, origin = known
                    if payload != item.payload_digest and (origin is None or item.origin is None
                                                           or origin == item.origin):
                        raise IntegrityError("a repeated observation carries a different payload")
                    results.append(False)
                    continue
                if self.mode == "frozen":
                    results.append(False)
                    continue
                base = self._states.get(item.key) or OnlineRidgeState.initial(self.anchor_rank, self.prior_strength)
                self._states[item.key] = base.updated(item.x, item.observed_rank)
                self._applied[ident] = (item.payload_digest, item.origin)
                self._sequence += 1
                self._log.append(ident)
                results.append(True)
        return tuple(results)

    def to_dict(self) -> dict[str, Any]:
        with self._lock:
            return {"schema": REGISTRY_SCHEMA, "registry_id": self.registry_id, "anchor_rank": self.anchor_rank,
                    "prior_strength": self.prior_strength, "sequence": self._sequence,
                    "learners": [{"key": k.to_dict(), "state": s.to_dict()}
                                 for k, s in sorted(self._states.items(), key=lambda kv: kv[0].digest)],
                    "applied": sorted(self._applied)}

    @classmethod
    def from_dict(cls, data: Mapping[str, Any], *, mode: str = "shared") -> RankPredictorRegistry:
        if data.get("schema") != REGISTRY_SCHEMA:
            raise ConfigurationError("unsupported predictor registry schema")
        registry = cls(data["registry_id"], anchor_rank=data["anchor_rank"], prior_strength=data["prior_strength"],
                       mode=mode)
        for item in data["learners"]:
            registry._states[PredictorKey.from_dict(item["key"])] = OnlineRidgeState.from_dict(item["state"])
        for ident in data.get("applied", ()):
            registry._applied[ident] = ("", None)
        registry._sequence = data["sequence"]
        return registry
