"""Experimental, source-bound online ranks with atomic scalar-state candidates (the counterpart of reference
reelcache/online_rank.py: ``RankPolicy`` :490, ``RankState`` :910, ``predict_rank`` :1061, ``RankDecision``
:1169, ``PreparedRankMatrix`` :1383, ``RankAbstention`` :1438, ``RankPreparation`` :1446).

A :class:`RankPolicy` binds a model, a chunk geometry, per-matrix allowed rank sets and a layer template of
expected ranks; optional *anchor* matrices are measured with the fixed anchor detector and scale the template
for the other layers (causally: an anchor of a lower layer of the same chunk, or the previous chunk's value).
:class:`RankPreparation` prepares one clean chunk matrix by matrix: predict a rank, fit candidate directions,
and guard the stored representation (FP16 rows, FP32 coefficients) against the declared pre-codec direct
residual ``sqrt(1 - E_t)``, growing through the allowed ranks; a matrix that exhausts its guard attempts
abstains (:class:`RankAbstention`). An accepted decision certifies only that residual, nothing about the
codec or perceptual quality. Preparation never publishes: the caller commits the prepared factors, the
decisions and :meth:`RankPreparation.next_state` atomically.
"""

from __future__ import annotations

import math
from dataclasses import asdict, dataclass, field
from types import MappingProxyType
from typing import Any, Mapping

import torch

from .errors import CapacityError, ConfigurationError, StateError
from .factorization import (DetectorSpec, Factors, acquire_anchor_directions, fit_rank_directions,
                            project_rank_directions, tensor_sha256, validate_matrix)
from .types import CodecSpec, MatrixKey, ModelIdentity, TensorContext, canonical_digest

POLICY_SCHEMA = "reelcache.rank_policy.v1"
STATE_SCHEMA = "reelcache.rank_state.v1"
DECISION_SCHEMA = "reelcache.rank_decision.v1"
PREPARED_SCHEMA = "reelcache.prepared_rank_matrix.v1"
PREDICTOR_SCHEMA = "reelcache.rank_predictor_profile.v1"
ANCHOR_MODES = ("none", "causal", "staged")
SOLVERS = ("qr_q2", "exact_oracle")


def _label(key: MatrixKey) -> str:
    return f"{key.layer}:{key.target}"


def _key(label: str) -> MatrixKey:
    layer, target = label.split(":")
    return MatrixKey(int(layer), target)


def _finite(value: Any, name: str) -> float:
    if isinstance(value, bool) or not isinstance(value, (int, float)) or not math.isfinite(float(value)):
        raise ConfigurationError(f"{name} must be a finite number")
    return float(value)


def _keyed(values: Mapping, name: str) -> Mapping:
    if not isinstance(values, Mapping) or any(not isinstance(k, MatrixKey) for k in values):
        raise ConfigurationError(f"{name} must be a MatrixKey-keyed mapping")
    return MappingProxyType(dict(values))


@dataclass(frozen=True)
class RankPredictorProfile:
    """Calibrated prediction of one target in one history regime (``startup`` = first chunk, ``later``)."""

    target: str
    history_regime: str
    layer_template: tuple[float, ...]
    anchor_layers: tuple[int, ...] = ()
    rank_buckets: tuple[int, ...] = ()
    rank_margin: float = 0.0
    uniform_rank: int | None = None
    schema_version: str = PREDICTOR_SCHEMA

    def __post_init__(self) -> None:
        if self.target not in ("K", "V") or self.history_regime not in ("startup", "later"):
            raise ConfigurationError("predictor profiles are per K/V and startup/later regime")
        object.__setattr__(self, "layer_template", tuple(_finite(v, "template rank") for v in self.layer_template))
        object.__setattr__(self, "anchor_layers", tuple(int(v) for v in self.anchor_layers))
        object.__setattr__(self, "rank_buckets", tuple(int(v) for v in self.rank_buckets))


@dataclass(frozen=True)
class RankPrediction:
    key: MatrixKey
    predicted: float
    initial_rank: int
    sources: tuple = ()


@dataclass(frozen=True)
class RankPolicy:
    policy_id: str
    model: ModelIdentity
    geometry: tuple[int, int, int]
    energy_target: float
    template_ranks: Mapping[MatrixKey, float]
    allowed_ranks: Mapping[MatrixKey, tuple[int, ...]]
    codec: CodecSpec = field(default_factory=lambda: CodecSpec("svd", 1))
    anchors: tuple[MatrixKey, ...] = ()
    anchor_mode: str = "none"
    solver: str = "qr_q2"
    seed: int = 0
    prediction_margin: float = 1.0
    additive_margin: float = 0.0
    hysteresis_fraction: float = 0.0
    history_min: int = 1
    history_max: int = 3
    tile_rows: int = 1024
    oversample: int = 8
    fit_growth: float = 2.0
    max_fit_attempts: int = 4
    max_guard_attempts: int = 16
    source_limit_bytes: int = 1 << 30
    energy_targets: Mapping[str, float] | None = None
    predictor_profiles: Mapping[str, RankPredictorProfile] = field(default_factory=dict)
    detector_spec: DetectorSpec = field(default_factory=DetectorSpec)
    schema_version: str = POLICY_SCHEMA

    def __post_init__(self) -> None:
        if self.schema_version != POLICY_SCHEMA:
            raise ConfigurationError("unsupported rank policy schema")
        if not isinstance(self.policy_id, str) or not self.policy_id:
            raise ConfigurationError("policy_id must be a nonempty string")
        if not isinstance(self.model, ModelIdentity):
            raise ConfigurationError("rank policy requires a ModelIdentity")
        if len(self.geometry) != 3 or any(int(g) < 1 for g in self.geometry):
            raise ConfigurationError("geometry must be frames, height, width")
        object.__setattr__(self, "geometry", tuple(int(g) for g in self.geometry))
        energy = _finite(self.energy_target, "energy_target")
        if not 0 < energy <= 1:
            raise ConfigurationError("energy_target must lie in (0, 1]")
        if self.energy_targets is not None:
            if set(self.energy_targets) != {"K", "V"}:
                raise ConfigurationError("energy_targets must cover exactly K and V")
            object.__setattr__(self, "energy_targets", MappingProxyType(
                {k: _finite(v, "target energy") for k, v in self.energy_targets.items()}))
        if self.codec.kind == "raw":
            raise ConfigurationError("adaptive ranks require a lossy codec, never a RAW fallback")
        templates = _keyed(self.template_ranks, "template_ranks")
        allowed = _keyed(self.allowed_ranks, "allowed_ranks")
        if set(templates) != set(allowed) or not templates:
            raise ConfigurationError("template and allowed ranks must cover the same matrices")
        for key, ranks in allowed.items():
            ranks = tuple(int(r) for r in ranks)
            limit = min(self.tokens, self.model.channels_for(key))
            if not ranks or any(b <= a for a, b in zip(ranks, ranks[1:])) or ranks[0] < 1 or ranks[-1] > limit:
                raise ConfigurationError("allowed ranks must increase strictly within the matrix dimensions")
        object.__setattr__(self, "template_ranks", templates)
        object.__setattr__(self, "allowed_ranks", MappingProxyType({k: tuple(int(r) for r in v)
                                                                   for k, v in allowed.items()}))
        anchors = tuple(self.anchors)
        if any(a not in templates for a in anchors) or len(set(anchors)) != len(anchors):
            raise ConfigurationError("anchors must be unique policy keys")
        object.__setattr__(self, "anchors", anchors)
        if self.anchor_mode not in ANCHOR_MODES:
            raise ConfigurationError(f"anchor_mode must be one of {ANCHOR_MODES}")
        if self.anchor_mode == "none" and anchors:
            raise ConfigurationError("no-anchor mode cannot declare anchors")
        if self.solver not in SOLVERS:
            raise ConfigurationError("solver must be qr_q2 or exact_oracle")
        if not 1 <= self.history_min <= self.history_max:
            raise ConfigurationError("history support interval is reversed")
        if self.fit_growth <= 1.0 or self.prediction_margin <= 0:
            raise ConfigurationError("fit_growth must exceed one and prediction_margin be positive")
        if max(self.source_bytes_for(k) for k in templates) > self.source_limit_bytes:
            raise CapacityError("policy matrix exceeds its source allowance")

    @property
    def keys(self) -> tuple[MatrixKey, ...]:
        return tuple(sorted(self.template_ranks, key=lambda k: (k.layer, k.target)))

    @property
    def tokens(self) -> int:
        frames, height, width = self.geometry
        return frames * height * width

    def source_bytes_for(self, key: MatrixKey) -> int:
        return self.tokens * self.model.channels_for(key) * 4

    def target_for(self, key: MatrixKey) -> float:
        return self.energy_target if self.energy_targets is None else self.energy_targets[key.target]

    def spec_for(self, key: MatrixKey, rank: int) -> CodecSpec:
        if rank not in self.allowed_ranks[key]:
            raise ConfigurationError(f"rank {rank} is not allowed for {key}")
        return CodecSpec(**{**self.codec.to_dict(), "rank": int(rank)})

    def active_anchors(self, ordinal: int) -> tuple[MatrixKey, ...]:
        return self.anchors if self.anchor_mode != "none" else ()

    def to_dict(self) -> dict[str, Any]:
        return {"schema": self.schema_version, "policy_id": self.policy_id, "model": self.model.to_dict(),
                "geometry": list(self.geometry), "energy_target": self.energy_target,
                "energy_targets": None if self.energy_targets is None else dict(self.energy_targets),
                "template_ranks": {_label(k): v for k, v in self.template_ranks.items()},
                "allowed_ranks": {_label(k): list(v) for k, v in self.allowed_ranks.items()},
                "codec": self.codec.to_dict(), "anchors": [_label(a) for a in self.anchors],
                "anchor_mode": self.anchor_mode, "solver": self.solver, "seed": self.seed,
                "prediction_margin": self.prediction_margin, "additive_margin": self.additive_margin,
                "hysteresis_fraction": self.hysteresis_fraction, "history_min": self.history_min,
                "history_max": self.history_max, "tile_rows": self.tile_rows, "oversample": self.oversample,
                "fit_growth": self.fit_growth, "max_fit_attempts": self.max_fit_attempts,
                "max_guard_attempts": self.max_guard_attempts, "source_limit_bytes": self.source_limit_bytes,
                "predictor_profiles": {name: asdict(p) for name, p in self.predictor_profiles.items()},
                "detector_spec": self.detector_spec.to_dict()}

    @classmethod
    def from_dict(cls, data: Mapping[str, Any]) -> "RankPolicy":
        if data.get("schema") != POLICY_SCHEMA:
            raise ConfigurationError("not a rank policy record")
        return cls(data["policy_id"], ModelIdentity.from_dict(data["model"]), tuple(data["geometry"]),
                   data["energy_target"], {_key(k): v for k, v in data["template_ranks"].items()},
                   {_key(k): tuple(v) for k, v in data["allowed_ranks"].items()}, CodecSpec.from_dict(data["codec"]),
                   tuple(_key(a) for a in data["anchors"]), data["anchor_mode"], data["solver"], data["seed"],
                   data["prediction_margin"], data["additive_margin"], data["hysteresis_fraction"],
                   data["history_min"], data["history_max"], data["tile_rows"], data["oversample"],
                   data["fit_growth"], data["max_fit_attempts"], data["max_guard_attempts"],
                   data["source_limit_bytes"], data.get("energy_targets"),
                   {n: RankPredictorProfile(**p) for n, p in data.get("predictor_profiles", {}).items()},
                   DetectorSpec.from_dict(data["detector_spec"]))

    @property
    def fingerprint(self) -> str:
        return canonical_digest(self.to_dict())

    @property
    def policy_hash(self) -> str:
        return self.fingerprint


def _snap(predicted: float, buckets: tuple[int, ...]) -> int:
    """Smallest allowed rank at or above the prediction (the largest when none is)."""
    for rank in buckets:
        if rank >= predicted - 1e-9:
            return rank
    return buckets[-1]


def predict_rank(policy: RankPolicy, key: MatrixKey, *, chunk_ordinal: int, current_anchors: Mapping[MatrixKey, float],
                 previous_anchors: Mapping[MatrixKey, float],
                 previous_anchor_chunks: Mapping[MatrixKey, int]) -> RankPrediction:
    """Pure prediction: the layer template of ``key`` scaled by the geometric mean of the available anchors'
    measured/template ratios (current anchors where the mode allows them -- ``staged`` any, ``causal`` lower
    layers only -- else the previous chunk's), times ``prediction_margin`` plus ``additive_margin``."""
    if key not in policy.template_ranks:
        raise ConfigurationError("prediction key is outside the policy")
    if not policy.history_min <= chunk_ordinal <= policy.history_max:
        raise StateError("prediction is outside the policy's history support")
    if set(previous_anchors) != set(previous_anchor_chunks):
        raise ConfigurationError("previous anchors need their source chunks")
    if any(chunk >= chunk_ordinal for chunk in previous_anchor_chunks.values()):
        raise ConfigurationError("previous anchors cannot come from the current or a future chunk")
    regime = "startup" if chunk_ordinal == 1 else "later"
    profile = policy.predictor_profiles.get(f"{regime}:{key.target}")
    if profile is not None and profile.uniform_rank is not None:
        buckets = policy.allowed_ranks[key]
        return RankPrediction(key, float(profile.uniform_rank), _snap(profile.uniform_rank, buckets),
                              ({"source": "uniform_rank"},))
    template = {k.layer: v for k, v in policy.template_ranks.items() if k.target == key.target}
    if profile is not None:
        template = dict(enumerate(profile.layer_template))
    ratios, sources = [], []
    if key not in policy.anchors:
        for anchor in policy.active_anchors(chunk_ordinal):
            if anchor.target != key.target or template.get(anchor.layer, 0) <= 0:
                continue
            current_ok = policy.anchor_mode == "staged" or (policy.anchor_mode == "causal" and anchor.layer < key.layer)
            if current_ok and anchor in current_anchors:
                value, origin = current_anchors[anchor], "current"
            elif anchor in previous_anchors:
                value, origin = previous_anchors[anchor], "previous"
            else:
                continue
            ratios.append(max(float(value), 1.0) / template[anchor.layer])
            sources.append({"anchor": _label(anchor), "value": float(value), "origin": origin})
    scale = math.exp(sum(math.log(r) for r in ratios) / len(ratios)) if ratios else 1.0
    margin = policy.additive_margin if profile is None else profile.rank_margin
    predicted = template[key.layer] * scale * policy.prediction_margin + margin
    return RankPrediction(key, predicted, _snap(predicted, policy.allowed_ranks[key]), tuple(sources))


@dataclass(frozen=True)
class RankState:
    """The scalar state carried from chunk to chunk (anchors and selected ranks), committed with each node."""

    policy_hash: str
    last_chunk_id: str | None = None
    parent_head: str | None = None
    token_end: int = 0
    completed_chunks: int = 0
    anchor_ranks: Mapping[MatrixKey, float] = field(default_factory=dict)
    anchor_chunks: Mapping[MatrixKey, int] = field(default_factory=dict)
    selected_ranks: Mapping[MatrixKey, int] = field(default_factory=dict)
    schema_version: str = STATE_SCHEMA

    def __post_init__(self) -> None:
        if self.schema_version != STATE_SCHEMA:
            raise ConfigurationError("unsupported rank state schema")
        for name in ("anchor_ranks", "anchor_chunks", "selected_ranks"):
            object.__setattr__(self, name, _keyed(getattr(self, name), name))
        if set(self.anchor_ranks) != set(self.anchor_chunks):
            raise ConfigurationError("anchor values and their chunks differ")
        if any(c > self.completed_chunks or c < 1 for c in self.anchor_chunks.values()):
            raise ConfigurationError("a saved anchor cannot come from the future")
        if self.completed_chunks == 0:
            if self.last_chunk_id is not None or self.parent_head is not None or self.selected_ranks:
                raise ConfigurationError("an empty rank state contains committed history")
        elif self.last_chunk_id is None or not self.selected_ranks or self.token_end < 1:
            raise ConfigurationError("a committed rank state is incomplete")

    def to_dict(self) -> dict[str, Any]:
        return {"schema": self.schema_version, "policy_hash": self.policy_hash, "last_chunk_id": self.last_chunk_id,
                "parent_head": self.parent_head, "token_end": self.token_end,
                "completed_chunks": self.completed_chunks,
                "anchor_ranks": {_label(k): v for k, v in self.anchor_ranks.items()},
                "anchor_chunks": {_label(k): v for k, v in self.anchor_chunks.items()},
                "selected_ranks": {_label(k): v for k, v in self.selected_ranks.items()}}

    @classmethod
    def from_dict(cls, data: Mapping[str, Any]) -> "RankState":
        if data.get("schema") != STATE_SCHEMA:
            raise ConfigurationError("not a rank state record")
        return cls(data["policy_hash"], data["last_chunk_id"], data["parent_head"], data["token_end"],
                   data["completed_chunks"], {_key(k): v for k, v in data["anchor_ranks"].items()},
                   {_key(k): v for k, v in data["anchor_chunks"].items()},
                   {_key(k): v for k, v in data["selected_ranks"].items()})

    @property
    def fingerprint(self) -> str:
        return canonical_digest(self.to_dict())


@dataclass(frozen=True)
class RankDecision:
    policy_hash: str
    chunk_id: str
    parent_head: str | None
    context: TensorContext
    input_sha256: str
    energy_target: float
    solver: str
    predicted_rank: float
    initial_rank: int
    status: str                         # "accepted" | "abstained"
    reason: str
    rank: int | None = None
    resolved_spec: CodecSpec | None = None
    fit_width: int = 0
    guard_threshold: float = 0.0
    guard_relative_residual: float | None = None
    guard_passed: bool = False
    zero_input: bool = False
    prediction_sources: tuple = ()
    attempts: tuple = ()
    metrics: Mapping[str, Any] = field(default_factory=dict)
    schema_version: str = DECISION_SCHEMA

    def __post_init__(self) -> None:
        if self.status not in ("accepted", "abstained"):
            raise ConfigurationError("decision status is accepted or abstained")
        if self.status == "accepted" and (self.rank is None or not self.guard_passed):
            raise ConfigurationError("an accepted decision carries a guarded rank")

    @property
    def key(self) -> MatrixKey:
        return self.context.key

    def to_dict(self) -> dict[str, Any]:
        return {"schema": self.schema_version, "policy_hash": self.policy_hash, "chunk_id": self.chunk_id,
                "parent_head": self.parent_head, "context": self.context.to_dict(), "input_sha256": self.input_sha256,
                "energy_target": self.energy_target, "solver": self.solver, "predicted_rank": self.predicted_rank,
                "initial_rank": self.initial_rank, "status": self.status, "reason": self.reason, "rank": self.rank,
                "resolved_spec": None if self.resolved_spec is None else self.resolved_spec.to_dict(),
                "fit_width": self.fit_width, "guard_threshold": self.guard_threshold,
                "guard_relative_residual": self.guard_relative_residual, "guard_passed": self.guard_passed,
                "zero_input": self.zero_input, "prediction_sources": list(self.prediction_sources),
                "attempts": list(self.attempts), "metrics": dict(self.metrics)}


@dataclass(frozen=True)
class PreparedRankMatrix:
    decision: RankDecision
    factors: Factors
    schema_version: str = PREPARED_SCHEMA

    @property
    def key(self) -> MatrixKey:
        return self.decision.key


class RankAbstention(StateError):
    """A matrix exhausted its guard attempts; the chunk cannot be prepared under the policy."""

    def __init__(self, decision: RankDecision):
        super().__init__(f"rank abstention for {decision.key}: {decision.reason}")
        self.decision = decision


class RankPreparation:
    """One clean-chunk attempt under a policy; never mutates the prior state. Use as a context manager or call
    :meth:`close`; :meth:`next_state` is available once every policy matrix is prepared."""

    def __init__(self, policy: RankPolicy, prior_state: RankState | None = None, *, chunk_id: str,
                 parent_head: str | None, token_start: int, device: Any = None):
        if not isinstance(policy, RankPolicy):
            raise ConfigurationError("preparation requires a RankPolicy")
        prior = RankState(policy.fingerprint) if prior_state is None else prior_state
        if not isinstance(prior, RankState) or prior.policy_hash != policy.fingerprint:
            raise ConfigurationError("the prior state belongs to another policy")
        if prior.completed_chunks:
            if parent_head is None or token_start != prior.token_end or chunk_id == prior.last_chunk_id:
                raise ConfigurationError("the prior rank state does not match the requested history boundary")
        elif parent_head is not None:
            raise ConfigurationError("adaptive history cannot start on an unbound existing head")
        ordinal = prior.completed_chunks + 1
        if not policy.history_min <= ordinal <= policy.history_max:
            raise StateError("the clean chunk is outside the policy's history support")
        self.policy, self.prior_state = policy, prior
        self.chunk_id, self.parent_head, self.token_start = chunk_id, parent_head, int(token_start)
        self.ordinal = ordinal
        self.device = device
        self._decisions: dict[MatrixKey, RankDecision] = {}
        self._anchors: dict[MatrixKey, float] = {}
        self._metrics = {"fits": 0, "guards": 0, "anchor_acquisitions": 0, "abstentions": 0}
        self._closed = False

    def __enter__(self) -> "RankPreparation":
        return self

    def __exit__(self, *_: Any) -> None:
        self.close()

    def close(self) -> None:
        self._closed = True

    @property
    def decisions(self) -> Mapping[MatrixKey, RankDecision]:
        return MappingProxyType(dict(self._decisions))

    def metrics(self) -> Mapping[str, Any]:
        return MappingProxyType(dict(self._metrics))

    def _check_context(self, context: TensorContext) -> None:
        policy = self.policy
        if context.model != policy.model or context.key not in policy.template_ranks:
            raise ConfigurationError("the matrix is outside the policy")
        if (context.frames, context.height, context.width) != policy.geometry:
            raise ConfigurationError("the matrix geometry differs from the policy")
        if context.token_start != self.token_start:
            raise ConfigurationError("the matrix does not start at the chunk's first token")
        if context.key in self._decisions:
            raise StateError("the matrix was prepared already")

    def prediction(self, key: MatrixKey) -> RankPrediction:
        return predict_rank(self.policy, key, chunk_ordinal=self.ordinal, current_anchors=self._anchors,
                            previous_anchors=self.prior_state.anchor_ranks,
                            previous_anchor_chunks=self.prior_state.anchor_chunks)

    def prepare_matrix(self, tensor: torch.Tensor, context: TensorContext) -> PreparedRankMatrix:
        """Predict, fit and guard one matrix; raises :class:`RankAbstention` when no allowed rank passes."""
        if self._closed:
            raise StateError("the preparation is closed")
        self._check_context(context)
        policy, key = self.policy, context.key
        x = validate_matrix(tensor, context)
        if self.device is not None:
            x = x.to(self.device)
        target = policy.target_for(key)
        threshold = math.sqrt(max(0.0, 1.0 - target))
        if key in policy.anchors:  # the fixed detector measures the anchor's rank at the target energy
            acquisition = acquire_anchor_directions(x, context, policy.detector_spec)
            self._metrics["anchor_acquisitions"] += 1
            rank_at = acquisition.rank_at(target)
            self._anchors[key] = float(rank_at if rank_at is not None else acquisition.width)
        prediction = self.prediction(key)
        buckets = policy.allowed_ranks[key]
        start = buckets.index(prediction.initial_rank)
        if policy.hysteresis_fraction > 0 and key in self.prior_state.selected_ranks:
            previous = self.prior_state.selected_ranks[key]
            if previous in buckets and abs(previous - prediction.predicted) <= policy.hysteresis_fraction * previous:
                start = buckets.index(previous)
        attempts = []
        fit = None
        fit_width = 0
        digest = tensor_sha256(x)
        total = float(x.double().square().sum())
        for index in range(start, min(len(buckets), start + policy.max_guard_attempts)):
            rank = buckets[index]
            if fit is None or rank > fit_width:
                if len([a for a in attempts if a["kind"] == "fit"]) >= policy.max_fit_attempts:
                    break
                fit_width = min(min(x.shape), max(rank + policy.oversample, int(math.ceil(rank * policy.fit_growth))))
                fit = fit_rank_directions(x, fit_width, seed=policy.seed, solver="topk_rr")
                self._metrics["fits"] += 1
                attempts.append({"kind": "fit", "width": fit_width})
            if total == 0.0:
                projection = None
                residual = 0.0
            else:
                projection = project_rank_directions(x, fit.directions, rank)
                residual = projection.relative_residual
            self._metrics["guards"] += 1
            attempts.append({"kind": "guard", "rank": rank, "relative_residual": residual})
            if residual <= threshold:
                rows = fit.directions[:, :rank].t().contiguous().to(torch.float16)
                coefficients = (projection.coefficients if projection is not None else
                                torch.zeros((x.shape[0], rank), dtype=torch.float32, device=x.device))
                decision = RankDecision(policy.fingerprint, self.chunk_id, self.parent_head, context, digest, target,
                                        policy.solver, prediction.predicted, prediction.initial_rank, "accepted",
                                        "guard_passed", rank, policy.spec_for(key, rank), fit_width, threshold,
                                        residual, True, total == 0.0, prediction.sources, tuple(attempts))
                self._decisions[key] = decision
                return PreparedRankMatrix(decision, Factors(rows, coefficients, rank, {"relative_residual": residual}))
        decision = RankDecision(policy.fingerprint, self.chunk_id, self.parent_head, context, digest, target,
                                policy.solver, prediction.predicted, prediction.initial_rank, "abstained",
                                "guard_attempts_exhausted", fit_width=fit_width, guard_threshold=threshold,
                                guard_relative_residual=attempts[-1].get("relative_residual") if attempts else None,
                                prediction_sources=prediction.sources, attempts=tuple(attempts))
        self._decisions[key] = decision
        self._metrics["abstentions"] += 1
        raise RankAbstention(decision)

    def prepare_staged(self, sources: Mapping[MatrixKey, torch.Tensor],
                       contexts: Mapping[MatrixKey, TensorContext]) -> dict[MatrixKey, PreparedRankMatrix]:
        """Prepare every matrix of the chunk, anchors first (their measurements feed the others)."""
        order = sorted(contexts, key=lambda k: (k not in self.policy.anchors, k.layer, k.target))
        return {key: self.prepare_matrix(sources[key], contexts[key]) for key in order}

    def next_state(self) -> RankState:
        """The scalar state after this chunk (every matrix accepted)."""
        missing = set(self.policy.keys) - set(self._decisions)
        if missing:
            raise StateError(f"{len(missing)} policy matrices are not prepared")
        if any(d.status != "accepted" for d in self._decisions.values()):
            raise StateError("an abstained chunk has no next state")
        anchors = dict(self.prior_state.anchor_ranks)
        chunks = dict(self.prior_state.anchor_chunks)
        for key, value in self._anchors.items():
            anchors[key] = value
            chunks[key] = self.ordinal
        return RankState(self.policy.fingerprint, self.chunk_id, self.parent_head,
                         self.token_start + self.policy.tokens, self.ordinal, anchors, chunks,
                         {k: d.rank for k, d in self._decisions.items()})


__all__ = ["PreparedRankMatrix", "RankAbstention", "RankDecision", "RankPolicy", "RankPrediction",
           "RankPredictorProfile", "RankPreparation", "RankState", "predict_rank"]
