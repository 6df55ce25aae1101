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
    number = isinstance(value, (int, float)) and not isinstance(value, bool)
    if number and math.isfinite(value):
        return float(value)
    raise ConfigurationError(f"{name}={value!r} is not a finite int or float")


def _keyed(values: Mapping, name: str) -> Mapping:
    """A read-only copy of a mapping whose keys are all :class:`MatrixKey`."""
    if isinstance(values, Mapping) and all(isinstance(key, MatrixKey) for key in values):
        return MappingProxyType(dict(values))
    raise ConfigurationError(f"{name} must map MatrixKey -> value")


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
        if (self.target, self.history_regime) not in {(t, r) for t in "KV" for r in ("startup", "later")}:
            raise ConfigurationError(f"predictor profile ({self.target!r}, {self.history_regime!r}): the target is K "
                                     f"or V and the regime startup or later")
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
        def reject(problem):
            raise ConfigurationError(f"RankPolicy {self.policy_id!r}: {problem}")

        if self.schema_version != POLICY_SCHEMA:
            reject(f"schema {self.schema_version!r} is not {POLICY_SCHEMA}")
        if not (isinstance(self.policy_id, str) and self.policy_id):
            raise ConfigurationError("RankPolicy: policy_id must be a non-empty string")
        if not isinstance(self.model, ModelIdentity):
            reject(f"model is {type(self.model).__name__}, not ModelIdentity")
        grid = tuple(int(g) for g in self.geometry)
        if len(grid) != 3 or min(grid) < 1:
            reject(f"geometry {self.geometry!r} is not a positive (frames, height, width)")
        object.__setattr__(self, "geometry", grid)
        if not 0 < _finite(self.energy_target, "energy_target") <= 1:
            reject(f"energy_target {self.energy_target} is outside (0, 1]")
        if self.energy_targets is not None:
            if set(self.energy_targets) != {"K", "V"}:
                reject(f"energy_targets names {sorted(self.energy_targets)}; it needs K and V")
            object.__setattr__(self, "energy_targets", MappingProxyType(
                {target: _finite(value, f"energy_targets[{target}]") for target, value in self.energy_targets.items()}))
        if self.codec.kind == "raw":
            reject("the codec is raw; adaptive ranks need svd or svd_hevc")
        templates = _keyed(self.template_ranks, "template_ranks")
        allowed = {key: tuple(int(r) for r in ranks) for key, ranks in _keyed(self.allowed_ranks, "allowed_ranks").items()}
        if not templates or set(templates) != set(allowed):
            reject("template_ranks and allowed_ranks must name the same non-empty set of matrices")
        for key, ranks in allowed.items():
            ceiling = min(self.tokens, self.model.channels_for(key))
            increasing = all(lo < hi for lo, hi in zip(ranks, ranks[1:]))
            if not (ranks and increasing and 1 <= ranks[0] and ranks[-1] <= ceiling):
                reject(f"allowed ranks {ranks} of {key} must increase strictly inside [1, {ceiling}]")
        object.__setattr__(self, "template_ranks", templates)
        object.__setattr__(self, "allowed_ranks", MappingProxyType(allowed))
        anchors = tuple(self.anchors)
        if len(set(anchors)) != len(anchors) or not set(anchors) <= set(templates):
            reject(f"anchors {anchors} must be distinct matrices of the policy")
        object.__setattr__(self, "anchors", anchors)
        if self.anchor_mode not in ANCHOR_MODES:
            reject(f"anchor_mode {self.anchor_mode!r} is not one of {ANCHOR_MODES}")
        if anchors and self.anchor_mode == "none":
            reject("anchor_mode 'none' declares anchors")
        if self.solver not in SOLVERS:
            reject(f"solver {self.solver!r} is not one of {SOLVERS}")
        if not 1 <= self.history_min <= self.history_max:
            reject(f"history window [{self.history_min}, {self.history_max}] is empty or starts below 1")
        if not (self.fit_growth > 1.0 and self.prediction_margin > 0):
            reject(f"fit_growth {self.fit_growth} must be > 1 and prediction_margin {self.prediction_margin} > 0")
        largest = max(self.source_bytes_for(key) for key in templates)
        if largest > self.source_limit_bytes:
            raise CapacityError(f"RankPolicy {self.policy_id!r}: a {largest}-byte source matrix exceeds "
                                f"source_limit_bytes={self.source_limit_bytes}")

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
            raise ConfigurationError(f"record schema {data.get('schema')!r} is not {POLICY_SCHEMA}")
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
        raise ConfigurationError(f"{key} has no template rank in policy {policy.policy_id!r}")
    if chunk_ordinal < policy.history_min or chunk_ordinal > policy.history_max:
        raise StateError(f"chunk {chunk_ordinal} lies outside the policy's history window "
                         f"[{policy.history_min}, {policy.history_max}]")
    if previous_anchors.keys() != previous_anchor_chunks.keys():
        raise ConfigurationError("every previous anchor value needs the chunk it was measured on, and only those")
    late = [chunk for chunk in previous_anchor_chunks.values() if chunk >= chunk_ordinal]
    if late:
        raise ConfigurationError(f"previous anchors measured on chunk {late[0]} are not before chunk {chunk_ordinal}")
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
            raise ConfigurationError(f"RankState schema {self.schema_version!r} is not {STATE_SCHEMA}")
        for name in ("anchor_ranks", "anchor_chunks", "selected_ranks"):
            object.__setattr__(self, name, _keyed(getattr(self, name), name))
        if self.anchor_ranks.keys() != self.anchor_chunks.keys():
            raise ConfigurationError("RankState: anchor_ranks and anchor_chunks name different matrices")
        if not all(1 <= chunk <= self.completed_chunks for chunk in self.anchor_chunks.values()):
            raise ConfigurationError(f"RankState: anchor chunks must lie in [1, {self.completed_chunks}]")
        history = (self.last_chunk_id, self.parent_head, dict(self.selected_ranks))
        if self.completed_chunks == 0 and history != (None, None, {}):
            raise ConfigurationError("RankState: zero completed chunks but a last chunk, parent head or ranks")
        if self.completed_chunks and (self.last_chunk_id is None or not self.selected_ranks or self.token_end < 1):
            raise ConfigurationError("RankState: a state after committed chunks needs last_chunk_id, selected ranks "
                                     "and token_end")

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
            raise ConfigurationError(f"record schema {data.get('schema')!r} is not {STATE_SCHEMA}")
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
        if self.status == "abstained":
            return
        if self.status != "accepted":
            raise ConfigurationError(f"RankDecision status {self.status!r}: expected accepted or abstained")
        if self.rank is None or not self.guard_passed:
            raise ConfigurationError(f"accepted RankDecision of {self.context.key} lacks a rank that passed its guard")

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
        super().__init__(f"{decision.key} abstained ({decision.reason}) after {len(decision.attempts)} fit/guard steps")
        self.decision = decision


class RankPreparation:
    """One clean-chunk attempt under a policy; never mutates the prior state. Use as a context manager or call
    :meth:`close`; :meth:`next_state` is available once every policy matrix is prepared."""

    def __init__(self, policy: RankPolicy, prior_state: RankState | None = None, *, chunk_id: str,
                 parent_head: str | None, token_start: int, device: Any = None):
        if not isinstance(policy, RankPolicy):
            raise ConfigurationError(f"RankPreparation needs a RankPolicy, got {type(policy).__name__}")
        prior = prior_state if prior_state is not None else RankState(policy.fingerprint)
        if not (isinstance(prior, RankState) and prior.policy_hash == policy.fingerprint):
            raise ConfigurationError(f"prior state was made under another policy than {policy.policy_id!r}")
        if not prior.completed_chunks and parent_head is not None:
            raise ConfigurationError(f"a first adaptive chunk cannot extend head {parent_head}, which has no rank state")
        continues = parent_head is not None and token_start == prior.token_end and chunk_id != prior.last_chunk_id
        if prior.completed_chunks and not continues:
            raise ConfigurationError(f"chunk {chunk_id!r} at token {token_start} does not continue the prior state "
                                     f"(ends at {prior.token_end} after {prior.last_chunk_id!r})")
        ordinal = prior.completed_chunks + 1
        if ordinal < policy.history_min or ordinal > policy.history_max:
            raise StateError(f"chunk {ordinal} lies outside the policy's history window "
                             f"[{policy.history_min}, {policy.history_max}]")
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
        policy, key = self.policy, context.key
        problems = []
        if context.model != policy.model or key not in policy.template_ranks:
            problems.append("is not a matrix of the policy")
        if (context.frames, context.height, context.width) != policy.geometry:
            problems.append(f"has grid {(context.frames, context.height, context.width)}, not {policy.geometry}")
        if context.token_start != self.token_start:
            problems.append(f"starts at token {context.token_start}, not {self.token_start}")
        if problems:
            raise ConfigurationError(f"{key} " + "; ".join(problems))
        if key in self._decisions:
            raise StateError(f"{key} was prepared already in this chunk")

    def prediction(self, key: MatrixKey) -> RankPrediction:
        return predict_rank(self.policy, key, chunk_ordinal=self.ordinal, current_anchors=self._anchors,
                            previous_anchors=self.prior_state.anchor_ranks,
                            previous_anchor_chunks=self.prior_state.anchor_chunks)

    def prepare_matrix(self, tensor: torch.Tensor, context: TensorContext) -> PreparedRankMatrix:
        """Predict, fit and guard one matrix; raises :class:`RankAbstention` when no allowed rank passes."""
        if self._closed:
            raise StateError(f"preparation of chunk {self.chunk_id!r} was closed")
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
        unprepared = [key for key in self.policy.keys if key not in self._decisions]
        if unprepared:
            raise StateError(f"{len(unprepared)} matrices (first {unprepared[0]}) are not prepared yet")
        abstained = [key for key, d in self._decisions.items() if d.status != "accepted"]
        if abstained:
            raise StateError(f"{abstained[0]} abstained; the chunk has no next rank state")
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
