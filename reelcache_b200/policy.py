"""Deterministic selection of measured whole-model representation profiles (the counterpart of reference
reelcache/policy.py: ``QualityEvidence`` :93, ``QualityBudget`` :130, ``Profile`` :164, ``Selection`` :244,
``qualification_failure`` :269, ``select_profile`` :299).

A :class:`Profile` is a static per-matrix codec vector measured offline (stored bytes, predicted distortion,
encode time) with its supported geometry, history depth and feature bounds, and optionally the quality
evidence that qualifies it (held-out, natively validated SSIM against a reference). :func:`select_profile`
never fits anything: it keeps the profiles whose support covers the request and whose evidence meets the
budget, picks the smallest stored size below RAW, and otherwise reports RAW explicitly. Unqualified lossy
profiles are only ever used when named explicitly with ``allow_experimental``. Evidence fields are operator
measurements, not per-request guarantees.
"""

from __future__ import annotations

import math
import re
from dataclasses import dataclass, field
from types import MappingProxyType
from typing import Any, Mapping, Sequence

from .errors import ConfigurationError
from .types import CodecSpec, MatrixKey, ModelIdentity

FEATURE_NAMES = frozenset({"K_residual_max", "V_residual_max", "K_range_imbalance", "V_range_imbalance",
                           "K_outlier_fraction", "V_outlier_fraction", "K_spatial_variation", "V_spatial_variation",
                           "basis_age"})
_SHA = re.compile(r"[0-9a-f]{64}")


def _finite(value, name: str, *, minimum=None, maximum=None) -> float:
    if isinstance(value, bool) or not isinstance(value, (int, float)) or not math.isfinite(float(value)):
        raise ConfigurationError(f"{name} must be a finite number")
    value = float(value)
    if (minimum is not None and value < minimum) or (maximum is not None and value > maximum):
        raise ConfigurationError(f"{name} is outside its valid range")
    return value


def _strings(values, name: str) -> tuple[str, ...]:
    values = tuple(values)
    if any(not isinstance(v, str) or not v for v in values) or len(set(values)) != len(values):
        raise ConfigurationError(f"{name} must be unique nonempty strings")
    return values


@dataclass(frozen=True)
class QualityEvidence:
    reference_id: str
    mean_ssim: float
    minimum_frame_ssim: float
    mean_ssim_drop: float
    calibration_prompts: tuple[str, ...]
    validation_prompts: tuple[str, ...]
    validation_cases: tuple[str, ...]
    source_sha256: tuple[str, ...]
    held_out: bool = False
    native_validated: bool = False

    def __post_init__(self):
        if not isinstance(self.reference_id, str) or not self.reference_id:
            raise ConfigurationError("quality evidence names its reference")
        _finite(self.mean_ssim, "mean_ssim", minimum=-1, maximum=1)
        _finite(self.minimum_frame_ssim, "minimum_frame_ssim", minimum=-1, maximum=1)
        _finite(self.mean_ssim_drop, "mean_ssim_drop", minimum=-2, maximum=2)
        if self.minimum_frame_ssim > self.mean_ssim:
            raise ConfigurationError("minimum frame SSIM exceeds the mean")
        for name in ("calibration_prompts", "validation_prompts", "validation_cases", "source_sha256"):
            object.__setattr__(self, name, _strings(getattr(self, name), name))
        if any(_SHA.fullmatch(v) is None for v in self.source_sha256):
            raise ConfigurationError("evidence sources are SHA-256 hex digests")
        if self.held_out and set(self.calibration_prompts) & set(self.validation_prompts):
            raise ConfigurationError("held-out prompts overlap the calibration prompts")


@dataclass(frozen=True)
class QualityBudget:
    reference_id: str = "per_channel"
    min_mean_ssim: float | None = None
    min_frame_ssim: float | None = None
    max_mean_ssim_drop: float | None = None
    min_calibration_prompts: int = 6
    min_validation_prompts: int = 6
    min_validation_cases: int = 6


@dataclass(frozen=True)
class Profile:
    profile_id: str
    model: ModelIdentity
    specs: Mapping[MatrixKey, CodecSpec]
    geometry: tuple[int, int, int]
    measured_stored_bytes: int
    predicted_distortion: float
    encode_seconds: float
    history_min: int = 1
    history_max: int = 1
    feature_bounds: Mapping[str, tuple[float, float]] = field(default_factory=dict)
    evidence: QualityEvidence | None = None
    implementation_fingerprint: str | None = None

    def __post_init__(self):
        if not isinstance(self.profile_id, str) or not self.profile_id or self.profile_id == "RAW":
            raise ConfigurationError("profile_id must be nonempty and not the reserved RAW")
        if not isinstance(self.model, ModelIdentity):
            raise ConfigurationError("a profile needs a ModelIdentity")
        specs = dict(self.specs)
        expected = {MatrixKey(layer, t) for layer in range(self.model.layers) for t in ("K", "V")}
        if set(specs) != expected or any(not isinstance(s, CodecSpec) for s in specs.values()):
            raise ConfigurationError("a profile gives one CodecSpec per model matrix")
        object.__setattr__(self, "specs", MappingProxyType(specs))
        if len(self.geometry) != 3 or any(int(g) < 1 for g in self.geometry):
            raise ConfigurationError("geometry must be frames, height, width")
        object.__setattr__(self, "geometry", tuple(int(g) for g in self.geometry))
        if type(self.measured_stored_bytes) is not int or self.measured_stored_bytes < 1:
            raise ConfigurationError("measured_stored_bytes must be a positive integer")
        _finite(self.predicted_distortion, "predicted_distortion", minimum=0)
        _finite(self.encode_seconds, "encode_seconds", minimum=0)
        if not 1 <= self.history_min <= self.history_max:
            raise ConfigurationError("history support interval is reversed")
        if not set(self.feature_bounds) <= FEATURE_NAMES:
            raise ConfigurationError("unsupported online feature in a profile")
        bounds = {}
        for name, (low, high) in self.feature_bounds.items():
            low, high = _finite(low, name, minimum=0), _finite(high, name, minimum=0)
            if low > high:
                raise ConfigurationError("feature support interval is reversed")
            bounds[name] = (low, high)
        object.__setattr__(self, "feature_bounds", MappingProxyType(bounds))
        if self.implementation_fingerprint is not None and _SHA.fullmatch(self.implementation_fingerprint) is None:
            raise ConfigurationError("implementation fingerprint must be SHA-256 hex")

    def to_dict(self) -> dict[str, Any]:
        evidence = None
        if self.evidence is not None:
            e = self.evidence
            evidence = {"reference_id": e.reference_id, "mean_ssim": e.mean_ssim,
                        "minimum_frame_ssim": e.minimum_frame_ssim, "mean_ssim_drop": e.mean_ssim_drop,
                        "calibration_prompts": list(e.calibration_prompts),
                        "validation_prompts": list(e.validation_prompts), "validation_cases": list(e.validation_cases),
                        "source_sha256": list(e.source_sha256), "held_out": e.held_out,
                        "native_validated": e.native_validated}
        return {"profile_id": self.profile_id, "model": self.model.to_dict(),
                "specs": {f"{k.layer}:{k.target}": v.to_dict() for k, v in sorted(
                    self.specs.items(), key=lambda kv: (kv[0].layer, kv[0].target))},
                "geometry": list(self.geometry), "measured_stored_bytes": self.measured_stored_bytes,
                "predicted_distortion": self.predicted_distortion, "encode_seconds": self.encode_seconds,
                "history_min": self.history_min, "history_max": self.history_max,
                "feature_bounds": {k: list(v) for k, v in sorted(self.feature_bounds.items())},
                "evidence": evidence, "implementation_fingerprint": self.implementation_fingerprint}

    @classmethod
    def from_dict(cls, data: Mapping[str, Any]) -> "Profile":
        specs = {}
        for label, spec in data["specs"].items():
            layer, target = label.split(":")
            specs[MatrixKey(int(layer), target)] = CodecSpec.from_dict(spec)
        evidence = data.get("evidence")
        if evidence is not None:
            evidence = QualityEvidence(**{k: tuple(v) if isinstance(v, list) else v for k, v in evidence.items()})
        return cls(data["profile_id"], ModelIdentity.from_dict(data["model"]), specs, tuple(data["geometry"]),
                   data["measured_stored_bytes"], data["predicted_distortion"], data["encode_seconds"],
                   data["history_min"], data["history_max"],
                   {k: tuple(v) for k, v in data.get("feature_bounds", {}).items()}, evidence,
                   data.get("implementation_fingerprint"))

    @property
    def lossy(self) -> bool:
        return any(spec.kind != "raw" for spec in self.specs.values())

    def support_failure(self, *, model, geometry, history_chunks, features, implementation_fingerprint) -> str | None:
        if self.model != model:
            return "model identity differs"
        if self.geometry != tuple(geometry):
            return "geometry differs"
        if not self.history_min <= history_chunks <= self.history_max:
            return "history depth is outside the measured support"
        for name, (low, high) in self.feature_bounds.items():
            if name not in features:
                return f"feature {name} was not measured"
            if not low <= features[name] <= high:
                return f"feature {name} is outside the measured support"
        if implementation_fingerprint is not None and self.implementation_fingerprint not in (
                None, implementation_fingerprint):
            return "measured with another implementation"
        return None


@dataclass(frozen=True)
class Selection:
    profile_id: str
    specs: Mapping[MatrixKey, CodecSpec]
    predicted_bytes: int
    predicted_distortion: float
    encode_seconds: float | None
    evidence_qualified: bool
    experimental: bool
    reason: str
    rejected: Mapping[str, str]

    def to_dict(self) -> dict[str, Any]:
        return {"profile_id": self.profile_id,
                "specs": {f"{k.layer}:{k.target}": v.to_dict() for k, v in self.specs.items()},
                "predicted_bytes": self.predicted_bytes, "predicted_distortion": self.predicted_distortion,
                "encode_seconds": self.encode_seconds, "evidence_qualified": self.evidence_qualified,
                "experimental": self.experimental, "reason": self.reason, "rejected": dict(self.rejected),
                "per_request_SSIM_guarantee": False, "costs_are_predictions_not_capacity_reservations": True}


def qualification_failure(profile: Profile, budget: QualityBudget) -> str | None:
    """Why the profile's evidence does not qualify it under ``budget`` (None: qualified)."""
    if None in (budget.min_mean_ssim, budget.min_frame_ssim, budget.max_mean_ssim_drop):
        return "automatic lossy selection requires an explicit absolute/relative SSIM budget"
    evidence = profile.evidence
    if evidence is None:
        return "no native quality evidence"
    if not evidence.native_validated or not evidence.held_out:
        return "native held-out validation is missing"
    if not evidence.source_sha256:
        return "quality evidence has no source identities"
    if evidence.reference_id != budget.reference_id:
        return "quality reference does not match the budget"
    if (len(evidence.calibration_prompts) < budget.min_calibration_prompts
            or len(evidence.validation_prompts) < budget.min_validation_prompts
            or len(evidence.validation_cases) < budget.min_validation_cases):
        return "insufficient independent calibration/validation support"
    if (evidence.mean_ssim < budget.min_mean_ssim or evidence.minimum_frame_ssim < budget.min_frame_ssim
            or evidence.mean_ssim_drop > budget.max_mean_ssim_drop):
        return "absolute or relative SSIM quality budget failed"
    return None


def _raw_specs(model: ModelIdentity) -> dict:
    return {MatrixKey(layer, t): CodecSpec("raw") for layer in range(model.layers) for t in ("K", "V")}


def select_profile(profiles: Sequence[Profile], *, model: ModelIdentity, geometry: tuple[int, int, int],
                   history_chunks: int, features: Mapping[str, float], raw_bytes: int,
                   budget: QualityBudget | None = None, explicit_profile: str | None = None,
                   allow_experimental: bool = False, implementation_fingerprint: str | None = None) -> Selection:
    """The smallest supported, qualified profile below RAW, or RAW with every rejection reason."""
    budget = QualityBudget() if budget is None else budget
    if type(history_chunks) is not int or history_chunks < 1 or type(raw_bytes) is not int or raw_bytes < 1:
        raise ConfigurationError("history_chunks and raw_bytes must be positive integers")
    if not set(features) <= FEATURE_NAMES:
        raise ConfigurationError("features must be declared current-tensor statistics")
    for name, value in features.items():
        _finite(value, name, minimum=0)
    if allow_experimental and explicit_profile is None:
        raise ConfigurationError("experimental selection requires an explicit profile")
    if any(not isinstance(p, Profile) for p in profiles):
        raise ConfigurationError("static selection accepts Profile vectors only")
    ids = [p.profile_id for p in profiles]
    if len(ids) != len(set(ids)):
        raise ConfigurationError("duplicate profile identifiers")
    if explicit_profile is not None and explicit_profile not in ids:
        raise ConfigurationError("the explicit profile is not registered")
    rejected: dict[str, str] = {}
    candidates = []
    for profile in profiles:
        if explicit_profile is not None and profile.profile_id != explicit_profile:
            continue
        failure = profile.support_failure(model=model, geometry=geometry, history_chunks=history_chunks,
                                          features=features, implementation_fingerprint=implementation_fingerprint)
        if failure is None and profile.measured_stored_bytes >= raw_bytes:
            failure = "not smaller than RAW"
        qualification = qualification_failure(profile, budget) if profile.lossy else None
        experimental = False
        if failure is None and qualification is not None:
            if allow_experimental and profile.profile_id == explicit_profile:
                experimental = True
            else:
                failure = qualification
        if failure is not None:
            rejected[profile.profile_id] = failure
            continue
        candidates.append((profile.measured_stored_bytes, profile.predicted_distortion, profile.profile_id,
                           profile, experimental))
    if not candidates:
        return Selection("RAW", MappingProxyType(_raw_specs(model)), raw_bytes, 0.0, None, False, False,
                         "no supported qualified profile is smaller than RAW", MappingProxyType(rejected))
    _, _, _, best, experimental = min(candidates, key=lambda item: item[:3])
    return Selection(best.profile_id, best.specs, best.measured_stored_bytes, best.predicted_distortion,
                     best.encode_seconds, not experimental and best.lossy, experimental,
                     "explicit experimental profile" if experimental else "smallest qualified profile",
                     MappingProxyType(rejected))


__all__ = ["FEATURE_NAMES", "Profile", "QualityBudget", "QualityEvidence", "Selection", "qualification_failure",
           "select_profile"]
