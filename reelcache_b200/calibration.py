"""Profile calibration and immutable registries (the counterpart of reference reelcache/calibration.py:
``package_fingerprint`` :29, ``configuration_fingerprint`` :45, ``Observation`` :55, ``fit_profile`` :108,
``save_registry`` / ``load_registry`` :188-255, ``save_rank_policy`` / ``load_rank_policy`` :256-330).

Measured observations of one frozen profile configuration (one per case; calibration and validation splits)
fit the profile's costs and feature support on the calibration split only; the validation split becomes its
quality evidence. Registries and rank policies are written once, atomically, bound to a SHA-256 of their
canonical JSON body, and refuse to be overwritten with different content.
"""

from __future__ import annotations

import hashlib
import json
import os
import tempfile
from dataclasses import dataclass, replace
from pathlib import Path
from typing import Mapping, Sequence

from .errors import ConfigurationError, IntegrityError, StateError
from .policy import FEATURE_NAMES, Profile, QualityEvidence

REGISTRY_SCHEMA = "reelcache_profile_registry_v1"
POLICY_FILE_SCHEMA = "reelcache_rank_policy_file_v1"


def _canonical(value) -> bytes:
    return json.dumps(value, sort_keys=True, separators=(",", ":"), allow_nan=False).encode("utf-8")


def package_fingerprint(*, package_root: Path | None = None, extra_identity: Mapping | None = None) -> str:
    """SHA-256 binding the package's Python and native sources (plus caller-supplied identities)."""
    root = Path(__file__).parent if package_root is None else Path(package_root)
    sources = {str(p.relative_to(root)): hashlib.sha256(p.read_bytes()).hexdigest()
               for pattern in ("*.py", "*.cu", "*.cuh", "*.cpp", "*.h")
               for p in sorted(root.rglob(pattern)) if "_build" not in p.parts}
    if not sources:
        raise ConfigurationError("an implementation fingerprint needs package sources")
    return hashlib.sha256(_canonical({"sources": sources, "extra_identity": dict(extra_identity or {})})).hexdigest()


def configuration_fingerprint(profile: Profile) -> str:
    data = profile.to_dict()
    fields = ("profile_id", "model", "specs", "geometry", "history_min", "history_max", "implementation_fingerprint")
    return hashlib.sha256(_canonical({k: data[k] for k in fields})).hexdigest()


@dataclass(frozen=True)
class Observation:
    profile_id: str
    case_id: str
    prompt_id: str
    split: str                        # "calibration" | "validation"
    configuration_sha256: str
    history_chunks: int
    stored_bytes: int
    distortion: float
    encode_seconds: float
    features: Mapping[str, float]
    mean_ssim: float | None = None
    minimum_frame_ssim: float | None = None
    mean_ssim_drop: float | None = None
    source_sha256: str | None = None

    def __post_init__(self):
        if self.split not in ("calibration", "validation"):
            raise ConfigurationError("observation split is calibration or validation")
        if not set(self.features) <= FEATURE_NAMES:
            raise ConfigurationError("unknown feature in an observation")
        if self.stored_bytes < 1 or self.history_chunks < 1:
            raise ConfigurationError("observations measure positive sizes and history depths")


def fit_profile(template: Profile, observations: Sequence[Observation], *, reference_id: str = "per_channel",
                native_validated: bool = False) -> Profile:
    """Costs (worst case bytes, mean distortion and encode time) and feature support from the calibration
    split; SSIM evidence from the validation split."""
    if not observations:
        raise ConfigurationError("profile fitting needs measured observations")
    digest = configuration_fingerprint(template)
    if len({o.case_id for o in observations}) != len(observations):
        raise ConfigurationError("duplicate cases must not inflate the support")
    if any(o.profile_id != template.profile_id or o.configuration_sha256 != digest for o in observations):
        raise ConfigurationError("observations do not match the frozen profile configuration")
    if any(not template.history_min <= o.history_chunks <= template.history_max for o in observations):
        raise ConfigurationError("an observation lies outside the frozen history support")
    fitting = [o for o in observations if o.split == "calibration"]
    validation = [o for o in observations if o.split == "validation"]
    if not fitting:
        raise ConfigurationError("no calibration observations")
    names = set().union(*(o.features for o in fitting))
    bounds = {n: (min(o.features[n] for o in fitting if n in o.features),
                  max(o.features[n] for o in fitting if n in o.features)) for n in sorted(names)}
    evidence = None
    if validation and all(o.mean_ssim is not None and o.minimum_frame_ssim is not None
                          and o.mean_ssim_drop is not None and o.source_sha256 for o in validation):
        calibration_prompts = tuple(sorted({o.prompt_id for o in fitting}))
        validation_prompts = tuple(sorted({o.prompt_id for o in validation}))
        evidence = QualityEvidence(
            reference_id, sum(o.mean_ssim for o in validation) / len(validation),
            min(o.minimum_frame_ssim for o in validation), max(o.mean_ssim_drop for o in validation),
            calibration_prompts, validation_prompts, tuple(sorted(o.case_id for o in validation)),
            tuple(sorted({o.source_sha256 for o in validation})),
            held_out=not set(calibration_prompts) & set(validation_prompts), native_validated=native_validated)
    return replace(template, measured_stored_bytes=max(o.stored_bytes for o in fitting),
                   predicted_distortion=sum(o.distortion for o in fitting) / len(fitting),
                   encode_seconds=sum(o.encode_seconds for o in fitting) / len(fitting), feature_bounds=bounds,
                   evidence=evidence)


def _publish(path: Path, payload: bytes, what: str) -> None:
    path = Path(path)
    path.parent.mkdir(parents=True, exist_ok=True)
    if path.is_symlink():
        raise IntegrityError(f"{what} must not be a symlink")
    if path.exists():
        if path.read_bytes() != payload:
            raise StateError(f"refusing to overwrite a frozen {what}")
        return
    descriptor, temporary = tempfile.mkstemp(prefix=".reelcache-", dir=path.parent)
    try:
        with os.fdopen(descriptor, "wb") as stream:
            stream.write(payload)
            stream.flush()
            os.fsync(stream.fileno())
        os.link(temporary, path)  # fails if another writer won the race
    finally:
        os.unlink(temporary)


def _read(path: Path, schema: str, expected_sha256: str | None, what: str) -> dict:
    path = Path(path)
    if path.is_symlink():
        raise IntegrityError(f"{what} must not be a symlink")
    data = json.loads(path.read_bytes())
    digest = data.pop("sha256", None)
    if data.get("schema") != schema:
        raise IntegrityError(f"not a {what}")
    actual = hashlib.sha256(_canonical(data)).hexdigest()
    if digest != actual or (expected_sha256 is not None and expected_sha256 != actual):
        raise IntegrityError(f"{what} checksum mismatch")
    return data


def save_registry(path: Path, profiles: Sequence[Profile]) -> str:
    if any(not isinstance(p, Profile) for p in profiles):
        raise ConfigurationError("static registries hold Profile vectors; use save_rank_policy for policies")
    ids = [p.profile_id for p in profiles]
    if len(set(ids)) != len(ids):
        raise ConfigurationError("the registry contains duplicate profiles")
    body = {"schema": REGISTRY_SCHEMA, "profiles": [p.to_dict() for p in sorted(profiles, key=lambda p: p.profile_id)]}
    digest = hashlib.sha256(_canonical(body)).hexdigest()
    _publish(Path(path), _canonical({**body, "sha256": digest}) + b"\n", "profile registry")
    return digest


def load_registry(path: Path, *, expected_sha256: str | None = None) -> list[Profile]:
    data = _read(path, REGISTRY_SCHEMA, expected_sha256, "profile registry")
    return [Profile.from_dict(p) for p in data["profiles"]]


def save_rank_policy(path: Path, policy) -> str:
    from .online_rank import RankPolicy
    if not isinstance(policy, RankPolicy):
        raise ConfigurationError("save_rank_policy takes a RankPolicy")
    body = {"schema": POLICY_FILE_SCHEMA, "policy": policy.to_dict()}
    digest = hashlib.sha256(_canonical(body)).hexdigest()
    _publish(Path(path), _canonical({**body, "sha256": digest}) + b"\n", "rank policy")
    return digest


def load_rank_policy(path: Path, *, expected_sha256: str | None = None):
    from .online_rank import RankPolicy
    data = _read(path, POLICY_FILE_SCHEMA, expected_sha256, "rank policy")
    return RankPolicy.from_dict(data["policy"])


__all__ = ["Observation", "configuration_fingerprint", "fit_profile", "load_rank_policy", "load_registry",
           "package_fingerprint", "save_rank_policy", "save_registry"]
