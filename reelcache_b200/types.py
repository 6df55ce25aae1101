"""Validated, immutable contracts of the runtime and their JSON forms.

The JSON produced by every ``to_dict`` is part of the on-disk format (node manifests, matrix
records, basis versions, epochs, predictor state), so field names, schema strings and the rules
for omitted optional fields are identical to the reference's (reelcache/types.py:80-1399):
``reelcache.energy_targets.v1`` (:566), ``reelcache.basis_version.v1`` (:726),
``reelcache.matrix_record.v1`` (:888), ``reelcache.cache_epoch.v1`` (:1032),
``reelcache.chunk_node.v1/.v2`` (:1143), ``reelcache.online_ridge_state.v1`` (:1306),
``reelcache.fit_observation.v1`` (:1383).
"""

from __future__ import annotations

import hashlib
import json
import math
import re
from dataclasses import dataclass
from types import MappingProxyType
from typing import Any, Mapping, Sequence

from .errors import ConfigurationError

_DTYPE_ALIASES = {
    "float16": "float16", "half": "float16", "bfloat16": "bfloat16", "bf16": "bfloat16",
    "float32": "float32", "float": "float32", "float64": "float64", "double": "float64",
}
RANK_BUCKET = 32
_OBJECT_REF = re.compile(r"^(blob|basis|manifest):[0-9a-f]{64}$")
_HEX64 = re.compile(r"^[0-9a-f]{64}$")
_ENERGY_SLACK = 1e-6
BASIS_DOMAINS = MappingProxyType({"K": "normalized_pre_rope_k", "V": "direct_v"})
NODE_KINDS = ("root", "chunk", "recache", "segment")
EPOCH_CAUSES = ("initial", "kv_recache", "longcat_segment")
PREDICTOR_REGIMES = ("fresh", "residual")
TARGETS = ("K", "V")


# ---------------------------------------------------------------------------------------------
# Field checks and canonical JSON
# ---------------------------------------------------------------------------------------------


def _count(value: Any, name: str, *, zero: bool = False) -> None:
    if type(value) is not int or value < (0 if zero else 1):
        raise ConfigurationError(f"{name} must be a {'nonnegative' if zero else 'positive'} integer")


def _nonempty(value: Any, name: str) -> None:
    if not isinstance(value, str) or not value.strip():
        raise ConfigurationError(f"{name} must be a nonempty string")


def _maybe_text(value: Any, name: str) -> None:
    if value is not None:
        _nonempty(value, name)


def _real(value: Any) -> bool:
    return not isinstance(value, bool) and isinstance(value, (int, float)) and math.isfinite(value)


def canonical_dtype(value: Any) -> str:
    name = str(value).removeprefix("torch.")
    if name not in _DTYPE_ALIASES:
        raise ConfigurationError(f"unsupported KV dtype: {value!r}")
    return _DTYPE_ALIASES[name]


def json_copy(value: Any, *, name: str = "metadata") -> Any:
    """A plain JSON copy; rejects NaN/inf, non-string keys and non-JSON objects."""

    def walk(item: Any) -> Any:
        if item is None or type(item) in (str, bool, int):
            return item
        if type(item) is float:
            if not math.isfinite(item):
                raise ConfigurationError(f"{name} contains a non-finite number")
            return item
        if isinstance(item, Mapping):
            out = {}
            for key, child in item.items():
                if not isinstance(key, str):
                    raise ConfigurationError(f"{name} keys must be strings")
                out[key] = walk(child)
            return out
        if isinstance(item, (list, tuple)):
            return [walk(child) for child in item]
        raise ConfigurationError(f"{name} contains a non-JSON value: {type(item).__name__}")

    try:
        return walk(value)
    except RecursionError as exc:
        raise ConfigurationError(f"{name} is not a finite acyclic JSON value") from exc


def _freeze(value: Any) -> Any:
    if isinstance(value, Mapping):
        return MappingProxyType({key: _freeze(item) for key, item in value.items()})
    if isinstance(value, (list, tuple)):
        return tuple(_freeze(item) for item in value)
    return value


def thaw_json(value: Any) -> Any:
    """Plain JSON copy of a frozen mapping/tuple structure."""
    if isinstance(value, Mapping):
        return {key: thaw_json(item) for key, item in value.items()}
    if isinstance(value, (list, tuple)):
        return [thaw_json(item) for item in value]
    return value


def frozen_json(value: Any, *, name: str = "metadata") -> Any:
    return _freeze(json_copy(thaw_json(value), name=name))


def canonical_json(value: Any) -> bytes:
    return json.dumps(json_copy(thaw_json(value)), sort_keys=True, separators=(",", ":"),
                      allow_nan=False).encode("utf-8")


def canonical_digest(value: Any) -> str:
    """SHA-256 of canonical JSON (sorted keys, no whitespace, no NaN)."""
    return hashlib.sha256(canonical_json(value)).hexdigest()


def object_ref(value: Any, name: str, *, kinds: tuple[str, ...] = ("manifest",)) -> str:
    if not isinstance(value, str) or _OBJECT_REF.fullmatch(value) is None or value.split(":", 1)[0] not in kinds:
        raise ConfigurationError(f"{name} must be an immutable {'/'.join(kinds)} object reference")
    return value


def _hex64(value: Any, name: str) -> str:
    if not isinstance(value, str) or _HEX64.fullmatch(value) is None:
        raise ConfigurationError(f"{name} must be a lowercase SHA256 hex digest")
    return value


def _fraction(value: Any, name: str) -> float:
    if not _real(value) or not 0 < value <= 1:
        raise ConfigurationError(f"{name} must be a finite fraction in (0, 1]")
    return float(value)


def _measured_energy(value: Any, name: str) -> float:
    if not _real(value) or value > 1 + _ENERGY_SLACK:
        raise ConfigurationError(f"{name} must be a finite measured energy fraction <= 1")
    return float(value)


def _build(cls, fields: Mapping[str, Any], what: str):
    try:
        return cls(**dict(fields))
    except (TypeError, KeyError) as exc:
        raise ConfigurationError(f"invalid {what} fields") from exc


# ---------------------------------------------------------------------------------------------
# Model and matrix identity
# ---------------------------------------------------------------------------------------------


@dataclass(frozen=True)
class ModelIdentity:
    name: str
    fingerprint: str
    layers: int
    kv_channels: int | Mapping[str, int]
    layout: str
    dtype: str | Mapping[str, str]

    def __post_init__(self) -> None:
        _nonempty(self.name, "model name")
        _nonempty(self.fingerprint, "model fingerprint")
        _count(self.layers, "layers")
        _nonempty(self.layout, "layout")
        if isinstance(self.dtype, Mapping):
            per_matrix = {f"{layer}:{target}" for layer in range(self.layers) for target in TARGETS}
            if set(self.dtype) not in ({"K", "V"}, per_matrix):
                raise ConfigurationError("dtype mapping must cover K/V or every layer:target matrix")
            object.__setattr__(self, "dtype",
                               MappingProxyType({k: canonical_dtype(v) for k, v in self.dtype.items()}))
        else:
            object.__setattr__(self, "dtype", canonical_dtype(self.dtype))
        if isinstance(self.kv_channels, Mapping):
            if set(self.kv_channels) != {"K", "V"}:
                raise ConfigurationError("kv_channels mapping must contain exactly K and V")
            for target, channels in self.kv_channels.items():
                _count(channels, f"{target} channels")
            object.__setattr__(self, "kv_channels", MappingProxyType(dict(self.kv_channels)))
        else:
            _count(self.kv_channels, "kv_channels")

    def channels_for(self, target: str | MatrixKey) -> int:
        if isinstance(target, MatrixKey):
            target = target.target
        if target not in TARGETS:
            raise ConfigurationError("target must be K or V")
        return self.kv_channels[target] if isinstance(self.kv_channels, Mapping) else self.kv_channels

    def dtype_for(self, target: str | MatrixKey) -> str:
        key = target if isinstance(target, MatrixKey) else None
        target = key.target if key is not None else target
        if target not in TARGETS:
            raise ConfigurationError("target must be K or V")
        if key is not None and key.layer >= self.layers:
            raise ConfigurationError("matrix layer is outside the model")
        if not isinstance(self.dtype, Mapping):
            return self.dtype
        if target in self.dtype:
            return self.dtype[target]
        if key is None:
            raise ConfigurationError("layer-specific dtype requires a MatrixKey")
        return self.dtype[f"{key.layer}:{key.target}"]

    def to_dict(self) -> dict[str, Any]:
        return {
            "name": self.name, "fingerprint": self.fingerprint, "layers": self.layers,
            "kv_channels": dict(self.kv_channels) if isinstance(self.kv_channels, Mapping) else self.kv_channels,
            "layout": self.layout, "dtype": dict(self.dtype) if isinstance(self.dtype, Mapping) else self.dtype,
        }

    @classmethod
    def from_dict(cls, data: Mapping[str, Any]) -> ModelIdentity:
        return _build(cls, data, "model identity")

    def __hash__(self) -> int:
        dtypes = tuple(self.dtype_for(MatrixKey(layer, t)) for layer in range(self.layers) for t in TARGETS)
        return hash((self.name, self.fingerprint, self.layers, self.channels_for("K"), self.channels_for("V"),
                     self.layout, dtypes))


@dataclass(frozen=True, order=True)
class MatrixKey:
    layer: int
    target: str

    def __post_init__(self) -> None:
        _count(self.layer, "layer", zero=True)
        if self.target not in TARGETS:
            raise ConfigurationError("matrix target must be K or V")

    def to_dict(self) -> dict[str, Any]:
        return {"layer": self.layer, "target": self.target}

    @classmethod
    def from_dict(cls, data: Mapping[str, Any]) -> MatrixKey:
        return _build(cls, data, "matrix key")


@dataclass(frozen=True)
class TensorContext:
    """Canonical coordinates of one ``[N, C]`` matrix; ``source_dtype`` optionally overrides the
    model's declared dtype (and is serialized only when set)."""

    model: ModelIdentity
    key: MatrixKey
    token_start: int
    frames: int
    height: int
    width: int
    key_space: str
    source_dtype: str | None = None

    def __post_init__(self) -> None:
        if not isinstance(self.model, ModelIdentity) or not isinstance(self.key, MatrixKey):
            raise ConfigurationError("context requires ModelIdentity and MatrixKey")
        if self.key.layer >= self.model.layers:
            raise ConfigurationError("matrix layer is outside the model")
        _count(self.token_start, "token_start", zero=True)
        for name in ("frames", "height", "width"):
            _count(getattr(self, name), name)
        if self.key_space not in ("pre_rope", "post_rope", "none"):
            raise ConfigurationError("key_space must be pre_rope, post_rope, or none")
        if self.key.target == "V" and self.key_space != "none":
            raise ConfigurationError("V matrices must use key_space='none'")
        if self.source_dtype is not None:
            object.__setattr__(self, "source_dtype", canonical_dtype(self.source_dtype))

    @property
    def channels(self) -> int:
        return self.model.channels_for(self.key)

    @property
    def dtype(self) -> str:
        return self.model.dtype_for(self.key) if self.source_dtype is None else self.source_dtype

    @property
    def token_count(self) -> int:
        return self.frames * self.height * self.width

    @property
    def token_end(self) -> int:
        return self.token_start + self.token_count

    @property
    def shape(self) -> tuple[int, int]:
        return self.token_count, self.channels

    def to_dict(self) -> dict[str, Any]:
        data = {"model": self.model.to_dict(), "key": self.key.to_dict(), "token_start": self.token_start,
                "frames": self.frames, "height": self.height, "width": self.width, "key_space": self.key_space}
        if self.source_dtype is not None:
            data["source_dtype"] = self.source_dtype
        return data

    @classmethod
    def from_dict(cls, data: Mapping[str, Any]) -> TensorContext:
        try:
            fields = dict(data)
            fields["model"] = ModelIdentity.from_dict(fields["model"])
            fields["key"] = MatrixKey.from_dict(fields["key"])
        except (TypeError, KeyError) as exc:
            raise ConfigurationError("invalid tensor context fields") from exc
        return _build(cls, fields, "tensor context")


@dataclass(frozen=True)
class CodecSpec:
    """Representation parameters (``raw``, ``svd``, ``svd_hevc``).

    Per-channel normalization canonicalizes ``protected_fraction`` to 1 and global to 0.
    ``inter_prediction`` (svd_hevc only) is serialized for version-2 records; ``None`` marks a
    version-1 svd_hevc record that predates the flag.
    """

    kind: str = "raw"
    rank: int | None = None
    normalization: str = "per_channel"
    protected_fraction: float = 1.0
    pix_fmt: str = "yuv444p"
    qp: int = 8
    preset: str = "ultrafast"
    ffmpeg_path: str | None = None
    inter_prediction: bool | None = False

    def __post_init__(self) -> None:
        if self.kind not in ("raw", "svd", "svd_hevc"):
            raise ConfigurationError("codec kind must be raw, svd, or svd_hevc")
        if self.kind == "raw":
            if self.rank is not None:
                raise ConfigurationError("raw encoding does not take a rank")
        else:
            _count(self.rank, "rank")
        if self.normalization not in ("per_channel", "global", "leading_columns"):
            raise ConfigurationError("unsupported normalization")
        if not _real(self.protected_fraction) or not 0 <= self.protected_fraction <= 1:
            raise ConfigurationError("protected_fraction must be in [0, 1]")
        if self.normalization == "global":
            object.__setattr__(self, "protected_fraction", 0.0)
        elif self.normalization == "per_channel":
            object.__setattr__(self, "protected_fraction", 1.0)
        _nonempty(self.pix_fmt, "pix_fmt")
        _nonempty(self.preset, "preset")
        if self.ffmpeg_path is not None:
            _nonempty(self.ffmpeg_path, "ffmpeg_path")
            if "\x00" in self.ffmpeg_path:
                raise ConfigurationError("ffmpeg_path must not contain NUL")
        if type(self.qp) is not int or not 0 <= self.qp <= 51:
            raise ConfigurationError("qp must be an integer in [0, 51]")
        if self.inter_prediction is not None and type(self.inter_prediction) is not bool:
            raise ConfigurationError("inter_prediction must be a boolean")
        if self.kind != "svd_hevc":
            if self.inter_prediction:
                raise ConfigurationError("inter prediction applies only to svd_hevc coefficient streams")
            object.__setattr__(self, "inter_prediction", False)

    @property
    def legacy_gop(self) -> bool:
        return self.inter_prediction is None

    def to_dict(self) -> dict[str, Any]:
        data = {"kind": self.kind, "rank": self.rank, "normalization": self.normalization,
                "protected_fraction": self.protected_fraction, "pix_fmt": self.pix_fmt, "qp": self.qp,
                "preset": self.preset, "ffmpeg_path": self.ffmpeg_path}
        if self.kind == "svd_hevc" and self.inter_prediction is not None:
            data["inter_prediction"] = self.inter_prediction
        return data

    @classmethod
    def from_dict(cls, data: Mapping[str, Any]) -> CodecSpec:
        fields = dict(data)
        if "inter_prediction" not in fields:
            fields["inter_prediction"] = None
        elif type(fields["inter_prediction"]) is not bool:
            raise ConfigurationError("serialized inter_prediction must be a boolean when present")
        return _build(cls, fields, "codec spec")


@dataclass(frozen=True)
class EncodedTensor:
    metadata: Mapping[str, Any]
    payloads: Mapping[str, bytes]
    basis: bytes | None = None
    metrics: Mapping[str, Any] | None = None

    def __post_init__(self) -> None:
        if not isinstance(self.metadata, Mapping) or not isinstance(self.payloads, Mapping):
            raise ConfigurationError("encoded metadata and payloads must be mappings")
        if not self.payloads:
            raise ConfigurationError("encoded tensors require at least one payload")
        for name, payload in self.payloads.items():
            _nonempty(name, "payload name")
            if not isinstance(payload, bytes):
                raise ConfigurationError("encoded payloads must be immutable bytes")
        if self.basis is not None and not isinstance(self.basis, bytes):
            raise ConfigurationError("encoded basis must be immutable bytes")
        if self.metrics is not None and not isinstance(self.metrics, Mapping):
            raise ConfigurationError("metrics must be a mapping")
        object.__setattr__(self, "metadata", json_copy(self.metadata))
        object.__setattr__(self, "payloads", MappingProxyType(dict(self.payloads)))
        if self.metrics is not None:
            object.__setattr__(self, "metrics", json_copy(self.metrics, name="metrics"))


# ---------------------------------------------------------------------------------------------
# Node entry keys (single stream: MatrixKey; CFG streams: (MatrixKey, label))
# ---------------------------------------------------------------------------------------------


def entry_key(value: Any, name: str = "matrix entry") -> Any:
    if isinstance(value, MatrixKey):
        return value
    if (isinstance(value, tuple) and len(value) == 2 and isinstance(value[0], MatrixKey)
            and isinstance(value[1], str) and value[1] and value[1] == value[1].strip()):
        return value
    raise ConfigurationError(f"{name} keys must be MatrixKey or (MatrixKey, stream label)")


def entry_parts(value: Any) -> tuple[MatrixKey, str | None]:
    value = entry_key(value)
    return (value, None) if isinstance(value, MatrixKey) else value


def entry_order(value: Any) -> tuple:
    key, stream = entry_parts(value)
    return key.layer, key.target, stream is not None, stream or ""


def _entry_dict(value: Any) -> dict[str, Any]:
    key, stream = entry_parts(value)
    return {"key": key.to_dict()} if stream is None else {"key": key.to_dict(), "stream": stream}


def _entry_from(item: Mapping[str, Any]) -> Any:
    key = MatrixKey.from_dict(item["key"])
    stream = item.get("stream")
    return key if stream is None else entry_key((key, stream))


def _sorted_pairs(values: Any, name: str, convert) -> tuple:
    items = values.items() if isinstance(values, Mapping) else values
    if not isinstance(items, (tuple, list)) and not isinstance(values, Mapping):
        raise ConfigurationError(f"{name} must be a MatrixKey mapping or pair sequence")
    pairs = []
    for item in items:
        if not isinstance(item, (tuple, list)) or len(item) != 2:
            raise ConfigurationError(f"{name} entries must be (MatrixKey, value) pairs")
        pairs.append((entry_key(item[0], name), convert(item[1])))
    pairs.sort(key=lambda pair: entry_order(pair[0]))
    if len({key for key, _ in pairs}) != len(pairs):
        raise ConfigurationError(f"{name} contains duplicate matrix keys")
    return tuple(pairs)


def _validate_streams(streams: Any, entries: Sequence[Any], name: str) -> tuple[str, ...]:
    streams = tuple(streams)
    if any(not isinstance(s, str) or not s or s != s.strip() for s in streams):
        raise ConfigurationError("stream labels must be nonempty strings without surrounding whitespace")
    if len(set(streams)) != len(streams) or list(streams) != sorted(streams):
        raise ConfigurationError("stream labels must be unique and sorted")
    labels = {entry_parts(item)[1] for item in entries}
    if not streams:
        if labels - {None}:
            raise ConfigurationError(f"{name} carry stream labels but the node declares no streams")
        return streams
    if None in labels or not labels <= set(streams):
        raise ConfigurationError(f"{name} of a multi-stream node must be labeled with declared streams")
    if entries:
        per_stream: dict[str, set] = {s: set() for s in streams}
        for item in entries:
            key, stream = entry_parts(item)
            per_stream[stream].add(key)
        first = per_stream[streams[0]]
        if any(keys != first for keys in per_stream.values()):
            raise ConfigurationError(f"{name} must cover the same matrices in every stream")
    return streams


# ---------------------------------------------------------------------------------------------
# Energy targets and reports
# ---------------------------------------------------------------------------------------------


@dataclass(frozen=True)
class EnergyTargets:
    """Pre-codec energy fractions for normalized pre-RoPE K and direct V (1.0 = full-width diagnostic)."""

    profile: str
    key: float
    value: float
    provisional: bool
    note: str | None = None

    def __post_init__(self) -> None:
        _nonempty(self.profile, "energy profile")
        object.__setattr__(self, "key", _fraction(self.key, "K energy target"))
        object.__setattr__(self, "value", _fraction(self.value, "V energy target"))
        if type(self.provisional) is not bool:
            raise ConfigurationError("provisional must be boolean")
        _maybe_text(self.note, "energy profile note")

    def for_target(self, target: str | MatrixKey) -> float:
        target = target.target if isinstance(target, MatrixKey) else target
        if target == "K":
            return self.key
        if target == "V":
            return self.value
        raise ConfigurationError("energy target selector must be K or V")

    def is_diagnostic(self, target: str | MatrixKey) -> bool:
        return self.for_target(target) == 1.0

    def to_dict(self) -> dict[str, Any]:
        return {"schema": "reelcache.energy_targets.v1", "profile": self.profile, "key": self.key,
                "value": self.value, "provisional": self.provisional, "note": self.note}

    @classmethod
    def from_dict(cls, data: Mapping[str, Any]) -> EnergyTargets:
        fields = dict(data)
        if fields.pop("schema", None) != "reelcache.energy_targets.v1":
            raise ConfigurationError("unsupported energy target schema")
        return _build(cls, fields, "energy target")

    @property
    def fingerprint(self) -> str:
        return canonical_digest(self.to_dict())


_PROVISIONAL = "provisional K98/V95 until the energy sweeps select a model-specific profile"
ENERGY_TARGET_PROFILES = MappingProxyType({
    "causvid": EnergyTargets("causvid", 0.98, 0.95, False, "final: pre-RoPE K 98%, V 95%"),
    "raven": EnergyTargets("raven", 0.98, 0.95, True, _PROVISIONAL),
    "longlive1": EnergyTargets("longlive1", 0.98, 0.95, True, _PROVISIONAL),
    "longlive2": EnergyTargets("longlive2", 0.98, 0.95, True, _PROVISIONAL),
    "longcat_720p": EnergyTargets("longcat_720p", 0.98, 0.95, True, _PROVISIONAL),
})


def energy_targets(profile: str) -> EnergyTargets:
    try:
        return ENERGY_TARGET_PROFILES[profile]
    except (KeyError, TypeError) as exc:
        raise ConfigurationError(f"no energy target profile is configured for {profile!r}") from exc


@dataclass(frozen=True)
class EnergyReport:
    """Ideal-subspace, stored-factor (FP32 ``P = A Q^T`` with FP16 rows) and post-codec measurements."""

    target: float
    ideal_subspace_energy: float
    stored_factor_energy: float
    post_codec_relative_error: float | None = None
    observed_rank: int | None = None
    bucket_rank: int = 0
    rank_view: int = 1
    zero_input: bool = False
    diagnostic_full_width: bool = False

    def __post_init__(self) -> None:
        object.__setattr__(self, "target", _fraction(self.target, "energy target"))
        object.__setattr__(self, "ideal_subspace_energy",
                           _measured_energy(self.ideal_subspace_energy, "ideal subspace energy"))
        object.__setattr__(self, "stored_factor_energy",
                           _measured_energy(self.stored_factor_energy, "stored-factor energy"))
        if self.post_codec_relative_error is not None:
            value = self.post_codec_relative_error
            if not _real(value) or value < 0:
                raise ConfigurationError("post-codec relative error must be finite and nonnegative or None")
            object.__setattr__(self, "post_codec_relative_error", float(value))
        if self.observed_rank is not None:
            _count(self.observed_rank, "observed rank", zero=True)
        _count(self.bucket_rank, "bucket rank", zero=True)
        _count(self.rank_view, "rank view")
        for name in ("zero_input", "diagnostic_full_width"):
            if type(getattr(self, name)) is not bool:
                raise ConfigurationError(f"{name} must be boolean")
        if self.zero_input and (self.ideal_subspace_energy != 1.0 or self.stored_factor_energy != 1.0):
            raise ConfigurationError("a zero input is represented exactly")

    @property
    def meets_target(self) -> bool:
        return self.zero_input or self.stored_factor_energy >= self.target

    def to_dict(self) -> dict[str, Any]:
        return {name: getattr(self, name) for name in (
            "target", "ideal_subspace_energy", "stored_factor_energy", "post_codec_relative_error",
            "observed_rank", "bucket_rank", "rank_view", "zero_input", "diagnostic_full_width")}

    @classmethod
    def from_dict(cls, data: Mapping[str, Any]) -> EnergyReport:
        return _build(cls, data, "energy report")


# ---------------------------------------------------------------------------------------------
# Basis versions and bindings
# ---------------------------------------------------------------------------------------------


@dataclass(frozen=True)
class BasisVersion:
    """One immutable node of a per-(layer, target) basis DAG: the parent's rows followed by this
    version's FP16 row block; ``view_sha256`` binds the assembled ``[total_rank, channels]`` bytes."""

    parent_ref: str | None
    added_rows_ref: str
    added_rank: int
    total_rank: int
    channels: int
    group_id: str
    key: MatrixKey
    model_fingerprint: str
    depth: int
    view_sha256: str
    dtype: str = "float16"

    def __post_init__(self) -> None:
        if self.parent_ref is not None:
            object_ref(self.parent_ref, "basis parent version")
        object_ref(self.added_rows_ref, "added basis row block", kinds=("basis",))
        _count(self.added_rank, "added rank")
        _count(self.total_rank, "total rank")
        _count(self.channels, "basis channels")
        _count(self.depth, "basis version depth", zero=True)
        if not isinstance(self.key, MatrixKey):
            raise ConfigurationError("basis version key must be a MatrixKey")
        _nonempty(self.model_fingerprint, "basis model fingerprint")
        _hex64(self.group_id, "basis group id")
        _hex64(self.view_sha256, "basis view digest")
        if self.dtype != "float16":
            raise ConfigurationError("stored basis rows are FP16")
        if self.total_rank > self.channels:
            raise ConfigurationError("basis rank cannot exceed its channel count")
        if (self.parent_ref is None) != (self.depth == 0):
            raise ConfigurationError("only a depth-zero root version has no parent")
        if self.parent_ref is None and self.total_rank != self.added_rank:
            raise ConfigurationError("a root version's total rank equals its block rank")
        if self.parent_ref is not None and self.total_rank <= self.added_rank:
            raise ConfigurationError("an extension version must add rows to a nonempty parent")

    @property
    def domain(self) -> str:
        return BASIS_DOMAINS[self.key.target]

    @property
    def parent_rank(self) -> int:
        return self.total_rank - self.added_rank

    @property
    def added_bytes(self) -> int:
        return self.added_rank * self.channels * 2

    @staticmethod
    def root_group_id(model_fingerprint: str, key: MatrixKey, rows_ref: str) -> str:
        return canonical_digest({"model": model_fingerprint, "key": key.to_dict(), "root_rows": rows_ref})

    def to_dict(self) -> dict[str, Any]:
        return {"schema": "reelcache.basis_version.v1", "parent": self.parent_ref, "added_rows": self.added_rows_ref,
                "added_rank": self.added_rank, "total_rank": self.total_rank, "channels": self.channels,
                "dtype": self.dtype, "group_id": self.group_id, "key": self.key.to_dict(), "domain": self.domain,
                "model_fingerprint": self.model_fingerprint, "depth": self.depth, "view_sha256": self.view_sha256}

    @classmethod
    def from_dict(cls, data: Mapping[str, Any]) -> BasisVersion:
        try:
            fields = dict(data)
            if fields.pop("schema") != "reelcache.basis_version.v1":
                raise ConfigurationError("unsupported basis version schema")
            domain = fields.pop("domain")
            version = cls(parent_ref=fields.pop("parent"), added_rows_ref=fields.pop("added_rows"),
                          key=MatrixKey.from_dict(fields.pop("key")), **fields)
        except (KeyError, TypeError) as exc:
            raise ConfigurationError("invalid basis version fields") from exc
        if domain != version.domain:
            raise ConfigurationError("basis version domain disagrees with its K/V key")
        return version


@dataclass(frozen=True)
class ActiveBasisBinding:
    """A lineage's active basis for one (layer, target) plus its refit memory (fresh rank, measured
    coefficient rate and the cumulative refit debt, serialized only when nonzero)."""

    version_ref: str | None = None
    total_rank: int = 0
    group_id: str | None = None
    fresh_rank: int | None = None
    fresh_chunk_id: str | None = None
    coefficient_rate: float | None = None
    rate_identity: str | None = None
    refit_debt: float = 0.0

    def __post_init__(self) -> None:
        if self.version_ref is None:
            if self.total_rank != 0 or self.group_id is not None:
                raise ConfigurationError("an empty binding has no rank or group")
        else:
            object_ref(self.version_ref, "active basis version")
            _count(self.total_rank, "active basis rank")
            _hex64(self.group_id, "active basis group")
        if (self.fresh_rank is None) != (self.fresh_chunk_id is None):
            raise ConfigurationError("fresh rank and its chunk are recorded together")
        if self.fresh_rank is not None:
            _count(self.fresh_rank, "fresh rank")
            _nonempty(self.fresh_chunk_id, "fresh chunk id")
        if (self.coefficient_rate is None) != (self.rate_identity is None):
            raise ConfigurationError("a coefficient rate requires its codec/geometry identity")
        if self.coefficient_rate is not None:
            if not _real(self.coefficient_rate) or self.coefficient_rate <= 0:
                raise ConfigurationError("coefficient rate must be finite and positive")
            object.__setattr__(self, "coefficient_rate", float(self.coefficient_rate))
            _hex64(self.rate_identity, "coefficient rate identity")
        debt = self.refit_debt
        if not _real(debt) or debt < 0:
            raise ConfigurationError("refit debt must be finite and nonnegative")
        object.__setattr__(self, "refit_debt", float(debt) if debt else 0.0)
        if self.refit_debt and (self.version_ref is None or self.fresh_rank is None):
            raise ConfigurationError("a refit debt needs an active basis and its fresh rank")

    def to_dict(self) -> dict[str, Any]:
        data = {name: getattr(self, name) for name in (
            "version_ref", "total_rank", "group_id", "fresh_rank", "fresh_chunk_id", "coefficient_rate",
            "rate_identity")}
        if self.refit_debt:
            data["refit_debt"] = self.refit_debt
        return data

    @classmethod
    def from_dict(cls, data: Mapping[str, Any]) -> ActiveBasisBinding:
        fields = dict(data)
        if "refit_debt" in fields and fields["refit_debt"] == 0:
            raise ConfigurationError("a zero refit debt is omitted")
        return _build(cls, fields, "active basis binding")


def _factor_pack_tile(codec: CodecSpec, decision: Any) -> bool:
    packet = decision.get("packet") if isinstance(decision, Mapping) else None
    canvas = packet.get("canvas") if isinstance(packet, Mapping) else None
    return codec.kind == "svd" and isinstance(canvas, Mapping) and canvas.get("policy") == "factor_tiles"


@dataclass(frozen=True)
class MatrixRecord:
    """One committed matrix: its packet (or tile of a node pack) plus its explicit basis view."""

    context: TensorContext
    codec: CodecSpec
    packet_ref: str
    basis_version_ref: str | None
    rank_view: int | None
    energy: EnergyReport | None
    predictor_revision_ref: str | None
    decision: Mapping[str, Any]
    packet_tile: int | None = None
    stream: str | None = None

    def __post_init__(self) -> None:
        if not isinstance(self.context, TensorContext) or not isinstance(self.codec, CodecSpec):
            raise ConfigurationError("matrix record requires a TensorContext and CodecSpec")
        object_ref(self.packet_ref, "matrix packet")
        if self.codec.kind == "raw":
            if self.basis_version_ref is not None or self.rank_view is not None or self.energy is not None:
                raise ConfigurationError("RAW records carry no basis, rank view or factor energy")
        else:
            object_ref(self.basis_version_ref, "matrix basis version")
            _count(self.rank_view, "rank view")
            if self.rank_view != self.codec.rank:
                raise ConfigurationError("rank view must equal the resolved codec rank")
            if not isinstance(self.energy, EnergyReport) or self.energy.rank_view != self.rank_view:
                raise ConfigurationError("lossy records require an energy report for their rank view")
            if self.context.key.target == "K" and self.context.key_space != "pre_rope":
                raise ConfigurationError("lossy K records must be normalized pre-RoPE K")
        if self.packet_tile is not None:
            _count(self.packet_tile, "packet tile", zero=True)
            if not _factor_pack_tile(self.codec, self.decision) and (
                    self.codec.kind != "svd_hevc" or self.codec.inter_prediction is not False):
                raise ConfigurationError("only all-intra svd_hevc matrices are tiles of a node pack")
        if self.stream is not None:
            entry_key((self.context.key, self.stream), "matrix record stream")
        if self.predictor_revision_ref is not None:
            _nonempty(self.predictor_revision_ref, "predictor revision reference")
        object.__setattr__(self, "decision", frozen_json(self.decision, name="matrix decision"))

    @property
    def entry(self) -> Any:
        return self.context.key if self.stream is None else (self.context.key, self.stream)

    def to_dict(self) -> dict[str, Any]:
        data = {"schema": "reelcache.matrix_record.v1", "context": self.context.to_dict(),
                "codec": self.codec.to_dict(), "packet": self.packet_ref, "basis_version": self.basis_version_ref,
                "rank_view": self.rank_view, "energy": None if self.energy is None else self.energy.to_dict(),
                "predictor_revision": self.predictor_revision_ref, "decision": thaw_json(self.decision)}
        if self.packet_tile is not None:
            data["packet_tile"] = self.packet_tile
        if self.stream is not None:
            data["stream"] = self.stream
        return data

    @classmethod
    def from_dict(cls, data: Mapping[str, Any]) -> MatrixRecord:
        try:
            fields = dict(data)
            if fields.pop("schema") != "reelcache.matrix_record.v1":
                raise ConfigurationError("unsupported matrix record schema")
            energy = fields.pop("energy")
            for optional in ("packet_tile", "stream"):
                if optional in fields and fields[optional] is None:
                    raise ConfigurationError(f"an unset {optional} is omitted, not null")
            return cls(context=TensorContext.from_dict(fields.pop("context")),
                       codec=CodecSpec.from_dict(fields.pop("codec")), packet_ref=fields.pop("packet"),
                       basis_version_ref=fields.pop("basis_version"), rank_view=fields.pop("rank_view"),
                       energy=None if energy is None else EnergyReport.from_dict(energy),
                       predictor_revision_ref=fields.pop("predictor_revision"), decision=fields.pop("decision"),
                       **fields)
        except (KeyError, TypeError) as exc:
            raise ConfigurationError("invalid matrix record fields") from exc


# ---------------------------------------------------------------------------------------------
# Epochs and nodes
# ---------------------------------------------------------------------------------------------


@dataclass(frozen=True)
class TokenRangeRecords:
    """Matrix records of one re-materialized (or segment-local) token range."""

    chunk_id: str
    token_start: int
    token_end: int
    frames: int
    height: int
    width: int
    records: tuple[tuple[Any, str], ...]
    streams: tuple[str, ...] = ()
    packet_ref: str | None = None

    def __post_init__(self) -> None:
        _nonempty(self.chunk_id, "range chunk id")
        if self.packet_ref is not None:
            object_ref(self.packet_ref, "range node pack")
        _count(self.token_start, "range token start", zero=True)
        for name in ("frames", "height", "width"):
            _count(getattr(self, name), f"range {name}")
        if self.token_end != self.token_start + self.frames * self.height * self.width:
            raise ConfigurationError("range token span must equal its geometry")
        object.__setattr__(self, "records", _sorted_pairs(
            self.records, "range records", lambda ref: object_ref(ref, "range matrix record")))
        if not self.records:
            raise ConfigurationError("a re-materialized range carries matrix records")
        object.__setattr__(self, "streams", _validate_streams(self.streams, [k for k, _ in self.records],
                                                              "range records"))

    def to_dict(self) -> dict[str, Any]:
        data = {"chunk_id": self.chunk_id, "token_start": self.token_start, "token_end": self.token_end,
                "frames": self.frames, "height": self.height, "width": self.width,
                "records": [{**_entry_dict(key), "record": ref} for key, ref in self.records]}
        if self.streams:
            data["streams"] = list(self.streams)
        if self.packet_ref is not None:
            data["packet"] = self.packet_ref
        return data

    @classmethod
    def from_dict(cls, data: Mapping[str, Any]) -> TokenRangeRecords:
        try:
            fields = dict(data)
            records = tuple((_entry_from(item), item["record"]) for item in fields.pop("records"))
            streams = tuple(fields.pop("streams", ()))
            if "streams" in data and not streams:
                raise ConfigurationError("an empty stream list is omitted")
            packet = fields.pop("packet", None)
            if "packet" in data and packet is None:
                raise ConfigurationError("an absent node pack is omitted")
            return cls(records=records, streams=streams, packet_ref=packet, **fields)
        except (KeyError, TypeError) as exc:
            raise ConfigurationError("invalid token range fields") from exc


@dataclass(frozen=True)
class CacheEpoch:
    """A cache version: ``initial``, a KV recache, or a LongCat segment (segment-local positions)."""

    epoch_id: str
    parent_epoch_ref: str | None
    cause: str
    position_space: str
    ranges: tuple[TokenRangeRecords, ...]
    details: Mapping[str, Any]

    def __post_init__(self) -> None:
        _nonempty(self.epoch_id, "epoch id")
        if self.parent_epoch_ref is not None:
            object_ref(self.parent_epoch_ref, "parent epoch")
        if self.cause not in EPOCH_CAUSES:
            raise ConfigurationError(f"epoch cause must be one of {EPOCH_CAUSES}")
        if self.position_space not in ("global", "segment_local"):
            raise ConfigurationError("epoch position space must be global or segment_local")
        ranges = tuple(self.ranges)
        if any(not isinstance(item, TokenRangeRecords) for item in ranges):
            raise ConfigurationError("epoch ranges must be TokenRangeRecords")
        ordered = sorted(ranges, key=lambda item: item.token_start)
        if ordered != list(ranges) or any(a.token_end > b.token_start for a, b in zip(ordered, ordered[1:])):
            raise ConfigurationError("epoch ranges must be ordered and non-overlapping")
        if self.cause == "initial":
            if ranges or self.parent_epoch_ref is not None or self.position_space != "global":
                raise ConfigurationError("an initial epoch has no parent and no re-materialized ranges")
        elif self.cause == "kv_recache":
            if not ranges or self.parent_epoch_ref is None or self.position_space != "global":
                raise ConfigurationError("a KV recache epoch re-materializes global ranges of a parent epoch")
        elif (self.position_space != "segment_local" or len(ranges) != 1 or ranges[0].token_start != 0
              or self.parent_epoch_ref is None):
            raise ConfigurationError("a LongCat segment epoch holds one segment-local range starting at zero")
        object.__setattr__(self, "ranges", ranges)
        object.__setattr__(self, "details", frozen_json(self.details, name="epoch details"))

    def to_dict(self) -> dict[str, Any]:
        return {"schema": "reelcache.cache_epoch.v1", "epoch_id": self.epoch_id, "parent_epoch": self.parent_epoch_ref,
                "cause": self.cause, "position_space": self.position_space,
                "ranges": [item.to_dict() for item in self.ranges], "details": thaw_json(self.details)}

    @classmethod
    def from_dict(cls, data: Mapping[str, Any]) -> CacheEpoch:
        try:
            fields = dict(data)
            if fields.pop("schema") != "reelcache.cache_epoch.v1":
                raise ConfigurationError("unsupported cache epoch schema")
            return cls(epoch_id=fields.pop("epoch_id"), parent_epoch_ref=fields.pop("parent_epoch"),
                       ranges=tuple(TokenRangeRecords.from_dict(item) for item in fields.pop("ranges")), **fields)
        except (KeyError, TypeError) as exc:
            raise ConfigurationError("invalid cache epoch fields") from exc


@dataclass(frozen=True)
class ChunkNode:
    """One immutable state-tree node (``root``, ``chunk``, ``recache`` or ``segment``); ``active_basis``
    is the complete per-key binding the next commit tests."""

    node_kind: str
    chunk_id: str
    parent_ref: str | None
    cache_epoch_id: str
    epoch_ref: str
    token_start: int
    token_end: int
    frames: int
    height: int
    width: int
    frontier: int
    matrix_records: tuple[tuple[Any, str], ...]
    active_basis: tuple[tuple[Any, ActiveBasisBinding], ...]
    execution_state_ref: str | None = None
    streams: tuple[str, ...] = ()
    packet_ref: str | None = None

    def __post_init__(self) -> None:
        if self.node_kind not in NODE_KINDS:
            raise ConfigurationError(f"node kind must be one of {NODE_KINDS}")
        _nonempty(self.chunk_id, "node chunk id")
        if self.parent_ref is not None:
            object_ref(self.parent_ref, "parent node")
        if (self.node_kind == "root") != (self.parent_ref is None):
            raise ConfigurationError("exactly the root node has no parent")
        _nonempty(self.cache_epoch_id, "cache epoch id")
        object_ref(self.epoch_ref, "cache epoch")
        for name in ("token_start", "token_end", "frames", "height", "width", "frontier"):
            _count(getattr(self, name), f"node {name}", zero=True)
        span = self.frames * self.height * self.width
        if self.token_end != self.token_start + span:
            raise ConfigurationError("node token span must equal its geometry")
        object.__setattr__(self, "matrix_records", _sorted_pairs(
            self.matrix_records, "node matrix records", lambda ref: object_ref(ref, "node matrix record")))
        object.__setattr__(self, "active_basis", _sorted_pairs(self.active_basis, "active basis bindings",
                                                               self._binding))
        streams = _validate_streams(self.streams, [k for k, _ in self.matrix_records], "node matrix records")
        _validate_streams(streams, [k for k, _ in self.active_basis], "active basis bindings")
        object.__setattr__(self, "streams", streams)
        if self.node_kind == "chunk":
            if not span or not self.matrix_records or self.frontier != self.token_end:
                raise ConfigurationError("a chunk node appends nonempty frames with matrix records")
        elif self.matrix_records:
            raise ConfigurationError("only chunk nodes carry their own matrix records")
        if self.node_kind in ("root", "recache") and span:
            raise ConfigurationError("root and recache nodes add no frames")
        if self.node_kind == "segment" and (self.token_start != 0 or not span or self.frontier != self.token_end):
            raise ConfigurationError("a segment node owns one segment-local range starting at zero")
        if self.execution_state_ref is not None:
            object_ref(self.execution_state_ref, "execution state", kinds=("blob",))
        if self.packet_ref is not None:
            object_ref(self.packet_ref, "node pack")
            if self.node_kind != "chunk":
                raise ConfigurationError("only chunk nodes carry their own node pack (epoch ranges carry theirs)")

    @staticmethod
    def _binding(value: Any) -> ActiveBasisBinding:
        if not isinstance(value, ActiveBasisBinding):
            raise ConfigurationError("active basis entries must be ActiveBasisBinding values")
        return value

    def binding(self, key: MatrixKey, stream: str | None = None) -> ActiveBasisBinding:
        entry = key if stream is None else (key, stream)
        for candidate, value in self.active_basis:
            if candidate == entry:
                return value
        return ActiveBasisBinding()

    def record_ref(self, key: MatrixKey, stream: str | None = None) -> str | None:
        entry = key if stream is None else (key, stream)
        for candidate, value in self.matrix_records:
            if candidate == entry:
                return value
        return None

    def to_dict(self) -> dict[str, Any]:
        data = {
            "schema": "reelcache.chunk_node.v2" if self.streams else "reelcache.chunk_node.v1",
            "node_kind": self.node_kind, "chunk_id": self.chunk_id, "parent": self.parent_ref,
            "cache_epoch_id": self.cache_epoch_id, "epoch": self.epoch_ref, "token_start": self.token_start,
            "token_end": self.token_end, "frames": self.frames, "height": self.height, "width": self.width,
            "frontier": self.frontier,
            "matrices": [{**_entry_dict(key), "record": ref} for key, ref in self.matrix_records],
            "active_basis": [{**_entry_dict(key), "binding": value.to_dict()} for key, value in self.active_basis],
            "execution_state": self.execution_state_ref,
        }
        if self.streams:
            data["streams"] = list(self.streams)
        if self.packet_ref is not None:
            data["packet"] = self.packet_ref
        return data

    @classmethod
    def from_dict(cls, data: Mapping[str, Any]) -> ChunkNode:
        try:
            fields = dict(data)
            schema = fields.pop("schema")
            if schema not in ("reelcache.chunk_node.v1", "reelcache.chunk_node.v2"):
                raise ConfigurationError("unsupported chunk node schema")
            streams = tuple(fields.pop("streams", ()))
            if (schema == "reelcache.chunk_node.v2") != bool(streams) or ("streams" in data and not streams):
                raise ConfigurationError("chunk node v2 (and only v2) declares its CFG streams")
            packet = fields.pop("packet", None)
            if "packet" in data and packet is None:
                raise ConfigurationError("an absent node pack is omitted")
            return cls(packet_ref=packet, parent_ref=fields.pop("parent"), epoch_ref=fields.pop("epoch"),
                       matrix_records=tuple((_entry_from(item), item["record"]) for item in fields.pop("matrices")),
                       active_basis=tuple((_entry_from(item), ActiveBasisBinding.from_dict(item["binding"]))
                                          for item in fields.pop("active_basis")),
                       execution_state_ref=fields.pop("execution_state"), streams=streams, **fields)
        except (KeyError, TypeError) as exc:
            raise ConfigurationError("invalid chunk node fields") from exc


# ---------------------------------------------------------------------------------------------
# Online rank predictor state
# ---------------------------------------------------------------------------------------------


@dataclass(frozen=True, order=True)
class PredictorKey:
    """Learner scope: model/source, layer, K|V, geometry, solver/detector and regime (fresh fits and
    augmentation-residual fits never share a learner)."""

    model_fingerprint: str
    layer: int
    target: str
    rows: int
    channels: int
    solver: str
    detector: str
    regime: str

    def __post_init__(self) -> None:
        _nonempty(self.model_fingerprint, "predictor model fingerprint")
        MatrixKey(self.layer, self.target)
        _count(self.rows, "predictor rows")
        _count(self.channels, "predictor channels")
        _nonempty(self.solver, "predictor solver")
        _nonempty(self.detector, "predictor detector")
        if self.regime not in PREDICTOR_REGIMES:
            raise ConfigurationError(f"predictor regime must be one of {PREDICTOR_REGIMES}")

    @property
    def matrix_key(self) -> MatrixKey:
        return MatrixKey(self.layer, self.target)

    @property
    def digest(self) -> str:
        return canonical_digest(self.to_dict())

    def to_dict(self) -> dict[str, Any]:
        return {name: getattr(self, name) for name in (
            "model_fingerprint", "layer", "target", "rows", "channels", "solver", "detector", "regime")}

    @classmethod
    def from_dict(cls, data: Mapping[str, Any]) -> PredictorKey:
        return _build(cls, data, "predictor key")


@dataclass(frozen=True)
class OnlineRidgeState:
    """2x2 online ridge regression of ``ln r = a + b x`` with prior ``M0 = s I``,
    ``v0 = M0 (ln m, 1)``; ``M`` stored as ``(m00, m01, m11)``."""

    m: tuple[float, float, float]
    v: tuple[float, float]
    observations: int = 0
    revision: int = 0
    anchor_rank: int = RANK_BUCKET
    prior_strength: float = 2.0

    def __post_init__(self) -> None:
        m, v = tuple(self.m), tuple(self.v)
        if len(m) != 3 or len(v) != 2 or not all(_real(item) for item in (*m, *v)):
            raise ConfigurationError("ridge state requires finite M (3 entries) and v (2 entries)")
        object.__setattr__(self, "m", tuple(float(item) for item in m))
        object.__setattr__(self, "v", tuple(float(item) for item in v))
        _count(self.observations, "ridge observations", zero=True)
        _count(self.revision, "ridge revision", zero=True)
        _count(self.anchor_rank, "anchor rank")
        if not _real(self.prior_strength) or self.prior_strength <= 0:
            raise ConfigurationError("ridge prior strength must be finite and positive")
        object.__setattr__(self, "prior_strength", float(self.prior_strength))
        m00, m01, m11 = self.m
        if m00 <= 0 or m00 * m11 - m01 * m01 <= 0:
            raise ConfigurationError("ridge M must be symmetric positive definite")

    @classmethod
    def initial(cls, anchor_rank: int = RANK_BUCKET, prior_strength: float = 2.0) -> OnlineRidgeState:
        _count(anchor_rank, "anchor rank")
        s = float(prior_strength)
        return cls((s, 0.0, s), (s * math.log(anchor_rank), s), 0, 0, anchor_rank, s)

    def coefficients(self) -> tuple[float, float]:
        m00, m01, m11 = self.m
        v0, v1 = self.v
        det = m00 * m11 - m01 * m01
        return (m11 * v0 - m01 * v1) / det, (m00 * v1 - m01 * v0) / det

    def log_rank(self, x: float) -> float:
        a, b = self.coefficients()
        return a + b * float(x)

    def predict(self, x: float) -> float:
        value = self.log_rank(x)
        return math.inf if value > 700 else math.exp(value)

    def updated(self, x: float, observed_rank: int | float) -> OnlineRidgeState:
        if not _real(x) or not _real(observed_rank) or observed_rank <= 0:
            raise ConfigurationError("ridge updates need a finite x and positive observed rank")
        x, label = float(x), math.log(float(observed_rank))
        m00, m01, m11 = self.m
        v0, v1 = self.v
        return OnlineRidgeState((m00 + 1.0, m01 + x, m11 + x * x), (v0 + label, v1 + x * label),
                                self.observations + 1, self.revision + 1, self.anchor_rank, self.prior_strength)

    @property
    def digest(self) -> str:
        return canonical_digest(self.to_dict())

    def to_dict(self) -> dict[str, Any]:
        return {"schema": "reelcache.online_ridge_state.v1", "m": list(self.m), "v": list(self.v),
                "observations": self.observations, "revision": self.revision, "anchor_rank": self.anchor_rank,
                "prior_strength": self.prior_strength}

    @classmethod
    def from_dict(cls, data: Mapping[str, Any]) -> OnlineRidgeState:
        try:
            fields = dict(data)
            if fields.pop("schema") != "reelcache.online_ridge_state.v1":
                raise ConfigurationError("unsupported ridge state schema")
            return cls(m=tuple(fields.pop("m")), v=tuple(fields.pop("v")), **fields)
        except (KeyError, TypeError) as exc:
            raise ConfigurationError("invalid ridge state fields") from exc


@dataclass(frozen=True)
class FitObservation:
    """A verified training observation of the rank predictor (never a retained KV matrix);
    ``observation_id`` binds the learner scope and the source identity, so replays are idempotent.
    ``origin`` is run context and never serialized."""

    key: PredictorKey
    source_id: str
    anchor_energy: float
    target_energy: float
    x: float
    observed_rank: int
    predicted_rank: float | None = None
    prediction_revision: int | None = None
    origin: str | None = None

    def __post_init__(self) -> None:
        if not isinstance(self.key, PredictorKey):
            raise ConfigurationError("observation key must be a PredictorKey")
        if self.origin is not None:
            _hex64(self.origin, "observation origin")
        _hex64(self.source_id, "observation source id")
        energy = self.anchor_energy
        if not _real(energy) or not 0 <= energy < 1:
            raise ConfigurationError("anchor energy must be in [0, 1)")
        target = _fraction(self.target_energy, "observation target")
        if target >= 1 or energy >= target:
            raise ConfigurationError("observations come from below-target anchors and sub-unit targets")
        if not _real(self.x) or self.x <= 0:
            raise ConfigurationError("observation x must be finite and positive")
        _count(self.observed_rank, "observed rank")
        if self.predicted_rank is not None and (
                isinstance(self.predicted_rank, bool) or not isinstance(self.predicted_rank, (int, float))
                or math.isnan(self.predicted_rank) or self.predicted_rank <= 0):
            raise ConfigurationError("predicted rank must be positive or None")
        if self.prediction_revision is not None:
            _count(self.prediction_revision, "prediction revision", zero=True)
        object.__setattr__(self, "anchor_energy", float(energy))
        object.__setattr__(self, "target_energy", target)
        object.__setattr__(self, "x", float(self.x))

    @property
    def observation_id(self) -> str:
        return canonical_digest({"key": self.key.to_dict(), "source_id": self.source_id})

    @property
    def payload_digest(self) -> str:
        return canonical_digest({"anchor_energy": self.anchor_energy, "target_energy": self.target_energy,
                                 "x": self.x, "observed_rank": self.observed_rank})

    def to_dict(self) -> dict[str, Any]:
        predicted = self.predicted_rank
        return {"schema": "reelcache.fit_observation.v1", "key": self.key.to_dict(), "source_id": self.source_id,
                "anchor_energy": self.anchor_energy, "target_energy": self.target_energy, "x": self.x,
                "observed_rank": self.observed_rank,
                "predicted_rank": None if predicted is None or not math.isfinite(predicted) else predicted,
                "prediction_revision": self.prediction_revision}

    @classmethod
    def from_dict(cls, data: Mapping[str, Any]) -> FitObservation:
        try:
            fields = dict(data)
            if fields.pop("schema") != "reelcache.fit_observation.v1":
                raise ConfigurationError("unsupported fit observation schema")
            return cls(key=PredictorKey.from_dict(fields.pop("key")), **fields)
        except (KeyError, TypeError) as exc:
            raise ConfigurationError("invalid fit observation fields") from exc
