"""Immutable, validated records of the runtime and their JSON forms.

What ``to_dict`` writes is the on-disk format (node manifests, matrix records, basis versions, cache epochs,
predictor state), shared with the reference implementation so that either reads the other's store: the key
names, the schema strings (``reelcache.energy_targets.v1``, ``reelcache.basis_version.v1``,
``reelcache.matrix_record.v1``, ``reelcache.cache_epoch.v1``, ``reelcache.chunk_node.v1`` / ``.v2``,
``reelcache.online_ridge_state.v1``, ``reelcache.fit_observation.v1``) and which optional keys are left out
when unset. Everything else here -- how a record is checked and how its JSON is produced and read back -- is
this module's own: every record class lists its JSON layout once (:class:`_Key` entries) and the shared
:func:`_encode` / :func:`_decode` helpers drive both directions from that list.
"""

from __future__ import annotations

import hashlib
import json
import math
import re
from dataclasses import dataclass
from types import MappingProxyType
from typing import Any, Callable, Mapping, Sequence

from .errors import ConfigurationError

RANK_BUCKET = 32
TARGETS = ("K", "V")
NODE_KINDS = ("root", "chunk", "recache", "segment")
EPOCH_CAUSES = ("initial", "kv_recache", "longcat_segment")
PREDICTOR_REGIMES = ("fresh", "residual")
BASIS_DOMAINS = MappingProxyType({"K": "normalized_pre_rope_k", "V": "direct_v"})
KEY_SPACES = ("pre_rope", "post_rope", "none")

_DTYPES = MappingProxyType({"float16": "float16", "half": "float16", "bfloat16": "bfloat16", "bf16": "bfloat16",
                            "float32": "float32", "float": "float32", "float64": "float64", "double": "float64"})
_REF_PATTERN = re.compile(r"(blob|basis|manifest):[0-9a-f]{64}")
_DIGEST_PATTERN = re.compile(r"[0-9a-f]{64}")
_ENERGY_TOLERANCE = 1e-6


# -------------------------------------------------------------------------------------------------------------
# Checks (each raises ConfigurationError with the offending value)
# -------------------------------------------------------------------------------------------------------------

def _fail(message: str):
    raise ConfigurationError(message)


def _whole(value: Any, what: str, *, allow_zero: bool = False) -> int:
    lowest = 0 if allow_zero else 1
    if type(value) is not int or value < lowest:
        _fail(f"{what}: expected an integer >= {lowest}, got {value!r}")
    return value


def _text(value: Any, what: str) -> str:
    if not isinstance(value, str) or value.strip() == "":
        _fail(f"{what}: expected a nonempty string, got {value!r}")
    return value


def _optional_text(value: Any, what: str) -> str | None:
    return None if value is None else _text(value, what)


def _finite(value: Any) -> bool:
    return isinstance(value, (int, float)) and not isinstance(value, bool) and math.isfinite(value)


def _share(value: Any, what: str) -> float:
    """A fraction in (0, 1]."""
    if not _finite(value) or value <= 0 or value > 1:
        _fail(f"{what}: expected a finite fraction in (0, 1], got {value!r}")
    return float(value)


def _measured_share(value: Any, what: str) -> float:
    """A measured energy fraction (at most 1 up to rounding)."""
    if not _finite(value) or value > 1 + _ENERGY_TOLERANCE:
        _fail(f"{what}: expected a finite measured fraction <= 1, got {value!r}")
    return float(value)


def _flag(value: Any, what: str) -> bool:
    if type(value) is not bool:
        _fail(f"{what}: expected true or false, got {value!r}")
    return value


def _digest(value: Any, what: str) -> str:
    if not isinstance(value, str) or _DIGEST_PATTERN.fullmatch(value) is None:
        _fail(f"{what}: expected a lowercase SHA-256 hex digest, got {value!r}")
    return value


def object_ref(value: Any, name: str, *, kinds: tuple[str, ...] = ("manifest",)) -> str:
    """``value`` if it names an immutable store object of one of ``kinds`` (``kind:<sha256>``)."""
    ok = isinstance(value, str) and _REF_PATTERN.fullmatch(value) is not None and value.partition(":")[0] in kinds
    if not ok:
        _fail(f"{name}: expected a {' or '.join(kinds)} object id, got {value!r}")
    return value


def canonical_dtype(value: Any) -> str:
    label = str(value)
    if label.startswith("torch."):
        label = label[len("torch."):]
    found = _DTYPES.get(label)
    if found is None:
        _fail(f"KV dtype {value!r} is not one of float16, bfloat16, float32, float64")
    return found


# -------------------------------------------------------------------------------------------------------------
# JSON values
# -------------------------------------------------------------------------------------------------------------

def json_copy(value: Any, *, name: str = "metadata") -> Any:
    """A plain JSON copy (dicts with string keys, lists, str/int/bool/None, finite floats)."""
    stack_limit = 10_000

    def copy(item: Any, depth: int) -> Any:
        if depth > stack_limit:
            _fail(f"{name} nests too deeply (or is cyclic)")
        if item is None or isinstance(item, (str, bool)) or type(item) is int:
            return item
        if type(item) is float:
            if not math.isfinite(item):
                _fail(f"{name} holds a non-finite number")
            return item
        if isinstance(item, Mapping):
            out = {}
            for key, child in item.items():
                if not isinstance(key, str):
                    _fail(f"{name} has a non-string key {key!r}")
                out[key] = copy(child, depth + 1)
            return out
        if isinstance(item, (list, tuple)):
            return [copy(child, depth + 1) for child in item]
        _fail(f"{name} holds a {type(item).__name__}, which is not JSON")

    try:
        return copy(value, 0)
    except RecursionError as exc:
        raise ConfigurationError(f"{name} nests too deeply (or is cyclic)") from exc


def thaw_json(value: Any) -> Any:
    """Plain dicts and lists from a frozen (mapping proxy / tuple) structure."""
    if isinstance(value, Mapping):
        return {key: thaw_json(item) for key, item in value.items()}
    if isinstance(value, (list, tuple)):
        return [thaw_json(item) for item in value]
    return value


def _frozen(value: Any) -> Any:
    if isinstance(value, Mapping):
        return MappingProxyType({key: _frozen(item) for key, item in value.items()})
    if isinstance(value, (list, tuple)):
        return tuple(_frozen(item) for item in value)
    return value


def frozen_json(value: Any, *, name: str = "metadata") -> Any:
    """An immutable copy of a JSON value (mapping proxies and tuples)."""
    return _frozen(json_copy(thaw_json(value), name=name))


def canonical_json(value: Any) -> bytes:
    return json.dumps(json_copy(thaw_json(value)), sort_keys=True, separators=(",", ":"),
                      allow_nan=False).encode("utf-8")


def canonical_digest(value: Any) -> str:
    """SHA-256 of the canonical JSON of ``value`` (sorted keys, no whitespace, no NaN)."""
    return hashlib.sha256(canonical_json(value)).hexdigest()


# -------------------------------------------------------------------------------------------------------------
# Declarative JSON layouts
# -------------------------------------------------------------------------------------------------------------

_ALWAYS = "always"     # the key is always written
_IF_SET = "if_set"     # written unless the value is None; a stored null is rejected
_IF_TRUE = "if_true"   # written only for truthy values; a stored falsy value is rejected


@dataclass(frozen=True)
class _Key:
    """One JSON key of a record: the attribute it holds, how the value is written and read back, and when
    the key is omitted."""

    attr: str
    key: str = ""
    write: Callable[[Any], Any] | None = None
    read: Callable[[Any], Any] | None = None
    omit: str = _ALWAYS

    @property
    def json_key(self) -> str:
        return self.key or self.attr


def _encode(record: Any, layout: Sequence[_Key], schema: str | None = None) -> dict[str, Any]:
    out: dict[str, Any] = {} if schema is None else {"schema": schema}
    for item in layout:
        value = getattr(record, item.attr)
        if item.omit == _IF_SET and value is None:
            continue
        if item.omit == _IF_TRUE and not value:
            continue
        out[item.json_key] = value if item.write is None else item.write(value)
    return out


def _decode(cls, data: Mapping[str, Any], layout: Sequence[_Key], what: str, *, schemas: tuple[str, ...] = (),
            extra: Mapping[str, Any] | None = None):
    """Build ``cls`` from its JSON; unknown keys, a wrong schema and stored nulls/zeros of omitted-when-unset
    keys are rejected."""
    if not isinstance(data, Mapping):
        _fail(f"{what}: expected a JSON object")
    fields = dict(data)
    if schemas:
        schema = fields.pop("schema", None)
        if schema not in schemas:
            _fail(f"{what}: schema {schema!r} is not one of {schemas}")
    kwargs = dict(extra or {})
    try:
        for item in layout:
            if item.json_key not in fields:
                if item.omit == _ALWAYS:
                    _fail(f"{what}: the key {item.json_key!r} is missing")
                continue
            raw = fields.pop(item.json_key)
            if item.omit == _IF_SET and raw is None:
                _fail(f"{what}: an unset {item.json_key!r} is left out, not stored as null")
            if item.omit == _IF_TRUE and not raw:
                _fail(f"{what}: a zero or empty {item.json_key!r} is left out, not stored")
            kwargs[item.attr] = raw if item.read is None else item.read(raw)
    except (KeyError, TypeError, AttributeError) as exc:
        raise ConfigurationError(f"{what}: malformed field ({exc})") from exc
    if fields:
        _fail(f"{what}: unknown keys {sorted(fields)}")
    try:
        return cls(**kwargs)
    except TypeError as exc:
        raise ConfigurationError(f"{what}: {exc}") from exc


# -------------------------------------------------------------------------------------------------------------
# Model and matrix identity
# -------------------------------------------------------------------------------------------------------------

def _per_target(value: Any) -> Any:
    return dict(value) if isinstance(value, Mapping) else value


@dataclass(frozen=True)
class ModelIdentity:
    """The model a store's matrices belong to: channel width and dtype per K/V (or per matrix)."""

    name: str
    fingerprint: str
    layers: int
    kv_channels: int | Mapping[str, int]
    layout: str
    dtype: str | Mapping[str, str]

    _JSON = (_Key("name"), _Key("fingerprint"), _Key("layers"), _Key("kv_channels", write=_per_target),
             _Key("layout"), _Key("dtype", write=_per_target))

    def __post_init__(self) -> None:
        _text(self.name, "model name")
        _text(self.fingerprint, "model fingerprint")
        _whole(self.layers, "model layers")
        _text(self.layout, "model layout")
        if isinstance(self.kv_channels, Mapping):
            if set(self.kv_channels) != set(TARGETS):
                _fail("per-target kv_channels name exactly K and V")
            for target in TARGETS:
                _whole(self.kv_channels[target], f"{target} channels")
            object.__setattr__(self, "kv_channels", MappingProxyType(dict(self.kv_channels)))
        else:
            _whole(self.kv_channels, "kv_channels")
        if isinstance(self.dtype, Mapping):
            by_target = set(TARGETS)
            by_matrix = {f"{layer}:{target}" for layer in range(self.layers) for target in TARGETS}
            if set(self.dtype) not in (by_target, by_matrix):
                _fail("a dtype mapping names K and V, or every layer:target matrix")
            object.__setattr__(self, "dtype", MappingProxyType({k: canonical_dtype(v) for k, v in self.dtype.items()}))
        else:
            object.__setattr__(self, "dtype", canonical_dtype(self.dtype))

    def channels_for(self, target: str | "MatrixKey") -> int:
        which = target.target if isinstance(target, MatrixKey) else target
        if which not in TARGETS:
            _fail(f"target {which!r} is not K or V")
        return self.kv_channels[which] if isinstance(self.kv_channels, Mapping) else self.kv_channels

    def dtype_for(self, target: str | "MatrixKey") -> str:
        key = target if isinstance(target, MatrixKey) else None
        which = key.target if key is not None else target
        if which not in TARGETS:
            _fail(f"target {which!r} is not K or V")
        if key is not None and key.layer >= self.layers:
            _fail(f"layer {key.layer} is outside the model's {self.layers} layers")
        table = self.dtype
        if not isinstance(table, Mapping):
            return table
        if which in table:
            return table[which]
        if key is None:
            _fail("a per-layer dtype is looked up by MatrixKey")
        return table[f"{key.layer}:{key.target}"]

    def to_dict(self) -> dict[str, Any]:
        return _encode(self, self._JSON)

    @classmethod
    def from_dict(cls, data: Mapping[str, Any]) -> "ModelIdentity":
        return _decode(cls, data, cls._JSON, "model identity")

    def __hash__(self) -> int:
        dtypes = tuple(self.dtype_for(MatrixKey(layer, t)) for layer in range(self.layers) for t in TARGETS)
        return hash((self.name, self.fingerprint, self.layers, self.channels_for("K"), self.channels_for("V"),
                     self.layout, dtypes))


@dataclass(frozen=True, order=True)
class MatrixKey:
    layer: int
    target: str

    _JSON = (_Key("layer"), _Key("target"))

    def __post_init__(self) -> None:
        _whole(self.layer, "matrix layer", allow_zero=True)
        if self.target not in TARGETS:
            _fail(f"matrix target {self.target!r} is not K or V")

    def to_dict(self) -> dict[str, Any]:
        return {"layer": self.layer, "target": self.target}

    @classmethod
    def from_dict(cls, data: Mapping[str, Any]) -> "MatrixKey":
        return _decode(cls, data, cls._JSON, "matrix key")


@dataclass(frozen=True)
class TensorContext:
    """Where one ``[tokens, channels]`` matrix sits: model, layer and K/V, first token, frame grid and key
    space. ``source_dtype`` overrides the model's declared dtype (written only when set)."""

    model: ModelIdentity
    key: MatrixKey
    token_start: int
    frames: int
    height: int
    width: int
    key_space: str
    source_dtype: str | None = None

    _JSON = (_Key("model", write=lambda m: m.to_dict(), read=lambda d: ModelIdentity.from_dict(d)),
             _Key("key", write=lambda k: k.to_dict(), read=lambda d: MatrixKey.from_dict(d)),
             _Key("token_start"), _Key("frames"), _Key("height"), _Key("width"), _Key("key_space"),
             _Key("source_dtype", omit=_IF_SET))

    def __post_init__(self) -> None:
        if not isinstance(self.model, ModelIdentity):
            _fail("a tensor context needs a ModelIdentity")
        if not isinstance(self.key, MatrixKey):
            _fail("a tensor context needs a MatrixKey")
        if self.key.layer >= self.model.layers:
            _fail(f"layer {self.key.layer} is outside the model's {self.model.layers} layers")
        _whole(self.token_start, "context token_start", allow_zero=True)
        for axis in ("frames", "height", "width"):
            _whole(getattr(self, axis), f"context {axis}")
        if self.key_space not in KEY_SPACES:
            _fail(f"key_space {self.key_space!r} is not one of {KEY_SPACES}")
        if self.key.target == "V" and self.key_space != "none":
            _fail("V matrices have no key space (key_space='none')")
        if self.source_dtype is not None:
            object.__setattr__(self, "source_dtype", canonical_dtype(self.source_dtype))

    @property
    def channels(self) -> int:
        return self.model.channels_for(self.key)

    @property
    def dtype(self) -> str:
        return self.source_dtype if self.source_dtype is not None else self.model.dtype_for(self.key)

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
        return _encode(self, self._JSON)

    @classmethod
    def from_dict(cls, data: Mapping[str, Any]) -> "TensorContext":
        return _decode(cls, data, cls._JSON, "tensor context")


_CODEC_KINDS = ("raw", "svd", "svd_hevc")
_NORMALIZATIONS = ("per_channel", "global", "leading_columns")


@dataclass(frozen=True)
class CodecSpec:
    """How a matrix is represented: ``raw``, ``svd`` (factors) or ``svd_hevc`` (factors, coefficients in an
    8-bit video stream). Per-channel normalization pins ``protected_fraction`` to 1 and global to 0.
    ``inter_prediction`` is written for svd_hevc records of version 2; ``None`` marks a version-1 record
    written before the flag existed."""

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
        if self.kind not in _CODEC_KINDS:
            _fail(f"codec kind {self.kind!r} is not one of {_CODEC_KINDS}")
        if self.kind == "raw" and self.rank is not None:
            _fail("a raw representation has no rank")
        if self.kind != "raw":
            _whole(self.rank, "codec rank")
        if self.normalization not in _NORMALIZATIONS:
            _fail(f"normalization {self.normalization!r} is not one of {_NORMALIZATIONS}")
        if not _finite(self.protected_fraction) or not 0 <= self.protected_fraction <= 1:
            _fail(f"protected_fraction {self.protected_fraction!r} is not in [0, 1]")
        pinned = {"global": 0.0, "per_channel": 1.0}.get(self.normalization)
        if pinned is not None:
            object.__setattr__(self, "protected_fraction", pinned)
        _text(self.pix_fmt, "pix_fmt")
        _text(self.preset, "preset")
        if self.ffmpeg_path is not None and ("\x00" in _text(self.ffmpeg_path, "ffmpeg_path")):
            _fail("ffmpeg_path holds a NUL byte")
        if type(self.qp) is not int or self.qp < 0 or self.qp > 51:
            _fail(f"qp {self.qp!r} is not an integer in [0, 51]")
        if self.inter_prediction is not None and type(self.inter_prediction) is not bool:
            _fail("inter_prediction is true, false or unset")
        if self.kind != "svd_hevc":
            if self.inter_prediction:
                _fail("inter prediction exists only for svd_hevc coefficient streams")
            object.__setattr__(self, "inter_prediction", False)

    @property
    def legacy_gop(self) -> bool:
        return self.inter_prediction is None

    def to_dict(self) -> dict[str, Any]:
        out = {name: getattr(self, name) for name in ("kind", "rank", "normalization", "protected_fraction",
                                                      "pix_fmt", "qp", "preset", "ffmpeg_path")}
        if self.kind == "svd_hevc" and self.inter_prediction is not None:
            out["inter_prediction"] = self.inter_prediction
        return out

    @classmethod
    def from_dict(cls, data: Mapping[str, Any]) -> "CodecSpec":
        fields = dict(data)
        flag = fields.get("inter_prediction", None)
        if "inter_prediction" in fields and type(flag) is not bool:
            _fail("a stored inter_prediction is true or false")
        fields["inter_prediction"] = flag
        try:
            return cls(**fields)
        except TypeError as exc:
            raise ConfigurationError(f"codec spec: {exc}") from exc


@dataclass(frozen=True)
class EncodedTensor:
    """An encoded packet: JSON metadata, named payloads, an optional attached basis and metrics."""

    metadata: Mapping[str, Any]
    payloads: Mapping[str, bytes]
    basis: bytes | None = None
    metrics: Mapping[str, Any] | None = None

    def __post_init__(self) -> None:
        if not isinstance(self.metadata, Mapping) or not isinstance(self.payloads, Mapping):
            _fail("an encoded packet has mapping metadata and payloads")
        if len(self.payloads) == 0:
            _fail("an encoded packet has at least one payload")
        for name, blob in self.payloads.items():
            _text(name, "payload name")
            if not isinstance(blob, bytes):
                _fail(f"payload {name!r} is not immutable bytes")
        if self.basis is not None and not isinstance(self.basis, bytes):
            _fail("an attached basis is immutable bytes")
        if self.metrics is not None and not isinstance(self.metrics, Mapping):
            _fail("packet metrics are a mapping")
        object.__setattr__(self, "metadata", json_copy(self.metadata))
        object.__setattr__(self, "payloads", MappingProxyType(dict(self.payloads)))
        if self.metrics is not None:
            object.__setattr__(self, "metrics", json_copy(self.metrics, name="metrics"))


# -------------------------------------------------------------------------------------------------------------
# Node entries: a MatrixKey, or (MatrixKey, CFG stream label) in multi-stream nodes
# -------------------------------------------------------------------------------------------------------------

def _label_ok(label: Any) -> bool:
    return isinstance(label, str) and label != "" and label == label.strip()


def entry_key(value: Any, name: str = "matrix entry") -> Any:
    if isinstance(value, MatrixKey):
        return value
    if isinstance(value, tuple) and len(value) == 2 and isinstance(value[0], MatrixKey) and _label_ok(value[1]):
        return value
    _fail(f"{name}: expected a MatrixKey or (MatrixKey, stream label), got {value!r}")


def entry_parts(value: Any) -> tuple[MatrixKey, str | None]:
    checked = entry_key(value)
    return (checked, None) if isinstance(checked, MatrixKey) else checked


def entry_order(value: Any) -> tuple:
    key, stream = entry_parts(value)
    return key.layer, key.target, stream is not None, stream or ""


def _entry_json(value: Any) -> dict[str, Any]:
    key, stream = entry_parts(value)
    out = {"key": key.to_dict()}
    if stream is not None:
        out["stream"] = stream
    return out


def _entry_read(item: Mapping[str, Any]) -> Any:
    key = MatrixKey.from_dict(item["key"])
    return key if item.get("stream") is None else entry_key((key, item["stream"]))


def _keyed_pairs(values: Any, what: str, check: Callable[[Any], Any]) -> tuple:
    """Sorted ``(entry, value)`` pairs with unique entries, from a mapping or a pair sequence."""
    if isinstance(values, Mapping):
        items = list(values.items())
    elif isinstance(values, (tuple, list)):
        items = list(values)
    else:
        _fail(f"{what}: expected a mapping or a sequence of (entry, value) pairs")
    pairs = []
    for item in items:
        if not isinstance(item, (tuple, list)) or len(item) != 2:
            _fail(f"{what}: {item!r} is not an (entry, value) pair")
        pairs.append((entry_key(item[0], what), check(item[1])))
    pairs.sort(key=lambda pair: entry_order(pair[0]))
    if len({entry for entry, _ in pairs}) != len(pairs):
        _fail(f"{what}: an entry appears twice")
    return tuple(pairs)


def _check_streams(streams: Any, entries: Sequence[Any], what: str) -> tuple[str, ...]:
    """Declared CFG streams (sorted, unique) and entries that cover the same matrices in every stream."""
    streams = tuple(streams)
    if not all(_label_ok(s) for s in streams):
        _fail("stream labels are nonempty and carry no surrounding whitespace")
    if list(streams) != sorted(set(streams)):
        _fail("stream labels are listed once each, sorted")
    labels = {entry_parts(item)[1] for item in entries}
    if not streams:
        if labels != set() and labels != {None}:
            _fail(f"{what}: labeled entries in a node that declares no streams")
        return streams
    if None in labels or not labels <= set(streams):
        _fail(f"{what}: every entry of a multi-stream node is labeled with a declared stream")
    if entries:
        keys_of: dict[str, set] = {s: set() for s in streams}
        for item in entries:
            key, stream = entry_parts(item)
            keys_of[stream].add(key)
        if len({frozenset(keys) for keys in keys_of.values()}) != 1:
            _fail(f"{what}: the streams cover different matrices")
    return streams


# -------------------------------------------------------------------------------------------------------------
# Energy targets and reports
# -------------------------------------------------------------------------------------------------------------

_ENERGY_SCHEMA = "reelcache.energy_targets.v1"


@dataclass(frozen=True)
class EnergyTargets:
    """The energy fractions a fit must keep: pre-RoPE K and direct V (1.0 marks a full-width diagnostic)."""

    profile: str
    key: float
    value: float
    provisional: bool
    note: str | None = None

    _JSON = (_Key("profile"), _Key("key"), _Key("value"), _Key("provisional"), _Key("note"))

    def __post_init__(self) -> None:
        _text(self.profile, "energy profile")
        object.__setattr__(self, "key", _share(self.key, "K energy target"))
        object.__setattr__(self, "value", _share(self.value, "V energy target"))
        _flag(self.provisional, "provisional")
        _optional_text(self.note, "energy profile note")

    def for_target(self, target: str | MatrixKey) -> float:
        which = target.target if isinstance(target, MatrixKey) else target
        if which not in TARGETS:
            _fail(f"energy targets exist for K and V, not {which!r}")
        return self.key if which == "K" else self.value

    def is_diagnostic(self, target: str | MatrixKey) -> bool:
        return self.for_target(target) == 1.0

    def to_dict(self) -> dict[str, Any]:
        return _encode(self, self._JSON, _ENERGY_SCHEMA)

    @classmethod
    def from_dict(cls, data: Mapping[str, Any]) -> "EnergyTargets":
        return _decode(cls, data, cls._JSON, "energy targets", schemas=(_ENERGY_SCHEMA,))

    @property
    def fingerprint(self) -> str:
        return canonical_digest(self.to_dict())


_UNTUNED = "provisional K98/V95 until the energy sweeps select a model-specific profile"
ENERGY_TARGET_PROFILES = MappingProxyType({
    name: EnergyTargets(name, 0.98, 0.95, name != "causvid",
                        "final: pre-RoPE K 98%, V 95%" if name == "causvid" else _UNTUNED)
    for name in ("causvid", "raven", "longlive1", "longlive2", "longcat_720p")})


def energy_targets(profile: str) -> EnergyTargets:
    found = ENERGY_TARGET_PROFILES.get(profile) if isinstance(profile, str) else None
    if found is None:
        _fail(f"there is no energy target profile named {profile!r}")
    return found


@dataclass(frozen=True)
class EnergyReport:
    """Energies of one fit: the ideal subspace, the stored factors (FP16 rows, FP32 ``P = A Q^T``) and,
    when measured, the relative error after the codec."""

    target: float
    ideal_subspace_energy: float
    stored_factor_energy: float
    post_codec_relative_error: float | None = None
    observed_rank: int | None = None
    bucket_rank: int = 0
    rank_view: int = 1
    zero_input: bool = False
    diagnostic_full_width: bool = False

    _JSON = tuple(_Key(name) for name in ("target", "ideal_subspace_energy", "stored_factor_energy",
                                          "post_codec_relative_error", "observed_rank", "bucket_rank", "rank_view",
                                          "zero_input", "diagnostic_full_width"))

    def __post_init__(self) -> None:
        object.__setattr__(self, "target", _share(self.target, "energy target"))
        for name in ("ideal_subspace_energy", "stored_factor_energy"):
            object.__setattr__(self, name, _measured_share(getattr(self, name), name.replace("_", " ")))
        error = self.post_codec_relative_error
        if error is not None:
            if not _finite(error) or error < 0:
                _fail(f"post-codec relative error {error!r} is not a finite nonnegative number")
            object.__setattr__(self, "post_codec_relative_error", float(error))
        if self.observed_rank is not None:
            _whole(self.observed_rank, "observed rank", allow_zero=True)
        _whole(self.bucket_rank, "bucket rank", allow_zero=True)
        _whole(self.rank_view, "rank view")
        _flag(self.zero_input, "zero_input")
        _flag(self.diagnostic_full_width, "diagnostic_full_width")
        if self.zero_input and (self.ideal_subspace_energy, self.stored_factor_energy) != (1.0, 1.0):
            _fail("an all-zero input is represented exactly (energies of 1)")

    @property
    def meets_target(self) -> bool:
        return self.zero_input or self.stored_factor_energy >= self.target

    def to_dict(self) -> dict[str, Any]:
        return _encode(self, self._JSON)

    @classmethod
    def from_dict(cls, data: Mapping[str, Any]) -> "EnergyReport":
        return _decode(cls, data, cls._JSON, "energy report")


# -------------------------------------------------------------------------------------------------------------
# Basis versions and the active basis of a lineage
# -------------------------------------------------------------------------------------------------------------

_BASIS_SCHEMA = "reelcache.basis_version.v1"


@dataclass(frozen=True)
class BasisVersion:
    """One immutable version of a per-(layer, K/V) basis: the parent's rows followed by this version's FP16
    row block. ``view_sha256`` binds the bytes of the whole ``[total_rank, channels]`` view."""

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

    _JSON = (_Key("parent_ref", "parent"), _Key("added_rows_ref", "added_rows"), _Key("added_rank"),
             _Key("total_rank"), _Key("channels"), _Key("dtype"), _Key("group_id"),
             _Key("key", write=lambda k: k.to_dict(), read=lambda d: MatrixKey.from_dict(d)),
             _Key("domain"), _Key("model_fingerprint"), _Key("depth"), _Key("view_sha256"))

    def __post_init__(self) -> None:
        if self.parent_ref is not None:
            object_ref(self.parent_ref, "parent basis version")
        object_ref(self.added_rows_ref, "basis row block", kinds=("basis",))
        for name in ("added_rank", "total_rank", "channels"):
            _whole(getattr(self, name), name.replace("_", " "))
        _whole(self.depth, "basis depth", allow_zero=True)
        if not isinstance(self.key, MatrixKey):
            _fail("a basis version belongs to one MatrixKey")
        _text(self.model_fingerprint, "basis model fingerprint")
        _digest(self.group_id, "basis group id")
        _digest(self.view_sha256, "basis view digest")
        if self.dtype != "float16":
            _fail("basis rows are stored as float16")
        if self.total_rank > self.channels:
            _fail(f"a basis of {self.channels} channels holds at most that many rows, not {self.total_rank}")
        root = self.parent_ref is None
        if root != (self.depth == 0):
            _fail("depth 0 and no parent go together")
        if root and self.total_rank != self.added_rank:
            _fail("a root version holds exactly its own block")
        if not root and self.total_rank <= self.added_rank:
            _fail("an extension appends to a nonempty parent")

    @property
    def domain(self) -> str:
        return BASIS_DOMAINS[self.key.target]

    @property
    def parent_rank(self) -> int:
        return self.total_rank - self.added_rank

    @property
    def added_bytes(self) -> int:
        return 2 * self.added_rank * self.channels

    @staticmethod
    def root_group_id(model_fingerprint: str, key: MatrixKey, rows_ref: str) -> str:
        return canonical_digest({"model": model_fingerprint, "key": key.to_dict(), "root_rows": rows_ref})

    def to_dict(self) -> dict[str, Any]:
        return _encode(self, self._JSON, _BASIS_SCHEMA)

    @classmethod
    def from_dict(cls, data: Mapping[str, Any]) -> "BasisVersion":
        fields = dict(data) if isinstance(data, Mapping) else None
        if fields is None or "domain" not in fields:
            _fail("basis version: the key 'domain' is missing")
        domain = fields.pop("domain")
        layout = tuple(item for item in cls._JSON if item.attr != "domain")
        version = _decode(cls, fields, layout, "basis version", schemas=(_BASIS_SCHEMA,))
        if domain != version.domain:
            _fail(f"basis version: domain {domain!r} does not match its {version.key.target} key")
        return version


@dataclass(frozen=True)
class ActiveBasisBinding:
    """A lineage's current basis for one matrix and what the refit rule remembers about it (the fresh
    rank, the measured coefficient rate, and the cumulative refit debt -- written only when nonzero)."""

    version_ref: str | None = None
    total_rank: int = 0
    group_id: str | None = None
    fresh_rank: int | None = None
    fresh_chunk_id: str | None = None
    coefficient_rate: float | None = None
    rate_identity: str | None = None
    refit_debt: float = 0.0

    _JSON = tuple(_Key(name) for name in ("version_ref", "total_rank", "group_id", "fresh_rank", "fresh_chunk_id",
                                          "coefficient_rate", "rate_identity")) + (_Key("refit_debt", omit=_IF_TRUE),)

    def __post_init__(self) -> None:
        if self.version_ref is not None:
            object_ref(self.version_ref, "active basis version")
            _whole(self.total_rank, "active basis rank")
            _digest(self.group_id, "active basis group")
        elif self.total_rank != 0 or self.group_id is not None:
            _fail("an empty binding carries no rank and no group")
        if (self.fresh_rank is None) is not (self.fresh_chunk_id is None):
            _fail("a fresh rank is recorded with the chunk that measured it")
        if self.fresh_rank is not None:
            _whole(self.fresh_rank, "fresh rank")
            _text(self.fresh_chunk_id, "fresh chunk id")
        if (self.coefficient_rate is None) is not (self.rate_identity is None):
            _fail("a coefficient rate is recorded with its codec and geometry identity")
        if self.coefficient_rate is not None:
            if not _finite(self.coefficient_rate) or self.coefficient_rate <= 0:
                _fail(f"coefficient rate {self.coefficient_rate!r} is not finite and positive")
            object.__setattr__(self, "coefficient_rate", float(self.coefficient_rate))
            _digest(self.rate_identity, "coefficient rate identity")
        if not _finite(self.refit_debt) or self.refit_debt < 0:
            _fail(f"refit debt {self.refit_debt!r} is not finite and nonnegative")
        object.__setattr__(self, "refit_debt", float(self.refit_debt) if self.refit_debt else 0.0)
        if self.refit_debt and (self.version_ref is None or self.fresh_rank is None):
            _fail("a refit debt belongs to an active basis with a recorded fresh rank")

    def to_dict(self) -> dict[str, Any]:
        return _encode(self, self._JSON)

    @classmethod
    def from_dict(cls, data: Mapping[str, Any]) -> "ActiveBasisBinding":
        layout = tuple(_Key(k.attr, omit=_IF_SET if k.attr == "refit_debt" else k.omit) for k in cls._JSON)
        if isinstance(data, Mapping) and "refit_debt" in data and data["refit_debt"] == 0:
            _fail("active basis binding: a zero refit debt is left out, not stored")
        fields = {name: None for name in ("version_ref", "group_id", "fresh_rank", "fresh_chunk_id",
                                          "coefficient_rate", "rate_identity")}
        fields["total_rank"] = 0
        fields.update(dict(data) if isinstance(data, Mapping) else {})
        return _decode(cls, fields, layout, "active basis binding")


def _is_factor_tile(codec: CodecSpec, decision: Any) -> bool:
    """An svd record stored as a tile of a factor pack (canvas policy ``factor_tiles``)."""
    packet = decision.get("packet") if isinstance(decision, Mapping) else None
    canvas = packet.get("canvas") if isinstance(packet, Mapping) else None
    return codec.kind == "svd" and isinstance(canvas, Mapping) and canvas.get("policy") == "factor_tiles"


_RECORD_SCHEMA = "reelcache.matrix_record.v1"


def _optional_dict(value):
    return None if value is None else value.to_dict()


@dataclass(frozen=True)
class MatrixRecord:
    """One committed matrix: its packet (or its tile of a node pack) and the exact basis view it uses."""

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

    _JSON = (_Key("context", write=lambda c: c.to_dict(), read=lambda d: TensorContext.from_dict(d)),
             _Key("codec", write=lambda c: c.to_dict(), read=lambda d: CodecSpec.from_dict(d)),
             _Key("packet_ref", "packet"), _Key("basis_version_ref", "basis_version"), _Key("rank_view"),
             _Key("energy", write=_optional_dict, read=lambda d: None if d is None else EnergyReport.from_dict(d)),
             _Key("predictor_revision_ref", "predictor_revision"), _Key("decision", write=thaw_json),
             _Key("packet_tile", omit=_IF_SET), _Key("stream", omit=_IF_SET))

    def __post_init__(self) -> None:
        if not isinstance(self.context, TensorContext) or not isinstance(self.codec, CodecSpec):
            _fail("a matrix record has a TensorContext and a CodecSpec")
        object_ref(self.packet_ref, "matrix packet")
        lossy = self.codec.kind != "raw"
        if not lossy:
            if (self.basis_version_ref, self.rank_view, self.energy) != (None, None, None):
                _fail("a raw record names no basis, no rank view and no energy")
        else:
            object_ref(self.basis_version_ref, "matrix basis version")
            _whole(self.rank_view, "rank view")
            if self.rank_view != self.codec.rank:
                _fail(f"rank view {self.rank_view} differs from the codec's rank {self.codec.rank}")
            if not isinstance(self.energy, EnergyReport) or self.energy.rank_view != self.rank_view:
                _fail("a lossy record carries the energy report of its rank view")
            if self.context.key.target == "K" and self.context.key_space != "pre_rope":
                _fail("lossy K records hold normalized pre-RoPE K")
        if self.packet_tile is not None:
            _whole(self.packet_tile, "packet tile", allow_zero=True)
            pack_tile = _is_factor_tile(self.codec, self.decision) or \
                (self.codec.kind == "svd_hevc" and self.codec.inter_prediction is False)
            if not pack_tile:
                _fail("only all-intra svd_hevc matrices and factor-pack tiles live in a pack")
        if self.stream is not None:
            entry_key((self.context.key, self.stream), "matrix record stream")
        if self.predictor_revision_ref is not None:
            _text(self.predictor_revision_ref, "predictor revision")
        object.__setattr__(self, "decision", frozen_json(self.decision, name="matrix decision"))

    @property
    def entry(self) -> Any:
        return self.context.key if self.stream is None else (self.context.key, self.stream)

    def to_dict(self) -> dict[str, Any]:
        return _encode(self, self._JSON, _RECORD_SCHEMA)

    @classmethod
    def from_dict(cls, data: Mapping[str, Any]) -> "MatrixRecord":
        return _decode(cls, data, cls._JSON, "matrix record", schemas=(_RECORD_SCHEMA,))


# -------------------------------------------------------------------------------------------------------------
# Cache epochs and chunk nodes
# -------------------------------------------------------------------------------------------------------------

def _record_id(ref: Any) -> str:
    return object_ref(ref, "matrix record")


def _pairs_json(field: str):
    def write(pairs):
        return [{**_entry_json(entry), field: (value.to_dict() if hasattr(value, "to_dict") else value)}
                for entry, value in pairs]
    return write


def _pairs_read(field: str, convert=None):
    def read(items):
        return tuple((_entry_read(item), item[field] if convert is None else convert(item[field])) for item in items)
    return read


@dataclass(frozen=True)
class TokenRangeRecords:
    """The matrix records of one re-materialized (or segment-local) token range of an epoch."""

    chunk_id: str
    token_start: int
    token_end: int
    frames: int
    height: int
    width: int
    records: tuple[tuple[Any, str], ...]
    streams: tuple[str, ...] = ()
    packet_ref: str | None = None

    _JSON = (_Key("chunk_id"), _Key("token_start"), _Key("token_end"), _Key("frames"), _Key("height"),
             _Key("width"), _Key("records", write=_pairs_json("record"), read=_pairs_read("record")),
             _Key("streams", write=list, read=tuple, omit=_IF_TRUE), _Key("packet_ref", "packet", omit=_IF_SET))

    def __post_init__(self) -> None:
        _text(self.chunk_id, "range chunk id")
        if self.packet_ref is not None:
            object_ref(self.packet_ref, "range node pack")
        _whole(self.token_start, "range token start", allow_zero=True)
        for axis in ("frames", "height", "width"):
            _whole(getattr(self, axis), f"range {axis}")
        if self.token_end - self.token_start != self.frames * self.height * self.width:
            _fail("a range spans exactly its frames x height x width tokens")
        records = _keyed_pairs(self.records, "range records", _record_id)
        object.__setattr__(self, "records", records)
        object.__setattr__(self, "streams", _check_streams(self.streams, [e for e, _ in records], "range records"))

    def to_dict(self) -> dict[str, Any]:
        return _encode(self, self._JSON)

    @classmethod
    def from_dict(cls, data: Mapping[str, Any]) -> "TokenRangeRecords":
        return _decode(cls, data, cls._JSON, "token range")


_EPOCH_SCHEMA = "reelcache.cache_epoch.v1"


@dataclass(frozen=True)
class CacheEpoch:
    """A version of the cache: ``initial``, a KV recache (global positions) or a LongCat segment
    (segment-local positions)."""

    epoch_id: str
    parent_epoch_ref: str | None
    cause: str
    position_space: str
    ranges: tuple[TokenRangeRecords, ...]
    details: Mapping[str, Any]

    _JSON = (_Key("epoch_id"), _Key("parent_epoch_ref", "parent_epoch"), _Key("cause"), _Key("position_space"),
             _Key("ranges", write=lambda rs: [r.to_dict() for r in rs],
                  read=lambda items: tuple(TokenRangeRecords.from_dict(i) for i in items)),
             _Key("details", write=thaw_json))

    def __post_init__(self) -> None:
        _text(self.epoch_id, "epoch id")
        if self.parent_epoch_ref is not None:
            object_ref(self.parent_epoch_ref, "parent epoch")
        if self.cause not in EPOCH_CAUSES:
            _fail(f"epoch cause {self.cause!r} is not one of {EPOCH_CAUSES}")
        if self.position_space not in ("global", "segment_local"):
            _fail(f"position space {self.position_space!r} is neither global nor segment_local")
        ranges = tuple(self.ranges)
        if not all(isinstance(r, TokenRangeRecords) for r in ranges):
            _fail("epoch ranges are TokenRangeRecords")
        starts = [r.token_start for r in ranges]
        if starts != sorted(starts) or any(a.token_end > b.token_start for a, b in zip(ranges, ranges[1:])):
            _fail("epoch ranges are sorted and disjoint")
        shape = (bool(ranges), self.parent_epoch_ref is not None, self.position_space)
        allowed = {"initial": (False, False, "global"), "kv_recache": (True, True, "global"),
                   "longcat_segment": (True, True, "segment_local")}[self.cause]
        if shape != allowed:
            _fail(f"a {self.cause} epoch has ranges={allowed[0]}, a parent={allowed[1]} and {allowed[2]} "
                  "positions")
        if self.cause == "longcat_segment" and (len(ranges) != 1 or ranges[0].token_start != 0):
            _fail("a segment epoch holds exactly one range starting at token 0")
        latents_only = isinstance(self.details, Mapping) and self.details.get("kv_objects") is False
        if any(not r.records for r in ranges) and not latents_only:
            _fail("a re-materialized range lists its matrix records (only a latents-only epoch, details "
                  "kv_objects=false, stores none)")
        object.__setattr__(self, "ranges", ranges)
        object.__setattr__(self, "details", frozen_json(self.details, name="epoch details"))

    def to_dict(self) -> dict[str, Any]:
        return _encode(self, self._JSON, _EPOCH_SCHEMA)

    @classmethod
    def from_dict(cls, data: Mapping[str, Any]) -> "CacheEpoch":
        return _decode(cls, data, cls._JSON, "cache epoch", schemas=(_EPOCH_SCHEMA,))


_NODE_V1, _NODE_V2 = "reelcache.chunk_node.v1", "reelcache.chunk_node.v2"


@dataclass(frozen=True)
class ChunkNode:
    """One immutable node of a session tree (``root``, ``chunk``, ``recache`` or ``segment``);
    ``active_basis`` is the complete per-matrix binding the next commit tests against."""

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

    _JSON = (_Key("node_kind"), _Key("chunk_id"), _Key("parent_ref", "parent"), _Key("cache_epoch_id"),
             _Key("epoch_ref", "epoch"), _Key("token_start"), _Key("token_end"), _Key("frames"), _Key("height"),
             _Key("width"), _Key("frontier"),
             _Key("matrix_records", "matrices", write=_pairs_json("record"), read=_pairs_read("record")),
             _Key("active_basis", write=_pairs_json("binding"),
                  read=_pairs_read("binding", lambda d: ActiveBasisBinding.from_dict(d))),
             _Key("execution_state_ref", "execution_state"),
             _Key("streams", write=list, read=tuple, omit=_IF_TRUE), _Key("packet_ref", "packet", omit=_IF_SET))

    def __post_init__(self) -> None:
        if self.node_kind not in NODE_KINDS:
            _fail(f"node kind {self.node_kind!r} is not one of {NODE_KINDS}")
        _text(self.chunk_id, "node chunk id")
        if self.parent_ref is not None:
            object_ref(self.parent_ref, "parent node")
        if (self.parent_ref is None) != (self.node_kind == "root"):
            _fail("the root, and only the root, has no parent")
        _text(self.cache_epoch_id, "cache epoch id")
        object_ref(self.epoch_ref, "cache epoch")
        for name in ("token_start", "token_end", "frames", "height", "width", "frontier"):
            _whole(getattr(self, name), f"node {name}", allow_zero=True)
        span = self.frames * self.height * self.width
        if self.token_end - self.token_start != span:
            _fail("a node spans exactly its frames x height x width tokens")

        def binding(value):
            if not isinstance(value, ActiveBasisBinding):
                _fail("active basis values are ActiveBasisBinding records")
            return value

        records = _keyed_pairs(self.matrix_records, "node matrix records", _record_id)
        bindings = _keyed_pairs(self.active_basis, "active basis bindings", binding)
        object.__setattr__(self, "matrix_records", records)
        object.__setattr__(self, "active_basis", bindings)
        streams = _check_streams(self.streams, [e for e, _ in records], "node matrix records")
        _check_streams(streams, [e for e, _ in bindings], "active basis bindings")
        object.__setattr__(self, "streams", streams)
        kind = self.node_kind
        if kind == "chunk" and (span == 0 or self.frontier != self.token_end
                                or (not records and self.execution_state_ref is None)):
            _fail("a chunk node appends frames and records their matrices (a latents-only node instead names "
                  "the execution state it is replayed from); its frontier is its end")
        if kind != "chunk" and records:
            _fail("only chunk nodes carry matrix records of their own")
        if kind in ("root", "recache") and span:
            _fail(f"a {kind} node adds no frames")
        if kind == "segment" and (self.token_start != 0 or span == 0 or self.frontier != self.token_end):
            _fail("a segment node owns one segment-local range from token 0")
        if self.execution_state_ref is not None:
            object_ref(self.execution_state_ref, "execution state", kinds=("blob",))
        if self.packet_ref is not None:
            object_ref(self.packet_ref, "node pack")
            if kind != "chunk":
                _fail("only chunk nodes name a node pack (epoch ranges name their own)")

    def binding(self, key: MatrixKey, stream: str | None = None) -> ActiveBasisBinding:
        entry = key if stream is None else (key, stream)
        return dict(self.active_basis).get(entry, ActiveBasisBinding())

    def record_ref(self, key: MatrixKey, stream: str | None = None) -> str | None:
        entry = key if stream is None else (key, stream)
        return dict(self.matrix_records).get(entry)

    def to_dict(self) -> dict[str, Any]:
        return _encode(self, self._JSON, _NODE_V2 if self.streams else _NODE_V1)

    @classmethod
    def from_dict(cls, data: Mapping[str, Any]) -> "ChunkNode":
        schema = data.get("schema") if isinstance(data, Mapping) else None
        node = _decode(cls, data, cls._JSON, "chunk node", schemas=(_NODE_V1, _NODE_V2))
        if (schema == _NODE_V2) != bool(node.streams):
            _fail("chunk node: version 2 (and only version 2) declares CFG streams")
        return node


# -------------------------------------------------------------------------------------------------------------
# Online rank predictor
# -------------------------------------------------------------------------------------------------------------

@dataclass(frozen=True, order=True)
class PredictorKey:
    """The scope of one rank learner: model, layer, K/V, geometry, solver, detector and regime (fresh fits
    and augmentation residuals never share a learner)."""

    model_fingerprint: str
    layer: int
    target: str
    rows: int
    channels: int
    solver: str
    detector: str
    regime: str

    _JSON = tuple(_Key(name) for name in ("model_fingerprint", "layer", "target", "rows", "channels", "solver",
                                          "detector", "regime"))

    def __post_init__(self) -> None:
        _text(self.model_fingerprint, "predictor model")
        MatrixKey(self.layer, self.target)
        _whole(self.rows, "predictor rows")
        _whole(self.channels, "predictor channels")
        _text(self.solver, "predictor solver")
        _text(self.detector, "predictor detector")
        if self.regime not in PREDICTOR_REGIMES:
            _fail(f"predictor regime {self.regime!r} is not one of {PREDICTOR_REGIMES}")

    @property
    def matrix_key(self) -> MatrixKey:
        return MatrixKey(self.layer, self.target)

    @property
    def digest(self) -> str:
        return canonical_digest(self.to_dict())

    def to_dict(self) -> dict[str, Any]:
        return _encode(self, self._JSON)

    @classmethod
    def from_dict(cls, data: Mapping[str, Any]) -> "PredictorKey":
        return _decode(cls, data, cls._JSON, "predictor key")


_RIDGE_SCHEMA = "reelcache.online_ridge_state.v1"


@dataclass(frozen=True)
class OnlineRidgeState:
    """Online ridge regression of ``ln r = a + b x``: the normal matrix ``M`` (stored as ``m00, m01,
    m11``) and the right-hand side ``v``, starting from the prior ``M0 = s I``, ``v0 = M0 (ln m, 1)``."""

    m: tuple[float, float, float]
    v: tuple[float, float]
    observations: int = 0
    revision: int = 0
    anchor_rank: int = RANK_BUCKET
    prior_strength: float = 2.0

    _JSON = (_Key("m", write=list, read=tuple), _Key("v", write=list, read=tuple), _Key("observations"),
             _Key("revision"), _Key("anchor_rank"), _Key("prior_strength"))

    def __post_init__(self) -> None:
        m, v = tuple(self.m), tuple(self.v)
        if (len(m), len(v)) != (3, 2) or not all(_finite(x) for x in m + v):
            _fail("a ridge state has three finite entries of M and two of v")
        object.__setattr__(self, "m", tuple(map(float, m)))
        object.__setattr__(self, "v", tuple(map(float, v)))
        _whole(self.observations, "ridge observations", allow_zero=True)
        _whole(self.revision, "ridge revision", allow_zero=True)
        _whole(self.anchor_rank, "anchor rank")
        if not _finite(self.prior_strength) or self.prior_strength <= 0:
            _fail(f"prior strength {self.prior_strength!r} is not finite and positive")
        object.__setattr__(self, "prior_strength", float(self.prior_strength))
        m00, m01, m11 = self.m
        if not (m00 > 0 and m00 * m11 > m01 * m01):
            _fail("the ridge normal matrix must be positive definite")

    @classmethod
    def initial(cls, anchor_rank: int = RANK_BUCKET, prior_strength: float = 2.0) -> "OnlineRidgeState":
        _whole(anchor_rank, "anchor rank")
        s = float(prior_strength)
        return cls((s, 0.0, s), (s * math.log(anchor_rank), s), 0, 0, anchor_rank, s)

    def coefficients(self) -> tuple[float, float]:
        """``(a, b)``: the 2x2 normal equations solved by Cramer's rule."""
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

    def updated(self, x: float, observed_rank: int | float) -> "OnlineRidgeState":
        """The state after one observation ``(x, ln observed_rank)`` (a rank-one update of M and v)."""
        if not (_finite(x) and _finite(observed_rank) and observed_rank > 0):
            _fail(f"a ridge observation needs finite x and a positive rank, got ({x!r}, {observed_rank!r})")
        x = float(x)
        y = math.log(float(observed_rank))
        m00, m01, m11 = self.m
        v0, v1 = self.v
        return OnlineRidgeState((m00 + 1.0, m01 + x, m11 + x * x), (v0 + y, v1 + x * y), self.observations + 1,
                                self.revision + 1, self.anchor_rank, self.prior_strength)

    @property
    def digest(self) -> str:
        return canonical_digest(self.to_dict())

    def to_dict(self) -> dict[str, Any]:
        return _encode(self, self._JSON, _RIDGE_SCHEMA)

    @classmethod
    def from_dict(cls, data: Mapping[str, Any]) -> "OnlineRidgeState":
        return _decode(cls, data, cls._JSON, "ridge state", schemas=(_RIDGE_SCHEMA,))


_OBSERVATION_SCHEMA = "reelcache.fit_observation.v1"


def _finite_or_none(value):
    return None if value is None or not math.isfinite(value) else value


@dataclass(frozen=True)
class FitObservation:
    """A verified training example of the rank predictor (never a stored KV matrix). ``observation_id`` binds
    the learner scope and the source, so replaying an observation changes nothing. ``origin`` is run context
    and is not written."""

    key: PredictorKey
    source_id: str
    anchor_energy: float
    target_energy: float
    x: float
    observed_rank: int
    predicted_rank: float | None = None
    prediction_revision: int | None = None
    origin: str | None = None

    _JSON = (_Key("key", write=lambda k: k.to_dict(), read=lambda d: PredictorKey.from_dict(d)), _Key("source_id"),
             _Key("anchor_energy"), _Key("target_energy"), _Key("x"), _Key("observed_rank"),
             _Key("predicted_rank", write=_finite_or_none), _Key("prediction_revision"))

    def __post_init__(self) -> None:
        if not isinstance(self.key, PredictorKey):
            _fail("an observation belongs to a PredictorKey")
        if self.origin is not None:
            _digest(self.origin, "observation origin")
        _digest(self.source_id, "observation source")
        anchor = self.anchor_energy
        if not _finite(anchor) or anchor < 0 or anchor >= 1:
            _fail(f"anchor energy {anchor!r} is not in [0, 1)")
        target = _share(self.target_energy, "observation target")
        if target >= 1 or anchor >= target:
            _fail("observations come from anchors below a target below 1")
        if not _finite(self.x) or self.x <= 0:
            _fail(f"observation x {self.x!r} is not finite and positive")
        _whole(self.observed_rank, "observed rank")
        predicted = self.predicted_rank
        if predicted is not None and (isinstance(predicted, bool) or not isinstance(predicted, (int, float))
                                      or predicted != predicted or predicted <= 0):
            _fail(f"predicted rank {predicted!r} is neither positive nor unset")
        if self.prediction_revision is not None:
            _whole(self.prediction_revision, "prediction revision", allow_zero=True)
        object.__setattr__(self, "anchor_energy", float(anchor))
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
        return _encode(self, self._JSON, _OBSERVATION_SCHEMA)

    @classmethod
    def from_dict(cls, data: Mapping[str, Any]) -> "FitObservation":
        return _decode(cls, data, cls._JSON, "fit observation", schemas=(_OBSERVATION_SCHEMA,))
