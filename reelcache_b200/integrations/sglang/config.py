"""``ReelCacheRuntimeConfig``: the serving bridge's frozen, validated configuration (field names,
defaults and the ``reelcache.sglang.runtime_config.v1`` JSON form follow reference
reelcache/integrations/sglang/config.py:544-664 and :947-1014, so existing configuration files and
session identities carry over).

``content_dict()`` is the archive-identifying subset (method, codec, targets) hashed into session
roots; everything else is run configuration. ``to_dict()`` omits the optional fields at their
defaults, as the reference's records do.
"""

from __future__ import annotations

import dataclasses
import math
import os
from dataclasses import dataclass
from typing import Any, Mapping

from ...errors import ConfigurationError

SCHEMA = "reelcache.sglang.runtime_config.v1"
MODES = ("archive_native",)
REPRESENTATIONS = ("raw", "svd_hevc", "svd", "hevc")
LATENTS_ONLY = "latents_only"
RAW_OFFLOAD = "raw_offload"
FIT_DEVICES = ("cuda", "cpu")
DECODERS = ("nvdec_packed", "software")
ROPE_MODES = ("fused", "native")
PIX_FMTS = ("yuv444p", "yuv420p")
NORMALIZATIONS = ("per_channel", "global")
CANVASES = ("canonical", "own_size")
ORTHOGONALIZERS = ("batched", "householder")
DURABILITY = ("pause", "always", "never")
OPEN_ERRORS = ("quarantine", "raise")
MATMUL_PRECISIONS = ("fp32", "fp32_verified_fp64")
RAW_RESTORES = ("prefer", "off")
ENCODERS = ("auto", "x265", "nvenc")
REFIT_RULES = ("cumulative", "paper")
TREE_RETENTIONS = ("head", "full")
TREE_SWITCHES = ("drain", "detach")
RESTORE_MODES = ("archive", "recompute")
STORE_IOS = ("buffered", "nocache")
RAW_TIER_RETAINS = ("drop", "lru")
RAW_TIER_PROMOTES = ("off", "host")
ARCHIVAL_CPUS = ("job", "inherit")
FITTER_STREAMS = ("dedicated", "pooled")
RANK_POLICIES = ("adaptive", "fixed_uniform", "fixed_fraction")
SVD_RANK_FRACTIONS = {"K": 1 / 6, "V": 1 / 4}
GENFIRST_INFLIGHT = ("wait", "overlap")

CONTENT_FIELDS = ("mode", "representation", "profile", "profile_fields", "energy_profile", "energy_key",
                  "energy_value", "predictor_registry_id", "reuse", "refit", "refit_rule", "rate_lag",
                  "hevc_inter_prediction", "hevc_qp", "hevc_pix_fmt", "hevc_preset", "normalization", "orthogonalizer",
                  "canvas", "matmul_precision", "rank_policy", "uniform_rank", "svd_rank_fraction_k",
                  "svd_rank_fraction_v")
# content fields that enter the identity only away from these values (older records stay identical)
LEGACY_CONTENT = {"refit_rule": "paper", "rank_policy": "adaptive", "uniform_rank": None,
                  "svd_rank_fraction_k": None, "svd_rank_fraction_v": None}
# run fields omitted from to_dict at their defaults
_OPTIONAL_AT_DEFAULT = ("tree_switch", "pipelined_restore", "verify_bases", "decoded_tier_bytes", "decoded_tier_route",
                        "decoded_tier_layer_ms", "raw_tier_retain", "raw_tier_promote", "archive_budget_bytes",
                        "defer_archival_during_generation", "archival_defer_backlog_fraction",
                        "archival_defer_max_age_seconds", "archival_defer_inflight", "fitter_green_context_sms",
                        "fitter_green_workqueue", "fitter_cuda_graphs", "fitter_graph_memory_bytes",
                        "fused_fingerprints", "finalize_on_fit_device", "fitter_fp64", "validation_decoder",
                        "hash_once", "seal_prepare_after_publish", "nvenc_device_input", "gil_fastpaths", "native_ext")
_BOOLS = ("reuse", "refit", "hevc_inter_prediction", "verify_reads", "verify_capture_rope", "verify_post_codec",
          "validate_decode", "seal_prepare", "prewarm", "resident_reuse", "observe_plain_requests",
          "defer_archival_during_decode", "decode_entry_guard", "audit_on_open", "staging_engine",
          "archival_pump_pause", "raw_tier", "host_raw_pinned", "overlap_restore", "pipelined_restore", "verify_bases",
          "workload_telemetry", "defer_archival_during_generation", "hash_once", "seal_prepare_after_publish",
          "nvenc_device_input", "gil_fastpaths", "native_ext", "fitter_cuda_graphs", "fused_fingerprints",
          "finalize_on_fit_device")


def available_cpus() -> int:
    try:
        return max(1, len(os.sched_getaffinity(0)))
    except (AttributeError, OSError):
        return max(1, os.cpu_count() or 1)


def derived_encode_workers(cpus: int | None = None) -> int:
    """Default parallel node encodes: one per 8 CPUs, 2 to 4."""
    cpus = available_cpus() if cpus is None else cpus
    return max(2, min(4, cpus // 8))


def derived_x265_threads(encode_workers: int, cpus: int | None = None) -> int:
    """Default encoder threads per node encode: the CPUs split over the workers, 2 to 6 each."""
    cpus = available_cpus() if cpus is None else cpus
    return max(2, min(6, cpus // max(1, encode_workers)))


@dataclass(frozen=True)
class ReelCacheRuntimeConfig:
    store_root: str
    mode: str = "archive_native"
    representation: str = "svd_hevc"
    profile: str | None = None
    profile_fields: Mapping[str, Any] | None = None
    energy_profile: str | None = None
    energy_key: float | None = None
    energy_value: float | None = None
    predictor_registry_id: str = "sglang"
    reuse: bool = True
    refit: bool = True
    refit_rule: str = "paper"
    rate_lag: int = 3
    matmul_precision: str | None = None
    hevc_inter_prediction: bool = False
    hevc_qp: int = 8
    hevc_pix_fmt: str = "yuv444p"
    hevc_preset: str = "ultrafast"
    normalization: str = "per_channel"
    rank_policy: str = "adaptive"
    uniform_rank: int | None = None
    svd_rank_fraction_k: float | None = None
    svd_rank_fraction_v: float | None = None
    x265_threads: int | None = None
    encode_workers: int | None = None
    fit_device: str = "cuda"
    orthogonalizer: str = "batched"
    max_source_chunks: int = 2
    max_unpublished: int = 4
    max_staged_canvases: int | None = None
    submit_timeout: float | None = None
    canvas: str = "canonical"
    validate_decode: bool = True
    validation_decoder: str = "ffmpeg"
    hash_once: bool = False
    seal_prepare_after_publish: bool = False
    nvenc_device_input: bool = False
    gil_fastpaths: bool = False
    native_ext: bool = False
    stream_priority: int | None = None
    fitter_green_context_sms: int | None = None
    fitter_green_workqueue: str | None = None
    fitter_cuda_graphs: bool = False
    fitter_graph_memory_bytes: int | None = None
    fused_fingerprints: bool = False
    finalize_on_fit_device: bool = False
    fitter_fp64: str = "on"
    archival_pump_pause: bool = True
    archival_cpu_priority: Any = None
    raw_tier: bool = True
    gpu_raw_budget_bytes: int | None = None
    gpu_raw_reserve_bytes: int | None = None
    host_raw_budget_bytes: int | None = None
    host_raw_pinned: bool = True
    raw_tier_workers: int | None = None
    raw_restore: str = "prefer"
    raw_tier_retain: str = "drop"
    raw_tier_promote: str = "off"
    archive_budget_bytes: int | None = None
    max_archival_lag_seconds: float | None = None
    encoder: str = "auto"
    durability: str = "pause"
    resident_reuse: bool = True
    tree_retention: str = "head"
    tree_switch: str = "drain"
    restore_mode: str = "archive"
    store_io: str = "buffered"
    decoder: str = "nvdec_packed"
    nvdec_workers: int = 8
    restore_arena_bytes: int = 4 << 30
    basis_budget_bytes: int = 4 << 30
    prepared_budget_bytes: int = 4 << 30
    staging_engine: bool = True
    staging_threads: int | None = None
    staging_prepare_threads: int | None = None
    staging_pinned_bytes: int = 512 << 20
    seal_prepare: bool = True
    prewarm: bool = True
    overlap_restore: bool = True
    pipelined_restore: bool = False
    warmup: bool | None = None
    rope_mode: str = "fused"
    max_store_bytes: int | None = None
    max_resident_bytes: int = 16 << 30
    verify_reads: bool = True
    verify_bases: bool = True
    decoded_tier_bytes: int = 0
    decoded_tier_route: str = "deficit"
    decoded_tier_layer_ms: Any = None
    audit_on_open: bool = False
    on_open_error: str = "quarantine"
    verify_capture_rope: bool = True
    verify_post_codec: bool = False
    observe_plain_requests: bool = False
    workload_telemetry: bool = False
    decode_context_latents: int = 40
    plan_memory_bytes: int | None = None
    defer_archival_during_decode: bool = False
    defer_archival_during_generation: bool = False
    archival_defer_backlog_fraction: float = 0.5
    archival_defer_max_age_seconds: float = 30.0
    archival_defer_inflight: str = "wait"
    decode_entry_guard: bool = True
    decode_reserve_prior_bytes: int | None = None
    decode_working_set_floor_bytes: int | None = None
    cuda_memory_limit_bytes: int | None = None
    archival_cpus: str = "job"
    fitter_stream: str = "dedicated"

    def __post_init__(self) -> None:
        if not isinstance(self.store_root, str) or not self.store_root.strip():
            raise ConfigurationError("store_root must name the archive directory")
        object.__setattr__(self, "store_root", os.path.abspath(os.path.expanduser(self.store_root)))
        enums = (("mode", MODES), ("representation", REPRESENTATIONS + (LATENTS_ONLY, RAW_OFFLOAD)),
                 ("fit_device", FIT_DEVICES), ("decoder", DECODERS), ("rope_mode", ROPE_MODES),
                 ("hevc_pix_fmt", PIX_FMTS), ("normalization", NORMALIZATIONS), ("canvas", CANVASES),
                 ("orthogonalizer", ORTHOGONALIZERS), ("durability", DURABILITY), ("on_open_error", OPEN_ERRORS),
                 ("refit_rule", REFIT_RULES), ("tree_retention", TREE_RETENTIONS), ("tree_switch", TREE_SWITCHES),
                 ("restore_mode", RESTORE_MODES), ("store_io", STORE_IOS), ("raw_restore", RAW_RESTORES),
                 ("raw_tier_retain", RAW_TIER_RETAINS), ("raw_tier_promote", RAW_TIER_PROMOTES),
                 ("encoder", ENCODERS), ("archival_cpus", ARCHIVAL_CPUS), ("fitter_stream", FITTER_STREAMS),
                 ("rank_policy", RANK_POLICIES), ("archival_defer_inflight", GENFIRST_INFLIGHT),
                 ("decoded_tier_route", ("deficit", "all")))
        for name, allowed in enums:
            if getattr(self, name) not in allowed:
                raise ConfigurationError(f"{name} must be one of {allowed}, got {getattr(self, name)!r}")
        for name in _BOOLS:
            if type(getattr(self, name)) is not bool:
                raise ConfigurationError(f"{name} must be a bool")
        if self.warmup is not None and type(self.warmup) is not bool:
            raise ConfigurationError("warmup must be a bool or None (automatic)")
        for name in ("profile", "energy_profile"):
            value = getattr(self, name)
            if value is not None and (not isinstance(value, str) or not value):
                raise ConfigurationError(f"{name} must be a nonempty string or None")
        if self.profile_fields is not None:
            if not isinstance(self.profile_fields, Mapping):
                raise ConfigurationError("profile_fields must be a JSON object or None")
            if self.profile is not None:
                raise ConfigurationError("give either a registered profile name or inline profile_fields")
        if (self.energy_key is None) != (self.energy_value is None):
            raise ConfigurationError("energy_key and energy_value are given together")
        for name in ("energy_key", "energy_value"):
            value = getattr(self, name)
            if value is not None and (isinstance(value, bool) or not isinstance(value, (int, float))
                                      or not math.isfinite(value) or not 0 < value <= 1):
                raise ConfigurationError(f"{name} must be a fraction in (0, 1]")
        if self.energy_key is not None and self.energy_profile is not None:
            raise ConfigurationError("give either an energy profile or explicit energy fractions")
        if self.matmul_precision is not None and self.matmul_precision not in MATMUL_PRECISIONS:
            raise ConfigurationError(f"matmul_precision must be None or one of {MATMUL_PRECISIONS}")
        if not isinstance(self.predictor_registry_id, str) or not self.predictor_registry_id:
            raise ConfigurationError("predictor_registry_id must be a nonempty string")
        for name in ("rate_lag", "max_source_chunks", "max_unpublished", "nvdec_workers", "decode_context_latents"):
            value = getattr(self, name)
            if type(value) is not int or value < 1:
                raise ConfigurationError(f"{name} must be a positive integer")
        for name in ("restore_arena_bytes", "basis_budget_bytes", "prepared_budget_bytes", "staging_pinned_bytes",
                     "max_resident_bytes", "decoded_tier_bytes"):
            value = getattr(self, name)
            if type(value) is not int or value < 0:
                raise ConfigurationError(f"{name} must be a nonnegative byte count")
        for name in ("archival_defer_backlog_fraction", "archival_defer_max_age_seconds"):
            value = getattr(self, name)
            high = 1.0 if name == "archival_defer_backlog_fraction" else math.inf
            if (isinstance(value, bool) or not isinstance(value, (int, float)) or not math.isfinite(value)
                    or not 0 < value <= high):
                raise ConfigurationError(f"{name} must be a positive number")
        if self.hevc_inter_prediction and self.representation == "svd_hevc":
            raise ConfigurationError("inter-coded coefficient streams are not supported by the serving bridge "
                                     "(node packs are all-intra)")
        if self.tree_switch == "detach" and self.tree_retention != "full":
            raise ConfigurationError("tree_switch='detach' needs tree_retention='full'")
        if self.representation == LATENTS_ONLY and self.restore_mode != "recompute":
            raise ConfigurationError("representation='latents_only' stores no KV: it needs restore_mode='recompute'")
        if self.restore_mode == "recompute" and self.representation not in (LATENTS_ONLY, "raw"):
            raise ConfigurationError("restore_mode='recompute' replays from stored clean latents")
        if self.representation == RAW_OFFLOAD and not self.raw_tier:
            raise ConfigurationError("representation='raw_offload' needs raw_tier=true")
        if not self.verify_bases and self.verify_reads:
            raise ConfigurationError("verify_bases=False needs verify_reads=False")
        if self.rank_policy == "fixed_uniform" and (type(self.uniform_rank) is not int or self.uniform_rank < 1):
            raise ConfigurationError("rank_policy='fixed_uniform' needs a positive uniform_rank")
        if self.rank_policy != "fixed_uniform" and self.uniform_rank is not None:
            raise ConfigurationError("uniform_rank belongs to rank_policy='fixed_uniform'")
        if self.rank_policy != "fixed_fraction" and (self.svd_rank_fraction_k is not None
                                                     or self.svd_rank_fraction_v is not None):
            raise ConfigurationError("svd_rank_fraction_* belong to rank_policy='fixed_fraction'")

    # -- derived values -----------------------------------------------------------------------------------------

    def resolved_encode_workers(self) -> int:
        return self.encode_workers if self.encode_workers is not None else derived_encode_workers()

    def resolved_x265_threads(self) -> int:
        if self.x265_threads is not None:
            return self.x265_threads
        return derived_x265_threads(self.resolved_encode_workers())

    def rank_fractions(self) -> dict[str, float]:
        return {"K": self.svd_rank_fraction_k if self.svd_rank_fraction_k is not None else SVD_RANK_FRACTIONS["K"],
                "V": self.svd_rank_fraction_v if self.svd_rank_fraction_v is not None else SVD_RANK_FRACTIONS["V"]}

    # -- JSON -----------------------------------------------------------------------------------------------------

    def to_dict(self) -> dict[str, Any]:
        data = dataclasses.asdict(self)
        if self.profile_fields is not None:
            data["profile_fields"] = dict(self.profile_fields)
        fields = type(self).__dataclass_fields__
        for name in _OPTIONAL_AT_DEFAULT:
            if data.get(name) == fields[name].default:
                del data[name]
        return {"schema": SCHEMA, **data}

    def content_dict(self) -> dict[str, Any]:
        """The archive-identifying subset of :meth:`to_dict`."""
        data = dataclasses.asdict(self)
        if self.profile_fields is not None:
            data["profile_fields"] = dict(self.profile_fields)
        return {"schema": SCHEMA, **{name: data[name] for name in CONTENT_FIELDS
                                     if name not in LEGACY_CONTENT or data[name] != LEGACY_CONTENT[name]}}

    @classmethod
    def from_dict(cls, data: Mapping[str, Any]) -> "ReelCacheRuntimeConfig":
        if not isinstance(data, Mapping):
            raise ConfigurationError("ReelCache runtime configuration must be a JSON object")
        values = dict(data)
        schema = values.pop("schema", SCHEMA)
        if schema != SCHEMA:
            raise ConfigurationError(f"unsupported ReelCache runtime configuration schema {schema!r}")
        known = {f.name for f in dataclasses.fields(cls)}
        unknown = sorted(set(values) - known)
        if unknown:
            raise ConfigurationError(f"unknown ReelCache runtime configuration keys: {unknown}")
        if "store_root" not in values:
            raise ConfigurationError("ReelCache runtime configuration requires store_root")
        return cls(**values)


__all__ = ["ReelCacheRuntimeConfig", "SCHEMA", "CONTENT_FIELDS", "derived_encode_workers", "derived_x265_threads"]
