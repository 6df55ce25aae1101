"""``ReelCacheRuntimeConfig``: the frozen, validated configuration of the serving bridge.

Field names, defaults and the ``reelcache.sglang.runtime_config.v1`` JSON form are the reference's
(reelcache/integrations/sglang/config.py:544-664), so configuration files and the session identities hashed
from them carry over. How the fields are checked is this module's own: every field has one entry in
:data:`FIELDS` (its check, whether it identifies archived content, whether ``to_dict`` leaves it out at its
default) and cross-field rules are listed in :data:`_RULES`.

No field is accepted and then ignored. A field is either honored by the bridge (:mod:`.lineage_archive`,
:mod:`.bridge`, :mod:`.session`), or it has a ``pinned`` reason: then only its default is accepted and any
other value raises :class:`~reelcache_b200.errors.ConfigurationError` naming that reason (for example an
NVENC/NVDEC engine or CPU green contexts this build does not have). The host "levers" of the reference
(``hash_once``, ``gil_fastpaths``, ``native_ext``, ``fused_fingerprints``, ``finalize_on_fit_device``,
``seal_prepare_after_publish``) switch between byte-identical code paths; this build always runs the fast
path, so both values are accepted and documented as such in :data:`LEVERS_ALWAYS_ON` (``pipelined_restore``
too: an overlapped restore always uploads each layer's packs just ahead of that layer's kernels).
"""

from __future__ import annotations

import dataclasses
import math
import os
from dataclasses import dataclass
from typing import Any, Callable, Mapping

from ...errors import ConfigurationError

SCHEMA = "reelcache.sglang.runtime_config.v1"
LATENTS_ONLY = "latents_only"
RAW_OFFLOAD = "raw_offload"
SVD_RANK_FRACTIONS = {"K": 1 / 6, "V": 1 / 4}
#: levers whose effect this build has built in (both values accepted; outputs are byte-identical either way)
LEVERS_ALWAYS_ON = ("hash_once", "seal_prepare_after_publish", "gil_fastpaths", "native_ext", "fused_fingerprints",
                    "finalize_on_fit_device", "pipelined_restore")


def available_cpus() -> int:
    try:
        return max(1, len(os.sched_getaffinity(0)))
    except (AttributeError, OSError):
        return max(1, os.cpu_count() or 1)


def derived_encode_workers(cpus: int | None = None) -> int:
    """Parallel node encodes by default: one per 8 CPUs, at least 2 and at most 4."""
    n = available_cpus() if cpus is None else cpus
    return min(4, max(2, n // 8))


def derived_x265_threads(encode_workers: int, cpus: int | None = None) -> int:
    """Encoder threads per node encode by default: the CPUs shared by the workers, 2 to 6 each."""
    n = available_cpus() if cpus is None else cpus
    return min(6, max(2, n // max(1, encode_workers)))


# -------------------------------------------------------------------------------------------------------------
# Checks
# -------------------------------------------------------------------------------------------------------------

Check = Callable[[str, Any], None]


def _choice(*allowed) -> Check:
    def check(name, value):
        if value not in allowed:
            raise ConfigurationError(f"{name}: {value!r} is not one of {allowed}")
    return check


def _flag(name, value):
    if type(value) is not bool:
        raise ConfigurationError(f"{name}: expected true or false, got {value!r}")


def _count(minimum: int) -> Check:
    def check(name, value):
        if type(value) is not int or value < minimum:
            raise ConfigurationError(f"{name}: expected an integer >= {minimum}, got {value!r}")
    return check


def _number(low: float, high: float, *, include_low: bool = False) -> Check:
    def check(name, value):
        ok = isinstance(value, (int, float)) and not isinstance(value, bool) and math.isfinite(value)
        if not ok or value > high or value < low or (value == low and not include_low):
            raise ConfigurationError(f"{name}: expected a number in {'[' if include_low else '('}{low}, {high}], "
                                     f"got {value!r}")
    return check


def _text(name, value):
    if not isinstance(value, str) or not value.strip():
        raise ConfigurationError(f"{name}: expected a nonempty string, got {value!r}")


def _mapping(name, value):
    if not isinstance(value, Mapping):
        raise ConfigurationError(f"{name}: expected a JSON object")


def _anything(name, value):
    return None


def _integer(name, value):
    if type(value) is not int:
        raise ConfigurationError(f"{name}: expected an integer, got {value!r}")


def _qp(name, value):
    if type(value) is not int or not 0 <= value <= 51:
        raise ConfigurationError(f"{name}: expected an integer in [0, 51], got {value!r}")


def _optional(check: Check) -> Check:
    def wrapped(name, value):
        if value is not None:
            check(name, value)
    return wrapped


@dataclass(frozen=True)
class Field:
    """How one configuration field is checked and recorded. ``pinned``: the field is not implemented by this
    build -- only its default is accepted, and the reason is part of the error for any other value."""

    check: Check
    content: bool = False
    omit_at_default: bool = False
    pinned: str | None = None


_NO_NVCODEC = "B200 has no NVENC/NVDEC engine and this build has no Video Codec SDK binding"
_NOT_BUILT = "not implemented by this build"

FIELDS: dict[str, Field] = {
    # method
    "store_root": Field(_text),
    "mode": Field(_choice("archive_native"), content=True),
    "representation": Field(_choice("raw", "svd_hevc", "svd", "hevc", LATENTS_ONLY, RAW_OFFLOAD), content=True),
    "profile": Field(_optional(_text), content=True),
    "profile_fields": Field(_optional(_mapping), content=True),
    "energy_profile": Field(_optional(_text), content=True),
    "energy_key": Field(_optional(_number(0.0, 1.0)), content=True),
    "energy_value": Field(_optional(_number(0.0, 1.0)), content=True),
    "predictor_registry_id": Field(_text, content=True),
    "reuse": Field(_flag, content=True),
    "refit": Field(_flag, content=True),
    "refit_rule": Field(_choice("cumulative", "paper"), content=True),
    "rate_lag": Field(_count(1), content=True),
    "matmul_precision": Field(_optional(_choice("fp32", "fp32_verified_fp64")), content=True),
    # codec
    "hevc_inter_prediction": Field(_flag, content=True),
    "hevc_qp": Field(_qp, content=True),
    "hevc_pix_fmt": Field(_choice("yuv444p", "yuv420p"), content=True),
    "hevc_preset": Field(_text, content=True),
    "normalization": Field(_choice("per_channel", "global"), content=True),
    "rank_policy": Field(_choice("adaptive", "fixed_uniform", "fixed_fraction"), content=True),
    "uniform_rank": Field(_optional(_count(1)), content=True),
    "svd_rank_fraction_k": Field(_optional(_number(0.0, 1.0)), content=True),
    "svd_rank_fraction_v": Field(_optional(_number(0.0, 1.0)), content=True),
    "x265_threads": Field(_optional(_count(1))),
    "encode_workers": Field(_optional(_count(1))),
    # fitter
    "fit_device": Field(_choice("cuda", "cpu")),
    "orthogonalizer": Field(_choice("batched", "householder"), content=True),
    "max_source_chunks": Field(_count(1)),
    "max_unpublished": Field(_count(1)),
    "max_staged_canvases": Field(_optional(_count(1)),
                                 pinned="canvases are staged inside each node's commit, not in a shared queue"),
    "submit_timeout": Field(_optional(_number(0.0, math.inf))),
    "canvas": Field(_choice("canonical", "own_size"), content=True),
    "validate_decode": Field(_flag),
    "validation_decoder": Field(_choice("ffmpeg", "nvdec"), omit_at_default=True, pinned=_NO_NVCODEC),
    # levers
    "hash_once": Field(_flag, omit_at_default=True),
    "seal_prepare_after_publish": Field(_flag, omit_at_default=True),
    "nvenc_device_input": Field(_flag, omit_at_default=True, pinned=_NO_NVCODEC),
    "gil_fastpaths": Field(_flag, omit_at_default=True),
    "native_ext": Field(_flag, omit_at_default=True),
    "stream_priority": Field(_optional(_integer)),
    "fitter_green_context_sms": Field(_optional(_count(1)), omit_at_default=True,
                                      pinned="green contexts are " + _NOT_BUILT),
    "fitter_green_workqueue": Field(_optional(_text), omit_at_default=True, pinned="green contexts are " + _NOT_BUILT),
    "fitter_cuda_graphs": Field(_flag, omit_at_default=True,
                                pinned="CUDA-graph replay of the fitter's FP64 passes is not built (the reference "
                                       "documents it as harmful)"),
    "fitter_graph_memory_bytes": Field(_optional(_count(0)), omit_at_default=True,
                                       pinned="CUDA-graph replay of the fitter is not built"),
    "fused_fingerprints": Field(_flag, omit_at_default=True),
    "finalize_on_fit_device": Field(_flag, omit_at_default=True),
    "fitter_fp64": Field(_choice("on", "off"), omit_at_default=True,
                         pinned="the planner's FP64 passes run on the FP32-accurate tensor-core path; the FP32 "
                                "replacements are not selectable"),
    "archival_pump_pause": Field(_flag),
    "archival_cpu_priority": Field(_anything, pinned="encode-thread CPU priorities are " + _NOT_BUILT),
    # tiers
    "raw_tier": Field(_flag),
    "gpu_raw_budget_bytes": Field(_optional(_count(0))),
    "gpu_raw_reserve_bytes": Field(_optional(_count(0))),
    "host_raw_budget_bytes": Field(_optional(_count(0))),
    "host_raw_pinned": Field(_flag),
    "raw_tier_workers": Field(_optional(_count(1)), pinned="raw-tier copies run on one side stream; a worker "
                                                           "count is " + _NOT_BUILT),
    "raw_restore": Field(_choice("prefer", "off")),
    "raw_tier_retain": Field(_choice("drop", "lru"), omit_at_default=True),
    "raw_tier_promote": Field(_choice("off", "host"), omit_at_default=True),
    "archive_budget_bytes": Field(_optional(_count(1)), omit_at_default=True),
    "max_archival_lag_seconds": Field(_optional(_number(0.0, math.inf)),
                                      pinned="age-based archival backpressure is " + _NOT_BUILT),
    "encoder": Field(_choice("auto", "x265", "nvenc"),
                     pinned="node packs are written with the 8-bit stream codec (raw8): no HEVC encoder is wired "
                            "(no NVENC on B200, no FFmpeg/libx265 on these machines)"),
    # store and sessions
    "durability": Field(_choice("pause", "always", "never")),
    "resident_reuse": Field(_flag),
    "tree_retention": Field(_choice("head", "full")),
    "tree_switch": Field(_choice("drain", "detach"), omit_at_default=True),
    "restore_mode": Field(_choice("archive", "recompute")),
    "store_io": Field(_choice("buffered", "nocache")),
    # restore
    "decoder": Field(_choice("nvdec_packed", "software")),
    "nvdec_workers": Field(_count(1), pinned=_NO_NVCODEC),
    "restore_arena_bytes": Field(_count(0)),
    "basis_budget_bytes": Field(_count(0)),
    "prepared_budget_bytes": Field(_count(0)),
    "staging_engine": Field(_flag),
    "staging_threads": Field(_optional(_count(1))),
    "staging_prepare_threads": Field(_optional(_count(1)),
                                     pinned="preparation runs on the staging threads; a separate pool is "
                                            + _NOT_BUILT),
    "staging_pinned_bytes": Field(_count(0)),
    "seal_prepare": Field(_flag),
    "prewarm": Field(_flag),
    "overlap_restore": Field(_flag),
    "pipelined_restore": Field(_flag, omit_at_default=True),
    "warmup": Field(_optional(_flag)),
    "rope_mode": Field(_choice("fused", "native"), pinned="RoPE is applied in the restore kernel's epilogue"),
    "max_store_bytes": Field(_optional(_count(0))),
    "max_resident_bytes": Field(_count(0)),
    "verify_reads": Field(_flag),
    "verify_bases": Field(_flag, omit_at_default=True),
    "decoded_tier_bytes": Field(_count(0), omit_at_default=True,
                                pinned="restores read 8-bit coefficients straight from the prepared packs; a separate "
                                       "decoded-picture tier is not wired into the bridge"),
    "decoded_tier_route": Field(_choice("deficit", "all"), omit_at_default=True,
                                pinned="the decoded-picture tier is not wired into the bridge"),
    "decoded_tier_layer_ms": Field(_anything, omit_at_default=True,
                                   pinned="the decoded tier's per-layer compute model is not configurable here"),
    "audit_on_open": Field(_flag),
    "on_open_error": Field(_choice("quarantine", "raise")),
    "verify_capture_rope": Field(_flag),
    "verify_post_codec": Field(_flag, pinned="post-codec error measurement at commit is " + _NOT_BUILT),
    # scheduling and diagnostics
    "observe_plain_requests": Field(_flag),
    "workload_telemetry": Field(_flag),
    "decode_context_latents": Field(_count(1), pinned="VAE decode context is the engine's, not configurable here"),
    "plan_memory_bytes": Field(_optional(_count(1))),
    "defer_archival_during_decode": Field(_flag),
    "defer_archival_during_generation": Field(_flag, omit_at_default=True),
    "archival_defer_backlog_fraction": Field(_number(0.0, 1.0), omit_at_default=True),
    "archival_defer_max_age_seconds": Field(_number(0.0, math.inf), omit_at_default=True),
    "archival_defer_inflight": Field(_choice("wait", "overlap"), omit_at_default=True),
    "decode_entry_guard": Field(_flag),
    "decode_reserve_prior_bytes": Field(_optional(_count(0))),
    "decode_working_set_floor_bytes": Field(_optional(_count(0))),
    "cuda_memory_limit_bytes": Field(_optional(_count(1))),
    "archival_cpus": Field(_choice("job", "inherit")),
    "fitter_stream": Field(_choice("dedicated", "pooled")),
}
# content fields that enter the session identity only away from these values (older records stay identical)
LEGACY_CONTENT = {"refit_rule": "paper", "rank_policy": "adaptive", "uniform_rank": None,
                  "svd_rank_fraction_k": None, "svd_rank_fraction_v": None}
CONTENT_FIELDS = tuple(name for name, spec in FIELDS.items() if spec.content)


# -------------------------------------------------------------------------------------------------------------
# Cross-field rules: (condition that is an error, message)
# -------------------------------------------------------------------------------------------------------------

_RULES: tuple[tuple[Callable[[Any], bool], str], ...] = (
    (lambda c: c.profile is not None and c.profile_fields is not None,
     "name a registered profile or give inline profile_fields, not both"),
    (lambda c: (c.energy_key is None) != (c.energy_value is None), "energy_key and energy_value come together"),
    (lambda c: c.energy_key is not None and c.energy_profile is not None,
     "give an energy profile or explicit energy fractions, not both"),
    (lambda c: c.hevc_inter_prediction and c.representation == "svd_hevc",
     "node packs are all-intra: inter-predicted coefficient streams are not supported"),
    (lambda c: c.representation == "hevc",
     "representation='hevc' (full-rank coded KV) is " + _NOT_BUILT + "; use svd_hevc, svd, raw or raw_offload"),
    (lambda c: c.encoder == "nvenc", "encoder='nvenc': " + _NO_NVCODEC),
    (lambda c: c.representation == LATENTS_ONLY and c.restore_mode != "recompute",
     "representation='latents_only' stores no KV and needs restore_mode='recompute'"),
    (lambda c: c.restore_mode == "recompute" and c.representation not in (LATENTS_ONLY, "raw"),
     "restore_mode='recompute' replays stored clean latents: representation must be 'raw' or 'latents_only'"),
    (lambda c: c.representation == RAW_OFFLOAD and not c.raw_tier, "representation='raw_offload' needs raw_tier"),
    (lambda c: c.verify_reads and not c.verify_bases, "verify_bases=false needs verify_reads=false"),
    (lambda c: c.rank_policy == "fixed_uniform" and c.uniform_rank is None,
     "rank_policy='fixed_uniform' needs uniform_rank"),
    (lambda c: c.rank_policy != "fixed_uniform" and c.uniform_rank is not None,
     "uniform_rank belongs to rank_policy='fixed_uniform'"),
    (lambda c: c.rank_policy != "fixed_fraction" and (c.svd_rank_fraction_k, c.svd_rank_fraction_v) != (None, None),
     "svd_rank_fraction_k/_v belong to rank_policy='fixed_fraction'"),
    (lambda c: c.pipelined_restore and not c.overlap_restore,
     "pipelined_restore splits an overlapped restore into per-layer uploads: it needs overlap_restore"),
)


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
        defaults = {f.name: f.default for f in dataclasses.fields(self)}
        for name, spec in FIELDS.items():
            value = getattr(self, name)
            spec.check(name, value)
            if spec.pinned is not None and value != defaults.get(name):
                raise ConfigurationError(f"{name}={value!r} is not available: {spec.pinned}")
        if set(FIELDS) != set(defaults):
            raise ConfigurationError("the configuration table and the dataclass fields differ")
        object.__setattr__(self, "store_root", os.path.abspath(os.path.expanduser(self.store_root)))
        for broken, message in _RULES:
            if broken(self):
                raise ConfigurationError(message)

    # -- derived values -----------------------------------------------------------------------------------------

    def resolved_encode_workers(self) -> int:
        return self.encode_workers if self.encode_workers is not None else derived_encode_workers()

    def resolved_x265_threads(self) -> int:
        return self.x265_threads if self.x265_threads is not None else \
            derived_x265_threads(self.resolved_encode_workers())

    def rank_fractions(self) -> dict[str, float]:
        chosen = {"K": self.svd_rank_fraction_k, "V": self.svd_rank_fraction_v}
        return {t: SVD_RANK_FRACTIONS[t] if v is None else v for t, v in chosen.items()}

    # -- JSON ---------------------------------------------------------------------------------------------------

    def _plain(self) -> dict[str, Any]:
        data = dataclasses.asdict(self)
        if self.profile_fields is not None:
            data["profile_fields"] = dict(self.profile_fields)
        return data

    def to_dict(self) -> dict[str, Any]:
        data = self._plain()
        defaults = {f.name: f.default for f in dataclasses.fields(self)}
        kept = {k: v for k, v in data.items() if not (FIELDS[k].omit_at_default and v == defaults[k])}
        return {"schema": SCHEMA, **kept}

    def content_dict(self) -> dict[str, Any]:
        """The fields that identify archived content (hashed into session roots)."""
        data = self._plain()
        chosen = {k: data[k] for k in CONTENT_FIELDS if k not in LEGACY_CONTENT or data[k] != LEGACY_CONTENT[k]}
        return {"schema": SCHEMA, **chosen}

    @classmethod
    def from_dict(cls, data: Mapping[str, Any]) -> "ReelCacheRuntimeConfig":
        if not isinstance(data, Mapping):
            raise ConfigurationError("a runtime configuration is a JSON object")
        values = dict(data)
        schema = values.pop("schema", SCHEMA)
        if schema != SCHEMA:
            raise ConfigurationError(f"configuration schema {schema!r} is not {SCHEMA}")
        unknown = sorted(set(values) - set(FIELDS))
        if unknown:
            raise ConfigurationError(f"unknown configuration keys {unknown}")
        if "store_root" not in values:
            raise ConfigurationError("a runtime configuration names store_root")
        return cls(**values)


__all__ = ["CONTENT_FIELDS", "FIELDS", "LEVERS_ALWAYS_ON", "SCHEMA", "Field", "ReelCacheRuntimeConfig",
           "derived_encode_workers", "derived_x265_threads"]
