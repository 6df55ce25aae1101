"""Per-session archival and restore for the serving bridge (the counterpart of reference
reelcache/integrations/sglang/lineage_archive.py:428-1626).

One lineage per session over one content-addressed store. Commits go through the asynchronous
:class:`ArchivePipeline` (rank method on the fit device, node packs, strict in-order publication);
captured sources wait in the :class:`RawChunkTier` until published and stay as an evictable lossless
cache. Restores prefer the raw tier (``raw_restore="prefer"``) and otherwise decode the archive: on a
GPU with the fused sm_100a restore (:class:`LineageRestorer`, layer by layer, overlapped with the
first forward), elsewhere with the reference decode.
"""

from __future__ import annotations

from typing import Any

import torch

from ...archive_pipeline import ArchivePipeline, RawArchive
from ...archive_restore import LineageRestorer, RawLineageRestorer, SoftwareLineageRestorer
from ...factor_packs import FactorLineageRestorer
from ...errors import ConfigurationError
from ...lineage import LineageRuntime
from ...lineage_commit import ArchiveOptions
from ...predictor_registry import RankPredictorRegistry
from ...rank_method import RankMethodConfig
from ...raw_tier import RawChunkTier
from ...store import ObjectStore
from ...types import CodecSpec, EnergyTargets, MatrixKey, ModelIdentity, energy_targets
from .config import LATENTS_ONLY, ReelCacheRuntimeConfig
from .profiles import ModelProfile


def method_for(config: ReelCacheRuntimeConfig, profile: ModelProfile, fit_device) -> RankMethodConfig:
    """The rank method of a session archive: energy targets (profile or explicit), fixed-rank policies, and the
    codec parameters recorded with every lossy matrix (QP, pixel format, preset, normalization)."""
    if config.energy_key is not None:
        targets = EnergyTargets("custom", config.energy_key, config.energy_value, True, "explicit energy fractions")
    else:
        targets = energy_targets(config.energy_profile or profile.energy_profile)
    fixed = {}
    if config.rank_policy == "fixed_uniform":
        fixed = {"fixed_rank_k": config.uniform_rank, "fixed_rank_v": config.uniform_rank}
    elif config.rank_policy == "fixed_fraction":
        fractions = config.rank_fractions()
        fixed = {"fixed_rank_k": max(1, round(fractions["K"] * profile.channels)),
                 "fixed_rank_v": max(1, round(fractions["V"] * profile.channels))}
    kind = "svd" if config.representation == "svd" else "svd_hevc"
    codec = CodecSpec(kind, 32, normalization=config.normalization, pix_fmt=config.hevc_pix_fmt, qp=config.hevc_qp,
                      preset=config.hevc_preset)
    return RankMethodConfig(targets, codec, reuse=config.reuse, refit=config.refit, refit_rule=config.refit_rule,
                            rate_lag=config.rate_lag, matmul_precision=config.matmul_precision or "fp32",
                            orthogonalizer=config.orthogonalizer, **fixed)


class LineageSessionArchive:
    """Every session's lineage in one store, with its archival pipeline, raw tier and restorer, built from the
    runtime configuration (each field is consumed here, in the bridge or in the session controller)."""

    def __init__(self, config: ReelCacheRuntimeConfig, identity: ModelIdentity, profile: ModelProfile, device):
        import os

        self.config = config
        self.profile = profile
        self.device = torch.device(device)
        cuda = self.device.type == "cuda"
        self.store = ObjectStore(config.store_root, max_bytes=config.max_store_bytes, verify_reads=config.verify_reads,
                                 on_damage="keep" if config.on_open_error == "quarantine" else "raise")
        self.store.set_io_policy(config.store_io)
        self.audit = self._audit() if config.audit_on_open else None
        self.registry = RankPredictorRegistry(config.predictor_registry_id)
        self.runtime = LineageRuntime(self.store, identity, registry=self.registry)
        self.runtime.basis.verify_blocks = config.verify_bases
        fit_device = self.device if config.fit_device == "cuda" and cuda else torch.device("cpu")
        self.method = method_for(config, profile, fit_device)
        self.raw_tier = None
        if config.raw_tier:
            gpu = config.gpu_raw_budget_bytes
            if gpu is None:
                gpu = (4 << 30) if cuda else (256 << 20)
            self.raw_tier = RawChunkTier(self.device, gpu_budget_bytes=gpu, host_budget_bytes=config.host_raw_budget_bytes,
                                         host_pinned=config.host_raw_pinned, retain=config.raw_tier_retain,
                                         promote=config.raw_tier_promote, reserve_bytes=config.gpu_raw_reserve_bytes)
        self.eviction = None
        if config.archive_budget_bytes is not None:
            from .archive_eviction import ArchiveEviction
            self.eviction = ArchiveEviction(self.store, config.archive_budget_bytes)
        representation = config.representation
        if representation in ("raw", "raw_offload", LATENTS_ONLY):
            self.pipeline = RawArchive(self.runtime, raw_tier=self.raw_tier,
                                       write_behind=representation == "raw_offload",
                                       max_unwritten=config.max_unpublished,
                                       kv_objects=representation != LATENTS_ONLY)
        else:
            options = ArchiveOptions(encode_threads=config.resolved_x265_threads(),
                                     plan_memory_bytes=config.plan_memory_bytes)
            cpus = set(os.sched_getaffinity(0)) if (config.archival_cpus == "job" and hasattr(os, "sched_getaffinity")) \
                else None
            self.pipeline = ArchivePipeline(self.runtime, method=self.method, device=fit_device, options=options,
                                            raw_tier=self.raw_tier, max_unpublished=config.max_unpublished,
                                            submit_timeout=config.submit_timeout,
                                            encode_workers=config.resolved_encode_workers(), registry=self.registry,
                                            max_source_chunks=config.max_source_chunks,
                                            stream_priority=config.stream_priority,
                                            dedicated_stream=config.fitter_stream == "dedicated", encode_cpus=cpus,
                                            on_publish=self._published)
        self.restorer = None
        if cuda:
            if representation in ("raw", "raw_offload"):
                self.restorer = RawLineageRestorer(self.runtime, self.device)
            elif representation == "svd":
                self.restorer = FactorLineageRestorer(self.runtime, self.device)
            elif representation == "svd_hevc" and config.decoder == "software":
                self.restorer = SoftwareLineageRestorer(self.runtime, self.device)
            elif representation == "svd_hevc":
                staging = None
                if config.staging_engine:
                    from ...restore_staging import StagingEngine
                    staging = StagingEngine(self.store, pinned_bytes=config.staging_pinned_bytes,
                                            threads=config.staging_threads or 8)
                self.restorer = LineageRestorer(self.runtime, self.device,
                                                prepared_budget_bytes=config.prepared_budget_bytes,
                                                basis_budget_bytes=config.basis_budget_bytes,
                                                plan_budget_bytes=config.restore_arena_bytes, staging=staging,
                                                verify_packs=config.validate_decode)
            if config.warmup or (config.warmup is None and self.restorer is not None):
                self._warm_kernels()
        self.stats_ = {"raw_installs": 0, "archive_installs": 0, "commits": 0, "prepared_on_publish": 0}

    def _audit(self) -> dict:
        """Hash every object every ref reaches (``audit_on_open``); damaged graphs are quarantined."""
        damaged = {}
        for name, ref in self.store.list_refs().items():
            try:
                self.store.verify(ref)
            except Exception as exc:  # noqa: BLE001 - recorded per ref; on_open_error decides below
                damaged[name] = str(exc)
        if damaged and self.config.on_open_error == "raise":
            raise ConfigurationError(f"store audit found damaged refs: {sorted(damaged)[:5]}")
        return {"refs": len(self.store.list_refs()), "damaged": damaged}

    def _warm_kernels(self) -> None:
        from ...restore_kernels import WarmupShape, warmup
        p = self.profile
        warmup(self.device, [WarmupShape(p.num_heads, p.head_dim)])

    def _published(self, lineage: str, node_ref: str) -> None:
        """After a node is published: account its payloads under the archive budget, and (``seal_prepare``)
        decode its pack into the restorer's prepared cache so a later restore skips that work."""
        node = self.runtime.load_node(node_ref)
        if self.eviction is not None and node.packet_ref is not None:
            payloads = frozenset(r for r in self.store.references(node.packet_ref) if r.startswith("blob:"))
            self.eviction.published(node_ref, payloads)
        if self.config.seal_prepare and isinstance(self.restorer, LineageRestorer) and node.packet_ref is not None:
            self.restorer.prepared_pack(node.packet_ref)
            self.stats_["prepared_on_publish"] += 1

    # -- lineages -------------------------------------------------------------------------------------------------

    def create(self, session_id: str) -> str:
        self.runtime.create_lineage(session_id)
        return self.runtime.lineage_head(session_id)

    def exists(self, session_id: str) -> bool:
        return ("lineages/" + session_id) in self.store.list_refs("lineages/")

    def head(self, session_id: str) -> str:
        return self.runtime.lineage_head(session_id)

    def fork(self, node_ref: str, session_id: str) -> None:
        self.runtime.fork_lineage(node_ref, session_id)

    def rewind(self, session_id: str, node_ref: str) -> None:
        self.pipeline.drain(session_id)
        self.runtime.rewind_lineage(session_id, node_ref)

    def delete(self, session_id: str) -> None:
        self.pipeline.forget(session_id)
        self.runtime.delete_lineage(session_id)
        if self.raw_tier is not None:
            self.raw_tier.release_holder(session_id, drop=True)

    def commit_chunk(self, session_id: str, chunk_id: str, matrices, contexts, *, execution_state=None,
                     capture_event=None):
        self.stats_["commits"] += 1
        return self.pipeline.submit(session_id, chunk_id, matrices, contexts, execution_state=execution_state,
                                    capture_event=capture_event, holder=session_id)

    def commit_recache(self, session_id: str, recache_id: str, ranges, *, epoch_id: str, details=None,
                       execution_state=None) -> str:
        """Publish a prompt switch's ``kv_recache`` epoch after the session's submitted chunks; returns its node."""
        self.stats_["recaches"] = self.stats_.get("recaches", 0) + 1
        return self.pipeline.commit_recache(session_id, recache_id, ranges, epoch_id=epoch_id, details=details,
                                            execution_state=execution_state, holder=session_id)

    def drain(self, session_id: str | None = None, timeout: float | None = None) -> float:
        return self.pipeline.drain(session_id, timeout)

    # -- restore --------------------------------------------------------------------------------------------------

    def _raw_span(self, node_ref: str, key: MatrixKey, offset: int, length: int):
        if self.raw_tier is None or self.config.raw_restore != "prefer":
            return None
        lease = self.raw_tier.lookup(node_ref)
        if lease is None:
            return None
        try:
            tensor = lease.tensors.get(key)
            return None if tensor is None else tensor[offset:offset + length].clone()
        finally:
            lease.release()

    def install_dense(self, cache: dict, head_ref: str, plan, layers: int) -> dict:
        """Dense pre-RoPE history into a synthetic engine's cache: raw tier first, then the archive."""
        raw = archive = 0
        for layer in range(layers):
            for target, rows in (("K", cache["k"][layer]), ("V", cache["v"][layer])):
                key = MatrixKey(layer, target)
                for span in plan.spans:
                    piece = self._raw_span(span.node_ref, key, span.node_offset, span.length)
                    if piece is None:
                        piece = self.runtime.acquire_node_history(
                            head_ref, key, ranges=[(span.token_start, span.token_start + span.length)],
                            device=rows.device, dtype=rows.dtype)
                        archive += 1
                    else:
                        raw += 1
                    rows[span.slot_start:span.slot_start + span.length] = piece.to(rows.dtype)
        cache["end"] = plan.spans[-1].slot_start + plan.spans[-1].length if plan.spans else 0
        self.stats_["raw_installs"] += raw
        self.stats_["archive_installs"] += archive
        return {"raw_spans": raw, "archive_spans": archive, "attended_tokens": plan.attended_tokens}

    def restore_into(self, head_ref: str, install, plan, *, overlapped: bool = True):
        """Install the plan's history into native caches (GPU): spans whose nodes the raw tier still holds go
        through the dense RoPE-and-store kernel (exact captured rows), the rest through the fused sm_100a
        restorer (``install`` is a :class:`~.restore.LineageInstall`). Returns a restore result whose
        readiness covers both sources; ``result.lease`` owns the raw-tier pins until the install completes."""
        from ...archive_restore import RestoreResult
        from ...overlapped_restore import LayerReadiness
        from .restore import AttentionKVLease, restore_dense
        from .visibility import VisibilityPlan
        if self.restorer is None:
            raise ConfigurationError("the fused restore needs a CUDA device")
        lease = AttentionKVLease(description={"head": head_ref, "attended_tokens": plan.attended_tokens})
        raw_spans, archive_spans, leases = [], [], {}
        for span in plan.spans:
            raw = None
            if self.raw_tier is not None and self.config.raw_restore == "prefer":
                raw = leases.get(span.node_ref) or self.raw_tier.lookup(span.node_ref)
            if raw is not None:
                if span.node_ref not in leases:
                    leases[span.node_ref] = raw
                    lease.track(finalizer=raw.release)
                raw_spans.append(span)
            else:
                archive_spans.append(span)
        sources = (("restore",) if archive_spans else ()) + (("raw",) if raw_spans else ())
        layers = self.profile.num_layers
        readiness = LayerReadiness(layers, sources=sources or ("restore",))
        stream = torch.cuda.Stream(self.device)
        result = None
        if raw_spans:
            sub = VisibilityPlan(plan.next_chunk, tuple(raw_spans))
            restore_dense(lease, plan=sub, destination=install.destination,
                          rope=lambda span: (install.table, install._rope_rows(span.chunk_index)),
                          rows_of=lambda span, key: leases[span.node_ref].tensors[key][
                              span.node_offset:span.node_offset + span.length],
                          grid=self.profile.grid, layers=layers, stream=stream, readiness=readiness)
            self.stats_["raw_installs"] += len(raw_spans)
        if archive_spans:
            sub = VisibilityPlan(plan.next_chunk, tuple(archive_spans))
            archive_install = type(install)(plan=sub, destination=install.destination, rope_rows=install._rope_rows,
                                            table=install.table, tokens_per_frame=install.tokens_per_frame)
            result = archive_install.restore(self.restorer, head_ref, overlapped=overlapped, thread=overlapped,
                                             readiness=readiness, stream=stream)
            result.lease = lease
            self.stats_["archive_installs"] += len(archive_spans)
        if result is None:
            result = RestoreResult(head_ref, readiness, None, {"raw_spans": len(raw_spans)})
            result.lease = lease
        result.stats["raw_spans"] = len(raw_spans)
        result.stats["archive_spans"] = len(archive_spans)
        return result

    # -- lifecycle ------------------------------------------------------------------------------------------------

    def gc(self) -> dict:
        self.drain()
        return self.store.collect_garbage()

    def stats(self) -> dict[str, Any]:
        return {**self.stats_, "pipeline": self.pipeline.stats(),
                "raw_tier": None if self.raw_tier is None else self.raw_tier.stats(),
                "restorer": None if self.restorer is None else self.restorer.stats()}

    def close(self) -> None:
        self.pipeline.close(drain=True)
        if self.raw_tier is not None:
            self.raw_tier.close()
        self.store.close()
