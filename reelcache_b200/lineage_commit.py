"""Staged commit of one lineage node (reference: reelcache/lineage_commit.py:124-989).

A :class:`CommitJob` is one node's archival work, split into stages that the archive pipeline can run
on different threads:

``plan``      the rank method on the planning device (share / augment / refit / fresh per matrix);
``finalize``  device quantization of every coefficient tile (per-column covering FP32 affine, FP64
              ``rint``) -- only uint8 tiles and affines cross PCIe;
``encode``    one node pack (``reelcache.tensor_pack.v2``) of all tiles;
``store``     basis versions, pack blobs/manifest, matrix records, execution state -- staged under a
              store lease so a crash before publication leaves only collectable garbage;
``build_node`` the immutable :class:`~reelcache_b200.types.ChunkNode` manifest.

Publication (CAS of the lineage head) and registry training happen in
:meth:`reelcache_b200.lineage.LineageRuntime.publish_job`.
"""

from __future__ import annotations

import hashlib
import time
from dataclasses import dataclass, field
from typing import Any, Mapping, Sequence

import numpy as np
import torch

from . import codecs
from .errors import ConfigurationError, IntegrityError
from .rank_method import MatrixPlan, RankMethodConfig, plan_chunk
from .serialization import serialize_tensors
from .types import (ActiveBasisBinding, CodecSpec, EnergyReport, FitObservation, MatrixKey, MatrixRecord,
                    TensorContext, canonical_digest, entry_order, entry_parts, json_copy)

_FINGERPRINT_PRIME = (1 << 61) - 1


@dataclass(frozen=True)
class ArchiveOptions:
    """Archival path options (reference :124): node packing, the coefficient stream codec, tile rows of
    the planner's verification, the planning memory budget and encode threads."""

    packed: bool = True
    stream_codec: str = "raw8"
    tile_rows: int = 4096
    plan_memory_bytes: int | None = None
    encode_threads: int = 1
    finalize_on_device: bool = True

    def __post_init__(self):
        if self.stream_codec not in codecs.STREAM_CODECS:
            raise ConfigurationError(f"stream_codec must be one of {codecs.STREAM_CODECS}")


FINGERPRINT_PRIME = 2147483629
#: Elements per fingerprint row tile of the host path (int64 temporaries cover one tile, not the matrix).
FINGERPRINT_TILE_ELEMENTS = 1 << 24
#: (column multiplier, row multiplier, square) of the three checksums of each 16-bit part.
FINGERPRINT_COMBINATIONS = ((37, 101, False), (613, 211, False), (1, 17, True))


def _fingerprint_terms_host(source: torch.Tensor) -> torch.Tensor:
    rows, columns = source.shape
    wide = source.element_size() == 4
    column = torch.arange(columns, dtype=torch.int64)
    weights = [(column * a + 7) % 1021 + 1 for a, _, _ in FINGERPRINT_COMBINATIONS]
    totals = torch.zeros(6 if wide else 3, dtype=torch.int64)
    tile_rows = max(1, FINGERPRINT_TILE_ELEMENTS // columns)
    for start in range(0, rows, tile_rows):
        bits = source[start:start + tile_rows].contiguous().view(torch.int32 if wide else torch.int16).to(torch.int64)
        parts = [bits & 0xFFFF, bits >> 16] if wide else [bits]
        row = torch.arange(start, start + bits.shape[0], dtype=torch.int64)
        index = 0
        for part in parts:
            for (_, b, square), weight in zip(FINGERPRINT_COMBINATIONS, weights):
                term = part * part if square else part
                per_row = (term * weight).sum(1).remainder(FINGERPRINT_PRIME)
                totals[index] += (per_row * ((row * b + 3) % 1019 + 1)).sum()
                index += 1
    return totals.remainder(FINGERPRINT_PRIME)


def fingerprint_terms(matrix: torch.Tensor) -> torch.Tensor:
    """Exact modular checksums of a matrix's bit patterns: for each 16-bit part (the value, or the low and high
    halves of a 32-bit pattern) and combination ``(a, b, square)``, ``sum_rows ((sum_c t(c) w_a(c)) mod p)
    w_b(row)`` with ``w_a(c) = (a c + 7) mod 1021 + 1`` and ``w_b(r) = (b r + 3) mod 1019 + 1``. CUDA matrices
    use the fused kernel (csrc/fit/fitter.cu); the host path computes the same integers."""
    if matrix.ndim != 2 or matrix.numel() == 0:
        raise ConfigurationError("source fingerprints take a nonempty matrix")
    if matrix.element_size() not in (2, 4):
        raise ConfigurationError("source fingerprints support 16- and 32-bit element types")
    rows, columns = matrix.shape
    if rows > (1 << 22) or columns > (1 << 14):
        raise ConfigurationError("source fingerprint geometry exceeds its overflow-free range")
    source = matrix.detach()
    if source.is_cuda:
        from .ops import _ext
        if _ext.available():
            from .ops.fitter import fingerprint_partials
            wide = source.element_size() == 4
            return fingerprint_partials(source, 0, FINGERPRINT_PRIME).sum(0)[:6 if wide else 3].remainder(
                FINGERPRINT_PRIME)
    return _fingerprint_terms_host(source.cpu())


def _fingerprint_text(matrix: torch.Tensor, values) -> str:
    rows, columns = matrix.shape
    return f"fp1:{rows}x{columns}:{matrix.dtype}:" + "".join(f"{int(v):08x}" for v in values)


def source_fingerprint(matrix: torch.Tensor) -> str:
    """Exact, device-independent integer fingerprint of a matrix's bit patterns (``fp1:RxC:dtype:hex``); it
    binds observations to their content without a host copy of the matrix (not an integrity hash). Same
    string form and checksums as reference reelcache/lineage_commit.py:197-271."""
    return _fingerprint_text(matrix, fingerprint_terms(matrix).tolist())


def source_fingerprints(matrices: Mapping[Any, torch.Tensor]) -> dict[Any, str]:
    """Fingerprints of many matrices with one device-to-host read per device."""
    terms = {entry: fingerprint_terms(matrix) for entry, matrix in matrices.items()}
    out = {}
    by_device: dict = {}
    for entry, value in terms.items():
        by_device.setdefault(value.device, []).append(entry)
    for entries in by_device.values():
        flat = torch.cat([terms[e] for e in entries]).tolist()
        offset = 0
        for entry in entries:
            count = int(terms[entry].numel())
            out[entry] = _fingerprint_text(matrices[entry], flat[offset:offset + count])
            offset += count
    return out


@dataclass
class ParentState:
    """The parent head's active bindings and the assembled FP16 rows of each active basis."""

    node_ref: str
    bindings: dict[Any, ActiveBasisBinding]
    rows: dict[Any, torch.Tensor | None] = field(default_factory=dict)


@dataclass
class StagedTile:
    entry: Any
    context: TensorContext
    plan: MatrixPlan
    pixels: np.ndarray | None = None
    factors: np.ndarray | None = None      # FP16 coefficients of the SVD-only representation
    affine: np.ndarray | None = None
    normalization: Mapping[str, Any] | None = None


class CommitJob:
    """One node's archival work (see the module docstring for the stages)."""

    def __init__(self, runtime, branch_id: str, node_kind: str, chunk_id: str, ranges, *, method: RankMethodConfig,
                 parent: ParentState, expected_head: str, execution_state: Mapping[str, torch.Tensor] | None,
                 device: Any, options: ArchiveOptions, epoch_id: str | None = None,
                 details: Mapping[str, Any] | None = None, view=None):
        self.runtime = runtime
        self.branch_id = branch_id
        self.node_kind = node_kind
        self.chunk_id = chunk_id
        self.ranges = ranges  # [(range_chunk_id, matrices, contexts)]
        self.method = method
        self.parent = parent
        self.expected_head = expected_head
        self.execution_state = execution_state
        self.device = torch.device(device)
        self.options = options
        self.epoch_id = epoch_id
        self.details = dict(details or {})
        self.view = view
        self.tiles: list[list[StagedTile]] = []
        self.timings: dict[str, float] = {}
        self.packs: list[codecs.EncodedTensor] = []
        self.stored: dict[str, Any] | None = None
        self.lease = None
        self.observations: list[FitObservation] = []

    # -- stages ------------------------------------------------------------------------------------------------

    def plan(self) -> "CommitJob":
        started = time.perf_counter()
        bindings = dict(self.parent.bindings)
        rows = dict(self.parent.rows)
        for range_id, matrices, contexts in self.ranges:
            plans = plan_chunk(matrices, contexts, self.method, self.view, bindings, rows, chunk_id=range_id,
                               device=self.device)
            staged = []
            for entry in sorted(plans, key=entry_order):
                plan = plans[entry]
                staged.append(StagedTile(entry, contexts[entry], plan))
                if plan.observation is not None:
                    self.observations.append(plan.observation)
                bindings[entry] = plan.binding
                rows[entry] = plan.rows
            self.tiles.append(staged)
        self.timings["plan"] = time.perf_counter() - started
        return self

    def finalize(self) -> "CommitJob":
        started = time.perf_counter()
        spec = self.method.codec
        for staged in self.tiles:
            for tile in staged:
                if spec.kind == "svd":  # SVD-only baseline: FP16 factors (FP32 per matrix), no quantization
                    dtype = torch.float16 if self.options.packed else torch.float32
                    tile.factors = tile.plan.coefficients.detach().to(dtype).cpu().numpy()
                    tile.plan.coefficients = None
                    continue
                pixels, affine, layout = codecs.quantize(tile.plan.coefficients, spec.normalization,
                                                         spec.protected_fraction)
                tile.pixels, tile.affine, tile.normalization = np.ascontiguousarray(pixels), affine, layout
                tile.plan.coefficients = None  # release the device coefficients
        self.timings["finalize"] = time.perf_counter() - started
        return self

    def encode(self) -> "CommitJob":
        started = time.perf_counter()
        spec = self.method.codec
        for staged in self.tiles:
            tiles = []
            for tile in staged:
                key, stream = entry_parts(tile.entry)
                rank = tile.plan.rank_view
                view_bytes = tile.plan.rows.detach().cpu().contiguous().numpy().tobytes()
                tiles.append({"entry": {"key": key.to_dict(), **({"stream": stream} if stream else {})},
                              "context": tile.context, "codec": CodecSpec(**{**spec.to_dict(), "rank": rank,
                                                                            "inter_prediction": spec.inter_prediction}),
                              "pixels": tile.pixels, "affine": tile.affine, "normalization": tile.normalization,
                              "basis": codecs.descriptor(view_bytes, rank, tile.context.channels),
                              "coefficients": tile.factors})
            if spec.kind == "svd" and not self.options.packed:
                # one reelcache.tensor.v1 packet per matrix (FP32 coefficients, basis = the version prefix)
                self.packs.append([codecs.encode_factorized(torch.from_numpy(t["coefficients"]),
                                                            tile.plan.rows.detach().cpu().contiguous().numpy().tobytes(),
                                                            t["context"], t["codec"])
                                   for t, tile in zip(tiles, staged)])
            elif spec.kind == "svd":
                self.packs.append(codecs.encode_factor_pack(tiles))
            else:
                self.packs.append(codecs.encode_node_pack(tiles, stream_codec=self.options.stream_codec,
                                                          details={"chunk_id": self.chunk_id}))
        self.timings["encode"] = time.perf_counter() - started
        return self

    def store(self) -> "CommitJob":
        """Write every object of the node (basis versions, packs, records, state) under a staging lease."""
        started = time.perf_counter()
        runtime = self.runtime
        store = runtime.store
        spec = self.method.codec
        created: list[str] = []
        results = []
        bindings = dict(self.parent.bindings)
        with store.transaction():
            for staged, pack in zip(self.tiles, self.packs):
                version_refs = {}
                for tile in staged:
                    plan = tile.plan
                    binding = bindings.get(tile.entry, ActiveBasisBinding())
                    if plan.decision in ("fresh", "refit", "zero_input"):
                        ref, version = runtime.basis.put_root(tile.context.key, plan.new_rows.detach().cpu())
                        new_binding = ActiveBasisBinding(ref, version.total_rank, version.group_id,
                                                         plan.rank_view if plan.decision != "zero_input" else None,
                                                         self.chunk_id if plan.decision != "zero_input" else None)
                    elif plan.decision == "augment":
                        ref, version = runtime.basis.put_extension(binding.version_ref, plan.new_rows.detach().cpu())
                        new_binding = ActiveBasisBinding(ref, version.total_rank, version.group_id, binding.fresh_rank,
                                                         binding.fresh_chunk_id, binding.coefficient_rate,
                                                         binding.rate_identity,
                                                         plan.binding.refit_debt if binding.fresh_rank else 0.0)
                    else:
                        ref = binding.version_ref
                        new_binding = binding
                    rate_identity = canonical_digest({"codec": spec.to_dict(), "stream": self.options.stream_codec,
                                                      "shape": list(tile.context.shape)})
                    # measured stream bytes per coefficient value of this pack (FP32 per-matrix packets: 4)
                    rate = 4.0 if isinstance(pack, list) else \
                        max(pack.metadata["stream_bytes"] / max(pack.metadata["raw_bytes"], 1), 1e-9)
                    if new_binding.version_ref is not None and new_binding.fresh_rank is not None:
                        new_binding = ActiveBasisBinding(new_binding.version_ref, new_binding.total_rank,
                                                         new_binding.group_id, new_binding.fresh_rank,
                                                         new_binding.fresh_chunk_id, rate, rate_identity,
                                                         new_binding.refit_debt)
                    version_refs[tile.entry] = ref
                    bindings[tile.entry] = new_binding
                if isinstance(pack, list):
                    results.append((None, self._store_per_matrix(staged, pack, version_refs)))
                    continue
                blobs = {name: store.put(value) for name, value in pack.payloads.items()}
                basis_refs = sorted({r for r in version_refs.values() if r is not None})
                packet_ref = runtime.put_content({"type": "packet", "version": 1, "model": runtime.model.to_dict(),
                                                  "metadata": pack.metadata, "payloads": blobs,
                                                  "metrics": json_copy(pack.metrics or {}),
                                                  "basis_storage": "external",
                                                  "basis_versions": [version_refs[t.entry] for t in staged]},
                                                 field="metrics", references=sorted(blobs.values()) + basis_refs)
                records = {}
                for index, tile in enumerate(staged):
                    plan = tile.plan
                    rank = plan.rank_view
                    codec = CodecSpec(**{**spec.to_dict(), "rank": rank, "inter_prediction": spec.inter_prediction})
                    key, stream = entry_parts(tile.entry)
                    energy = plan.energy if plan.energy.rank_view == rank else EnergyReport(
                        **{**plan.energy.to_dict(), "rank_view": rank})
                    record = MatrixRecord(tile.context, codec, packet_ref, version_refs[tile.entry], rank, energy, None,
                                          {**json_copy(plan.decision_record()),
                                           "packet": {"tile": index, "stream_codec": "fp16" if spec.kind == "svd"
                                                     else self.options.stream_codec}},
                                          packet_tile=index if codec.kind == "svd_hevc" and codec.inter_prediction is False
                                          else None, stream=stream)
                    records[tile.entry] = runtime.put_record(record)
                results.append((packet_ref, records))
            state_ref = None
            if self.execution_state:
                state_ref = store.put(serialize_tensors(dict(self.execution_state)))
            created = list(store.created_objects)
        if created:
            self.lease = store.lease(created, purpose="staging", verify=False)
        self.stored = {"ranges": results, "bindings": bindings, "execution_state": state_ref}
        self.timings["store"] = time.perf_counter() - started
        return self

    def _store_per_matrix(self, staged, packets, version_refs) -> dict:
        """Per-matrix SVD packets and their records, in the layout both implementations read: a packet manifest
        holds exactly ``type, version, model, metadata, payloads, metrics, basis_storage`` and references only its
        payload blobs; the record names the basis version whose prefix the packet's basis descriptor covers."""
        runtime, store, spec = self.runtime, self.runtime.store, self.method.codec
        records = {}
        for tile, packet in zip(staged, packets):
            blobs = {name: store.put(value) for name, value in packet.payloads.items()}
            packet_ref = runtime.put_content({"type": "packet", "version": 1, "model": runtime.model.to_dict(),
                                              "metadata": packet.metadata, "payloads": blobs,
                                              "metrics": json_copy(packet.metrics or {}),
                                              "basis_storage": "external_version_prefix"},
                                             field="metrics", references=sorted(blobs.values()))
            plan = tile.plan
            rank = plan.rank_view
            codec = CodecSpec(**{**spec.to_dict(), "rank": rank, "inter_prediction": spec.inter_prediction})
            energy = plan.energy if plan.energy.rank_view == rank else EnergyReport(
                **{**plan.energy.to_dict(), "rank_view": rank})
            record = MatrixRecord(tile.context, codec, packet_ref, version_refs[tile.entry], rank, energy, None,
                                  json_copy(plan.decision_record()), stream=entry_parts(tile.entry)[1])
            records[tile.entry] = runtime.put_record(record)
        return records

    def release(self) -> None:
        if self.lease is not None:
            self.lease.release()
            self.lease = None

    def plan_summary(self) -> dict[str, Any]:
        decisions: dict[str, int] = {}
        ranks = []
        for staged in self.tiles:
            for tile in staged:
                decisions[tile.plan.decision] = decisions.get(tile.plan.decision, 0) + 1
                ranks.append(tile.plan.rank_view)
        return {"decisions": decisions, "mean_rank": float(np.mean(ranks)) if ranks else 0.0,
                "max_rank": int(max(ranks)) if ranks else 0, "matrices": len(ranks)}


def warm_commit_path(method: RankMethodConfig, contexts: Mapping[Any, TensorContext], *,
                     options: ArchiveOptions | None = None, device: Any = "cpu", max_frames: int | None = None,
                     seed: int = 0) -> dict[str, Any]:
    """Pay a commit path's first-use costs before the first real chunk: plan and finalize two synthetic chunks of
    ``contexts``' geometry on this thread (the fresh path, then the active-basis paths against the first one's rows);
    nothing is stored and nothing is learned. ``max_frames`` caps the frames of each context (less transient memory,
    the same kernels and library handles warmed). Returns per-phase seconds, the decisions and the synthetic bytes."""
    import time
    from dataclasses import replace as _replace

    from .rank_method import plan_chunk
    from .types import ActiveBasisBinding
    options = ArchiveOptions() if options is None else options
    if not isinstance(method, RankMethodConfig) or not isinstance(options, ArchiveOptions):
        raise ConfigurationError("a commit warm-up needs a RankMethodConfig and ArchiveOptions")
    if max_frames is not None and (type(max_frames) is not int or max_frames < 1):
        raise ConfigurationError("max_frames must be None or a positive integer")
    if not contexts:
        raise ConfigurationError("a commit warm-up needs the commit's contexts")
    device = torch.device(device)
    gen = torch.Generator().manual_seed(seed)
    capped, matrices = {}, {}
    for entry, context in contexts.items():
        if max_frames is not None and context.frames > max_frames:
            context = _replace(context, frames=max_frames)
        capped[entry] = context
        rows, channels = context.token_count, context.channels
        rank = max(1, min(channels // 4, 64))
        x = torch.randn(rows, rank, generator=gen) @ torch.randn(rank, channels, generator=gen)
        matrices[entry] = (x + 1e-2 * torch.randn(rows, channels, generator=gen)).to(torch.bfloat16).to(device)
    report: dict[str, Any] = {"source_bytes": sum(m.numel() * m.element_size() for m in matrices.values())}
    started = time.perf_counter()

    def finalize(plans):
        for plan in plans.values():
            if method.codec.kind == "svd":
                plan.coefficients.to(torch.float16).cpu()
            else:
                codecs.quantize(plan.coefficients, method.codec.normalization, method.codec.protected_fraction)

    clock = time.perf_counter()
    fresh = plan_chunk(matrices, capped, method, None, {}, {}, chunk_id="warm-0", device=device)
    report["fresh_plan_seconds"] = time.perf_counter() - clock
    clock = time.perf_counter()
    finalize(fresh)
    report["fresh_finalize_seconds"] = time.perf_counter() - clock
    bindings = {e: ActiveBasisBinding("manifest:" + "0" * 64, p.rows.shape[0], "0" * 64, p.rows.shape[0], "warm-0")
                for e, p in fresh.items() if p.decision in ("fresh", "refit")}
    clock = time.perf_counter()
    reuse = plan_chunk(matrices, capped, method, None, bindings, {e: fresh[e].rows for e in bindings},
                       chunk_id="warm-1", device=device)
    report["reuse_plan_seconds"] = time.perf_counter() - clock
    clock = time.perf_counter()
    finalize(reuse)
    report["reuse_finalize_seconds"] = time.perf_counter() - clock
    if device.type == "cuda":
        torch.cuda.synchronize(device)
    decisions: dict[str, int] = {}
    for plan in list(fresh.values()) + list(reuse.values()):
        decisions[plan.decision] = decisions.get(plan.decision, 0) + 1
    report.update(decisions=decisions, total_seconds=time.perf_counter() - started)
    return report
