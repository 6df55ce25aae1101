"""Lineages over the immutable node graph (reference: reelcache/lineage.py:66-1351).

A lineage is a named head ref (``lineages/<id>``) over immutable nodes. Nodes, epochs, matrix records
and packets are content-addressed manifests:

* node     ``{"type": "node", "version": 1, "model", "node": ChunkNode, "commit": report}``
* epoch    ``{"type": "cache_epoch", "version": 1, "model", "epoch": CacheEpoch}``
* record   ``{"type": "matrix_record", "version": 1, "model", "record": MatrixRecord}``
* packet   ``{"type": "packet", "version": 1, "model", "metadata", "payloads": {name: blob id},
             "metrics", "basis_storage", ...}``

Scheduling-dependent fields (timings) are split into the store's unhashed telemetry sidecar, so
identical content always yields identical ids. Commits run the staged :class:`CommitJob`
(plan -> finalize -> encode -> store) and publish with a compare-and-swap of the head; forks and
rewinds only move refs. History resolution returns, for any node, the newest KV version of every
attended token range on its ancestor path.
"""

from __future__ import annotations

import threading
import time
from dataclasses import dataclass
from typing import Callable, Any, Mapping, Sequence

import numpy as np
import torch

from . import codecs
from .basis_versions import BasisVersionStore
from .cache_epochs import ResolvedPiece, resolve
from .errors import ConfigurationError, IntegrityError, PendingError, StateError, UnsupportedError
from .lineage_commit import ArchiveOptions, CommitJob, ParentState, source_fingerprint
from .predictor_registry import RankPredictorRegistry, observation_origin
from .rank_method import RankMethodConfig
from .serialization import deserialize_tensors, serialize_tensors, tensor_bytes
from .store import ObjectStore
from .types import (ActiveBasisBinding, CacheEpoch, ChunkNode, CodecSpec, MatrixKey, MatrixRecord, ModelIdentity,
                    TensorContext, TokenRangeRecords, entry_order, entry_parts, json_copy)

LINEAGE_PREFIX = "lineages/"
#: Manifest ``type`` names each loader accepts: the names both implementations write (``cache_epoch``,
#: ``matrix_record``), and the short names of stores this package wrote before the layouts were aligned.
_MANIFEST_TYPES = {"node": ("node",), "epoch": ("cache_epoch", "epoch"), "record": ("matrix_record", "record"),
                   "packet": ("packet",)}
_TELEMETRY_KEYS = ("timings", "seconds", "planner_seconds", "started", "published")


def split_run_telemetry(value: Any) -> tuple[Any, Any]:
    """(content, telemetry) of a commit report: timing keys move to the unhashed sidecar."""
    if not isinstance(value, Mapping):
        return value, None
    content = {k: v for k, v in value.items() if k not in _TELEMETRY_KEYS}
    telemetry = {k: v for k, v in value.items() if k in _TELEMETRY_KEYS}
    return content, (telemetry or None)


@dataclass
class LineageCommit:
    """Result of one published commit."""

    node_ref: str
    node: ChunkNode
    records: dict
    plan: dict
    timings: dict


class LineageRuntime:
    """Lineage operations over one store and model (thread-safe; commits of one lineage serialize)."""

    def __init__(self, store: ObjectStore, model: ModelIdentity, *, registry: RankPredictorRegistry | None = None):
        self.store = store
        self.model = model
        self.basis = BasisVersionStore(store, model)
        self.registry = registry
        self._lock = threading.RLock()
        self._manifests: dict[str, Any] = {}
        self._lineage_pending: set[str] = set()
        self._lineage_owned_prefix = None

    # -- content manifests ---------------------------------------------------------------------------------------

    def put_content(self, data: Mapping[str, Any], *, field: str, references: Sequence[str]) -> str:
        content, telemetry = split_run_telemetry(data[field])
        ref = self.store.put_manifest({**data, field: content}, references=references)
        if telemetry is not None:
            self.store.put_telemetry(ref, {field: telemetry})
        return ref

    def put_record(self, record: MatrixRecord) -> str:
        references = [record.packet_ref] + ([record.basis_version_ref] if record.basis_version_ref else [])
        return self.store.put_manifest({"type": "matrix_record", "version": 1, "model": self.model.to_dict(),
                                        "record": record.to_dict()}, references=sorted(set(references)))

    def _put_epoch(self, epoch: CacheEpoch) -> str:
        references = [epoch.parent_epoch_ref] if epoch.parent_epoch_ref else []
        for item in epoch.ranges:
            references.extend(ref for _, ref in item.records)
            if item.packet_ref:
                references.append(item.packet_ref)
        return self.store.put_manifest({"type": "cache_epoch", "version": 1, "model": self.model.to_dict(),
                                        "epoch": epoch.to_dict()}, references=sorted(set(references)))

    def _put_node(self, node: ChunkNode, commit: Mapping[str, Any]) -> str:
        references = [node.parent_ref, node.epoch_ref, node.execution_state_ref, node.packet_ref,
                      *(ref for _, ref in node.matrix_records),
                      *(binding.version_ref for _, binding in node.active_basis)]
        return self.put_content({"type": "node", "version": 1, "model": self.model.to_dict(), "node": node.to_dict(),
                                 "commit": json_copy(dict(commit), name="node commit report")},
                                field="commit", references=sorted({r for r in references if r is not None}))

    def _cached(self, ref: str, kind: str):
        hit = self._manifests.get(ref)
        if hit is not None:
            return hit
        data = self.store.get_manifest(ref)
        if data.get("type") not in _MANIFEST_TYPES[kind] or data.get("version") != 1:
            raise IntegrityError(f"{ref} is not a {kind} manifest")
        if "model" in data and kind in ("epoch", "record") and ModelIdentity.from_dict(data["model"]) != self.model:
            raise IntegrityError(f"{kind} manifest {ref} belongs to another model")
        if kind == "node":
            if ModelIdentity.from_dict(data["model"]) != self.model:
                raise IntegrityError("node belongs to another model")
            value = ChunkNode.from_dict(data["node"])
        elif kind == "epoch":
            value = CacheEpoch.from_dict(data["epoch"])
        elif kind == "record":
            value = MatrixRecord.from_dict(data["record"])
        else:
            value = data
        if len(self._manifests) > 200000:
            self._manifests.clear()
        self._manifests[ref] = value
        return value

    def drop_manifest_caches(self) -> None:
        self._manifests.clear()
        self.basis.drop_caches()

    def load_node(self, ref: str) -> ChunkNode:
        return self._cached(ref, "node")

    def load_epoch(self, ref: str) -> CacheEpoch:
        return self._cached(ref, "epoch")

    def load_record(self, ref: str) -> MatrixRecord:
        return self._cached(ref, "record")

    def load_packet(self, ref: str) -> Mapping[str, Any]:
        return self._cached(ref, "packet")

    def load_basis_version(self, ref: str):
        return self.basis.load(ref)

    def node_path(self, ref: str) -> list[tuple[str, ChunkNode, CacheEpoch]]:
        """Root-first ancestor path of a node with each node's epoch."""
        path = []
        current = ref
        while current is not None:
            node = self.load_node(current)
            path.append((current, node, self.load_epoch(node.epoch_ref)))
            current = node.parent_ref
        return path[::-1]

    def node_commit_report(self, ref: str) -> Mapping[str, Any]:
        return self.store.get_manifest(ref)["commit"]

    def run_telemetry(self, ref: str) -> dict[str, Any] | None:
        return self.store.telemetry(ref)

    # -- lineage heads -------------------------------------------------------------------------------------------

    @staticmethod
    def _lineage_name(branch_id: str) -> str:
        if isinstance(branch_id, str) and branch_id and "\x00" not in branch_id:
            return LINEAGE_PREFIX + branch_id
        raise ConfigurationError(f"lineage id {branch_id!r} is not a non-empty string without NUL")

    def _entries(self, streams: Sequence[str]) -> list:
        keys = [MatrixKey(layer, target) for layer in range(self.model.layers) for target in ("K", "V")]
        return [(key, stream) for key in keys for stream in streams] if streams else keys

    def _idle(self, branch_id: str, action: str) -> None:
        if branch_id in self._lineage_pending:
            raise PendingError(f"lineage {branch_id!r} has a commit in flight; {action} after it publishes")

    def create_lineage(self, branch_id: str, *, epoch_id: str = "e0", details: Mapping[str, Any] | None = None,
                       streams: Sequence[str] = ()) -> str:
        """A new lineage whose head is a root node: zero tokens, the initial global epoch ``epoch_id`` and no
        active basis for any matrix (of any of ``streams``)."""
        streams = tuple(streams)
        with self._lock:
            name = self._lineage_name(branch_id)
            with self.store.transaction():
                if self.store.get_ref(name) is not None:
                    raise StateError(f"lineage {branch_id!r} exists already")
                epoch_ref = self._put_epoch(CacheEpoch(epoch_id, None, "initial", "global", (), details or {}))
                unbound = tuple((entry, ActiveBasisBinding()) for entry in self._entries(streams))
                root = ChunkNode("root", "root", None, epoch_id, epoch_ref, 0, 0, 0, 0, 0, 0, (), unbound,
                                 streams=streams)
                root_ref = self._put_node(root, {"kind": "root"})
                self.store.set_ref(name, root_ref, expected=None)
                return root_ref

    def lineage_head(self, branch_id: str) -> str:
        head = self.store.get_ref(self._lineage_name(branch_id))
        if head is None:
            raise StateError(f"no lineage named {branch_id!r}")
        return head

    def list_lineages(self) -> dict[str, str]:
        return {name.removeprefix(LINEAGE_PREFIX): ref for name, ref in self.store.list_refs(LINEAGE_PREFIX).items()}

    def fork_lineage(self, node_ref: str, branch_id: str) -> None:
        """Start lineage ``branch_id`` at ``node_ref`` (any readable node); other lineages do not move."""
        with self._lock:
            name = self._lineage_name(branch_id)
            with self.store.transaction():
                self.load_node(node_ref)
                if self.store.get_ref(name) is not None:
                    raise StateError(f"cannot fork into {branch_id!r}: the lineage exists")
                self.store.set_ref(name, node_ref, expected=None)

    def set_lineage_ownership(self, prefix: Any) -> None:
        """``prefix(branch_id)`` names a ref folder whose heads count as the lineage's own for rewinds (a
        detached side lineage keeps the chunks it took over reachable to the lineage it came from)."""
        self._lineage_owned_prefix = prefix

    def _reachable(self, node_ref: str, heads) -> bool:
        return any(node_ref in {ref for ref, _, _ in self.node_path(head)} for head in heads)

    def rewind_lineage(self, branch_id: str, node_ref: str) -> None:
        """Move the lineage's head back to one of its ancestors (or to a node of a lineage it owns)."""
        with self._lock:
            name = self._lineage_name(branch_id)
            self._idle(branch_id, "rewind")
            with self.store.transaction():
                head = self.lineage_head(branch_id)
                allowed = self._reachable(node_ref, [head])
                if not allowed and self._lineage_owned_prefix is not None:
                    prefix = self._lineage_owned_prefix(branch_id)
                    allowed = prefix is not None and self._reachable(node_ref, self.store.list_refs(prefix).values())
                if not allowed:
                    raise StateError(f"{node_ref} is not on lineage {branch_id!r}'s path; fork to reach it")
                self.store.set_ref(name, node_ref, expected=head)

    def delete_lineage(self, branch_id: str) -> None:
        with self._lock:
            self._idle(branch_id, "delete it")
            self.store.delete_ref(self._lineage_name(branch_id))

    # -- commits -------------------------------------------------------------------------------------------------

    def _parent_state(self, head_ref: str, device: Any) -> ParentState:
        node = self.load_node(head_ref)
        bindings = {entry: binding for entry, binding in node.active_basis}
        rows = {}
        cache: dict[str, torch.Tensor] = {}
        for entry, binding in bindings.items():
            if binding.version_ref is None:
                rows[entry] = None
                continue
            if binding.version_ref not in cache:
                cache[binding.version_ref] = self.basis.assemble(binding.version_ref).to(device)
            rows[entry] = cache[binding.version_ref]
        return ParentState(head_ref, bindings, rows)

    def _check_inputs(self, node: ChunkNode, matrices: Mapping[Any, torch.Tensor],
                      contexts: Mapping[Any, TensorContext]) -> None:
        expected = set(self._entries(node.streams))
        if set(matrices) != expected or set(contexts) != expected:
            raise ConfigurationError(f"a commit names {len(matrices)} matrices and {len(contexts)} contexts; the "
                                     f"node expects exactly its {len(expected)} (layer, K/V[, stream]) entries")
        for entry, context in contexts.items():
            key, _ = entry_parts(entry)
            if context.key != key or context.model != self.model:
                raise ConfigurationError(f"context of {entry} describes {context.key} of {context.model.name!r}")
            if tuple(matrices[entry].reshape(-1, context.channels).shape) != context.shape:
                raise ConfigurationError(f"{entry}: matrix does not reshape to its context's {context.shape}")

    def prepare_commit(self, node_kind: str, branch_id: str, chunk_id: str, ranges, *, method: RankMethodConfig,
                       registry: RankPredictorRegistry | None, epoch_id: str | None = None,
                       details: Mapping[str, Any] | None = None,
                       execution_state: Mapping[str, torch.Tensor] | None = None, device: Any = "cpu",
                       expected_head: str | None = None, options: ArchiveOptions | None = None,
                       parent: ParentState | None = None, view=None) -> CommitJob:
        """A staged :class:`CommitJob` against the current (or ``expected_head``) head; not yet run."""
        with self._lock:
            head = self.lineage_head(branch_id) if expected_head is None else expected_head
            node = self.load_node(head)
            if node_kind == "chunk":
                self._check_inputs(node, ranges[0][1], ranges[0][2])
                start = node.frontier
                context = next(iter(ranges[0][2].values()))
                if context.token_start != start:
                    raise ConfigurationError(f"chunk starts at token {context.token_start}, the head's frontier is {start}")
            registry = registry or self.registry
            if view is None and registry is not None:
                view = registry.pin()
            if parent is None:
                parent = self._parent_state(head, device)
            return CommitJob(self, branch_id, node_kind, chunk_id, ranges, method=method, parent=parent,
                             expected_head=head, execution_state=execution_state, device=device,
                             options=options or ArchiveOptions(), epoch_id=epoch_id, details=details, view=view)

    def _commit(self, node_kind, branch_id, chunk_id, ranges, *, method, registry, epoch_id, details,
                execution_state, device, expected_head, options) -> LineageCommit:
        job = self.prepare_commit(node_kind, branch_id, chunk_id, ranges, method=method, registry=registry,
                                  epoch_id=epoch_id, details=details, execution_state=execution_state,
                                  device=device, expected_head=expected_head, options=options)
        with self._lock:
            self._lineage_pending.add(branch_id)
        try:
            job.plan().finalize().encode().store()
            return self.publish_job(job, job.expected_head, registry=registry or self.registry)
        finally:
            with self._lock:
                self._lineage_pending.discard(branch_id)
            job.release()

    def commit_node(self, branch_id: str, chunk_id: str, matrices: Mapping[Any, torch.Tensor],
                    contexts: Mapping[Any, TensorContext], *, method: RankMethodConfig,
                    registry: RankPredictorRegistry | None = None,
                    execution_state: Mapping[str, torch.Tensor] | None = None, device: Any = "cpu",
                    expected_head: str | None = None, options: ArchiveOptions | None = None) -> LineageCommit:
        """Commit one complete clean chunk (all layers' pre-RoPE K and V, every stream) as a child node."""
        return self._commit("chunk", branch_id, chunk_id, [(chunk_id, matrices, contexts)], method=method,
                            registry=registry, epoch_id=None, details=None, execution_state=execution_state,
                            device=device, expected_head=expected_head, options=options)

    def commit_recache(self, branch_id: str, recache_id: str, ranges, *, method: RankMethodConfig,
                       registry: RankPredictorRegistry | None = None, epoch_id: str,
                       details: Mapping[str, Any] | None = None,
                       execution_state: Mapping[str, torch.Tensor] | None = None, device: Any = "cpu",
                       expected_head: str | None = None, options: ArchiveOptions | None = None) -> LineageCommit:
        """Publish a zero-frame node whose ``kv_recache`` epoch re-materializes earlier chunks."""
        return self._commit("recache", branch_id, recache_id, list(ranges), method=method, registry=registry,
                            epoch_id=epoch_id, details=details or {}, execution_state=execution_state,
                            device=device, expected_head=expected_head, options=options)

    def commit_segment(self, branch_id: str, segment_id: str, matrices, contexts, *, method: RankMethodConfig,
                       registry: RankPredictorRegistry | None = None, epoch_id: str,
                       details: Mapping[str, Any] | None = None,
                       execution_state: Mapping[str, torch.Tensor] | None = None, device: Any = "cpu",
                       expected_head: str | None = None, options: ArchiveOptions | None = None) -> LineageCommit:
        """Publish a LongCat segment: a new segment-local conditioning-cache epoch."""
        return self._commit("segment", branch_id, segment_id, [(segment_id, matrices, contexts)], method=method,
                            registry=registry, epoch_id=epoch_id, details=details or {},
                            execution_state=execution_state, device=device, expected_head=expected_head,
                            options=options)

    def publish_job(self, job: CommitJob, expected_head: str, *, registry: RankPredictorRegistry | None = None,
                    started: float | None = None) -> LineageCommit:
        """Build the node manifest from a stored job and CAS the lineage head; trains the registry."""
        if job.stored is None:
            raise StateError("a commit job must be stored before it is published")
        with self._lock, self.store.transaction():
            head_node = self.load_node(expected_head)
            bindings = job.stored["bindings"]
            active = tuple(sorted(((entry, binding) for entry, binding in bindings.items()),
                                  key=lambda pair: entry_order(pair[0])))
            ranges = job.stored["ranges"]
            if job.node_kind == "chunk":
                (packet_ref, records), = ranges
                context = next(iter(job.ranges[0][2].values()))
                node = ChunkNode("chunk", job.chunk_id, expected_head, head_node.cache_epoch_id, head_node.epoch_ref,
                                 context.token_start, context.token_end, context.frames, context.height, context.width,
                                 context.token_end, tuple(records.items()), active, job.stored["execution_state"],
                                 head_node.streams, packet_ref)
            else:
                epoch_ranges = []
                for (range_id, matrices, contexts), (packet_ref, records) in zip(job.ranges, ranges):
                    context = next(iter(contexts.values()))
                    start = 0 if job.node_kind == "segment" else context.token_start
                    epoch_ranges.append(TokenRangeRecords(range_id, start, start + context.token_count,
                                                          context.frames, context.height, context.width,
                                                          tuple(records.items()), head_node.streams, packet_ref))
                epoch = CacheEpoch(job.epoch_id, head_node.epoch_ref,
                                   "kv_recache" if job.node_kind == "recache" else "longcat_segment",
                                   "global" if job.node_kind == "recache" else "segment_local",
                                   tuple(sorted(epoch_ranges, key=lambda r: r.token_start)), job.details)
                epoch_ref = self._put_epoch(epoch)
                if job.node_kind == "recache":
                    node = ChunkNode("recache", job.chunk_id, expected_head, job.epoch_id, epoch_ref,
                                     head_node.frontier, head_node.frontier, 0, 0, 0, head_node.frontier, (), active,
                                     job.stored["execution_state"], head_node.streams)
                else:
                    first = epoch_ranges[0]
                    node = ChunkNode("segment", job.chunk_id, expected_head, job.epoch_id, epoch_ref, 0,
                                     first.token_end, first.frames, first.height, first.width, first.token_end, (),
                                     active, job.stored["execution_state"], head_node.streams)
            commit = {"kind": job.node_kind, "method": job.method.to_dict(), "plan": job.plan_summary(),
                      "stream_codec": job.options.stream_codec, "timings": dict(job.timings)}
            node_ref = self._put_node(node, commit)
            self.store.set_ref(self._lineage_name(job.branch_id), node_ref, expected=expected_head)
        registry = registry or self.registry
        if registry is not None and job.observations:
            origin = observation_origin(job.branch_id, job.node_kind, job.chunk_id, job.view) \
                if job.view is not None else None
            registry.observe([obs if origin is None else type(obs)(**{**obs.__dict__, "origin": origin})
                              for obs in job.observations])
        records = dict(job.stored["ranges"][0][1]) if job.stored["ranges"] else {}
        return LineageCommit(node_ref, node, records, job.plan_summary(), dict(job.timings))

    def _raw_records(self, matrices: Mapping[Any, torch.Tensor], contexts: Mapping[Any, TensorContext]) -> dict:
        """Exact RAW packets and records of one range (inside the caller's store transaction)."""
        raw = CodecSpec(kind="raw")
        records = {}
        for entry in sorted(contexts, key=entry_order):
            context = contexts[entry]
            encoded = codecs.encode_raw(matrices[entry].detach().to("cpu").reshape(context.shape), context)
            blobs = {name: self.store.put(value) for name, value in encoded.payloads.items()}
            packet_ref = self.put_content({"type": "packet", "version": 1, "model": self.model.to_dict(),
                                           "metadata": encoded.metadata, "payloads": blobs,
                                           "metrics": json_copy(encoded.metrics), "basis_storage": "none"},
                                          field="metrics", references=sorted(blobs.values()))
            record = MatrixRecord(context, raw, packet_ref, None, None, None, None,
                                  {"schema": "reelcache.raw_record.v1", "representation": "raw"},
                                  stream=entry_parts(entry)[1])
            records[entry] = self.put_record(record)
        return records

    def commit_raw_node(self, branch_id: str, chunk_id: str, matrices: Mapping[Any, torch.Tensor],
                        contexts: Mapping[Any, TensorContext], *,
                        execution_state: Mapping[str, torch.Tensor] | None = None,
                        expected_head: str | None = None, kv_objects: bool = True) -> LineageCommit:
        """Commit one chunk as exact RAW packets (the identity reference; extends RAW lineages only).
        ``kv_objects=False`` stores no KV at all: a latents-only node that a restore replays from its execution
        state (which must then be given)."""
        started = time.perf_counter()
        if not kv_objects and not execution_state:
            raise ConfigurationError("kv_objects=False stores no KV: pass the execution_state the node is replayed from")
        with self._lock:
            head = self.lineage_head(branch_id) if expected_head is None else expected_head
            head_node = self.load_node(head)
            self._check_inputs(head_node, matrices, contexts)
            if any(binding.version_ref is not None for _, binding in head_node.active_basis):
                raise UnsupportedError(f"head {head} binds lossy bases; exact RAW nodes go on RAW lineages")
            with self.store.transaction():
                records = self._raw_records(matrices, contexts) if kv_objects else {}
                state_ref = self.store.put(serialize_tensors(dict(execution_state))) if execution_state else None
                context = next(iter(contexts.values()))
                if context.token_start != head_node.frontier:
                    raise ConfigurationError(f"RAW chunk starts at {context.token_start}; the head ends at {head_node.frontier}")
                node = ChunkNode("chunk", chunk_id, head, head_node.cache_epoch_id, head_node.epoch_ref,
                                 context.token_start, context.token_end, context.frames, context.height, context.width,
                                 context.token_end, tuple(records.items()), head_node.active_basis, state_ref,
                                 head_node.streams)
                node_ref = self._put_node(node, {"kind": "raw_chunk" if kv_objects else "latents_chunk",
                                                 "timings": {"store": time.perf_counter() - started}})
                self.store.set_ref(self._lineage_name(branch_id), node_ref, expected=head)
        return LineageCommit(node_ref, node, records, {"decisions": {"raw": len(records)}}, {})

    def commit_raw_recache(self, branch_id: str, recache_id: str, ranges, *, epoch_id: str,
                           details: Mapping[str, Any] | None = None,
                           execution_state: Mapping[str, torch.Tensor] | None = None,
                           expected_head: str | None = None, kv_objects: bool = True) -> LineageCommit:
        """Publish a ``kv_recache`` epoch of exact RAW ranges (``ranges``: ``(range_id, matrices, contexts)`` per
        re-materialized chunk range). ``kv_objects=False`` records the ranges without KV (a latents-only
        lineage re-runs the recache on replay); the epoch's details then say ``kv_objects: false``."""
        details = dict(details or {})
        if not kv_objects:
            details["kv_objects"] = False
        with self._lock:
            head = self.lineage_head(branch_id) if expected_head is None else expected_head
            head_node = self.load_node(head)
            if any(binding.version_ref is not None for _, binding in head_node.active_basis):
                raise UnsupportedError(f"head {head} binds lossy bases; exact RAW recaches go on RAW lineages")
            with self.store.transaction():
                epoch_ranges = []
                for range_id, matrices, contexts in ranges:
                    self._check_inputs(head_node, matrices, contexts)
                    context = next(iter(contexts.values()))
                    if context.token_end > head_node.frontier:
                        raise ConfigurationError(f"range {range_id!r} ends at {context.token_end}, past the generated "
                                                 f"{head_node.frontier} tokens")
                    records = self._raw_records(matrices, contexts) if kv_objects else {}
                    epoch_ranges.append(TokenRangeRecords(range_id, context.token_start, context.token_end,
                                                          context.frames, context.height, context.width,
                                                          tuple(records.items()), head_node.streams))
                epoch = CacheEpoch(epoch_id, head_node.epoch_ref, "kv_recache", "global",
                                   tuple(sorted(epoch_ranges, key=lambda r: r.token_start)), details)
                epoch_ref = self._put_epoch(epoch)
                state_ref = self.store.put(serialize_tensors(dict(execution_state))) if execution_state else None
                node = ChunkNode("recache", recache_id, head, epoch_id, epoch_ref, head_node.frontier,
                                 head_node.frontier, 0, 0, 0, head_node.frontier, (), head_node.active_basis, state_ref,
                                 head_node.streams)
                node_ref = self._put_node(node, {"kind": "raw_recache" if kv_objects else "latents_recache"})
                self.store.set_ref(self._lineage_name(branch_id), node_ref, expected=head)
        return LineageCommit(node_ref, node, {}, {"decisions": {"raw_ranges": len(epoch_ranges)}}, {})

    # -- history -------------------------------------------------------------------------------------------------

    def resolve_history(self, node_ref: str, ranges: Sequence[tuple[int, int]] | None = None) -> list[ResolvedPiece]:
        """Newest KV version of each attended range on the node's path (default: the whole frontier)."""
        node = self.load_node(node_ref)
        if ranges is None:
            ranges = [(0, node.frontier)] if node.frontier else []
        return resolve(self.node_path(node_ref), ranges)

    def node_pack(self, packet_ref: str, *, verify: bool = True,
                  reader: Callable[[list[str]], Mapping[str, bytes]] | None = None
                  ) -> tuple[Mapping[str, Any], codecs.DecodedPack]:
        """(packet manifest, decoded coefficient pack) of a node pack; ``reader(ids)`` reads its payload objects
        (default: the store's parallel reads; a restore staging engine passes its own)."""
        packet = self.load_packet(packet_ref)
        metadata = packet["metadata"]
        if metadata.get("schema") != codecs.PACK_SCHEMA:
            raise IntegrityError("packet is not a node pack")
        ids = [packet["payloads"]["stream"], packet["payloads"]["affines"]]
        blobs = (reader or self.store.get_many)(ids)
        pack = codecs.DecodedPack(metadata, blobs[packet["payloads"]["stream"]], blobs[packet["payloads"]["affines"]],
                                  verify=verify)
        return packet, pack

    def factor_pack(self, packet_ref: str, *, verify: bool = True) -> tuple[Mapping[str, Any], codecs.FactorPack]:
        """(packet manifest, decoded FP16 factor pack) of an SVD-only node."""
        packet = self.load_packet(packet_ref)
        if packet["metadata"].get("schema") != codecs.FACTOR_PACK_SCHEMA:
            raise IntegrityError("packet is not a factor pack")
        return packet, codecs.FactorPack(packet["metadata"], self.store.get(packet["payloads"]["factors"]),
                                         verify=verify)

    def execution_state(self, node_ref: str, *, device: Any = "cpu") -> dict[str, torch.Tensor]:
        node = self.load_node(node_ref)
        if node.execution_state_ref is None:
            return {}
        return deserialize_tensors(self.store.get(node.execution_state_ref), device=device)

    def acquire_node_history(self, node_ref: str, key: MatrixKey, *, ranges: Sequence[tuple[int, int]] | None = None,
                             stream: str | None = None, device: Any = "cpu",
                             dtype: torch.dtype = torch.float32, packs: dict | None = None) -> torch.Tensor:
        """Dense pre-RoPE history ``[T, C]`` of one matrix (FP32 ``dequantize(P) @ Q``; RAW bitwise). ``packs``
        carries the parsed packets from one call to the next, so restoring every matrix of a node parses each
        packet once instead of once per matrix."""
        pieces = self.resolve_history(node_ref, ranges)
        parts = []
        packs = {} if packs is None else packs
        for piece in pieces:
            record_ref = piece.record(key, stream)
            record = self.load_record(record_ref)
            packet = self.load_packet(record.packet_ref)
            if record.codec.kind == "raw":
                blobs = {name: self.store.get(ref) for name, ref in packet["payloads"].items()}
                from .types import EncodedTensor
                values = codecs.decode_tensor(EncodedTensor(packet["metadata"], blobs), device=device).float()
            elif record.codec.kind == "svd":
                if packet["metadata"].get("schema") == codecs.TENSOR_V1:
                    # a per-matrix SVD packet: FP32 coefficients, the basis is the record's version prefix
                    blobs = {name: self.store.get(ref) for name, ref in packet["payloads"].items()}
                    from .types import EncodedTensor
                    coefficients, _ = codecs.decode_v1(EncodedTensor(packet["metadata"], blobs), device=device)
                else:
                    if record.packet_ref not in packs:
                        packs[record.packet_ref] = self.factor_pack(record.packet_ref)[1]
                    factors = packs[record.packet_ref].factors(record.decision["packet"]["tile"])
                    coefficients = torch.from_numpy(factors.astype(np.float32)).to(device)
                basis = self.basis.assemble(record.basis_version_ref, record.rank_view).to(device).float()
                values = coefficients @ basis
            else:
                if record.packet_ref not in packs:
                    packs[record.packet_ref] = self.node_pack(record.packet_ref)[1]
                pack = packs[record.packet_ref]
                index = record.decision["packet"]["tile"]
                pixels = pack.pixels(index)
                scale, offset = pack.scale_offset(index)
                coefficients = torch.from_numpy(pixels.astype(np.float32) * scale + offset).to(device)
                basis = self.basis.assemble(record.basis_version_ref, record.rank_view).to(device).float()
                values = coefficients @ basis
            parts.append(values[piece.offset:piece.offset + (piece.token_end - piece.token_start)])
        if not parts:
            return torch.zeros((0, self.model.channels_for(key)), dtype=dtype, device=device)
        return torch.cat(parts).to(dtype)

    def node_storage(self, node_ref: str) -> dict[str, Any]:
        """Bytes a node adds: coefficient streams, affines, new basis blocks and manifests."""
        node = self.load_node(node_ref)
        total = {"stream_bytes": 0, "affine_bytes": 0, "basis_bytes": 0, "raw_bytes": 0}
        packets = {self.load_record(ref).packet_ref for _, ref in node.matrix_records}
        for packet_ref in packets:
            packet = self.load_packet(packet_ref)
            sizes = self.store.object_sizes(packet["payloads"].values())
            for name, ref in packet["payloads"].items():
                key = {"stream": "stream_bytes", "affines": "affine_bytes", "factors": "stream_bytes"}.get(
                    name, "raw_bytes")
                total[key] += sizes.get(ref, 0)
        parent = self.load_node(node.parent_ref) if node.parent_ref else None
        before = {b.version_ref for _, b in parent.active_basis} if parent else set()
        for _, binding in node.active_basis:
            if binding.version_ref and binding.version_ref not in before:
                version = self.basis.load(binding.version_ref)
                total["basis_bytes"] += version.added_bytes
        total["total_bytes"] = sum(total.values())
        return total
