"""KVRuntime: the general single-host durable runtime over canonical full-KV-channel matrices
(the counterpart of reference reelcache/manager.py:357-2444; BASELINE config 1 drives it).

A *branch* is a named ref ``branches/<id>`` to an immutable *head* manifest listing committed chunk
manifests; every chunk holds one tensor manifest per (layer, K/V) matrix. Commits publish a new head
with a compare-and-set on the branch ref, so concurrent writers never lose history. Snapshots
(``snapshots/<sha>``) bind a head to portable metadata and a tensor-state blob (RNG, latents);
``restore`` points a branch (new or existing) at a snapshot's head, ``fork`` only a new one.
``acquire_history`` decodes a key's history into a residency-bounded lease.

Manifest shapes (identical to the reference so stores stay interchangeable):

* ``{"type": "model", "version": 1, "model": ...}`` at ref ``runtime/model``;
* ``{"type": "head", "version": 1, "model", "chunks": [chunk ids]}``;
* ``{"type": "chunk", "version": 1, "chunk_id", "model", "clean": true, "token_start", "token_end",
  "frames", "height", "width", "matrices": [{"key": {...}, "tensor": manifest id}]}``;
* ``{"type": "tensor", "version": 1, "context", "spec", "encoded": {"metadata", "payloads": {name: blob
  id}, "basis": basis id | null, "metrics"}}``;
* ``{"type": "snapshot", "version": 1, "model", "head", "metadata", "tensor_state": blob id}``.

The adaptive rank method (per-matrix energy-targeted ranks, basis versions) commits through the
lineage API this class inherits (:class:`reelcache_b200.lineage.LineageRuntime`); the static
``seal_chunk`` path encodes each matrix with a caller-chosen :class:`CodecSpec`.
"""

from __future__ import annotations

import threading
import time
from collections import OrderedDict
from dataclasses import dataclass, field
from typing import Any, Callable, Mapping, Sequence

import torch

from .errors import (CapacityError, ConfigurationError, IntegrityError, PendingError, QuarantinedError,
                     StateError, UnsupportedError)
from .execution import BoundedExecutor
from .lineage import LINEAGE_PREFIX, LineageRuntime
from .residency import HistoryLease, ResidencyPool
from .serialization import deserialize_tensors, serialize_tensors, tensor_nbytes
from .store import ObjectStore
from .types import CodecSpec, EncodedTensor, MatrixKey, ModelIdentity, TensorContext, json_copy

OPEN_ERROR_POLICIES = ("raise", "quarantine")
SNAPSHOT_CONTRACTS = ("clean_boundary", "conditioning", "execution", "rng", "latent", "vae")
BRANCH_PREFIX = "branches/"
SNAPSHOT_PREFIX = "snapshots/"


@dataclass(frozen=True)
class SnapshotState:
    snapshot_id: str
    metadata: dict
    tensors: dict
    rank_policy: Any = None
    rank_state: Any = None


@dataclass(frozen=True)
class RestoredState:
    snapshot_id: str
    branch_id: str
    head_id: str
    metadata: dict
    tensors: Mapping[str, torch.Tensor]


@dataclass
class _CommitState:
    branch_id: str
    parent: str
    staging_bytes: int
    phase: str = "queued"
    error: str | None = None
    result_id: str | None = None
    cancelled: bool = False
    started: float = field(default_factory=time.monotonic)


class PendingCommit:
    """Handle of an asynchronous ``submit_chunk`` publication."""

    def __init__(self, runtime: "KVRuntime", state: _CommitState, job):
        self._runtime = runtime
        self._state = state
        self._job = job

    def done(self) -> bool:
        return self._job.done()

    def cancel(self) -> bool:
        """Cancel before publication; returns False once the chunk is (being) published."""
        with self._runtime._lock:
            if self._state.phase in ("ready", "published"):
                return False
            self._state.cancelled = True
        return True

    def status(self) -> dict:
        return {"branch_id": self._state.branch_id, "parent": self._state.parent, "phase": self._state.phase,
                "error": self._state.error, "result": self._state.result_id,
                "staging_bytes": self._state.staging_bytes}

    def result(self, timeout: float | None = None) -> str:
        return self._job.result(timeout)


class StreamingChunk:
    """Layer-wise publication of one chunk: ``add`` encodes and stores each matrix as it arrives (the
    tensor objects are pinned by a staging lease), ``commit`` publishes the chunk atomically, ``abort``
    drops it. The branch accepts no other commit until then."""

    def __init__(self, runtime: "KVRuntime", branch_id: str, chunk_id: Any, contexts: Mapping[MatrixKey, TensorContext],
                 specs: Mapping[MatrixKey, CodecSpec], head_id: str, chunks: list, reuse_threshold):
        self._runtime = runtime
        self.branch_id = branch_id
        self.chunk_id = chunk_id
        self._contexts = dict(contexts)
        self._specs = dict(specs)
        self._head_id = head_id
        self._chunks = chunks
        self._reuse = reuse_threshold
        self._records: dict[MatrixKey, str] = {}
        self._leases = []
        self._state = "open"
        self._lock = threading.Lock()

    @property
    def state(self) -> str:
        return self._state

    def add(self, key: MatrixKey, tensor: torch.Tensor) -> None:
        with self._lock:
            if self._state != "open":
                raise StateError(f"streaming chunk is {self._state}")
            if key not in self._contexts:
                raise ConfigurationError("matrix key is outside the chunk's contexts")
            if key in self._records:
                raise ConfigurationError("matrix already added to this chunk")
            object_id = self._runtime._encode_and_store(key, tensor, self._contexts[key], self._specs[key],
                                                        self._chunks, self._reuse)
            self._leases.append(self._runtime.store.lease(object_id, purpose="staging", verify=False))
            self._records[key] = object_id

    def commit(self, chunk_id: Any = None) -> str:
        with self._lock:
            if self._state != "open":
                raise StateError(f"streaming chunk is {self._state}")
            if chunk_id is not None and chunk_id != self.chunk_id:
                raise ConfigurationError("commit chunk_id differs from the opened chunk")
            if set(self._records) != set(self._runtime._keys):
                raise StateError("streaming chunk is missing matrices")
            try:
                chunk = self._runtime._publish(self.branch_id, self.chunk_id, self._head_id, self._records,
                                               self._contexts)
            finally:
                self._release()
            self._state = "committed"
            return chunk

    def abort(self) -> None:
        with self._lock:
            if self._state == "open":
                self._release()
                self._state = "aborted"

    def _release(self):
        for lease in self._leases:
            lease.release()
        self._leases.clear()
        with self._runtime._lock:
            self._runtime._streams.discard(self.branch_id)


class KVRuntime(LineageRuntime):
    """Durable branches of chunked KV matrices over one content-addressed store (see module docstring).

    ``max_resident_bytes`` bounds decoded history leases; ``executor`` (a :class:`BoundedExecutor`) runs
    ``submit_chunk`` publications; ``encoder``/``decoder`` replace the codec functions
    (``codecs.encode_tensor`` / ``codecs.decode_tensor`` signatures). ``verify_reads`` hash-checks every
    object read for use; ``on_open_error="quarantine"`` lists damaged heads in :attr:`quarantined` and lets
    every other head work (their loads raise :class:`QuarantinedError`). ``history_read_ahead_bytes``
    bounds payloads read ahead for sequential ``acquire_history`` calls (layer-major, K before V).
    """

    HISTORY_READ_AHEAD_BYTES = 512 << 20

    def __init__(self, root, model: ModelIdentity, *, max_resident_bytes: int = 1 << 30,
                 max_store_bytes: int | None = None, encoder: Callable[..., EncodedTensor] | None = None,
                 decoder: Callable[..., torch.Tensor] | None = None, executor: Any = None,
                 encode_concurrency: int = 1, encode_workspace_bytes: int = 0,
                 max_pending_source_bytes: int = 1 << 30, verify_reads: bool = False, prefit=None,
                 audit_on_open: bool | None = None, on_open_error: str = "raise",
                 verify_references: bool | None = None, history_read_ahead_bytes: int | None = None,
                 registry=None) -> None:
        if not isinstance(model, ModelIdentity):
            raise ConfigurationError("runtime model must be a ModelIdentity")
        if on_open_error not in OPEN_ERROR_POLICIES:
            raise ConfigurationError(f"on_open_error must be one of {OPEN_ERROR_POLICIES}")
        if audit_on_open is not None and type(audit_on_open) is not bool:
            raise ConfigurationError("audit_on_open must be a bool or None (follow verify_reads)")
        if history_read_ahead_bytes is not None and (type(history_read_ahead_bytes) is not int
                                                     or history_read_ahead_bytes < 0):
            raise ConfigurationError("history_read_ahead_bytes must be a nonnegative integer or None")
        if executor is not None and not callable(getattr(executor, "submit", None)):
            raise ConfigurationError("executor must implement bounded submit")
        if type(encode_concurrency) is not int or encode_concurrency < 1:
            raise ConfigurationError("encode_concurrency must be a positive integer")
        if encode_concurrency > 1 and (not isinstance(executor, BoundedExecutor) or not encode_workspace_bytes):
            raise ConfigurationError("parallel encoding requires BoundedExecutor and a positive workspace reservation")
        if type(max_pending_source_bytes) is not int or max_pending_source_bytes < 0:
            raise ConfigurationError("max_pending_source_bytes must be a nonnegative integer")
        from .codecs import decode_tensor, encode_tensor
        self.encoder = encode_tensor if encoder is None else encoder
        self.decoder = decode_tensor if decoder is None else decoder
        if not callable(self.encoder) or not callable(self.decoder):
            raise ConfigurationError("encoder and decoder must be callable")
        self.executor = executor
        self.prefit = prefit
        self.encode_concurrency = encode_concurrency
        self.encode_workspace_bytes = encode_workspace_bytes
        self.max_pending_source_bytes = max_pending_source_bytes
        self._pending_source_bytes = 0
        self.residency = ResidencyPool(max_resident_bytes)
        store = ObjectStore(root, max_bytes=max_store_bytes, verify_reads=verify_reads,
                            verify_references=verify_references,
                            on_damage="keep" if on_open_error == "quarantine" else "raise")
        super().__init__(store, model, registry=registry)
        self.verify_reads = verify_reads
        self.audit_on_open = verify_reads if audit_on_open is None else audit_on_open
        self.on_open_error = on_open_error
        self.history_read_ahead_bytes = (self.HISTORY_READ_AHEAD_BYTES if history_read_ahead_bytes is None
                                         else history_read_ahead_bytes)
        self._keys = tuple(MatrixKey(layer, target) for layer in range(model.layers) for target in ("K", "V"))
        self._key_index = {key: i for i, key in enumerate(self._keys)}
        self._pending: set[str] = set()
        self._streams: set[str] = set()
        self._async: dict[str, _CommitState] = {}
        self._async_failures: dict[str, _CommitState] = {}
        self._async_counts = {"submitted": 0, "published": 0, "failed": 0, "cancelled": 0}
        self._quarantine: dict[str, tuple[str, str]] = {}
        self._tracks: OrderedDict = OrderedDict()
        self._window = None
        self._ra_stats = {"windows": 0, "taken": 0, "taken_bytes": 0, "dropped": 0}
        self._closed = False
        try:
            with self.store.transaction():
                identity = self.store.get_ref("runtime/model")
                if identity is None:
                    if self.store.list_refs():
                        raise IntegrityError("runtime identity is missing from a populated store")
                    identity = self.store.put_manifest({"type": "model", "version": 1, "model": model.to_dict()})
                    self.store.set_ref("runtime/model", identity, expected=None)
                else:
                    self._same_model(self._typed(identity, "model").get("model"))
            for name, head, error in self._check_heads():
                if on_open_error == "raise":
                    raise IntegrityError(f"damaged head {name}: {error}")
                self._quarantine[name] = (head, error)
        except BaseException:
            self.store.close()
            self.residency.close()
            raise

    # -- validation helpers -------------------------------------------------------------------------------------

    def _open(self):
        if self._closed:
            raise StateError("runtime is closed")

    def _same_model(self, data):
        if data != self.model.to_dict():
            raise IntegrityError("stored object belongs to another model identity")

    def _typed(self, object_id: str, kind: str) -> dict:
        self._check_quarantined(object_id)
        data = self.store.get_manifest(object_id)
        versions = {1, 2} if kind == "chunk" else {1}
        if data.get("type") != kind or data.get("version") not in versions:
            raise IntegrityError(f"unsupported {kind} manifest")
        return data

    def _check_quarantined(self, object_id: str):
        for name, (head, error) in self._quarantine.items():
            if head == object_id:
                raise QuarantinedError(f"{name} is quarantined: {error}")

    @staticmethod
    def _branch_name(branch_id: str) -> str:
        if (not isinstance(branch_id, str) or not branch_id or "\x00" in branch_id or "/" in branch_id
                or branch_id in (".", "..")):
            raise ConfigurationError("branch_id must be a nonempty single-component name")
        return BRANCH_PREFIX + branch_id

    @staticmethod
    def _chunk_id(chunk_id: Any) -> None:
        if (not isinstance(chunk_id, str) or not chunk_id) and (type(chunk_id) is not int or chunk_id < 0):
            raise ConfigurationError("chunk_id must be a nonempty string or nonnegative integer")

    def _ready(self, branch_id: str) -> str:
        self._open()
        name = self._branch_name(branch_id)
        if branch_id in self._pending:
            raise PendingError(f"branch has an uncommitted chunk: {branch_id}")
        head = self.store.get_ref(name)
        if head is None:
            raise StateError(f"branch does not exist: {branch_id}")
        return head

    def _check_heads(self):
        """(ref name, head, error) of every damaged branch / snapshot / lineage head."""
        damaged = []
        refs = {**self.store.list_refs(BRANCH_PREFIX), **self.store.list_refs(SNAPSHOT_PREFIX)}
        for name, head in refs.items():
            try:
                if name.startswith(BRANCH_PREFIX):
                    self._load_head(head)
                else:
                    self._snapshot_record(head)
                self.store.verify(head) if self.audit_on_open else self.store.check(head)
            except (IntegrityError, ConfigurationError) as error:
                damaged.append((name, head, str(error)))
        for name, head in self.store.list_refs(LINEAGE_PREFIX).items():
            try:
                self.store.verify(head) if self.audit_on_open else self.store.check(head)
            except IntegrityError as error:
                damaged.append((name, head, str(error)))
        return damaged

    # -- heads and chunks ---------------------------------------------------------------------------------------

    def _load_head(self, head_id: str) -> list[dict]:
        head = self._typed(head_id, "head")
        self._same_model(head.get("model"))
        ids = head.get("chunks")
        if not isinstance(ids, list) or any(not isinstance(i, str) for i in ids):
            raise IntegrityError("invalid branch chunk sequence")
        chunks, end, names, geometry = [], 0, set(), None
        for chunk_object in ids:
            chunk = self._typed(chunk_object, "chunk")
            try:
                self._same_model(chunk.get("model"))
                if chunk["version"] != 1:
                    raise UnsupportedError("adaptive (version 2) chunks are read through the lineage API")
                fields = ("token_start", "token_end", "frames", "height", "width")
                if any(type(chunk.get(f)) is not int for f in fields) or chunk["token_start"] != end \
                        or chunk["token_end"] != end + chunk["frames"] * chunk["height"] * chunk["width"]:
                    raise IntegrityError("branch history has a gap, overlap or invalid geometry")
                if chunk["chunk_id"] in names or chunk.get("clean") is not True:
                    raise IntegrityError("branch contains duplicate or unclean chunks")
                if geometry is not None and geometry != (chunk["height"], chunk["width"]):
                    raise IntegrityError("spatial geometry changes within a branch")
                geometry = (chunk["height"], chunk["width"])
                names.add(chunk["chunk_id"])
                records = {}
                for entry in chunk["matrices"]:
                    key = MatrixKey.from_dict(entry["key"])
                    tensor = entry["tensor"]
                    if key in records or not isinstance(tensor, str) or not tensor.startswith("manifest:"):
                        raise IntegrityError("duplicate matrix or mutable tensor reference in a chunk")
                    records[key] = tensor
                if set(records) != set(self._keys):
                    raise IntegrityError("committed chunk does not contain every layer's K and V")
            except (KeyError, TypeError, ValueError) as error:
                raise IntegrityError("invalid committed chunk") from error
            end = chunk["token_end"]
            chunks.append({**chunk, "object_id": chunk_object, "records": records})
        return chunks

    def _tensor_record(self, object_id: str) -> tuple[TensorContext, CodecSpec, dict]:
        data = self._typed(object_id, "tensor")
        try:
            return TensorContext.from_dict(data["context"]), CodecSpec.from_dict(data["spec"]), data["encoded"]
        except (KeyError, TypeError, ValueError) as error:
            raise IntegrityError("invalid tensor manifest") from error

    def _new_head(self, chunks: list[str]) -> str:
        return self.store.put_manifest({"type": "head", "version": 1, "model": self.model.to_dict(),
                                        "chunks": chunks}, references=chunks)

    def create_branch(self, branch_id: str) -> None:
        with self._lock:
            self._open()
            with self.store.transaction():
                name = self._branch_name(branch_id)
                if self.store.get_ref(name) is not None:
                    raise StateError(f"branch already exists: {branch_id}")
                self.store.set_ref(name, self._new_head([]), expected=None)

    def branch_info(self, branch_id: str) -> dict[str, Any]:
        with self._lock, self.store.transaction():
            head = self._ready(branch_id)
            chunks = self._load_head(head)
            return {"branch_id": branch_id, "head_id": head, "chunk_ids": [c["chunk_id"] for c in chunks],
                    "chunk_manifests": [c["object_id"] for c in chunks], "token_start": 0,
                    "token_end": chunks[-1]["token_end"] if chunks else 0,
                    "chunk_id": chunks[-1]["chunk_id"] if chunks else None, "clean": True}

    def require_head(self, branch_id: str, expected_head: str) -> None:
        with self._lock:
            if self._ready(branch_id) != expected_head:
                raise StateError("branch head changed")

    def history_contexts(self, branch_id: str, key: MatrixKey) -> tuple[TensorContext, ...]:
        with self._lock, self.store.transaction():
            chunks = self._load_head(self._ready(branch_id))
            return tuple(self._tensor_record(c["records"][key])[0] for c in chunks)

    def history_specs(self, branch_id: str, key: MatrixKey) -> tuple[CodecSpec, ...]:
        with self._lock, self.store.transaction():
            chunks = self._load_head(self._ready(branch_id))
            return tuple(self._tensor_record(c["records"][key])[1] for c in chunks)

    # -- commits ------------------------------------------------------------------------------------------------

    def _validate(self, chunk_id, matrices, contexts, specs, chunks, *, require_matrices=True):
        self._chunk_id(chunk_id)
        if any(c["chunk_id"] == chunk_id for c in chunks):
            raise ConfigurationError("chunk_id already exists in the branch history")
        if set(contexts) != set(self._keys):
            raise ConfigurationError("contexts must cover every layer's K and V")
        if isinstance(specs, CodecSpec):
            specs = {key: specs for key in self._keys}
        if set(specs) != set(self._keys) or any(not isinstance(s, CodecSpec) for s in specs.values()):
            raise ConfigurationError("specs must be one CodecSpec or one per matrix")
        end = chunks[-1]["token_end"] if chunks else 0
        first = contexts[self._keys[0]]
        for key, context in contexts.items():
            if not isinstance(context, TensorContext) or context.key != key or context.model != self.model:
                raise ConfigurationError("context key/model differs from the runtime")
            if (context.token_start, context.frames, context.height, context.width) != \
                    (first.token_start, first.frames, first.height, first.width):
                raise ConfigurationError("chunk positions or geometry disagree across matrices")
        if first.token_start != end:
            raise ConfigurationError(f"chunk must start at the branch end ({end})")
        if chunks and (chunks[-1]["height"], chunks[-1]["width"]) != (first.height, first.width):
            raise ConfigurationError("spatial geometry changes within a branch")
        if require_matrices:
            if set(matrices) != set(self._keys):
                raise ConfigurationError("matrices must cover every layer's K and V")
            for key, tensor in matrices.items():
                if not isinstance(tensor, torch.Tensor) or tuple(tensor.shape) != contexts[key].shape:
                    raise ConfigurationError(f"matrix {key} shape differs from its context")
        return specs

    def _parent_basis(self, chunks, key, rank):
        for chunk in reversed(chunks):
            _, spec, encoded = self._tensor_record(chunk["records"][key])
            if encoded.get("basis") and spec.rank == rank:
                data = self.store.get(encoded["basis"])
                channels = self.model.kv_channels
                return torch.frombuffer(bytearray(data), dtype=torch.float16).reshape(-1, channels)[:rank]
        return None

    def _encode_and_store(self, key, tensor, context, spec, chunks, reuse_threshold) -> str:
        basis = None
        if spec.kind != "raw" and reuse_threshold is not None and chunks:
            parent = self._parent_basis(chunks, key, spec.rank)
            if parent is not None:
                x = tensor.detach().double().cpu().reshape(context.shape)
                q = parent.double()
                error = torch.linalg.vector_norm(x - (x @ q.t()) @ q) / max(torch.linalg.vector_norm(x).item(), 1e-300)
                if float(error) <= reuse_threshold:
                    basis = parent
        encoded = self.encoder(tensor, context, spec, basis=basis) if spec.kind != "raw" else \
            self.encoder(tensor, context, spec)
        if not isinstance(encoded, EncodedTensor):
            raise IntegrityError("representation provider must return EncodedTensor")
        payloads = {name: self.store.put(payload) for name, payload in encoded.payloads.items()}
        basis_id = None if encoded.basis is None else self.store.put(encoded.basis, kind="basis")
        references = sorted(set(payloads.values()) | ({basis_id} if basis_id else set()))
        return self.store.put_manifest({"type": "tensor", "version": 1, "context": context.to_dict(),
                                        "spec": spec.to_dict(),
                                        "encoded": {"metadata": json_copy(encoded.metadata), "payloads": payloads,
                                                    "basis": basis_id,
                                                    "metrics": json_copy(dict(encoded.metrics or {}))}},
                                       references=references)

    def _publish(self, branch_id, chunk_id, expected_head, records: Mapping[MatrixKey, str], contexts) -> str:
        with self._lock:
            self._open()
            with self.store.transaction():
                head = self.store.get_ref(self._branch_name(branch_id))
                if head != expected_head:
                    raise StateError("branch head changed during the commit")
                chunks = self._load_head(head)
                context = contexts[self._keys[0]]
                data = {"type": "chunk", "version": 1, "chunk_id": chunk_id, "model": self.model.to_dict(),
                        "clean": True, "token_start": context.token_start, "token_end": context.token_end,
                        "frames": context.frames, "height": context.height, "width": context.width,
                        "matrices": [{"key": key.to_dict(), "tensor": records[key]} for key in self._keys]}
                chunk = self.store.put_manifest(data, references=[records[key] for key in self._keys])
                self.store.set_ref(self._branch_name(branch_id),
                                   self._new_head([c["object_id"] for c in chunks] + [chunk]), expected=head)
                return chunk

    def seal_chunk(self, branch_id: str, chunk_id: Any, matrices: Mapping[MatrixKey, torch.Tensor],
                   contexts: Mapping[MatrixKey, TensorContext], specs=CodecSpec(), *, clean: bool = True,
                   reuse_threshold: float | None = None, rank_policy=None, staging_bytes: int | None = None) -> str:
        """Encode every matrix of one clean chunk and publish it (CAS on the branch head)."""
        if clean is not True:
            raise ConfigurationError("only clean chunks are committed")
        if rank_policy is not None:
            raise UnsupportedError("adaptive rank policies commit through the lineage API (commit_node)")
        with self._lock:
            head = self._ready(branch_id)
            if branch_id in self._streams:
                raise PendingError(f"branch has an open streaming chunk: {branch_id}")
            with self.store.transaction():
                chunks = self._load_head(head)
            specs = self._validate(chunk_id, matrices, contexts, specs, chunks)
            self._pending.add(branch_id)
        leases = []
        try:
            records = {}
            for key in self._keys:
                records[key] = self._encode_and_store(key, matrices[key], contexts[key], specs[key], chunks,
                                                      reuse_threshold)
                leases.append(self.store.lease(records[key], purpose="staging", verify=False))
            with self._lock:
                self._pending.discard(branch_id)
            return self._publish(branch_id, chunk_id, head, records, contexts)
        finally:
            with self._lock:
                self._pending.discard(branch_id)
            for lease in leases:
                lease.release()

    def open_chunk(self, branch_id: str, chunk_id: Any, contexts: Mapping[MatrixKey, TensorContext],
                   specs=CodecSpec(), *, reuse_threshold: float | None = None) -> StreamingChunk:
        """Reserve ``branch_id`` for a layer-wise :class:`StreamingChunk`."""
        with self._lock:
            head = self._ready(branch_id)
            if branch_id in self._streams:
                raise PendingError(f"branch has an open streaming chunk: {branch_id}")
            with self.store.transaction():
                chunks = self._load_head(head)
            specs = self._validate(chunk_id, {}, contexts, specs, chunks, require_matrices=False)
            self._streams.add(branch_id)
        return StreamingChunk(self, branch_id, chunk_id, contexts, specs, head, chunks, reuse_threshold)

    def submit_chunk(self, branch_id: str, chunk_id: Any, matrices, contexts, specs=CodecSpec(), *,
                     reuse_threshold: float | None = None, timeout: float | None = None) -> PendingCommit:
        """Copy the inputs to host memory and enqueue the publication on the executor."""
        if self.executor is None:
            raise ConfigurationError("submit_chunk requires an executor")
        with self._lock:
            self._check_async_errors()
            head = self._ready(branch_id)
            if branch_id in self._streams:
                raise PendingError(f"branch has an open streaming chunk: {branch_id}")
            with self.store.transaction():
                chunks = self._load_head(head)
            specs = self._validate(chunk_id, matrices, contexts, specs, chunks)
            required = sum(t.numel() * t.element_size() for t in matrices.values())
            if self._pending_source_bytes + required > self.max_pending_source_bytes:
                raise CapacityError("pending source bytes exceed max_pending_source_bytes")
            owned = {key: t.detach().to("cpu", copy=True) for key, t in matrices.items()}
            state = _CommitState(branch_id, head, required)
            self._async[branch_id] = state
            self._pending.add(branch_id)
            self._pending_source_bytes += required
            self._async_counts["submitted"] += 1

        def run():
            try:
                if state.cancelled:
                    raise StateError("commit cancelled")
                state.phase = "encoding"
                records, leases = {}, []
                try:
                    for key in self._keys:
                        if state.cancelled:
                            raise StateError("commit cancelled")
                        records[key] = self._encode_and_store(key, owned[key], contexts[key], specs[key], chunks,
                                                              reuse_threshold)
                        leases.append(self.store.lease(records[key], purpose="staging", verify=False))
                    with self._lock:
                        if state.cancelled:
                            raise StateError("commit cancelled")
                        state.phase = "ready"
                        self._pending.discard(branch_id)
                    chunk = self._publish(branch_id, chunk_id, head, records, contexts)
                finally:
                    for lease in leases:
                        lease.release()
                state.phase, state.result_id = "published", chunk
                with self._lock:
                    self._async_counts["published"] += 1
                return chunk
            except BaseException as error:
                with self._lock:
                    state.phase = "cancelled" if state.cancelled else "failed"
                    state.error = f"{type(error).__name__}: {error}"
                    self._async_counts["cancelled" if state.cancelled else "failed"] += 1
                    if not state.cancelled:
                        self._async_failures[branch_id] = state
                raise
            finally:
                with self._lock:
                    self._pending.discard(branch_id)
                    self._async.pop(branch_id, None)
                    self._pending_source_bytes -= required

        try:
            job = self.executor.submit(run, staging_bytes=required, label=f"commit:{branch_id}:{chunk_id}",
                                       block=timeout is not None, timeout=timeout)
        except BaseException:
            with self._lock:
                self._pending.discard(branch_id)
                self._async.pop(branch_id, None)
                self._pending_source_bytes -= required
            raise
        return PendingCommit(self, state, job)

    def _check_async_errors(self):
        if self._async_failures:
            detail = "; ".join(f"{b}: {s.error}" for b, s in self._async_failures.items())
            self._async_failures.clear()
            raise StateError(f"asynchronous commits failed: {detail}")

    def async_stats(self) -> dict:
        with self._lock:
            return {**self._async_counts, "pending": len(self._async),
                    "pending_source_bytes": self._pending_source_bytes}

    # -- snapshots ----------------------------------------------------------------------------------------------

    def _snapshot_metadata(self, metadata, chunks, *, stored=False) -> dict:
        error = IntegrityError if stored else ConfigurationError
        if not isinstance(metadata, Mapping):
            raise error("snapshot metadata must be a mapping")
        copied = json_copy(metadata)
        if not set(SNAPSHOT_CONTRACTS) <= set(copied):
            raise error("snapshot metadata must record boundary/conditioning/execution/RNG/latent/VAE contracts")
        boundary = copied["clean_boundary"]
        end = chunks[-1]["token_end"] if chunks else 0
        last = chunks[-1]["chunk_id"] if chunks else None
        if (not isinstance(boundary, dict) or "chunk_id" not in boundary or boundary.get("chunk_id") != last
                or type(boundary.get("token_end")) is not int or boundary["token_end"] != end
                or boundary.get("clean", True) is not True):
            raise error("snapshot boundary does not match the committed clean history")
        if copied.get("pending", False) or (isinstance(copied["execution"], dict)
                                            and copied["execution"].get("pending", False)):
            raise PendingError("pending native execution cannot be snapshotted")
        for name in SNAPSHOT_CONTRACTS[1:]:
            if copied[name] is None:
                raise error(f"snapshot {name} contract must be explicit, not null")
        return copied

    def snapshot(self, branch_id: str, *, metadata: Mapping[str, Any],
                 tensors: Mapping[str, torch.Tensor] | None = None) -> str:
        """Persist a clean history root with portable metadata and named tensor state."""
        with self._lock, self.store.transaction():
            head = self._ready(branch_id)
            chunks = self._load_head(head)
            checked = self._snapshot_metadata(metadata, chunks)
            state = self.store.put(serialize_tensors({} if tensors is None else dict(tensors)))
            snapshot_id = self.store.put_manifest({"type": "snapshot", "version": 1, "model": self.model.to_dict(),
                                                   "head": head, "metadata": checked, "tensor_state": state},
                                                  references=[head, state])
            self.store.set_ref(SNAPSHOT_PREFIX + snapshot_id.split(":")[1], snapshot_id)
            return snapshot_id

    def _snapshot_record(self, snapshot_id: str) -> tuple[dict, dict]:
        data = self._typed(snapshot_id, "snapshot")
        self._same_model(data.get("model"))
        try:
            if not isinstance(data["tensor_state"], str) or not data["tensor_state"].startswith("blob:"):
                raise IntegrityError("snapshot tensor state must be an immutable blob")
            chunks = self._load_head(data["head"])
            return data, self._snapshot_metadata(data["metadata"], chunks, stored=True)
        except (KeyError, TypeError, ValueError) as error:
            raise IntegrityError("invalid snapshot record") from error

    def load_snapshot(self, snapshot_id: str) -> SnapshotState:
        with self._lock, self.store.transaction():
            self._open()
            data, metadata = self._snapshot_record(snapshot_id)
            return SnapshotState(snapshot_id, metadata, deserialize_tensors(self.store.get(data["tensor_state"])))

    def _restore(self, snapshot_id, branch_id, *, new_only, validator, metadata_validator) -> RestoredState:
        for callback in (validator, metadata_validator):
            if callback is not None and not callable(callback):
                raise ConfigurationError("validators must be callable")
        with self._lock:
            self._open()
            name = self._branch_name(branch_id)
            if branch_id in self._pending or branch_id in self._streams:
                raise PendingError(f"branch has an uncommitted chunk: {branch_id}")
            with self.store.transaction():
                data, metadata = self._snapshot_record(snapshot_id)
                current = self.store.get_ref(name)
                if new_only and current is not None:
                    raise StateError(f"fork target branch already exists: {branch_id}")
            if metadata_validator is not None:
                if metadata_validator(RestoredState(snapshot_id, branch_id, data["head"], json_copy(metadata), {}))\
                        is not None:
                    raise ConfigurationError("metadata_validator must return None")
            tensors = deserialize_tensors(self.store.get(data["tensor_state"]))
            state = RestoredState(snapshot_id, branch_id, data["head"], metadata, tensors)
            if validator is not None and validator(state) is not None:
                raise ConfigurationError("validator must return None")
            with self.store.transaction():
                self.store.set_ref(name, data["head"], expected=current)
            return state

    def restore(self, snapshot_id: str, branch_id: str, *, validator=None, metadata_validator=None,
                rank_policy=None) -> RestoredState:
        """Point ``branch_id`` (new or existing) at the snapshot's head after validation (CAS)."""
        return self._restore(snapshot_id, branch_id, new_only=False, validator=validator,
                             metadata_validator=metadata_validator)

    def fork(self, snapshot_id: str, branch_id: str, *, validator=None, metadata_validator=None,
             rank_policy=None) -> RestoredState:
        """Like :meth:`restore`, but never replaces an existing branch."""
        return self._restore(snapshot_id, branch_id, new_only=True, validator=validator,
                             metadata_validator=metadata_validator)

    # -- history ------------------------------------------------------------------------------------------------

    def _encoded(self, encoded: Mapping[str, Any], read_ahead=None) -> EncodedTensor:
        def read(object_id):
            data = None if read_ahead is None else read_ahead.take(object_id)
            if data is not None:
                self._ra_stats["taken"] += 1
                self._ra_stats["taken_bytes"] += len(data)
                return data
            return self.store.get(object_id)

        payloads = {name: read(object_id) for name, object_id in encoded["payloads"].items()}
        basis = None if encoded.get("basis") is None else read(encoded["basis"])
        return EncodedTensor(encoded["metadata"], payloads, basis=basis, metrics=encoded.get("metrics") or {})

    def _columns(self, columns, channels):
        if columns is None:
            return slice(0, channels), channels
        if isinstance(columns, tuple):
            if len(columns) != 2:
                raise ConfigurationError("tuple columns must be a (start, stop) interval; use a list for indices")
            columns = slice(*columns)
        if isinstance(columns, list):
            if (not columns or len(set(columns)) != len(columns)
                    or any(type(c) is not int or not 0 <= c < channels for c in columns)):
                raise ConfigurationError("channel indices must be nonempty, unique, and inside the canonical domain")
            return list(columns), len(columns)
        if not isinstance(columns, slice) or columns.step not in (None, 1):
            raise ConfigurationError("columns must be a contiguous slice or unique channel indices")
        start = 0 if columns.start is None else columns.start
        stop = channels if columns.stop is None else columns.stop
        if type(start) is not int or type(stop) is not int or not 0 <= start < stop <= channels:
            raise ConfigurationError("channel slice is outside the canonical KV domain")
        return slice(start, stop), stop - start

    def _read_ahead_for(self, head, start, end, key, chunks, covering):
        """Sequential-key detection: the second consecutive key of one (head, range) opens a window that
        reads the following keys' payloads ahead."""
        if not self.history_read_ahead_bytes:
            return None
        track = (head, start, end)
        index = self._key_index[key]
        previous = self._tracks.pop(track, None)
        self._tracks[track] = index
        while len(self._tracks) > 64:
            self._tracks.popitem(last=False)
        if self._window is not None and self._window[0] == track:
            return self._window[1]
        if previous is None or previous + 1 != index:
            return None
        self._drop_read_ahead()
        ids = []
        for following in self._keys[index + 1:]:
            for chunk in covering:
                _, _, encoded = self._tensor_record(chunk["records"][following])
                ids.extend(encoded["payloads"].values())
                if encoded.get("basis"):
                    ids.append(encoded["basis"])
        window = self.store.read_ahead(ids, max_bytes=self.history_read_ahead_bytes)
        self._window = (track, window)
        self._ra_stats["windows"] += 1
        return window

    def _drop_read_ahead(self):
        if self._window is not None:
            self._window[1].close()
            self._window = None
            self._ra_stats["dropped"] += 1

    def read_ahead_stats(self) -> dict[str, Any]:
        return dict(self._ra_stats, active=self._window is not None)

    def acquire_history(self, branch_id: str, key: MatrixKey, *, token_start: int | None = None,
                        token_end: int | None = None, device: Any = "cpu", dtype: Any = None, columns: Any = None,
                        column_groups: Any = None, decoder: Callable[..., torch.Tensor] | None = None,
                        head_id: str | None = None) -> HistoryLease:
        """Decode the key's history over ``[token_start, token_end)`` into an active residency lease."""
        if not isinstance(key, MatrixKey) or key not in self._key_index:
            raise ConfigurationError("history key is outside the model")
        if column_groups is not None:
            raise UnsupportedError("column_groups are not supported; pass columns")
        decode = self.decoder if decoder is None else decoder
        with self._lock, self.store.transaction():
            if head_id is None:
                head = self._ready(branch_id)
            else:
                self._open()
                head = head_id
            chunks = self._load_head(head)
            end_all = chunks[-1]["token_end"] if chunks else 0
            start = 0 if token_start is None else token_start
            end = end_all if token_end is None else token_end
            if type(start) is not int or type(end) is not int or not 0 <= start < end <= end_all:
                raise ConfigurationError("token range is not covered by the committed history")
            covering = [c for c in chunks if c["token_end"] > start and c["token_start"] < end]
            records = [(c, self._tensor_record(c["records"][key])) for c in covering]
            window = self._read_ahead_for(head, start, end, key, chunks, covering)
        context0 = records[0][1][0]
        out_dtype = getattr(torch, context0.dtype) if dtype is None else dtype
        selector, width = self._columns(columns, self.model.kv_channels)
        nbytes = tensor_nbytes((end - start, width), str(out_dtype).removeprefix("torch."))

        def load():
            parts = []
            for chunk, (context, spec, encoded) in records:
                matrix = decode(self._encoded(encoded, window), device=device, dtype=out_dtype)
                lo = max(start, chunk["token_start"]) - chunk["token_start"]
                hi = min(end, chunk["token_end"]) - chunk["token_start"]
                parts.append(matrix[lo:hi, selector])
            return torch.cat(parts).contiguous() if len(parts) > 1 else parts[0].contiguous()

        return self.residency.acquire(nbytes, load, metadata={"head": head, "key": key.to_dict(),
                                                              "token_start": start, "token_end": end})

    def history_packet(self, branch_id: str, key: MatrixKey, *, token_start: int, token_end: int) -> EncodedTensor:
        """The committed packet of exactly one chunk (for decoding elsewhere)."""
        if not isinstance(key, MatrixKey) or key not in self._key_index:
            raise ConfigurationError("history key is outside the model")
        with self._lock, self.store.transaction():
            chunks = self._load_head(self._ready(branch_id))
            matches = [c for c in chunks if c["token_start"] == token_start and c["token_end"] == token_end]
            if len(matches) != 1:
                raise StateError("requested range is not exactly one committed chunk")
            return self._encoded(self._tensor_record(matches[0]["records"][key])[2])

    # -- lifecycle ----------------------------------------------------------------------------------------------

    @property
    def resident_bytes(self) -> int:
        return self.residency.resident_bytes

    @property
    def active_leases(self) -> int:
        return self.residency.active_leases

    @property
    def quarantined(self) -> dict[str, str]:
        return {name: error for name, (_, error) in self._quarantine.items()}

    def audit(self, *, deep: bool = True, quarantine: bool = False) -> dict[str, str]:
        """Check every head (``deep``: hash every reachable object); returns {ref name: error}.
        ``quarantine=True`` adds newly damaged heads to :attr:`quarantined`."""
        with self._lock:
            self._open()
            saved = self.audit_on_open
            self.audit_on_open = deep
            try:
                damaged = self._check_heads()
            finally:
                self.audit_on_open = saved
            if quarantine:
                for name, head, error in damaged:
                    self._quarantine[name] = (head, error)
            return {name: error for name, _, error in damaged}

    def delete_branch(self, branch_id: str) -> None:
        with self._lock:
            with self.store.transaction():
                name = self._branch_name(branch_id)
                if branch_id in self._streams:
                    raise PendingError(f"branch has an open streaming chunk: {branch_id}")
                head = self.store.get_ref(name)
                if head is None or branch_id in self._pending:
                    self._ready(branch_id)
                self.store.delete_ref(name, expected=head)
            self._quarantine.pop(name, None)

    def delete_snapshot(self, snapshot_id: str) -> None:
        name = SNAPSHOT_PREFIX + snapshot_id.split(":")[1]
        with self._lock:
            self._open()
            with self.store.transaction():
                if name not in self._quarantine:
                    self._snapshot_record(snapshot_id)
                self.store.delete_ref(name, expected=snapshot_id)
            self._quarantine.pop(name, None)

    def collect_garbage(self) -> dict[str, Any]:
        with self._lock:
            self._open()
            self._drop_read_ahead()
            result = self.store.collect_garbage()
            self.drop_manifest_caches()
            return result

    gc = collect_garbage

    def close(self) -> None:
        with self._lock:
            if self._closed:
                return
            if self._pending or self._streams or self._lineage_pending:
                raise PendingError("cannot close a runtime with encoding still in flight")
            self._check_async_errors()
            self._closed = True
            self._drop_read_ahead()
            self.residency.close()
            self.store.close()

    def __enter__(self) -> "KVRuntime":
        self._open()
        return self

    def __exit__(self, *args: Any) -> None:
        self.close()


__all__ = ["KVRuntime", "PendingCommit", "RestoredState", "SnapshotState", "StreamingChunk", "HistoryLease"]
