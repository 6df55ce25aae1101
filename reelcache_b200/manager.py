"""KVRuntime: durable, branchable chunk histories of full-width KV matrices on one host (the runtime the
CPU demo drives; reference counterpart: reelcache/manager.py:357-2444).

Model of the state
------------------
* A **branch** is a mutable ref ``branches/<id>`` naming an immutable **head** manifest, which lists the
  branch's chunk manifests oldest first. A **chunk** lists one **tensor** manifest per (layer, K/V) matrix.
  Every commit writes the new chunk and a new head, then moves the branch ref with compare-and-set, so a
  concurrent writer can fail but never drop history.
* A **snapshot** (ref ``snapshots/<digest>``) pins one head together with JSON metadata (six named contracts)
  and one serialized blob of named tensors (RNG state, latents, ...). ``restore`` points a branch at a
  snapshot's head; ``fork`` does the same but only for a branch that does not exist yet.
* ``acquire_history`` decodes one matrix's history over a token range into a lease whose bytes are charged
  against ``max_resident_bytes``.

The manifest shapes are the reference's (stores written by either implementation open in the other):

* ``{"type": "model", "version": 1, "model": ...}`` at ref ``runtime/model``;
* ``{"type": "head", "version": 1, "model", "chunks": [chunk ids]}``;
* ``{"type": "chunk", "version": 1, "chunk_id", "model", "clean": true, "token_start", "token_end",
  "frames", "height", "width", "matrices": [{"key": {...}, "tensor": manifest id}]}``;
* ``{"type": "tensor", "version": 1, "context", "spec", "encoded": {"metadata", "payloads": {name: blob
  id}, "basis": basis id | null, "metrics"}}``;
* ``{"type": "snapshot", "version": 1, "model", "head", "metadata", "tensor_state": blob id}``.

Energy-targeted, per-matrix ranks (the rank method, basis versions) commit through the lineage API this
class inherits (:class:`reelcache_b200.lineage.LineageRuntime`); ``seal_chunk`` and friends encode every
matrix with a caller-chosen :class:`CodecSpec`.

Concurrency: one re-entrant lock (inherited) guards the bookkeeping; encoding runs outside it. A branch is
*busy* while a commit of any kind (sealed, streaming or asynchronous) is between reservation and
publication, and every other commit, restore or delete of that branch raises :class:`PendingError`.
"""

from __future__ import annotations

import threading
import time
from collections import OrderedDict
from dataclasses import dataclass, field
from typing import Any, Callable, Mapping

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
#: Metadata sections every snapshot must carry (all but the boundary may hold any non-null JSON value).
SNAPSHOT_CONTRACTS = ("clean_boundary", "conditioning", "execution", "rng", "latent", "vae")
BRANCH_PREFIX = "branches/"
SNAPSHOT_PREFIX = "snapshots/"
MODEL_REF = "runtime/model"
_GEOMETRY = ("token_start", "token_end", "frames", "height", "width")


# -- argument checks ---------------------------------------------------------------------------------------------

def _nonnegative_int(value) -> bool:
    return type(value) is int and value >= 0


def _positive_int(value) -> bool:
    return type(value) is int and value > 0


#: (argument, accepts, what it must be); ``None`` is accepted where the argument means "use the default".
_CONSTRUCTOR_RULES = (
    ("on_open_error", lambda v: v in OPEN_ERROR_POLICIES, f"one of {OPEN_ERROR_POLICIES}"),
    ("audit_on_open", lambda v: v is None or type(v) is bool, "True, False or None (None follows verify_reads)"),
    ("history_read_ahead_bytes", lambda v: v is None or _nonnegative_int(v), "a byte count >= 0, or None"),
    ("executor", lambda v: v is None or callable(getattr(v, "submit", None)), "None or an object with submit()"),
    ("encode_concurrency", _positive_int, "an int >= 1"),
    ("max_pending_source_bytes", _nonnegative_int, "a byte count >= 0"),
)


def _check_arguments(rules, values: Mapping[str, Any], owner: str) -> None:
    for name, accepts, wanted in rules:
        if not accepts(values[name]):
            raise ConfigurationError(f"{owner}: {name}={values[name]!r} is not {wanted}")


def _branch_ref(branch_id: Any) -> str:
    """``branches/<id>`` of a branch name that is one path component."""
    valid = isinstance(branch_id, str) and branch_id not in ("", ".", "..") and not (set(branch_id) & {"/", "\x00"})
    if not valid:
        raise ConfigurationError(f"branch name {branch_id!r} is not a single non-empty path component")
    return BRANCH_PREFIX + branch_id


def _check_chunk_id(chunk_id: Any) -> None:
    if (isinstance(chunk_id, str) and chunk_id) or _nonnegative_int(chunk_id):
        return
    raise ConfigurationError(f"chunk id {chunk_id!r} is neither a non-empty string nor an int >= 0")


def _snapshot_ref(snapshot_id: str) -> str:
    return SNAPSHOT_PREFIX + snapshot_id.split(":", 1)[1]


# -- parsed branch state -----------------------------------------------------------------------------------------

@dataclass(frozen=True)
class _Chunk:
    """One committed chunk of a branch, parsed from its manifest."""

    object_id: str
    chunk_id: Any
    token_start: int
    token_end: int
    frames: int
    height: int
    width: int
    records: Mapping[MatrixKey, str]     # tensor manifest of every (layer, K/V)

    def overlaps(self, start: int, end: int) -> bool:
        return self.token_start < end and start < self.token_end


@dataclass(frozen=True)
class _History:
    """A head and its chunks, contiguous from token 0."""

    head_id: str
    chunks: tuple[_Chunk, ...]

    @property
    def end(self) -> int:
        return self.chunks[-1].token_end if self.chunks else 0

    @property
    def last_chunk_id(self):
        return self.chunks[-1].chunk_id if self.chunks else None

    @property
    def grid(self) -> tuple[int, int] | None:
        return (self.chunks[-1].height, self.chunks[-1].width) if self.chunks else None

    def chunk_ids(self) -> list:
        return [c.chunk_id for c in self.chunks]

    def object_ids(self) -> list[str]:
        return [c.object_id for c in self.chunks]


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


# -- asynchronous commit bookkeeping -----------------------------------------------------------------------------

@dataclass
class _CommitState:
    branch_id: str
    parent: str
    staging_bytes: int
    phase: str = "queued"          # queued -> encoding -> ready -> published | failed | cancelled
    error: str | None = None
    result_id: str | None = None
    cancelled: bool = False
    started: float = field(default_factory=time.monotonic)


class _AsyncLedger:
    """Counts, in-flight states and unreported failures of ``submit_chunk`` publications, plus the source
    bytes they hold in host memory. Callers hold the runtime lock."""

    def __init__(self, max_source_bytes: int):
        self.max_source_bytes = max_source_bytes
        self.source_bytes = 0
        self.in_flight: dict[str, _CommitState] = {}
        self.failures: dict[str, _CommitState] = {}
        self.counts = {"submitted": 0, "published": 0, "failed": 0, "cancelled": 0}

    def admit(self, state: _CommitState) -> None:
        if self.source_bytes + state.staging_bytes > self.max_source_bytes:
            raise CapacityError(f"queued commits would hold {self.source_bytes + state.staging_bytes} source bytes, "
                                f"over max_pending_source_bytes={self.max_source_bytes}")
        self.in_flight[state.branch_id] = state
        self.source_bytes += state.staging_bytes
        self.counts["submitted"] += 1

    def settle(self, state: _CommitState, error: BaseException | None) -> None:
        if error is None:
            self.counts["published"] += 1
        else:
            state.phase = "cancelled" if state.cancelled else "failed"
            state.error = f"{type(error).__name__}: {error}"
            self.counts[state.phase] += 1
            if not state.cancelled:
                self.failures[state.branch_id] = state

    def release(self, state: _CommitState) -> None:
        if self.in_flight.get(state.branch_id) is state:
            del self.in_flight[state.branch_id]
            self.source_bytes -= state.staging_bytes

    def raise_failures(self) -> None:
        if self.failures:
            lines = [f"{branch}: {state.error}" for branch, state in self.failures.items()]
            self.failures.clear()
            raise StateError("earlier asynchronous commits failed -- " + "; ".join(lines))

    def stats(self) -> dict:
        return {**self.counts, "pending": len(self.in_flight), "pending_source_bytes": self.source_bytes}


class PendingCommit:
    """Handle of one ``submit_chunk`` publication running on the runtime's executor."""

    def __init__(self, runtime: "KVRuntime", state: _CommitState, job):
        self._runtime = runtime
        self._state = state
        self._job = job

    def done(self) -> bool:
        return self._job.done()

    def cancel(self) -> bool:
        """Ask the publication to stop; False once it has reached publication (``ready`` or later)."""
        with self._runtime._lock:
            if self._state.phase in ("ready", "published"):
                return False
            self._state.cancelled = True
            return True

    def status(self) -> dict:
        s = self._state
        return {"branch_id": s.branch_id, "parent": s.parent, "phase": s.phase, "error": s.error,
                "result": s.result_id, "staging_bytes": s.staging_bytes}

    def result(self, timeout: float | None = None) -> str:
        return self._job.result(timeout)


class StreamingChunk:
    """A chunk published layer by layer: ``add`` encodes and stores one matrix as soon as it exists (a staging
    lease keeps its objects alive until the chunk is published or dropped), ``commit`` publishes the whole chunk
    at once, ``abort`` drops it. The branch stays busy until one of the two."""

    def __init__(self, runtime: "KVRuntime", branch_id: str, chunk_id: Any, contexts: Mapping[MatrixKey, TensorContext],
                 specs: Mapping[MatrixKey, CodecSpec], history: _History, reuse_threshold):
        self._runtime = runtime
        self.branch_id = branch_id
        self.chunk_id = chunk_id
        self._contexts = dict(contexts)
        self._specs = dict(specs)
        self._history = history
        self._reuse = reuse_threshold
        self._stored: dict[MatrixKey, str] = {}
        self._leases = []
        self._state = "open"
        self._lock = threading.Lock()

    @property
    def state(self) -> str:
        return self._state

    def _require_open(self) -> None:
        if self._state != "open":
            raise StateError(f"chunk {self.chunk_id!r} of branch {self.branch_id!r} is already {self._state}")

    def add(self, key: MatrixKey, tensor: torch.Tensor) -> None:
        with self._lock:
            self._require_open()
            if key not in self._contexts:
                raise ConfigurationError(f"{key} has no context in this chunk")
            if key in self._stored:
                raise ConfigurationError(f"{key} was already added to this chunk")
            object_id = self._runtime._store_matrix(key, tensor, self._contexts[key], self._specs[key],
                                                    self._history, self._reuse)
            self._leases.append(self._runtime.store.lease(object_id, purpose="staging", verify=False))
            self._stored[key] = object_id

    def commit(self, chunk_id: Any = None) -> str:
        with self._lock:
            self._require_open()
            if chunk_id is not None and chunk_id != self.chunk_id:
                raise ConfigurationError(f"this chunk was opened as {self.chunk_id!r}, not {chunk_id!r}")
            missing = [key for key in self._runtime._keys if key not in self._stored]
            if missing:
                raise StateError(f"{len(missing)} matrices were never added, first {missing[0]}")
            try:
                published = self._runtime._publish(self.branch_id, self.chunk_id, self._history.head_id,
                                                   self._stored, self._contexts)
            finally:
                self._finish()
            self._state = "committed"
            return published

    def abort(self) -> None:
        with self._lock:
            if self._state == "open":
                self._finish()
                self._state = "aborted"

    def _finish(self) -> None:
        while self._leases:
            self._leases.pop().release()
        self._runtime._release_branch(self.branch_id, "stream")


class _ReadAhead:
    """Payload read-ahead for histories read key after key (layer-major, K before V). The second consecutive
    key of one (head, token range) opens a window that reads the payloads of the keys after it, up to a byte
    budget; a request for another range drops the window."""

    MAX_TRACKS = 64

    def __init__(self, budget: int, keys: tuple[MatrixKey, ...]):
        self.budget = budget
        self.keys = keys
        self.position = {key: i for i, key in enumerate(keys)}
        self.last_key: OrderedDict = OrderedDict()     # (head, start, end) -> index of the last key read
        self.window = None                             # ((head, start, end), store read-ahead handle)
        self.stats = {"windows": 0, "taken": 0, "taken_bytes": 0, "dropped": 0}

    def window_for(self, runtime: "KVRuntime", track, key, covering: list[_Chunk]):
        if not self.budget:
            return None
        index = self.position[key]
        before = self.last_key.pop(track, None)
        self.last_key[track] = index
        if len(self.last_key) > self.MAX_TRACKS:
            self.last_key.popitem(last=False)
        if self.window is not None and self.window[0] == track:
            return self.window[1]
        if before is None or before != index - 1:
            return None
        self.drop()
        wanted = []
        for later in self.keys[index + 1:]:
            for chunk in covering:
                encoded = runtime._tensor_manifest(chunk.records[later])[2]
                wanted.extend(encoded["payloads"].values())
                if encoded.get("basis"):
                    wanted.append(encoded["basis"])
        self.window = (track, runtime.store.read_ahead(wanted, max_bytes=self.budget))
        self.stats["windows"] += 1
        return self.window[1]

    def take(self, window, object_id: str):
        data = None if window is None else window.take(object_id)
        if data is not None:
            self.stats["taken"] += 1
            self.stats["taken_bytes"] += len(data)
        return data

    def drop(self) -> None:
        if self.window is not None:
            self.window[1].close()
            self.window = None
            self.stats["dropped"] += 1


def _select_columns(columns, channels: int):
    """``(selector, width)`` of a column request: None (all), a ``(start, stop)`` tuple, a unit-step slice or a
    list of distinct channel indices."""
    if columns is None:
        return slice(0, channels), channels
    if isinstance(columns, list):
        valid = bool(columns) and len(set(columns)) == len(columns) and all(
            type(c) is int and 0 <= c < channels for c in columns)
        if not valid:
            raise ConfigurationError(f"column list must hold distinct ints in [0, {channels})")
        return list(columns), len(columns)
    if isinstance(columns, tuple):
        if len(columns) != 2:
            raise ConfigurationError("a column tuple is one (start, stop) interval; pass a list for indices")
        columns = slice(*columns)
    if not isinstance(columns, slice) or columns.step not in (None, 1):
        raise ConfigurationError("columns must be None, a unit-step slice, a (start, stop) tuple or a list")
    lo = 0 if columns.start is None else columns.start
    hi = channels if columns.stop is None else columns.stop
    if not (type(lo) is int and type(hi) is int and 0 <= lo < hi <= channels):
        raise ConfigurationError(f"column interval [{lo}, {hi}) is empty or leaves [0, {channels})")
    return slice(lo, hi), hi - lo


class KVRuntime(LineageRuntime):
    """Durable branches of chunked KV matrices over one content-addressed store (module docstring).

    ``max_resident_bytes`` bounds the bytes of live history leases. ``executor`` (a :class:`BoundedExecutor`)
    runs ``submit_chunk`` publications. ``encoder`` / ``decoder`` replace ``codecs.encode_tensor`` /
    ``codecs.decode_tensor`` (same signatures). ``verify_reads`` hashes every object read for use.
    ``on_open_error="quarantine"`` opens a store with damaged heads: they are listed in :attr:`quarantined`
    and raise :class:`QuarantinedError` when used, everything else works. ``history_read_ahead_bytes`` caps
    the payload bytes read ahead while ``acquire_history`` walks the keys in order.
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
            raise ConfigurationError(f"KVRuntime needs a ModelIdentity, got {type(model).__name__}")
        _check_arguments(_CONSTRUCTOR_RULES, locals(), "KVRuntime")
        if encode_concurrency > 1 and not (isinstance(executor, BoundedExecutor) and encode_workspace_bytes):
            raise ConfigurationError("KVRuntime: encode_concurrency > 1 runs on a BoundedExecutor and reserves "
                                     "encode_workspace_bytes > 0 per encode")
        from .codecs import decode_tensor, encode_tensor
        self.encoder = encoder or encode_tensor
        self.decoder = decoder or decode_tensor
        if not (callable(self.encoder) and callable(self.decoder)):
            raise ConfigurationError("KVRuntime: encoder and decoder must be callables")
        self.executor = executor
        self.prefit = prefit
        self.encode_concurrency = encode_concurrency
        self.encode_workspace_bytes = encode_workspace_bytes
        self.max_pending_source_bytes = max_pending_source_bytes
        self.verify_reads = verify_reads
        self.audit_on_open = verify_reads if audit_on_open is None else audit_on_open
        self.on_open_error = on_open_error
        self.history_read_ahead_bytes = (self.HISTORY_READ_AHEAD_BYTES if history_read_ahead_bytes is None
                                         else history_read_ahead_bytes)
        self.residency = ResidencyPool(max_resident_bytes)
        store = ObjectStore(root, max_bytes=max_store_bytes, verify_reads=verify_reads,
                            verify_references=verify_references,
                            on_damage="keep" if on_open_error == "quarantine" else "raise")
        super().__init__(store, model, registry=registry)
        self._keys = tuple(MatrixKey(layer, target) for layer in range(model.layers) for target in ("K", "V"))
        self._busy: dict[str, str] = {}                 # branch -> "commit" | "stream" | "async"
        self._ledger = _AsyncLedger(max_pending_source_bytes)
        self._quarantine: dict[str, tuple[str, str]] = {}  # ref name -> (object id, reason)
        self._reader = _ReadAhead(self.history_read_ahead_bytes, self._keys)
        self._closed = False
        try:
            self._bind_model()
            for name, object_id, reason in self._scan_heads():
                if on_open_error == "raise":
                    raise IntegrityError(f"{name} -> {object_id} is damaged: {reason}")
                self._quarantine[name] = (object_id, reason)
        except BaseException:
            self.store.close()
            self.residency.close()
            raise

    @property
    def _pending_source_bytes(self) -> int:
        return self._ledger.source_bytes

    def _bind_model(self) -> None:
        """Record the model identity in a new store, or check it against the one a store was created for."""
        with self.store.transaction():
            existing = self.store.get_ref(MODEL_REF)
            if existing is not None:
                self._check_model(self._manifest(existing, "model").get("model"))
            elif self.store.list_refs():
                raise IntegrityError(f"store has refs but no {MODEL_REF}: not a KVRuntime store")
            else:
                identity = self.store.put_manifest({"type": "model", "version": 1, "model": self.model.to_dict()})
                self.store.set_ref(MODEL_REF, identity, expected=None)

    # -- manifests -----------------------------------------------------------------------------------------------

    def _require_open(self) -> None:
        if self._closed:
            raise StateError("this KVRuntime was closed")

    def _check_model(self, recorded) -> None:
        if recorded != self.model.to_dict():
            name = recorded.get("name") if isinstance(recorded, dict) else recorded
            raise IntegrityError(f"object was written for model {name!r}, not {self.model.name!r}")

    def _manifest(self, object_id: str, kind: str) -> dict:
        for name, (quarantined, reason) in self._quarantine.items():
            if quarantined == object_id:
                raise QuarantinedError(f"{name} is quarantined ({reason})")
        data = self.store.get_manifest(object_id)
        if data.get("type") != kind or data.get("version") not in ((1, 2) if kind == "chunk" else (1,)):
            raise IntegrityError(f"{object_id} is not a supported {kind} manifest "
                                 f"(type {data.get('type')!r}, version {data.get('version')!r})")
        return data

    def _parse_chunk(self, object_id: str, expected_start: int) -> _Chunk:
        data = self._manifest(object_id, "chunk")
        self._check_model(data.get("model"))
        if data["version"] != 1:
            raise UnsupportedError(f"{object_id} is an adaptive (version 2) chunk; read it through the lineage API")
        try:
            if not all(type(data.get(name)) is int for name in _GEOMETRY):
                raise IntegrityError(f"{object_id}: geometry fields must be ints")
            start, end = data["token_start"], data["token_end"]
            if start != expected_start or end - start != data["frames"] * data["height"] * data["width"]:
                raise IntegrityError(f"{object_id} covers [{start}, {end}) with grid "
                                     f"{data['frames']}x{data['height']}x{data['width']}; expected it to start at "
                                     f"{expected_start} and span the grid")
            if data.get("clean") is not True:
                raise IntegrityError(f"{object_id} is not a clean chunk")
            records: dict[MatrixKey, str] = {}
            for entry in data["matrices"]:
                key, tensor = MatrixKey.from_dict(entry["key"]), entry["tensor"]
                if key in records:
                    raise IntegrityError(f"{object_id} lists {key} twice")
                if not (isinstance(tensor, str) and tensor.startswith("manifest:")):
                    raise IntegrityError(f"{object_id}: {key} does not name a tensor manifest")
                records[key] = tensor
            if set(records) != set(self._keys):
                raise IntegrityError(f"{object_id} has {len(records)} matrices, the model has {len(self._keys)}")
            return _Chunk(object_id, data["chunk_id"], start, end, data["frames"], data["height"], data["width"],
                          records)
        except (KeyError, TypeError, ValueError) as error:
            raise IntegrityError(f"{object_id} is a malformed chunk manifest") from error

    def _history(self, head_id: str) -> _History:
        head = self._manifest(head_id, "head")
        self._check_model(head.get("model"))
        ids = head.get("chunks")
        if not (isinstance(ids, list) and all(isinstance(i, str) for i in ids)):
            raise IntegrityError(f"{head_id}: chunks must be a list of manifest ids")
        chunks: list[_Chunk] = []
        for object_id in ids:
            chunk = self._parse_chunk(object_id, chunks[-1].token_end if chunks else 0)
            if chunks and (chunk.height, chunk.width) != (chunks[0].height, chunks[0].width):
                raise IntegrityError(f"{head_id}: chunk {chunk.chunk_id!r} changes the spatial grid")
            if any(c.chunk_id == chunk.chunk_id for c in chunks):
                raise IntegrityError(f"{head_id}: chunk id {chunk.chunk_id!r} appears twice")
            chunks.append(chunk)
        return _History(head_id, tuple(chunks))

    def _tensor_manifest(self, object_id: str) -> tuple[TensorContext, CodecSpec, dict]:
        data = self._manifest(object_id, "tensor")
        try:
            return TensorContext.from_dict(data["context"]), CodecSpec.from_dict(data["spec"]), data["encoded"]
        except (KeyError, TypeError, ValueError) as error:
            raise IntegrityError(f"{object_id} is a malformed tensor manifest") from error

    def _scan_heads(self) -> list[tuple[str, str, str]]:
        """``(ref, object id, reason)`` of every damaged branch, snapshot and lineage head (hashing every
        reachable object when ``audit_on_open`` is set, else checking that it exists)."""
        check = self.store.verify if self.audit_on_open else self.store.check
        refs = [(name, oid, self._history) for name, oid in self.store.list_refs(BRANCH_PREFIX).items()]
        refs += [(name, oid, self._snapshot) for name, oid in self.store.list_refs(SNAPSHOT_PREFIX).items()]
        refs += [(name, oid, None) for name, oid in self.store.list_refs(LINEAGE_PREFIX).items()]
        damaged = []
        for name, object_id, parse in refs:
            try:
                if parse is not None:
                    parse(object_id)
                check(object_id)
            except (IntegrityError, ConfigurationError) as error:
                damaged.append((name, object_id, str(error)))
        return damaged

    # -- branch reservations -------------------------------------------------------------------------------------

    def _head_of(self, branch_id: str) -> str:
        """The branch's head; the branch must exist and not be busy."""
        self._require_open()
        name = _branch_ref(branch_id)
        busy = self._busy.get(branch_id)
        if busy is not None and busy != "stream":
            raise PendingError(f"branch {branch_id!r} has a {busy} in progress")
        head = self.store.get_ref(name)
        if head is None:
            raise StateError(f"no branch named {branch_id!r}")
        return head

    def _reserve_branch(self, branch_id: str, kind: str) -> _History:
        """Parse the branch's history and mark it busy with ``kind`` (caller holds the lock)."""
        head = self._head_of(branch_id)
        if branch_id in self._busy:
            raise PendingError(f"branch {branch_id!r} has an open streaming chunk")
        with self.store.transaction():
            history = self._history(head)
        self._busy[branch_id] = kind
        return history

    def _release_branch(self, branch_id: str, kind: str) -> None:
        with self._lock:
            if self._busy.get(branch_id) == kind:
                del self._busy[branch_id]

    # -- branches ------------------------------------------------------------------------------------------------

    def _write_head(self, chunk_ids: list[str]) -> str:
        return self.store.put_manifest({"type": "head", "version": 1, "model": self.model.to_dict(),
                                        "chunks": chunk_ids}, references=chunk_ids)

    def create_branch(self, branch_id: str) -> None:
        with self._lock:
            self._require_open()
            name = _branch_ref(branch_id)
            with self.store.transaction():
                if self.store.get_ref(name) is not None:
                    raise StateError(f"branch {branch_id!r} exists already")
                self.store.set_ref(name, self._write_head([]), expected=None)

    def _branch_history(self, branch_id: str) -> _History:
        with self._lock, self.store.transaction():
            return self._history(self._head_of(branch_id))

    def branch_info(self, branch_id: str) -> dict[str, Any]:
        history = self._branch_history(branch_id)
        return {"branch_id": branch_id, "head_id": history.head_id, "chunk_ids": history.chunk_ids(),
                "chunk_manifests": history.object_ids(), "token_start": 0, "token_end": history.end,
                "chunk_id": history.last_chunk_id, "clean": True}

    def require_head(self, branch_id: str, expected_head: str) -> None:
        with self._lock:
            current = self._head_of(branch_id)
        if current != expected_head:
            raise StateError(f"branch {branch_id!r} moved to {current}, expected {expected_head}")

    def history_contexts(self, branch_id: str, key: MatrixKey) -> tuple[TensorContext, ...]:
        with self._lock, self.store.transaction():
            history = self._history(self._head_of(branch_id))
            return tuple(self._tensor_manifest(c.records[key])[0] for c in history.chunks)

    def history_specs(self, branch_id: str, key: MatrixKey) -> tuple[CodecSpec, ...]:
        with self._lock, self.store.transaction():
            history = self._history(self._head_of(branch_id))
            return tuple(self._tensor_manifest(c.records[key])[1] for c in history.chunks)

    # -- commits -------------------------------------------------------------------------------------------------

    def _chunk_plan(self, chunk_id, matrices, contexts, specs, history: _History, *, with_matrices: bool = True):
        """Check one chunk against the branch it extends; returns its per-key :class:`CodecSpec`."""
        _check_chunk_id(chunk_id)
        if chunk_id in history.chunk_ids():
            raise ConfigurationError(f"branch already has a chunk {chunk_id!r}")
        keys = set(self._keys)
        if set(contexts) != keys:
            raise ConfigurationError(f"contexts name {len(contexts)} matrices; the model has {len(keys)}")
        per_key = dict.fromkeys(self._keys, specs) if isinstance(specs, CodecSpec) else dict(specs)
        if set(per_key) != keys or not all(isinstance(s, CodecSpec) for s in per_key.values()):
            raise ConfigurationError("specs must be a CodecSpec, or a mapping of every matrix to one")
        placement = None
        for key, context in contexts.items():
            if not (isinstance(context, TensorContext) and context.key == key and context.model == self.model):
                raise ConfigurationError(f"context of {key} names another matrix or model")
            here = (context.token_start, context.frames, context.height, context.width)
            if placement is None:
                placement = here
            elif here != placement:
                raise ConfigurationError(f"context of {key} places the chunk at {here}, others at {placement}")
        start, _, height, width = placement
        if start != history.end:
            raise ConfigurationError(f"chunk starts at token {start}; the branch ends at {history.end}")
        if history.grid is not None and history.grid != (height, width):
            raise ConfigurationError(f"chunk grid {height}x{width} differs from the branch's "
                                     f"{history.grid[0]}x{history.grid[1]}")
        if with_matrices:
            if set(matrices) != keys:
                raise ConfigurationError(f"matrices name {len(matrices)} keys; the model has {len(keys)}")
            for key, tensor in matrices.items():
                if not isinstance(tensor, torch.Tensor) or tuple(tensor.shape) != contexts[key].shape:
                    shape = tuple(tensor.shape) if isinstance(tensor, torch.Tensor) else type(tensor).__name__
                    raise ConfigurationError(f"{key} is {shape}; its context wants {contexts[key].shape}")
        return per_key

    def _reusable_basis(self, history: _History, key: MatrixKey, rank: int):
        """The newest stored FP16 basis of ``key`` with exactly ``rank`` rows, as ``[rank, channels]``."""
        for chunk in reversed(history.chunks):
            _, spec, encoded = self._tensor_manifest(chunk.records[key])
            if spec.rank == rank and encoded.get("basis"):
                raw = bytearray(self.store.get(encoded["basis"]))
                return torch.frombuffer(raw, dtype=torch.float16).view(-1, self.model.kv_channels)[:rank]
        return None

    def _store_matrix(self, key, tensor, context, spec, history: _History, reuse_threshold) -> str:
        """Encode one matrix (reusing the branch's basis when its projection residual is within
        ``reuse_threshold``) and store its payloads and tensor manifest."""
        if spec.kind == "raw":
            encoded = self.encoder(tensor, context, spec)
        else:
            basis = None
            if reuse_threshold is not None:
                candidate = self._reusable_basis(history, key, spec.rank)
                if candidate is not None:
                    x = tensor.detach().cpu().double().reshape(context.shape)
                    q = candidate.double()
                    residual = torch.linalg.vector_norm(x - x @ q.t() @ q)
                    scale = max(float(torch.linalg.vector_norm(x)), 1e-300)
                    basis = candidate if float(residual) / scale <= reuse_threshold else None
            encoded = self.encoder(tensor, context, spec, basis=basis)
        if not isinstance(encoded, EncodedTensor):
            raise IntegrityError(f"encoder returned {type(encoded).__name__}, not EncodedTensor")
        payloads = {name: self.store.put(data) for name, data in encoded.payloads.items()}
        basis_id = self.store.put(encoded.basis, kind="basis") if encoded.basis is not None else None
        refs = set(payloads.values()) | ({basis_id} - {None})
        manifest = {"type": "tensor", "version": 1, "context": context.to_dict(), "spec": spec.to_dict(),
                    "encoded": {"metadata": json_copy(encoded.metadata), "payloads": payloads, "basis": basis_id,
                                "metrics": json_copy(dict(encoded.metrics or {}))}}
        return self.store.put_manifest(manifest, references=sorted(refs))

    def _store_all(self, matrices, contexts, specs, history, reuse_threshold, *, stop=None):
        """Store every matrix under a staging lease; returns ``(tensor manifests, leases)``."""
        stored, leases = {}, []
        try:
            for key in self._keys:
                if stop is not None:
                    stop()
                stored[key] = self._store_matrix(key, matrices[key], contexts[key], specs[key], history,
                                                 reuse_threshold)
                leases.append(self.store.lease(stored[key], purpose="staging", verify=False))
        except BaseException:
            for lease in leases:
                lease.release()
            raise
        return stored, leases

    def _publish(self, branch_id, chunk_id, parent_head, stored: Mapping[MatrixKey, str], contexts) -> str:
        """Write the chunk manifest and a new head, and move the branch from ``parent_head`` to it."""
        with self._lock:
            self._require_open()
            name = _branch_ref(branch_id)
            with self.store.transaction():
                current = self.store.get_ref(name)
                if current != parent_head:
                    raise StateError(f"branch {branch_id!r} moved while chunk {chunk_id!r} was encoded")
                history = self._history(current)
                where = contexts[self._keys[0]]
                tensors = [stored[key] for key in self._keys]
                chunk = self.store.put_manifest(
                    {"type": "chunk", "version": 1, "chunk_id": chunk_id, "model": self.model.to_dict(),
                     "clean": True, "token_start": where.token_start, "token_end": where.token_end,
                     "frames": where.frames, "height": where.height, "width": where.width,
                     "matrices": [{"key": key.to_dict(), "tensor": oid} for key, oid in zip(self._keys, tensors)]},
                    references=tensors)
                self.store.set_ref(name, self._write_head(history.object_ids() + [chunk]), expected=current)
                return chunk

    def seal_chunk(self, branch_id: str, chunk_id: Any, matrices: Mapping[MatrixKey, torch.Tensor],
                   contexts: Mapping[MatrixKey, TensorContext], specs=CodecSpec(), *, clean: bool = True,
                   reuse_threshold: float | None = None, rank_policy=None, staging_bytes: int | None = None) -> str:
        """Encode every matrix of one clean chunk and publish it on ``branch_id``."""
        if clean is not True:
            raise ConfigurationError("KVRuntime commits clean chunks only")
        if rank_policy is not None:
            raise UnsupportedError("rank policies (adaptive ranks) commit through commit_node")
        with self._lock:
            history = self._reserve_branch(branch_id, "commit")
            try:
                per_key = self._chunk_plan(chunk_id, matrices, contexts, specs, history)
            except BaseException:
                del self._busy[branch_id]
                raise
        try:
            stored, leases = self._store_all(matrices, contexts, per_key, history, reuse_threshold)
        except BaseException:
            self._release_branch(branch_id, "commit")
            raise
        try:
            self._release_branch(branch_id, "commit")
            return self._publish(branch_id, chunk_id, history.head_id, stored, contexts)
        finally:
            for lease in leases:
                lease.release()

    def open_chunk(self, branch_id: str, chunk_id: Any, contexts: Mapping[MatrixKey, TensorContext],
                   specs=CodecSpec(), *, reuse_threshold: float | None = None) -> StreamingChunk:
        """Reserve ``branch_id`` for one chunk published layer by layer (:class:`StreamingChunk`)."""
        with self._lock:
            history = self._reserve_branch(branch_id, "stream")
            try:
                per_key = self._chunk_plan(chunk_id, {}, contexts, specs, history, with_matrices=False)
            except BaseException:
                del self._busy[branch_id]
                raise
        return StreamingChunk(self, branch_id, chunk_id, contexts, per_key, history, reuse_threshold)

    def submit_chunk(self, branch_id: str, chunk_id: Any, matrices, contexts, specs=CodecSpec(), *,
                     reuse_threshold: float | None = None, timeout: float | None = None) -> PendingCommit:
        """Take a host copy of the matrices and publish the chunk on the executor; the branch stays busy until
        the publication ends (``PendingCommit`` follows it)."""
        if self.executor is None:
            raise ConfigurationError("submit_chunk runs on the executor given to KVRuntime(executor=...)")
        with self._lock:
            self._ledger.raise_failures()
            history = self._reserve_branch(branch_id, "async")
            try:
                per_key = self._chunk_plan(chunk_id, matrices, contexts, specs, history)
                nbytes = sum(t.numel() * t.element_size() for t in matrices.values())
                state = _CommitState(branch_id, history.head_id, nbytes)
                self._ledger.admit(state)
            except BaseException:
                del self._busy[branch_id]
                raise
            owned = {key: t.detach().to("cpu", copy=True) for key, t in matrices.items()}

        def stop_if_cancelled():
            if state.cancelled:
                raise StateError(f"commit of {chunk_id!r} on {branch_id!r} was cancelled")

        def publish():
            error = None
            try:
                stop_if_cancelled()
                state.phase = "encoding"
                stored, leases = self._store_all(owned, contexts, per_key, history, reuse_threshold,
                                                 stop=stop_if_cancelled)
                try:
                    with self._lock:
                        stop_if_cancelled()
                        state.phase = "ready"
                        self._busy.pop(branch_id, None)
                    state.result_id = self._publish(branch_id, chunk_id, history.head_id, stored, contexts)
                    state.phase = "published"
                finally:
                    for lease in leases:
                        lease.release()
                return state.result_id
            except BaseException as raised:
                error = raised
                raise
            finally:
                with self._lock:
                    self._ledger.settle(state, error)
                    self._ledger.release(state)
                    if self._busy.get(branch_id) == "async":
                        del self._busy[branch_id]

        try:
            job = self.executor.submit(publish, staging_bytes=nbytes, label=f"commit:{branch_id}:{chunk_id}",
                                       block=timeout is not None, timeout=timeout)
        except BaseException:
            with self._lock:
                self._ledger.release(state)
                self._busy.pop(branch_id, None)
            raise
        return PendingCommit(self, state, job)

    def async_stats(self) -> dict:
        with self._lock:
            return self._ledger.stats()

    # -- snapshots -----------------------------------------------------------------------------------------------

    @staticmethod
    def _snapshot_contracts(metadata, history: _History, *, stored: bool) -> dict:
        """A JSON copy of snapshot metadata that names every contract and whose clean boundary is the end of
        ``history``. Caller errors raise :class:`ConfigurationError`, damaged stored records
        :class:`IntegrityError`; a snapshot of pending execution raises :class:`PendingError`."""
        bad = IntegrityError if stored else ConfigurationError
        if not isinstance(metadata, Mapping):
            raise bad(f"snapshot metadata is {type(metadata).__name__}, not a mapping")
        copied = json_copy(metadata)
        absent = [name for name in SNAPSHOT_CONTRACTS if name not in copied]
        if absent:
            raise bad(f"snapshot metadata lacks the contracts {absent}")
        boundary = copied["clean_boundary"]
        matches = (isinstance(boundary, dict) and "chunk_id" in boundary
                   and boundary["chunk_id"] == history.last_chunk_id
                   and type(boundary.get("token_end")) is int and boundary["token_end"] == history.end
                   and boundary.get("clean", True) is True)
        if not matches:
            raise bad(f"clean_boundary {boundary!r} is not the branch end (chunk {history.last_chunk_id!r}, "
                      f"token {history.end})")
        execution = copied["execution"]
        if copied.get("pending", False) or (isinstance(execution, dict) and execution.get("pending", False)):
            raise PendingError("execution is pending; snapshot at a clean boundary")
        nulls = [name for name in SNAPSHOT_CONTRACTS[1:] if copied[name] is None]
        if nulls:
            raise bad(f"snapshot contracts {nulls} are null; record them explicitly")
        return copied

    def snapshot(self, branch_id: str, *, metadata: Mapping[str, Any],
                 tensors: Mapping[str, torch.Tensor] | None = None) -> str:
        """Pin the branch's current head with portable metadata and named tensors; returns the snapshot id."""
        with self._lock, self.store.transaction():
            history = self._history(self._head_of(branch_id))
            contracts = self._snapshot_contracts(metadata, history, stored=False)
            blob = self.store.put(serialize_tensors(dict(tensors or {})))
            snapshot_id = self.store.put_manifest(
                {"type": "snapshot", "version": 1, "model": self.model.to_dict(), "head": history.head_id,
                 "metadata": contracts, "tensor_state": blob}, references=[history.head_id, blob])
            self.store.set_ref(_snapshot_ref(snapshot_id), snapshot_id)
            return snapshot_id

    def _snapshot(self, snapshot_id: str) -> tuple[dict, dict]:
        """``(manifest, checked metadata)`` of a stored snapshot."""
        data = self._manifest(snapshot_id, "snapshot")
        self._check_model(data.get("model"))
        try:
            blob = data["tensor_state"]
            if not (isinstance(blob, str) and blob.startswith("blob:")):
                raise IntegrityError(f"{snapshot_id}: tensor_state must name a blob")
            return data, self._snapshot_contracts(data["metadata"], self._history(data["head"]), stored=True)
        except (KeyError, TypeError, ValueError) as error:
            raise IntegrityError(f"{snapshot_id} is a malformed snapshot manifest") from error

    def load_snapshot(self, snapshot_id: str) -> SnapshotState:
        with self._lock, self.store.transaction():
            self._require_open()
            data, contracts = self._snapshot(snapshot_id)
            return SnapshotState(snapshot_id, contracts, deserialize_tensors(self.store.get(data["tensor_state"])))

    def _point_branch(self, snapshot_id, branch_id, *, create_only, validator, metadata_validator) -> RestoredState:
        """Point ``branch_id`` at a snapshot's head once the validators accept it (compare-and-set against the
        ref read before validation)."""
        if any(v is not None and not callable(v) for v in (validator, metadata_validator)):
            raise ConfigurationError("validator and metadata_validator must be callables or None")
        with self._lock:
            self._require_open()
            name = _branch_ref(branch_id)
            if branch_id in self._busy:
                raise PendingError(f"branch {branch_id!r} has a {self._busy[branch_id]} in progress")
            with self.store.transaction():
                data, contracts = self._snapshot(snapshot_id)
                before = self.store.get_ref(name)
            if create_only and before is not None:
                raise StateError(f"cannot fork into {branch_id!r}: the branch exists")
            if metadata_validator is not None:
                preview = RestoredState(snapshot_id, branch_id, data["head"], json_copy(contracts), {})
                if metadata_validator(preview) is not None:
                    raise ConfigurationError("metadata_validator returned a value; it must raise or return None")
            state = RestoredState(snapshot_id, branch_id, data["head"], contracts,
                                  deserialize_tensors(self.store.get(data["tensor_state"])))
            if validator is not None and validator(state) is not None:
                raise ConfigurationError("validator returned a value; it must raise or return None")
            with self.store.transaction():
                self.store.set_ref(name, data["head"], expected=before)
            return state

    def restore(self, snapshot_id: str, branch_id: str, *, validator=None, metadata_validator=None,
                rank_policy=None) -> RestoredState:
        """Point ``branch_id`` (new or existing) at the snapshot's head."""
        return self._point_branch(snapshot_id, branch_id, create_only=False, validator=validator,
                                  metadata_validator=metadata_validator)

    def fork(self, snapshot_id: str, branch_id: str, *, validator=None, metadata_validator=None,
             rank_policy=None) -> RestoredState:
        """:meth:`restore` into a branch that must not exist yet."""
        return self._point_branch(snapshot_id, branch_id, create_only=True, validator=validator,
                                  metadata_validator=metadata_validator)

    # -- history -------------------------------------------------------------------------------------------------

    def _encoded(self, encoded: Mapping[str, Any], window=None) -> EncodedTensor:
        def read(object_id):
            data = self._reader.take(window, object_id)
            return self.store.get(object_id) if data is None else data

        payloads = {name: read(object_id) for name, object_id in encoded["payloads"].items()}
        basis = read(encoded["basis"]) if encoded.get("basis") is not None else None
        return EncodedTensor(encoded["metadata"], payloads, basis=basis, metrics=encoded.get("metrics") or {})

    def read_ahead_stats(self) -> dict[str, Any]:
        return dict(self._reader.stats, active=self._reader.window is not None)

    def _known_key(self, key) -> None:
        if not (isinstance(key, MatrixKey) and key in self._reader.position):
            raise ConfigurationError(f"{key!r} is not a (layer, K/V) matrix of {self.model.name!r}")

    def acquire_history(self, branch_id: str, key: MatrixKey, *, token_start: int | None = None,
                        token_end: int | None = None, device: Any = "cpu", dtype: Any = None, columns: Any = None,
                        column_groups: Any = None, decoder: Callable[..., torch.Tensor] | None = None,
                        head_id: str | None = None) -> HistoryLease:
        """Decode ``key``'s history over ``[token_start, token_end)`` (default: all of it) into a residency
        lease; ``head_id`` reads a given head instead of the branch's current one."""
        self._known_key(key)
        if column_groups is not None:
            raise UnsupportedError("column_groups is not supported; select channels with columns")
        decode = decoder or self.decoder
        with self._lock, self.store.transaction():
            if head_id is None:
                head_id = self._head_of(branch_id)
            else:
                self._require_open()
            history = self._history(head_id)
            start = 0 if token_start is None else token_start
            end = history.end if token_end is None else token_end
            if not (type(start) is int and type(end) is int and 0 <= start < end <= history.end):
                raise ConfigurationError(f"tokens [{start}, {end}) are not inside the committed [0, {history.end})")
            parts = [(c, self._tensor_manifest(c.records[key])) for c in history.chunks if c.overlaps(start, end)]
            window = self._reader.window_for(self, (head_id, start, end), key,
                                             [c for c, _ in parts])
        first_context = parts[0][1][0]
        out_dtype = dtype if dtype is not None else getattr(torch, first_context.dtype)
        selector, width = _select_columns(columns, self.model.kv_channels)
        nbytes = tensor_nbytes((end - start, width), str(out_dtype).removeprefix("torch."))

        def load():
            pieces = []
            for chunk, (_, _, encoded) in parts:
                matrix = decode(self._encoded(encoded, window), device=device, dtype=out_dtype)
                lo, hi = max(start, chunk.token_start), min(end, chunk.token_end)
                pieces.append(matrix[lo - chunk.token_start:hi - chunk.token_start, selector])
            return (torch.cat(pieces) if len(pieces) > 1 else pieces[0]).contiguous()

        return self.residency.acquire(nbytes, load, metadata={"head": head_id, "key": key.to_dict(),
                                                              "token_start": start, "token_end": end})

    def history_packet(self, branch_id: str, key: MatrixKey, *, token_start: int, token_end: int) -> EncodedTensor:
        """The stored packet of the one chunk that covers exactly ``[token_start, token_end)``."""
        self._known_key(key)
        history = self._branch_history(branch_id)
        exact = [c for c in history.chunks if (c.token_start, c.token_end) == (token_start, token_end)]
        if len(exact) != 1:
            raise StateError(f"no single chunk of {branch_id!r} spans exactly [{token_start}, {token_end})")
        with self._lock, self.store.transaction():
            return self._encoded(self._tensor_manifest(exact[0].records[key])[2])

    # -- lifecycle -----------------------------------------------------------------------------------------------

    @property
    def resident_bytes(self) -> int:
        return self.residency.resident_bytes

    @property
    def active_leases(self) -> int:
        return self.residency.active_leases

    @property
    def quarantined(self) -> dict[str, str]:
        return {name: reason for name, (_, reason) in self._quarantine.items()}

    def audit(self, *, deep: bool = True, quarantine: bool = False) -> dict[str, str]:
        """Check every head (``deep``: hash every object it reaches); returns ``{ref: reason}`` of the damaged
        ones and, with ``quarantine=True``, quarantines them."""
        with self._lock:
            self._require_open()
            remembered, self.audit_on_open = self.audit_on_open, deep
            try:
                damaged = self._scan_heads()
            finally:
                self.audit_on_open = remembered
            if quarantine:
                self._quarantine.update({name: (oid, reason) for name, oid, reason in damaged})
            return {name: reason for name, _, reason in damaged}

    def delete_branch(self, branch_id: str) -> None:
        with self._lock:
            name = _branch_ref(branch_id)
            if branch_id in self._busy:
                raise PendingError(f"branch {branch_id!r} has a {self._busy[branch_id]} in progress")
            with self.store.transaction():
                head = self.store.get_ref(name)
                if head is None:
                    self._head_of(branch_id)      # raises: closed runtime or no such branch
                self.store.delete_ref(name, expected=head)
            self._quarantine.pop(name, None)

    def delete_snapshot(self, snapshot_id: str) -> None:
        name = _snapshot_ref(snapshot_id)
        with self._lock:
            self._require_open()
            with self.store.transaction():
                if name not in self._quarantine:
                    self._snapshot(snapshot_id)
                self.store.delete_ref(name, expected=snapshot_id)
            self._quarantine.pop(name, None)

    def collect_garbage(self) -> dict[str, Any]:
        with self._lock:
            self._require_open()
            self._reader.drop()
            swept = self.store.collect_garbage()
            self.drop_manifest_caches()
            return swept

    gc = collect_garbage

    def close(self) -> None:
        with self._lock:
            if self._closed:
                return
            if self._busy or self._lineage_pending:
                busy = sorted(set(self._busy) | set(self._lineage_pending))
                raise PendingError(f"commits are still encoding on {busy}; finish or abort them before close")
            self._ledger.raise_failures()
            self._closed = True
            self._reader.drop()
            self.residency.close()
            self.store.close()

    def __enter__(self) -> "KVRuntime":
        self._require_open()
        return self

    def __exit__(self, *args: Any) -> None:
        self.close()


__all__ = ["KVRuntime", "PendingCommit", "RestoredState", "SnapshotState", "StreamingChunk", "HistoryLease"]
