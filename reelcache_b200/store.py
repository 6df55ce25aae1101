"""Content-addressed object store (reference: reelcache/store.py:203-1273; on-disk layout identical).

Layout under ``root``::

    objects/{blob,basis,manifest}/<sha256>   immutable objects, id = "<kind>:<sha256 of the bytes>"
    staging/pending-<uuid>                   written + fsynced, then hard-linked into objects/
    store.lock                               advisory flock serializing publication and GC across processes
    index.sqlite3                            WAL, synchronous=FULL; tables settings (format
                                             reelcache.store.v1), objects, edges, refs, owners, leases,
                                             telemetry, and (only after an eviction) evicted

Manifests are canonical JSON ``{"format": "reelcache.manifest.v1", "references": [sorted ids],
"data": {...}}`` whose references become index edges. Named refs move with compare-and-swap. Leases
pin graphs for a live process (owners with dead pids are reaped). Garbage collection keeps what refs
and leases reach. Reads may be hash-verified; a failed check quarantines the object (every later
read is verified until its bytes verify again). Run telemetry is an unhashed sidecar that never
enters content ids.
"""

from __future__ import annotations

import contextlib
import fcntl
import hashlib
import os
import re
import sqlite3
import threading
import time
import uuid
import weakref
from concurrent.futures import ThreadPoolExecutor
from pathlib import Path
from typing import Any, Iterable, Iterator, Mapping

from .errors import CapacityError, ConfigurationError, IntegrityError, QuarantinedError, StateError
from .serialization import canonical_json, parse_json

_OBJECT_ID = re.compile(r"^(blob|basis|manifest):([0-9a-f]{64})$")
_ANY = object()
_ROOT_LOCKS: dict[str, threading.RLock] = {}
_ROOT_GUARD = threading.Lock()
FORMAT = "reelcache.store.v1"
MANIFEST_FORMAT = "reelcache.manifest.v1"
IO_POLICIES = ("buffered", "nocache")

_SCHEMA = """
CREATE TABLE IF NOT EXISTS settings (key TEXT PRIMARY KEY, value TEXT NOT NULL);
CREATE TABLE IF NOT EXISTS objects (id TEXT PRIMARY KEY, kind TEXT NOT NULL, size INTEGER NOT NULL);
CREATE TABLE IF NOT EXISTS edges (
    parent TEXT NOT NULL REFERENCES objects(id), child TEXT NOT NULL REFERENCES objects(id),
    PRIMARY KEY(parent, child));
CREATE TABLE IF NOT EXISTS refs (name TEXT PRIMARY KEY, object_id TEXT NOT NULL REFERENCES objects(id));
CREATE TABLE IF NOT EXISTS owners (id TEXT PRIMARY KEY, pid INTEGER NOT NULL, stamp TEXT);
CREATE TABLE IF NOT EXISTS leases (
    id TEXT NOT NULL, owner TEXT NOT NULL REFERENCES owners(id),
    object_id TEXT NOT NULL REFERENCES objects(id), PRIMARY KEY(id, object_id));
CREATE TABLE IF NOT EXISTS telemetry (
    object_id TEXT PRIMARY KEY REFERENCES objects(id) ON DELETE CASCADE, data TEXT NOT NULL);
"""


class EvictedObjectError(StateError):
    """The payload of this object was evicted under an archive budget (its index row remains)."""


def _process_stamp(pid: int) -> str | None:
    """Start time of a process (Linux /proc), distinguishing a reused pid from the original owner."""
    try:
        with open(f"/proc/{pid}/stat", "rb") as handle:
            fields = handle.read().rsplit(b")", 1)[1].split()
        return fields[19].decode()
    except (OSError, IndexError):
        return None


def _alive(pid: int, stamp: str | None) -> bool:
    try:
        os.kill(pid, 0)
    except ProcessLookupError:
        return False
    except PermissionError:
        pass
    return stamp is None or _process_stamp(pid) in (None, stamp)


class ObjectLease:
    """A pin on a set of objects (and everything they reference) for this process."""

    def __init__(self, store: ObjectStore, lease_id: str, object_ids: tuple[str, ...]) -> None:
        self._store = store
        self.lease_id = lease_id
        self.object_ids = object_ids
        self._active = True

    @property
    def active(self) -> bool:
        return self._active

    def release(self) -> None:
        if self._active:
            self._active = False
            if not self._store.closed:
                self._store._release_lease(self.lease_id)

    def __enter__(self) -> ObjectLease:
        return self

    def __exit__(self, *args: Any) -> None:
        self.release()

    def __del__(self) -> None:
        try:
            self.release()
        except Exception:  # noqa: BLE001 - interpreter shutdown or closed store
            pass


class ReadAhead:
    """Background reads of object payloads into a bounded buffer; ``take`` hands one over."""

    def __init__(self, store: ObjectStore, max_bytes: int) -> None:
        if type(max_bytes) is not int or max_bytes < 0:
            raise ConfigurationError("read-ahead max_bytes must be a nonnegative integer")
        self._store = store
        self._max = max_bytes
        self._lock = threading.Lock()
        self._held: dict[str, bytes] = {}
        self._held_bytes = 0
        self._pending: list[str] = []
        self._futures = []
        self.hits = 0
        self.misses = 0
        self._closed = False

    def schedule(self, object_ids: Iterable[str]) -> int:
        ids = [i for i in object_ids if i not in self._held]
        sizes = self._store.object_sizes(ids)
        count = 0
        with self._lock:
            budget = self._max - self._held_bytes
            for object_id in ids:
                size = sizes.get(object_id, 0)
                if size > budget:
                    break
                budget -= size
                self._pending.append(object_id)
                count += 1
        if count:
            self._futures.append(self._store._ahead_pool().submit(self._fill))
        return count

    def _fill(self) -> None:
        while True:
            with self._lock:
                if self._closed or not self._pending:
                    return
                object_id = self._pending.pop(0)
            try:
                data = self._store.get(object_id)
            except Exception:  # noqa: BLE001 - the consumer reads (and reports) it again on a miss
                continue
            with self._lock:
                if not self._closed:
                    self._held[object_id] = data
                    self._held_bytes += len(data)

    def take(self, object_id: str) -> bytes | None:
        with self._lock:
            data = self._held.pop(object_id, None)
            if data is None:
                self.misses += 1
                return None
            self._held_bytes -= len(data)
            self.hits += 1
            return data

    @property
    def held_bytes(self) -> int:
        return self._held_bytes

    def stats(self) -> dict[str, int]:
        return {"hits": self.hits, "misses": self.misses, "held_bytes": self._held_bytes}

    def close(self) -> None:
        with self._lock:
            self._closed = True
            self._held.clear()
            self._held_bytes = 0
            self._pending.clear()


class ObjectStore:
    """Owns the immutable blob/basis/manifest namespaces and atomic named roots.

    ``verify_reads`` hash-checks every object read for use; ``verify_references`` (default: follows
    ``verify_reads``) makes graph operations read and hash what they reach instead of trusting the
    index. ``on_damage`` ("raise" or "keep") is the GC policy for damaged graphs.
    """

    def __init__(self, root: str | os.PathLike[str], *, max_bytes: int | None = None, verify_reads: bool = False,
                 verify_references: bool | None = None, on_damage: str = "raise") -> None:
        if max_bytes is not None and (type(max_bytes) is not int or max_bytes < 0):
            raise ConfigurationError("max_bytes must be a nonnegative integer")
        if type(verify_reads) is not bool:
            raise ConfigurationError("verify_reads must be boolean")
        if verify_references is not None and type(verify_references) is not bool:
            raise ConfigurationError("verify_references must be boolean or None")
        if on_damage not in ("raise", "keep"):
            raise ConfigurationError("on_damage must be 'raise' or 'keep'")
        self.verify_reads = verify_reads
        self.verify_references = verify_reads if verify_references is None else verify_references
        self.on_damage = on_damage
        self.max_bytes = max_bytes
        self.root = Path(root).resolve()
        self.root.mkdir(parents=True, exist_ok=True)
        for kind in ("blob", "basis", "manifest"):
            (self.root / "objects" / kind).mkdir(parents=True, exist_ok=True)
        (self.root / "staging").mkdir(exist_ok=True)
        with _ROOT_GUARD:
            self._lock = _ROOT_LOCKS.setdefault(str(self.root), threading.RLock())
        had_lock_file = (self.root / "store.lock").exists()
        self._lock_file = (self.root / "store.lock").open("a+b")
        self._closed = False
        self._depth = 0
        self._rollback_only = False
        self._created: list[str] = []
        self._touched: dict[str, None] = {}
        self._events: list[tuple[str, str]] = []
        self.hooks: Any = None
        self._dirty_dirs: set[Path] = set()
        self._damaged: dict[str, str] = {}
        self._quarantined: dict[str, str] = {}
        self._quarantine_lock = threading.Lock()
        self._verified_count = threading.local()
        self._recovered_staging: set[str] = set()
        self._owner = uuid.uuid4().hex
        self._leases: weakref.WeakSet[ObjectLease] = weakref.WeakSet()
        self._readers: ThreadPoolExecutor | None = None
        self._pool_guard = threading.Lock()
        self.io_policy = "buffered"
        self._io_lock = threading.Lock()
        self.io_stats_ = {"read_calls": 0, "read_bytes": 0, "write_calls": 0, "write_bytes": 0,
                          "existing_calls": 0, "existing_bytes": 0, "errors": 0, "last_error": None}
        self._evicted: set[str] = set()
        self._unevicted: list[str] = []
        # objects whose whole subtree a reference update already checked in this process (immutable content:
        # the next update only walks what is new below them)
        self._verified: set[str] = set()
        try:
            with self._lock:
                fcntl.flock(self._lock_file, fcntl.LOCK_EX)
                try:
                    self._open_index(had_lock_file)
                finally:
                    fcntl.flock(self._lock_file, fcntl.LOCK_UN)
            with self.transaction():
                self._reap_owners()
                self._db.execute("INSERT INTO owners VALUES (?, ?, ?)",
                                 (self._owner, os.getpid(), _process_stamp(os.getpid())))
                self._recover_files()
            if self._recovered_staging:
                self.collect_garbage(candidates=self._recovered_staging)
        except sqlite3.Error as exc:
            self._abort_open()
            raise IntegrityError("cannot open the object store index") from exc
        except BaseException:
            self._abort_open()
            raise

    def _open_index(self, had_lock_file: bool) -> None:
        index = self.root / "index.sqlite3"
        existing = index.exists()
        if not existing and (had_lock_file or any((self.root / "objects").glob("*/*"))
                             or any((self.root / "staging").iterdir())):
            raise IntegrityError("object store index is missing; refusing to reset existing state")
        if existing and index.stat().st_size < 100:
            raise IntegrityError("object store index is truncated")
        self._db = sqlite3.connect(index, timeout=60, isolation_level=None, check_same_thread=False)
        if existing:
            tables = {row[0] for row in self._db.execute("SELECT name FROM sqlite_master WHERE type='table'")}
            if not {"settings", "objects", "edges", "refs", "owners", "leases"} <= tables:
                raise IntegrityError("object store index schema is incomplete")
            if self._db.execute("SELECT value FROM settings WHERE key='format'").fetchone() != (FORMAT,):
                raise IntegrityError("unsupported or missing object store format")
        self._db.execute("PRAGMA foreign_keys=ON")
        self._db.execute("PRAGMA journal_mode=WAL")
        self._db.execute("PRAGMA synchronous=FULL")
        self._db.executescript(_SCHEMA)
        self._db.execute("INSERT OR IGNORE INTO settings VALUES ('format', ?)", (FORMAT,))
        if self._db.execute("SELECT 1 FROM sqlite_master WHERE type='table' AND name='evicted'").fetchone():
            self._evicted = {row[0] for row in self._db.execute("SELECT id FROM evicted")}

    def _abort_open(self) -> None:
        self._closed = True
        if hasattr(self, "_db"):
            self._db.close()
        self._lock_file.close()

    # -- transactions ------------------------------------------------------------------------------------------

    @property
    def closed(self) -> bool:
        return self._closed

    @contextlib.contextmanager
    def transaction(self) -> Iterator[ObjectStore]:
        """Nested transactions join the outermost one (one SQLite IMMEDIATE transaction + flock)."""
        events: list[tuple[str, str]] = []
        with self._lock:
            if self._closed:
                raise StateError("object store is closed")
            outermost = self._depth == 0
            if outermost:
                fcntl.flock(self._lock_file, fcntl.LOCK_EX)
                try:
                    self._db.execute("BEGIN IMMEDIATE")
                except sqlite3.Error as exc:
                    fcntl.flock(self._lock_file, fcntl.LOCK_UN)
                    raise IntegrityError("cannot start an object store transaction") from exc
                self._rollback_only = False
                self._created, self._touched, self._events, self._unevicted = [], {}, [], []
            self._depth += 1
            try:
                yield self
                if outermost:
                    if self._rollback_only:
                        raise StateError("a failed nested store operation invalidated the transaction")
                    for directory in sorted(self._dirty_dirs):
                        self._sync_directory(directory)
                    self._db.execute("COMMIT")
                    if self._unevicted:
                        self._evicted.difference_update(self._unevicted)
                    if self.hooks is not None:
                        events = self._events
            except BaseException as exc:
                self._rollback_only = True
                if outermost and self._db.in_transaction:
                    self._db.execute("ROLLBACK")
                if isinstance(exc, sqlite3.Error):
                    raise IntegrityError("object store index operation failed") from exc
                raise
            finally:
                self._depth -= 1
                if outermost:
                    self._dirty_dirs.clear()
                    self._events = []
                    fcntl.flock(self._lock_file, fcntl.LOCK_UN)
        for event, object_id in events:
            self.hooks(event, object_id)

    @property
    def created_objects(self) -> tuple[str, ...]:
        with self._lock:
            if not self._depth:
                raise StateError("created_objects requires an active store transaction")
            return tuple(self._created)

    @property
    def touched_objects(self) -> tuple[str, ...]:
        with self._lock:
            if not self._depth:
                raise StateError("touched_objects requires an active store transaction")
            return tuple(self._touched)

    # -- paths and io --------------------------------------------------------------------------------------------

    def path_for(self, object_id: str) -> Path:
        match = _OBJECT_ID.fullmatch(object_id) if isinstance(object_id, str) else None
        if match is None:
            raise IntegrityError(f"invalid immutable object id: {object_id!r}")
        return self.root / "objects" / match[1] / match[2]

    def set_io_policy(self, policy: str, *, drop_existing: bool = False) -> dict[str, Any]:
        if policy not in IO_POLICIES:
            raise ConfigurationError(f"store io policy must be one of {IO_POLICIES}")
        self.io_policy = policy
        dropped = 0
        if drop_existing and policy == "nocache":
            for kind in ("blob", "basis", "manifest"):
                for path in (self.root / "objects" / kind).iterdir():
                    with contextlib.suppress(OSError):
                        fd = os.open(path, os.O_RDONLY)
                        try:
                            os.posix_fadvise(fd, 0, 0, os.POSIX_FADV_DONTNEED)
                            dropped += 1
                        finally:
                            os.close(fd)
        return {"policy": policy, "dropped_files": dropped}

    def io_stats(self) -> dict[str, Any]:
        with self._io_lock:
            return dict(self.io_stats_, policy=self.io_policy)

    def _read_file(self, path: Path) -> bytes:
        with open(path, "rb") as handle:
            data = handle.read()
            if self.io_policy == "nocache":
                with contextlib.suppress(OSError):
                    os.posix_fadvise(handle.fileno(), 0, 0, os.POSIX_FADV_DONTNEED)
        with self._io_lock:
            self.io_stats_["read_calls"] += 1
            self.io_stats_["read_bytes"] += len(data)
        return data

    def _write_file(self, path: Path, data: bytes) -> None:
        staged = self.root / "staging" / f"pending-{uuid.uuid4().hex}"
        try:
            with staged.open("xb") as handle:
                handle.write(data)
                handle.flush()
                os.fsync(handle.fileno())
                if self.io_policy == "nocache":
                    with contextlib.suppress(OSError):
                        os.posix_fadvise(handle.fileno(), 0, 0, os.POSIX_FADV_DONTNEED)
            if path.exists():
                path.unlink()
            os.link(staged, path)
            self._dirty_dirs.add(path.parent)
        finally:
            staged.unlink(missing_ok=True)
        with self._io_lock:
            self.io_stats_["write_calls"] += 1
            self.io_stats_["write_bytes"] += len(data)

    def _sync_directory(self, directory: Path) -> None:
        fd = os.open(directory, os.O_RDONLY | os.O_DIRECTORY)
        try:
            os.fsync(fd)
        finally:
            os.close(fd)

    # -- quarantine ----------------------------------------------------------------------------------------------

    def quarantine(self, object_id: str, reason: str) -> None:
        self.path_for(object_id)
        with self._quarantine_lock:
            self._quarantined[object_id] = str(reason)

    def lift_quarantine(self, object_id: str) -> bool:
        with self._quarantine_lock:
            return self._quarantined.pop(object_id, None) is not None

    @property
    def quarantined_objects(self) -> dict[str, str]:
        with self._quarantine_lock:
            return dict(self._quarantined)

    def check_quarantined(self, object_ids: Iterable[str]) -> None:
        for object_id in object_ids:
            if object_id in self._quarantined:
                self._get(object_id, verify=True)

    @property
    def verified_payloads(self) -> int:
        return getattr(self._verified_count, "value", 0)

    # -- reads ---------------------------------------------------------------------------------------------------

    def _require(self, object_id: str) -> None:
        path = self.path_for(object_id)
        row = self._db.execute("SELECT kind FROM objects WHERE id=?", (object_id,)).fetchone()
        if row is None:
            raise IntegrityError(f"missing immutable object: {object_id}")
        if object_id in self._evicted:
            return
        if not path.exists():
            raise IntegrityError(f"missing immutable object file: {object_id}")

    def _index_row(self, object_id: str):
        """The object's index row (kind, size); caller holds the store lock (SQLite runs on the caller's
        thread only: the connection is shared)."""
        row = self._db.execute("SELECT kind, size FROM objects WHERE id=?", (object_id,)).fetchone()
        if row is None:
            raise IntegrityError(f"missing immutable object: {object_id}")
        if object_id in self._evicted:
            raise EvictedObjectError(f"object payload was evicted: {object_id}")
        return row

    def _read_object(self, object_id: str) -> bytes:
        """File read of one object (no index access: safe on the reader pool)."""
        try:
            return self._read_file(self.path_for(object_id))
        except OSError as exc:
            with self._io_lock:
                self.io_stats_["errors"] += 1
                self.io_stats_["last_error"] = str(exc)
            raise IntegrityError(f"cannot read immutable object: {object_id}") from exc

    def _get(self, object_id: str, *, verify: bool | None = None, data: bytes | None = None, row=None) -> bytes:
        self.path_for(object_id)
        if row is None:
            row = self._index_row(object_id)
        verify = (self.verify_reads if verify is None else verify) or object_id in self._quarantined
        if data is None:
            data = self._read_object(object_id)
        if len(data) != row[1]:
            self._fail(object_id, "size differs from the index")
        if verify:
            self._verified_count.value = getattr(self._verified_count, "value", 0) + 1
            if hashlib.sha256(data).hexdigest() != object_id.split(":", 1)[1]:
                self._fail(object_id, "content hash mismatch")
            self.lift_quarantine(object_id)
        return data

    def _fail(self, object_id: str, reason: str) -> None:
        was = object_id in self._quarantined
        self.quarantine(object_id, reason)
        if was:
            raise QuarantinedError(f"quarantined object still fails verification: {object_id} ({reason})")
        raise IntegrityError(f"corrupt immutable object: {object_id} ({reason})")

    def get(self, object_id: str) -> bytes:
        with self.transaction():
            return self._get(object_id)

    get_bytes = get

    def _pool(self) -> ThreadPoolExecutor:
        """File reads of get_many (they never take the store lock)."""
        with self._pool_guard:
            if self._readers is None:
                self._readers = ThreadPoolExecutor(max_workers=8, thread_name_prefix="reelcache-store-read")
            return self._readers

    def _ahead_pool(self) -> ThreadPoolExecutor:
        """Read-ahead workers (they take the store lock per object, so they never share get_many's pool,
        whose caller holds that lock while it waits for its reads)."""
        with self._pool_guard:
            if getattr(self, "_ahead", None) is None:
                self._ahead = ThreadPoolExecutor(max_workers=4, thread_name_prefix="reelcache-store-ahead")
            return self._ahead

    def get_many(self, object_ids: Iterable[str], *, verify: bool | None = None,
                 read_ahead: ReadAhead | None = None) -> dict[str, bytes]:
        """Read several objects with parallel file reads (one index transaction)."""
        ids = list(dict.fromkeys(object_ids))
        result: dict[str, bytes] = {}
        if read_ahead is not None:
            for object_id in ids:
                data = read_ahead.take(object_id)
                if data is not None:
                    result[object_id] = data
        rest = [i for i in ids if i not in result]
        with self.transaction():
            rows = {object_id: (self.path_for(object_id), self._index_row(object_id))[1] for object_id in rest}
            if len(rest) <= 1:
                for object_id in rest:
                    result[object_id] = self._get(object_id, verify=verify, row=rows[object_id])
            else:
                # parallel file reads; index lookups and checks stay on this thread
                for object_id, data in zip(rest, self._pool().map(self._read_object, rest)):
                    result[object_id] = self._get(object_id, verify=verify, data=data, row=rows[object_id])
        return {object_id: result[object_id] for object_id in ids}

    def read_ahead(self, object_ids: Iterable[str] = (), *, max_bytes: int) -> ReadAhead:
        reader = ReadAhead(self, max_bytes)
        reader.schedule(object_ids)
        return reader

    def object_size(self, object_id: str) -> int:
        self.path_for(object_id)
        with self.transaction():
            row = self._db.execute("SELECT size FROM objects WHERE id=?", (object_id,)).fetchone()
            if row is None:
                raise IntegrityError(f"missing immutable object: {object_id}")
            return row[0]

    def object_sizes(self, object_ids: Iterable[str]) -> dict[str, int]:
        ids = list(object_ids)
        with self.transaction():
            result = {}
            for object_id in ids:
                row = self._db.execute("SELECT size FROM objects WHERE id=?", (object_id,)).fetchone()
                if row is not None:
                    result[object_id] = row[0]
            return result

    def indexed(self, object_ids: Iterable[str]) -> set[str]:
        return set(self.object_sizes(object_ids))

    # -- writes --------------------------------------------------------------------------------------------------

    def _put(self, data: bytes, kind: str) -> str:
        if kind not in ("blob", "basis", "manifest"):
            raise ConfigurationError("object kind must be blob, basis, or manifest")
        if not isinstance(data, bytes):
            raise ConfigurationError("immutable objects require bytes")
        object_id = f"{kind}:{hashlib.sha256(data).hexdigest()}"
        path = self.path_for(object_id)
        exists = self._db.execute("SELECT 1 FROM objects WHERE id=?", (object_id,)).fetchone()
        if exists is not None and object_id in self._evicted:
            self._write_file(path, data)
            self._db.execute("DELETE FROM evicted WHERE id=?", (object_id,))
            self._unevicted.append(object_id)
            self._touched[object_id] = None
            self._events.append(("created", object_id))
            return object_id
        if exists is not None:
            self._require(object_id)
            self._touched[object_id] = None
            self._events.append(("existing", object_id))
            with self._io_lock:
                self.io_stats_["existing_calls"] += 1
                self.io_stats_["existing_bytes"] += len(data)
            return object_id
        if self.max_bytes is not None:
            used = self._db.execute("SELECT COALESCE(SUM(size), 0) FROM objects").fetchone()[0]
            if used + len(data) > self.max_bytes:
                raise CapacityError(f"object store requires {used + len(data)} bytes, budget is {self.max_bytes}")
        if path.exists():
            try:
                existing = self._read_file(path)
            except OSError as exc:
                raise IntegrityError(f"cannot read orphaned immutable object: {object_id}") from exc
            if existing != data:
                raise IntegrityError(f"corrupt orphaned immutable object: {object_id}")
        else:
            self._write_file(path, data)
        self.lift_quarantine(object_id)
        self._db.execute("INSERT INTO objects VALUES (?, ?, ?)", (object_id, kind, len(data)))
        self._created.append(object_id)
        self._touched[object_id] = None
        self._events.append(("created", object_id))
        return object_id

    def put(self, data: bytes, *, kind: str = "blob") -> str:
        if kind == "manifest":
            raise ConfigurationError("use put_manifest to register manifest references")
        with self.transaction():
            return self._put(data, kind)

    put_bytes = put

    def put_manifest(self, data: Mapping[str, Any], *, references: Iterable[str] = ()) -> str:
        if not isinstance(data, Mapping):
            raise ConfigurationError("manifest data must be a JSON mapping")
        references = tuple(sorted(set(references)))
        with self.transaction():
            for reference in references:
                self._require(reference)
            encoded = canonical_json({"format": MANIFEST_FORMAT, "references": list(references), "data": data})
            object_id = self._put(encoded, "manifest")
            for reference in references:
                self._db.execute("INSERT OR IGNORE INTO edges VALUES (?, ?)", (object_id, reference))
            return object_id

    def _manifest(self, object_id: str) -> tuple[dict[str, Any], tuple[str, ...]]:
        if not isinstance(object_id, str) or not object_id.startswith("manifest:"):
            raise IntegrityError("expected a manifest object")
        value = parse_json(self._get(object_id))
        if (not isinstance(value, dict) or set(value) != {"format", "references", "data"}
                or value["format"] != MANIFEST_FORMAT or not isinstance(value["data"], dict)
                or not isinstance(value["references"], list)
                or any(not isinstance(item, str) for item in value["references"])
                or value["references"] != sorted(set(value["references"]))):
            raise IntegrityError("invalid immutable manifest")
        references = tuple(value["references"])
        for reference in references:
            self.path_for(reference)
        edges = tuple(row[0] for row in self._db.execute(
            "SELECT child FROM edges WHERE parent=? ORDER BY child", (object_id,)))
        if edges != references:
            raise IntegrityError("manifest references disagree with the store index")
        return value["data"], references

    def get_manifest(self, object_id: str) -> dict[str, Any]:
        with self.transaction():
            return self._manifest(object_id)[0]

    def get_manifest_with_references(self, object_id: str) -> tuple[dict[str, Any], tuple[str, ...]]:
        with self.transaction():
            return self._manifest(object_id)

    def get_manifests_with_references(self, object_ids: Iterable[str]):
        with self.transaction():
            return [self._manifest(object_id) for object_id in object_ids]

    def references(self, object_id: str) -> tuple[str, ...]:
        with self.transaction():
            return self._manifest(object_id)[1]

    def put_telemetry(self, object_id: str, data: Mapping[str, Any]) -> None:
        """Attach unhashed run telemetry to a stored object (latest write wins; removed by GC)."""
        self.path_for(object_id)
        if not isinstance(data, Mapping):
            raise ConfigurationError("object telemetry must be a JSON mapping")
        encoded = canonical_json(data).decode("utf-8")
        with self.transaction():
            if self._db.execute("SELECT 1 FROM objects WHERE id=?", (object_id,)).fetchone() is None:
                raise IntegrityError(f"missing immutable object: {object_id}")
            self._db.execute("INSERT INTO telemetry VALUES (?, ?) ON CONFLICT(object_id) DO UPDATE SET "
                             "data=excluded.data", (object_id, encoded))

    def telemetry(self, object_id: str) -> dict[str, Any] | None:
        self.path_for(object_id)
        with self.transaction():
            row = self._db.execute("SELECT data FROM telemetry WHERE object_id=?", (object_id,)).fetchone()
        return None if row is None else parse_json(row[0].encode("utf-8"))

    # -- graph walks, audits -------------------------------------------------------------------------------------

    def _walk(self, object_ids: Iterable[str], *, verify: bool, damaged: dict[str, str] | None = None,
              force: bool = False, cached: bool = False) -> set[str]:
        """Every object reachable from ``object_ids``; checks existence (and content when verifying).

        ``cached`` (reference updates only; the returned set is then not the full reachable set): an object
        whose subtree an earlier cached walk of this process checked is only checked to still exist -- the
        collector never removes a child that an existing manifest references -- and its subtree is not
        walked again, so publishing a node costs the new objects, not the whole history."""
        seen: set[str] = set()
        stack = list(object_ids)
        while stack:
            object_id = stack.pop()
            if object_id in seen:
                continue
            seen.add(object_id)
            if cached and object_id in self._verified:
                self._require(object_id)
                continue
            try:
                self.path_for(object_id)
                if object_id.startswith("manifest:"):
                    if verify and (self.verify_references or force):
                        _, refs = self._manifest(object_id)
                    else:
                        self._require(object_id)
                        refs = tuple(row[0] for row in self._db.execute(
                            "SELECT child FROM edges WHERE parent=?", (object_id,)))
                    stack.extend(refs)
                else:
                    if verify and (self.verify_references or force) and object_id not in self._evicted:
                        self._get(object_id, verify=True)
                    else:
                        self._require(object_id)
            except IntegrityError as exc:
                if damaged is None:
                    raise
                damaged[object_id] = str(exc)
                stack.extend(row[0] for row in self._db.execute(
                    "SELECT child FROM edges WHERE parent=?", (object_id,)))
        if cached:
            self._verified |= seen
        return seen

    def verify(self, object_id: str, *, recursive: bool = True) -> None:
        """Full forced audit: read and hash every reachable object."""
        with self.transaction():
            if recursive:
                self._walk([object_id], verify=True, force=True)
            else:
                self._get(object_id, verify=True)

    def check(self, object_id: str) -> None:
        with self.transaction():
            self._walk([object_id], verify=False)

    @property
    def damaged(self) -> dict[str, str]:
        return dict(self._damaged)

    # -- refs and leases -----------------------------------------------------------------------------------------

    def _ref_name(self, name: str) -> None:
        if not isinstance(name, str) or not name or "\x00" in name:
            raise ConfigurationError("reference names must be nonempty strings without NUL")

    def get_ref(self, name: str) -> str | None:
        self._ref_name(name)
        with self.transaction():
            row = self._db.execute("SELECT object_id FROM refs WHERE name=?", (name,)).fetchone()
            return None if row is None else row[0]

    def set_ref(self, name: str, object_id: str, *, expected: Any = _ANY) -> None:
        """Point ``name`` at ``object_id`` (compare-and-swap against ``expected`` when given)."""
        self._ref_name(name)
        with self.transaction():
            current = self.get_ref(name)
            if expected is not _ANY and current != expected:
                raise StateError(f"reference changed concurrently: {name}")
            self._walk([object_id], verify=True, cached=True)
            self._db.execute("INSERT INTO refs VALUES (?, ?) ON CONFLICT(name) DO UPDATE SET "
                             "object_id=excluded.object_id", (name, object_id))

    def delete_ref(self, name: str, *, expected: Any = _ANY) -> None:
        self._ref_name(name)
        with self.transaction():
            current = self.get_ref(name)
            if expected is not _ANY and current != expected:
                raise StateError(f"reference changed concurrently: {name}")
            if current is None:
                raise StateError(f"reference does not exist: {name}")
            self._db.execute("DELETE FROM refs WHERE name=?", (name,))

    def list_refs(self, prefix: str = "") -> dict[str, str]:
        with self.transaction():
            return {name: object_id for name, object_id in
                    self._db.execute("SELECT name, object_id FROM refs ORDER BY name") if name.startswith(prefix)}

    def lease(self, object_ids: str | Iterable[str], *, purpose: str = "read", verify: bool = True) -> ObjectLease:
        """Pin a graph for this process; ``purpose="staging"`` marks pending publications (recovered
        and collected when their owner dies)."""
        if purpose not in ("read", "staging"):
            raise ConfigurationError("object lease purpose must be read or staging")
        if type(verify) is not bool:
            raise ConfigurationError("lease verification must be boolean")
        if isinstance(object_ids, str):
            object_ids = [object_ids]
        ids = tuple(sorted(set(object_ids)))
        if not ids:
            raise ConfigurationError("an object lease requires at least one object")
        with self.transaction():
            self._walk(ids, verify=verify)
            lease_id = ("staging-" if purpose == "staging" else "") + uuid.uuid4().hex
            for object_id in ids:
                self._db.execute("INSERT INTO leases VALUES (?, ?, ?)", (lease_id, self._owner, object_id))
            lease = ObjectLease(self, lease_id, ids)
            self._leases.add(lease)
            return lease

    def _release_lease(self, lease_id: str) -> None:
        with self.transaction():
            self._db.execute("DELETE FROM leases WHERE id=? AND owner=?", (lease_id, self._owner))

    def _reap_owners(self) -> None:
        for owner, pid, stamp in list(self._db.execute("SELECT id, pid, stamp FROM owners")):
            if _alive(pid, stamp):
                continue
            pending = [object_id for lease_id, object_id in
                       self._db.execute("SELECT id, object_id FROM leases WHERE owner=?", (owner,))
                       if lease_id.startswith("staging-")]
            while pending:
                object_id = pending.pop()
                if object_id in self._recovered_staging:
                    continue
                self._recovered_staging.add(object_id)
                pending.extend(row[0] for row in self._db.execute("SELECT child FROM edges WHERE parent=?",
                                                                  (object_id,)))
            self._db.execute("DELETE FROM leases WHERE owner=?", (owner,))
            self._db.execute("DELETE FROM owners WHERE id=?", (owner,))

    def _recover_files(self) -> tuple[int, int]:
        removed = reclaimed = 0
        for path in (self.root / "staging").glob("pending-*"):
            if path.is_file() and re.fullmatch(r"pending-[0-9a-f]{32}", path.name):
                reclaimed += path.stat().st_size
                path.unlink()
                removed += 1
        known = {row[0] for row in self._db.execute("SELECT id FROM objects")}
        known -= self._evicted - set(self._unevicted)
        for kind in ("blob", "basis", "manifest"):
            for path in (self.root / "objects" / kind).iterdir():
                if path.is_file() and re.fullmatch(r"[0-9a-f]{64}", path.name) and f"{kind}:{path.name}" not in known:
                    reclaimed += path.stat().st_size
                    path.unlink()
                    removed += 1
        return removed, reclaimed

    # -- garbage collection and eviction -------------------------------------------------------------------------

    def collect_garbage(self, *, candidates: Iterable[str] | None = None) -> dict[str, int]:
        """Delete every object that no ref or lease reaches (restricted to ``candidates`` when given).
        Index rows go first; files are removed after the commit, so a crash leaves only garbage."""
        candidate_ids = None if candidates is None else set(candidates)
        if candidate_ids is not None:
            for object_id in candidate_ids:
                self.path_for(object_id)
        damaged = None
        with self.transaction():
            self._reap_owners()
            recovered = set(self._recovered_staging)
            if candidate_ids is not None:
                candidate_ids |= recovered
            roots = [row[0] for row in self._db.execute("SELECT object_id FROM refs")]
            roots += [row[0] for row in self._db.execute("SELECT object_id FROM leases")]
            damaged = {} if self.on_damage == "keep" else None
            live = self._walk(roots, verify=True, damaged=damaged)
            if damaged is not None:
                self._damaged = damaged
            objects = dict(self._db.execute("SELECT id, size FROM objects"))
            dead = set(objects) - live
            if candidate_ids is not None:
                dead &= candidate_ids
                edges = tuple(self._db.execute("SELECT parent, child FROM edges"))
                while True:
                    referenced = {child for parent, child in edges if parent not in dead and child in dead}
                    if not referenced:
                        break
                    dead -= referenced
            for object_id in dead:
                self._db.execute("DELETE FROM edges WHERE parent=?", (object_id,))
                self._db.execute("DELETE FROM telemetry WHERE object_id=?", (object_id,))
            for object_id in dead:
                if object_id in self._evicted:
                    self._db.execute("DELETE FROM evicted WHERE id=?", (object_id,))
                self._db.execute("DELETE FROM objects WHERE id=?", (object_id,))
                self._events.append(("deleted", object_id))
            self._evicted.difference_update(dead)
            self._verified.difference_update(dead)
        with self.transaction():
            removed, reclaimed = self._recover_files()
            self._recovered_staging.difference_update(recovered)
        result = {"objects_removed": removed, "bytes_reclaimed": reclaimed, "live_objects": len(live)}
        if damaged:
            result["damaged_objects"] = len(damaged)
        return result

    gc = collect_garbage

    def _protected(self, object_ids: Iterable[str]) -> set[str]:
        wanted = set(object_ids)
        direct = {row[0] for row in self._db.execute("SELECT object_id FROM leases")}
        staging = [row[0] for row in self._db.execute("SELECT object_id FROM leases WHERE id LIKE 'staging-%'")]
        reach = self._walk(staging, verify=False) if staging else set()
        return wanted & (direct | reach)

    def evict(self, object_ids: Iterable[str]) -> dict[str, Any]:
        """Evict payload objects (blob/basis) all or nothing: files go, index rows and edges stay, reads raise
        :class:`EvictedObjectError`. Protected (leased) objects make the call evict nothing."""
        ids = sorted({i for i in object_ids if not i.startswith("manifest:")})
        for object_id in ids:
            self.path_for(object_id)
        with self.transaction():
            protected = self._protected(ids)
            if protected:
                return {"evicted": 0, "bytes": 0, "leased": sorted(protected)}
            self._db.execute("CREATE TABLE IF NOT EXISTS evicted (id TEXT PRIMARY KEY REFERENCES objects(id) "
                             "ON DELETE CASCADE)")
            sizes = dict(self._db.execute(f"SELECT id, size FROM objects WHERE id IN ({','.join('?' * len(ids))})",
                                          ids)) if ids else {}
            fresh = [i for i in ids if i in sizes and i not in self._evicted]
            for object_id in fresh:
                self._db.execute("INSERT OR IGNORE INTO evicted VALUES (?)", (object_id,))
            self._evicted.update(fresh)
        freed = 0
        for object_id in fresh:
            path = self.path_for(object_id)
            with contextlib.suppress(FileNotFoundError):
                path.unlink()
                freed += sizes[object_id]
        return {"evicted": len(fresh), "bytes": freed, "leased": []}

    def evicted_ids(self, object_ids: Iterable[str] | None = None) -> set[str]:
        return set(self._evicted) if object_ids is None else set(object_ids) & self._evicted

    # -- stats and lifetime ----------------------------------------------------------------------------------------

    def stats(self) -> dict[str, int]:
        with self.transaction():
            objects, size = self._db.execute("SELECT COUNT(*), COALESCE(SUM(size), 0) FROM objects").fetchone()
            refs = self._db.execute("SELECT COUNT(*) FROM refs").fetchone()[0]
            leases = self._db.execute("SELECT COUNT(DISTINCT id) FROM leases").fetchone()[0]
            by_kind = dict(self._db.execute("SELECT kind, COALESCE(SUM(size), 0) FROM objects GROUP BY kind"))
        return {"objects": objects, "bytes": size, "refs": refs, "leases": leases,
                "blob_bytes": by_kind.get("blob", 0), "basis_bytes": by_kind.get("basis", 0),
                "manifest_bytes": by_kind.get("manifest", 0), "evicted": len(self._evicted)}

    def close(self) -> None:
        with self._lock:
            if self._closed:
                return
            for lease in list(self._leases):
                lease._active = False
            try:
                with self.transaction():
                    self._db.execute("DELETE FROM leases WHERE owner=?", (self._owner,))
                    self._db.execute("DELETE FROM owners WHERE id=?", (self._owner,))
            except (StateError, IntegrityError):
                pass
            self._closed = True
            self._db.close()
            self._lock_file.close()
        if self._readers is not None:
            self._readers.shutdown(wait=False)
        if getattr(self, "_ahead", None) is not None:
            self._ahead.shutdown(wait=False)

    def __enter__(self) -> ObjectStore:
        return self

    def __exit__(self, *args: Any) -> None:
        self.close()
