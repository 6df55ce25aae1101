"""Content-addressed object store.

On-disk layout (shared with the reference implementation so that either opens the other's stores)::

    objects/{blob,basis,manifest}/<sha256>   immutable objects; an id is "<kind>:<sha256 of the bytes>"
    staging/pending-<32 hex>                 a new object is written and fsynced here, then hard-linked in
    store.lock                               advisory flock: one writer (publication, GC) at a time
    index.sqlite3                            WAL, synchronous=FULL; tables settings (format
                                             reelcache.store.v1), objects, edges, refs, owners, leases,
                                             telemetry, and (after the first eviction) evicted

A manifest is the canonical JSON ``{"format": "reelcache.manifest.v1", "references": [sorted ids],
"data": {...}}``; its references become index edges, so garbage collection sees the graph.

This module is built from three parts: :class:`_Index` (every SQL statement), :class:`_Files` (paths, atomic
writes, page-cache policy, I/O counters) and :class:`_Quarantine` (objects whose bytes failed a check; every
later read of them verifies until they pass). :class:`ObjectStore` composes them under one re-entrant lock
and one flock-guarded SQLite transaction: named refs move by compare-and-swap, leases pin graphs for a live
process (rows of dead owners are reaped at open and before GC), GC keeps what refs and leases reach, eviction
drops payload files under a budget while their index rows stay, and run telemetry is an unhashed sidecar.
"""

from __future__ import annotations

import contextlib
import fcntl
import hashlib
import os
import re
import sqlite3
import threading
import uuid
import weakref
from concurrent.futures import ThreadPoolExecutor
from pathlib import Path
from typing import Any, Iterable, Iterator, Mapping

from .errors import CapacityError, ConfigurationError, IntegrityError, QuarantinedError, StateError
from .serialization import canonical_json, parse_json

FORMAT = "reelcache.store.v1"
MANIFEST_FORMAT = "reelcache.manifest.v1"
IO_POLICIES = ("buffered", "nocache")
KINDS = ("blob", "basis", "manifest")
_ID = re.compile(r"(blob|basis|manifest):([0-9a-f]{64})")
_UNSET = object()
_PROCESS_LOCKS: dict[str, threading.RLock] = {}
_PROCESS_LOCKS_GUARD = threading.Lock()

# table and column names are part of the shared format
_TABLES = """
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
_REQUIRED_TABLES = {"settings", "objects", "edges", "refs", "owners", "leases"}
_EVICTED_TABLE = "CREATE TABLE IF NOT EXISTS evicted (id TEXT PRIMARY KEY REFERENCES objects(id) ON DELETE CASCADE)"


class EvictedObjectError(StateError):
    """The object's payload was evicted under an archive budget; its index row remains."""


def split_id(object_id: Any) -> tuple[str, str]:
    """``(kind, digest)`` of a well-formed object id."""
    match = _ID.fullmatch(object_id) if isinstance(object_id, str) else None
    if match is None:
        raise IntegrityError(f"{object_id!r} is not an object id (kind:sha256)")
    return match[1], match[2]


def _start_time(pid: int) -> str | None:
    """The process's start time from /proc (tells a reused pid from the original owner)."""
    try:
        with open(f"/proc/{pid}/stat", "rb") as handle:
            tail = handle.read().rsplit(b")", 1)[1].split()
        return tail[19].decode()
    except (OSError, IndexError):
        return None


def _owner_alive(pid: int, stamp: str | None) -> bool:
    try:
        os.kill(pid, 0)
    except ProcessLookupError:
        return False
    except PermissionError:
        pass
    if stamp is None:
        return True
    now = _start_time(pid)
    return now is None or now == stamp


class _Index:
    """The SQLite index: every statement the store runs lives here."""

    def __init__(self, path: Path, *, existed: bool):
        self.db = sqlite3.connect(path, timeout=60, isolation_level=None, check_same_thread=False)
        if existed:
            present = {name for (name,) in self.db.execute("SELECT name FROM sqlite_master WHERE type = 'table'")}
            if not _REQUIRED_TABLES.issubset(present):
                raise IntegrityError(f"the store index lacks tables {sorted(_REQUIRED_TABLES - present)}")
            stored = self.db.execute("SELECT value FROM settings WHERE key = 'format'").fetchone()
            if stored is None or stored[0] != FORMAT:
                raise IntegrityError(f"the store index has format {stored!r}, not {FORMAT}")
        for pragma in ("foreign_keys=ON", "journal_mode=WAL", "synchronous=FULL"):
            self.db.execute(f"PRAGMA {pragma}")
        self.db.executescript(_TABLES)
        self.db.execute("INSERT OR IGNORE INTO settings (key, value) VALUES ('format', :f)", {"f": FORMAT})

    # transactions
    def begin(self) -> None:
        self.db.execute("BEGIN IMMEDIATE")

    def commit(self) -> None:
        self.db.execute("COMMIT")

    def rollback(self) -> None:
        if self.db.in_transaction:
            self.db.execute("ROLLBACK")

    def close(self) -> None:
        self.db.close()

    # objects
    def row(self, object_id: str):
        return self.db.execute("SELECT kind, size FROM objects WHERE id = :i", {"i": object_id}).fetchone()

    def add_object(self, object_id: str, kind: str, size: int) -> None:
        self.db.execute("INSERT INTO objects (id, kind, size) VALUES (:i, :k, :s)", {"i": object_id, "k": kind,
                                                                                     "s": size})

    def drop_objects(self, ids: Iterable[str], *, evicted: set[str]) -> None:
        """Delete index rows of ``ids``: first every outgoing edge and telemetry row of all of them, then the
        object rows (an edge between two dropped objects would otherwise block the row it points at)."""
        ids = list(ids)
        for object_id in ids:
            self.db.execute("DELETE FROM edges WHERE parent = :i", {"i": object_id})
            self.db.execute("DELETE FROM telemetry WHERE object_id = :i", {"i": object_id})
        for object_id in ids:
            if object_id in evicted:
                self.db.execute("DELETE FROM evicted WHERE id = :i", {"i": object_id})
            self.db.execute("DELETE FROM objects WHERE id = :i", {"i": object_id})

    def all_sizes(self) -> dict[str, int]:
        return dict(self.db.execute("SELECT id, size FROM objects"))

    def total_bytes(self) -> int:
        return self.db.execute("SELECT COALESCE(SUM(size), 0) FROM objects").fetchone()[0]

    def ids(self) -> set[str]:
        return {object_id for (object_id,) in self.db.execute("SELECT id FROM objects")}

    def summary(self) -> tuple[int, int, int, int, dict[str, int]]:
        count, size = self.db.execute("SELECT COUNT(*), COALESCE(SUM(size), 0) FROM objects").fetchone()
        refs = self.db.execute("SELECT COUNT(*) FROM refs").fetchone()[0]
        leases = self.db.execute("SELECT COUNT(DISTINCT id) FROM leases").fetchone()[0]
        kinds = dict(self.db.execute("SELECT kind, COALESCE(SUM(size), 0) FROM objects GROUP BY kind"))
        return count, size, refs, leases, kinds

    # edges
    def link(self, parent: str, child: str) -> None:
        self.db.execute("INSERT OR IGNORE INTO edges (parent, child) VALUES (:p, :c)", {"p": parent, "c": child})

    def children(self, parent: str) -> tuple[str, ...]:
        return tuple(c for (c,) in self.db.execute("SELECT child FROM edges WHERE parent = :p ORDER BY child",
                                                   {"p": parent}))

    def all_edges(self) -> tuple[tuple[str, str], ...]:
        return tuple(self.db.execute("SELECT parent, child FROM edges"))

    # refs
    def ref(self, name: str) -> str | None:
        found = self.db.execute("SELECT object_id FROM refs WHERE name = :n", {"n": name}).fetchone()
        return None if found is None else found[0]

    def put_ref(self, name: str, object_id: str) -> None:
        self.db.execute("INSERT INTO refs (name, object_id) VALUES (:n, :o) "
                        "ON CONFLICT(name) DO UPDATE SET object_id = excluded.object_id", {"n": name, "o": object_id})

    def remove_ref(self, name: str) -> None:
        self.db.execute("DELETE FROM refs WHERE name = :n", {"n": name})

    def refs(self) -> list[tuple[str, str]]:
        return list(self.db.execute("SELECT name, object_id FROM refs ORDER BY name"))

    # owners and leases
    def add_owner(self, owner: str, pid: int, stamp: str | None) -> None:
        self.db.execute("INSERT INTO owners (id, pid, stamp) VALUES (:o, :p, :s)", {"o": owner, "p": pid, "s": stamp})

    def owners(self) -> list[tuple[str, int, str | None]]:
        return list(self.db.execute("SELECT id, pid, stamp FROM owners"))

    def drop_owner(self, owner: str) -> None:
        self.db.execute("DELETE FROM leases WHERE owner = :o", {"o": owner})
        self.db.execute("DELETE FROM owners WHERE id = :o", {"o": owner})

    def add_lease(self, lease: str, owner: str, object_id: str) -> None:
        self.db.execute("INSERT INTO leases (id, owner, object_id) VALUES (:l, :o, :i)",
                        {"l": lease, "o": owner, "i": object_id})

    def drop_lease(self, lease: str, owner: str) -> None:
        self.db.execute("DELETE FROM leases WHERE id = :l AND owner = :o", {"l": lease, "o": owner})

    def leases_of(self, owner: str) -> list[tuple[str, str]]:
        return list(self.db.execute("SELECT id, object_id FROM leases WHERE owner = :o", {"o": owner}))

    def leased(self, *, staging_only: bool = False) -> list[str]:
        sql = "SELECT object_id FROM leases" + (" WHERE id LIKE 'staging-%'" if staging_only else "")
        return [object_id for (object_id,) in self.db.execute(sql)]

    # telemetry
    def put_telemetry(self, object_id: str, text: str) -> None:
        self.db.execute("INSERT INTO telemetry (object_id, data) VALUES (:i, :d) "
                        "ON CONFLICT(object_id) DO UPDATE SET data = excluded.data", {"i": object_id, "d": text})

    def telemetry(self, object_id: str) -> str | None:
        found = self.db.execute("SELECT data FROM telemetry WHERE object_id = :i", {"i": object_id}).fetchone()
        return None if found is None else found[0]

    # eviction
    def evicted(self) -> set[str]:
        present = self.db.execute("SELECT 1 FROM sqlite_master WHERE type = 'table' AND name = 'evicted'").fetchone()
        return set() if present is None else {i for (i,) in self.db.execute("SELECT id FROM evicted")}

    def mark_evicted(self, ids: Iterable[str]) -> None:
        self.db.execute(_EVICTED_TABLE)
        for object_id in ids:
            self.db.execute("INSERT OR IGNORE INTO evicted (id) VALUES (:i)", {"i": object_id})

    def unmark_evicted(self, object_id: str) -> None:
        self.db.execute("DELETE FROM evicted WHERE id = :i", {"i": object_id})


class _Files:
    """Object files: paths, atomic creation (staging file, fsync, hard link), page-cache policy, counters."""

    def __init__(self, root: Path):
        self.root = root
        self.policy = "buffered"
        self.dirty: set[Path] = set()
        self.lock = threading.Lock()
        self.counters = {"read_calls": 0, "read_bytes": 0, "write_calls": 0, "write_bytes": 0, "existing_calls": 0,
                         "existing_bytes": 0, "errors": 0, "last_error": None}

    def path(self, object_id: str) -> Path:
        kind, digest = split_id(object_id)
        return self.root / "objects" / kind / digest

    def _drop_cache(self, fd: int) -> None:
        if self.policy == "nocache":
            with contextlib.suppress(OSError):
                os.posix_fadvise(fd, 0, 0, os.POSIX_FADV_DONTNEED)

    def _count(self, name: str, nbytes: int) -> None:
        with self.lock:
            self.counters[f"{name}_calls"] += 1
            self.counters[f"{name}_bytes"] += nbytes

    def read(self, path: Path) -> bytes:
        with open(path, "rb") as handle:
            data = handle.read()
            self._drop_cache(handle.fileno())
        self._count("read", len(data))
        return data

    def read_object(self, object_id: str) -> bytes:
        try:
            return self.read(self.path(object_id))
        except OSError as exc:
            with self.lock:
                self.counters["errors"] += 1
                self.counters["last_error"] = str(exc)
            raise IntegrityError(f"object {object_id} cannot be read: {exc}") from exc

    def write(self, path: Path, data: bytes) -> None:
        temp = self.root / "staging" / f"pending-{uuid.uuid4().hex}"
        try:
            with temp.open("xb") as handle:
                handle.write(data)
                handle.flush()
                os.fsync(handle.fileno())
                self._drop_cache(handle.fileno())
            path.unlink(missing_ok=True)
            os.link(temp, path)
            self.dirty.add(path.parent)
        finally:
            temp.unlink(missing_ok=True)
        self._count("write", len(data))

    def sync_dirty(self) -> None:
        for directory in sorted(self.dirty):
            fd = os.open(directory, os.O_RDONLY | os.O_DIRECTORY)
            try:
                os.fsync(fd)
            finally:
                os.close(fd)

    def drop_all_cached(self) -> int:
        count = 0
        for kind in KINDS:
            for path in (self.root / "objects" / kind).iterdir():
                with contextlib.suppress(OSError):
                    fd = os.open(path, os.O_RDONLY)
                    try:
                        os.posix_fadvise(fd, 0, 0, os.POSIX_FADV_DONTNEED)
                        count += 1
                    finally:
                        os.close(fd)
        return count

    def sweep(self, indexed: set[str]) -> tuple[int, int]:
        """Delete leftover staging files and object files the index does not list."""
        removed = freed = 0
        for path in (self.root / "staging").glob("pending-*"):
            if path.is_file() and re.fullmatch(r"pending-[0-9a-f]{32}", path.name):
                freed += path.stat().st_size
                path.unlink()
                removed += 1
        for kind in KINDS:
            for path in (self.root / "objects" / kind).iterdir():
                if path.is_file() and re.fullmatch(r"[0-9a-f]{64}", path.name) and f"{kind}:{path.name}" not in indexed:
                    freed += path.stat().st_size
                    path.unlink()
                    removed += 1
        return removed, freed


class _Quarantine:
    """Objects whose bytes failed a check, with the reason; a passing verification lifts the mark."""

    def __init__(self):
        self.lock = threading.Lock()
        self.marked: dict[str, str] = {}

    def mark(self, object_id: str, reason: str) -> bool:
        """Mark ``object_id``; returns whether it was already marked."""
        with self.lock:
            before = object_id in self.marked
            self.marked[object_id] = str(reason)
            return before

    def lift(self, object_id: str) -> bool:
        with self.lock:
            return self.marked.pop(object_id, None) is not None

    def __contains__(self, object_id: str) -> bool:
        return object_id in self.marked

    def snapshot(self) -> dict[str, str]:
        with self.lock:
            return dict(self.marked)


class ObjectLease:
    """A pin on a set of objects and everything they reference, held by this process until released."""

    def __init__(self, store: "ObjectStore", lease_id: str, object_ids: tuple[str, ...]) -> None:
        self._store = store
        self.lease_id = lease_id
        self.object_ids = object_ids
        self._active = True

    @property
    def active(self) -> bool:
        return self._active

    def release(self) -> None:
        if not self._active:
            return
        self._active = False
        if not self._store.closed:
            self._store._release_lease(self.lease_id)

    def __enter__(self) -> "ObjectLease":
        return self

    def __exit__(self, *args: Any) -> None:
        self.release()

    def __del__(self) -> None:
        with contextlib.suppress(Exception):
            self.release()


class ReadAhead:
    """Background reads of object payloads into a byte-bounded buffer; ``take`` hands a payload over."""

    def __init__(self, store: "ObjectStore", max_bytes: int) -> None:
        if type(max_bytes) is not int or max_bytes < 0:
            raise ConfigurationError(f"read-ahead max_bytes must be a nonnegative integer, got {max_bytes!r}")
        self._store = store
        self._limit = max_bytes
        self._lock = threading.Lock()
        self._buffer: dict[str, bytes] = {}
        self._buffered = 0
        self._queue: list[str] = []
        self._futures = []
        self.hits = self.misses = 0
        self._closed = False

    def schedule(self, object_ids: Iterable[str]) -> int:
        """Queue payloads (in order) while they fit the remaining budget; returns how many were queued."""
        wanted = [i for i in object_ids if i not in self._buffer]
        sizes = self._store.object_sizes(wanted)
        queued = 0
        with self._lock:
            room = self._limit - self._buffered
            for object_id in wanted:
                size = sizes.get(object_id, 0)
                if size > room:
                    break
                room -= size
                self._queue.append(object_id)
                queued += 1
        if queued:
            self._futures.append(self._store._ahead_pool().submit(self._drain))
        return queued

    def _drain(self) -> None:
        while True:
            with self._lock:
                if self._closed or not self._queue:
                    return
                object_id = self._queue.pop(0)
            try:
                data = self._store.get(object_id)
            except Exception:  # noqa: BLE001 - a miss makes the consumer read (and report) it itself
                continue
            with self._lock:
                if not self._closed:
                    self._buffer[object_id] = data
                    self._buffered += len(data)

    def take(self, object_id: str) -> bytes | None:
        with self._lock:
            data = self._buffer.pop(object_id, None)
            if data is None:
                self.misses += 1
            else:
                self._buffered -= len(data)
                self.hits += 1
            return data

    @property
    def held_bytes(self) -> int:
        return self._buffered

    def stats(self) -> dict[str, int]:
        return {"hits": self.hits, "misses": self.misses, "held_bytes": self._buffered}

    def close(self) -> None:
        with self._lock:
            self._closed = True
            self._buffer.clear()
            self._buffered = 0
            self._queue.clear()


class ObjectStore:
    """The immutable blob / basis / manifest namespaces of one root, with atomic named refs.

    ``verify_reads``: hash every object read for use. ``verify_references`` (default: ``verify_reads``): graph
    operations read and hash what they reach instead of trusting the index. ``on_damage``: what GC does with a
    damaged graph -- ``"raise"``, or ``"keep"`` (record it in :attr:`damaged` and keep going).
    """

    def __init__(self, root: str | os.PathLike[str], *, max_bytes: int | None = None, verify_reads: bool = False,
                 verify_references: bool | None = None, on_damage: str = "raise") -> None:
        if max_bytes is not None and (type(max_bytes) is not int or max_bytes < 0):
            raise ConfigurationError(f"max_bytes must be a nonnegative integer or None, got {max_bytes!r}")
        if type(verify_reads) is not bool or (verify_references is not None and type(verify_references) is not bool):
            raise ConfigurationError("verify_reads and verify_references are booleans")
        if on_damage not in ("raise", "keep"):
            raise ConfigurationError(f"on_damage is 'raise' or 'keep', not {on_damage!r}")
        self.verify_reads = verify_reads
        self.verify_references = verify_reads if verify_references is None else verify_references
        self.on_damage = on_damage
        self.max_bytes = max_bytes
        self.root = Path(root).resolve()
        for sub in [Path("objects") / kind for kind in KINDS] + [Path("staging")]:
            (self.root / sub).mkdir(parents=True, exist_ok=True)
        with _PROCESS_LOCKS_GUARD:
            self._lock = _PROCESS_LOCKS.setdefault(str(self.root), threading.RLock())
        lock_path = self.root / "store.lock"
        lock_existed = lock_path.exists()
        self._flock = lock_path.open("a+b")
        self._files = _Files(self.root)
        self._quarantine = _Quarantine()
        self._closed = False
        self._depth = 0
        self._doomed = False               # a nested failure: the outermost transaction must roll back
        self._created: list[str] = []
        self._touched: dict[str, None] = {}
        self._events: list[tuple[str, str]] = []
        self.hooks: Any = None             # callable(event, object_id) after each commit
        self._damaged: dict[str, str] = {}
        self._verify_count = threading.local()
        self._recovered: set[str] = set()  # staging objects of dead owners, collected after open
        self._owner = uuid.uuid4().hex
        self._leases: weakref.WeakSet[ObjectLease] = weakref.WeakSet()
        self._readers: ThreadPoolExecutor | None = None
        self._ahead: ThreadPoolExecutor | None = None
        self._pools_lock = threading.Lock()
        self._evicted: set[str] = set()
        self._restored: list[str] = []     # evicted objects rewritten by the open transaction
        # objects whose subtree a reference update of this process already checked (immutable content: later
        # updates only walk what is new below them)
        self._checked: set[str] = set()
        try:
            with self._lock:
                fcntl.flock(self._flock, fcntl.LOCK_EX)
                try:
                    self._index = self._open_index(lock_existed)
                    self._evicted = self._index.evicted()
                finally:
                    fcntl.flock(self._flock, fcntl.LOCK_UN)
            with self.transaction():
                self._reap_dead_owners()
                self._index.add_owner(self._owner, os.getpid(), _start_time(os.getpid()))
                self._sweep_files()
            if self._recovered:
                self.collect_garbage(candidates=self._recovered)
        except sqlite3.Error as exc:
            self._shut()
            raise IntegrityError(f"the store index at {self.root} cannot be opened: {exc}") from exc
        except BaseException:
            self._shut()
            raise

    def _open_index(self, lock_existed: bool) -> _Index:
        path = self.root / "index.sqlite3"
        existed = path.exists()
        if not existed:
            leftovers = lock_existed or any((self.root / "objects").glob("*/*")) or \
                any((self.root / "staging").iterdir())
            if leftovers:
                raise IntegrityError(f"{self.root} holds store state but no index; it will not be reinitialized")
        elif path.stat().st_size < 100:
            raise IntegrityError(f"the store index at {path} is truncated")
        return _Index(path, existed=existed)

    def _shut(self) -> None:
        self._closed = True
        if getattr(self, "_index", None) is not None:
            self._index.close()
        self._flock.close()

    # -- transactions ----------------------------------------------------------------------------------------

    @property
    def closed(self) -> bool:
        return self._closed

    @contextlib.contextmanager
    def transaction(self) -> Iterator["ObjectStore"]:
        """One SQLite IMMEDIATE transaction under the store flock; nested calls join the outermost one."""
        fired: list[tuple[str, str]] = []
        with self._lock:
            if self._closed:
                raise StateError(f"the store at {self.root} is closed")
            outermost = self._depth == 0
            if outermost:
                fcntl.flock(self._flock, fcntl.LOCK_EX)
                try:
                    self._index.begin()
                except sqlite3.Error as exc:
                    fcntl.flock(self._flock, fcntl.LOCK_UN)
                    raise IntegrityError(f"a store transaction cannot start: {exc}") from exc
                self._doomed = False
                self._created, self._touched, self._events, self._restored = [], {}, [], []
            self._depth += 1
            try:
                yield self
                if outermost:
                    if self._doomed:
                        raise StateError("an operation inside this transaction failed; it was rolled back")
                    self._files.sync_dirty()
                    self._index.commit()
                    self._evicted.difference_update(self._restored)
                    if self.hooks is not None:
                        fired = self._events
            except BaseException as exc:
                self._doomed = True
                if outermost:
                    self._index.rollback()
                if isinstance(exc, sqlite3.Error):
                    raise IntegrityError(f"a store index operation failed: {exc}") from exc
                raise
            finally:
                self._depth -= 1
                if outermost:
                    self._files.dirty.clear()
                    self._events = []
                    fcntl.flock(self._flock, fcntl.LOCK_UN)
        for event, object_id in fired:
            self.hooks(event, object_id)

    def _inside(self, what: str) -> None:
        if not self._depth:
            raise StateError(f"{what} is only known inside a store transaction")

    @property
    def created_objects(self) -> tuple[str, ...]:
        with self._lock:
            self._inside("created_objects")
            return tuple(self._created)

    @property
    def touched_objects(self) -> tuple[str, ...]:
        with self._lock:
            self._inside("touched_objects")
            return tuple(self._touched)

    # -- files and I/O policy --------------------------------------------------------------------------------

    def path_for(self, object_id: str) -> Path:
        return self._files.path(object_id)

    @property
    def io_policy(self) -> str:
        return self._files.policy

    @property
    def io_stats_(self) -> dict:
        return self._files.counters

    def set_io_policy(self, policy: str, *, drop_existing: bool = False) -> dict[str, Any]:
        """``buffered`` or ``nocache`` (drop written and read pages from the page cache)."""
        if policy not in IO_POLICIES:
            raise ConfigurationError(f"store I/O policy {policy!r} is not one of {IO_POLICIES}")
        self._files.policy = policy
        dropped = self._files.drop_all_cached() if (drop_existing and policy == "nocache") else 0
        return {"policy": policy, "dropped_files": dropped}

    def io_stats(self) -> dict[str, Any]:
        with self._files.lock:
            return dict(self._files.counters, policy=self._files.policy)

    # -- quarantine ------------------------------------------------------------------------------------------

    def quarantine(self, object_id: str, reason: str) -> None:
        split_id(object_id)
        self._quarantine.mark(object_id, reason)

    def lift_quarantine(self, object_id: str) -> bool:
        return self._quarantine.lift(object_id)

    @property
    def quarantined_objects(self) -> dict[str, str]:
        return self._quarantine.snapshot()

    def check_quarantined(self, object_ids: Iterable[str]) -> None:
        """Re-verify the quarantined ones among ``object_ids`` (raises while they still fail)."""
        for object_id in object_ids:
            if object_id in self._quarantine:
                self._get(object_id, verify=True)

    @property
    def verified_payloads(self) -> int:
        return getattr(self._verify_count, "value", 0)

    # -- reads -----------------------------------------------------------------------------------------------

    def _present(self, object_id: str) -> None:
        """The object is indexed and (unless evicted) its file exists."""
        path = self.path_for(object_id)
        if self._index.row(object_id) is None:
            raise IntegrityError(f"object {object_id} is not in the store")
        if object_id not in self._evicted and not path.exists():
            raise IntegrityError(f"object {object_id} is indexed but its file is gone")

    def _row_for_read(self, object_id: str):
        row = self._index.row(object_id)
        if row is None:
            raise IntegrityError(f"object {object_id} is not in the store")
        if object_id in self._evicted:
            raise EvictedObjectError(f"the payload of {object_id} was evicted")
        return row

    def _get(self, object_id: str, *, verify: bool | None = None, data: bytes | None = None, row=None) -> bytes:
        split_id(object_id)
        row = self._row_for_read(object_id) if row is None else row
        check = (self.verify_reads if verify is None else verify) or object_id in self._quarantine
        data = self._files.read_object(object_id) if data is None else data
        if len(data) != row[1]:
            self._reject(object_id, f"{len(data)} bytes on disk, {row[1]} in the index")
        if check:
            self._verify_count.value = getattr(self._verify_count, "value", 0) + 1
            if hashlib.sha256(data).hexdigest() != split_id(object_id)[1]:
                self._reject(object_id, "its bytes do not hash to its id")
            self._quarantine.lift(object_id)
        return data

    def _reject(self, object_id: str, reason: str) -> None:
        if self._quarantine.mark(object_id, reason):
            raise QuarantinedError(f"quarantined object {object_id} failed verification again: {reason}")
        raise IntegrityError(f"object {object_id} is corrupt: {reason}")

    def get(self, object_id: str) -> bytes:
        with self.transaction():
            return self._get(object_id)

    get_bytes = get

    def _reader_pool(self) -> ThreadPoolExecutor:
        """Workers for the file reads of :meth:`get_many` (they never touch the index)."""
        with self._pools_lock:
            if self._readers is None:
                self._readers = ThreadPoolExecutor(max_workers=8, thread_name_prefix="reelcache-store-read")
            return self._readers

    def _ahead_pool(self) -> ThreadPoolExecutor:
        """Read-ahead workers: they take the store lock per object, so they must not share the reader pool
        (whose caller holds that lock while it waits)."""
        with self._pools_lock:
            if self._ahead is None:
                self._ahead = ThreadPoolExecutor(max_workers=4, thread_name_prefix="reelcache-store-ahead")
            return self._ahead

    def get_many(self, object_ids: Iterable[str], *, verify: bool | None = None,
                 read_ahead: ReadAhead | None = None) -> dict[str, bytes]:
        """Several objects in one index transaction; their files are read in parallel."""
        ordered = list(dict.fromkeys(object_ids))
        found: dict[str, bytes] = {}
        if read_ahead is not None:
            for object_id in ordered:
                data = read_ahead.take(object_id)
                if data is not None:
                    found[object_id] = data
        missing = [i for i in ordered if i not in found]
        with self.transaction():
            rows = {}
            for object_id in missing:
                split_id(object_id)
                rows[object_id] = self._row_for_read(object_id)
            if len(missing) > 1:
                blobs = self._reader_pool().map(self._files.read_object, missing)
                for object_id, data in zip(missing, blobs):
                    found[object_id] = self._get(object_id, verify=verify, data=data, row=rows[object_id])
            else:
                for object_id in missing:
                    found[object_id] = self._get(object_id, verify=verify, row=rows[object_id])
        return {object_id: found[object_id] for object_id in ordered}

    def read_ahead(self, object_ids: Iterable[str] = (), *, max_bytes: int) -> ReadAhead:
        reader = ReadAhead(self, max_bytes)
        reader.schedule(object_ids)
        return reader

    def object_size(self, object_id: str) -> int:
        split_id(object_id)
        with self.transaction():
            row = self._index.row(object_id)
        if row is None:
            raise IntegrityError(f"object {object_id} is not in the store")
        return row[1]

    def object_sizes(self, object_ids: Iterable[str]) -> dict[str, int]:
        wanted = list(object_ids)
        with self.transaction():
            rows = {object_id: self._index.row(object_id) for object_id in wanted}
        return {object_id: row[1] for object_id, row in rows.items() if row is not None}

    def indexed(self, object_ids: Iterable[str]) -> set[str]:
        return set(self.object_sizes(object_ids))

    # -- writes ----------------------------------------------------------------------------------------------

    def _put(self, data: bytes, kind: str) -> str:
        if kind not in KINDS:
            raise ConfigurationError(f"object kind {kind!r} is not one of {KINDS}")
        if not isinstance(data, bytes):
            raise ConfigurationError("objects are stored from bytes")
        object_id = f"{kind}:{hashlib.sha256(data).hexdigest()}"
        path = self.path_for(object_id)
        self._touched[object_id] = None
        if self._index.row(object_id) is not None:
            if object_id in self._evicted:          # an evicted payload written again: restore its file
                self._files.write(path, data)
                self._index.unmark_evicted(object_id)
                self._restored.append(object_id)
                self._events.append(("created", object_id))
            else:
                self._present(object_id)
                self._events.append(("existing", object_id))
                with self._files.lock:
                    self._files.counters["existing_calls"] += 1
                    self._files.counters["existing_bytes"] += len(data)
            return object_id
        if self.max_bytes is not None:
            needed = self._index.total_bytes() + len(data)
            if needed > self.max_bytes:
                raise CapacityError(f"the store would hold {needed} bytes, above its budget of {self.max_bytes}")
        if path.exists():                             # a file without an index row: must hold these bytes
            try:
                on_disk = self._files.read(path)
            except OSError as exc:
                raise IntegrityError(f"an unindexed file for {object_id} cannot be read: {exc}") from exc
            if on_disk != data:
                raise IntegrityError(f"an unindexed file for {object_id} holds other bytes")
        else:
            self._files.write(path, data)
        self._quarantine.lift(object_id)
        self._index.add_object(object_id, kind, len(data))
        self._created.append(object_id)
        self._events.append(("created", object_id))
        return object_id

    def put(self, data: bytes, *, kind: str = "blob") -> str:
        if kind == "manifest":
            raise ConfigurationError("manifests go through put_manifest, which records their references")
        with self.transaction():
            return self._put(data, kind)

    put_bytes = put

    def put_manifest(self, data: Mapping[str, Any], *, references: Iterable[str] = ()) -> str:
        if not isinstance(data, Mapping):
            raise ConfigurationError("manifest data is a JSON object")
        refs = sorted(set(references))
        with self.transaction():
            for ref in refs:
                self._present(ref)
            body = canonical_json({"format": MANIFEST_FORMAT, "references": refs, "data": data})
            object_id = self._put(body, "manifest")
            for ref in refs:
                self._index.link(object_id, ref)
            return object_id

    def _manifest(self, object_id: str) -> tuple[dict[str, Any], tuple[str, ...]]:
        if not isinstance(object_id, str) or not object_id.startswith("manifest:"):
            raise IntegrityError(f"{object_id!r} is not a manifest")
        value = parse_json(self._get(object_id))
        well_formed = (isinstance(value, dict) and set(value) == {"format", "references", "data"}
                       and value["format"] == MANIFEST_FORMAT and isinstance(value["data"], dict)
                       and isinstance(value["references"], list)
                       and all(isinstance(ref, str) for ref in value["references"])
                       and value["references"] == sorted(set(value["references"])))
        if not well_formed:
            raise IntegrityError(f"manifest {object_id} is malformed")
        refs = tuple(value["references"])
        for ref in refs:
            split_id(ref)
        if self._index.children(object_id) != refs:
            raise IntegrityError(f"manifest {object_id} lists other references than the index records")
        return value["data"], refs

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
        """Attach unhashed run telemetry to an object (the latest write wins; GC removes it with the object)."""
        split_id(object_id)
        if not isinstance(data, Mapping):
            raise ConfigurationError("object telemetry is a JSON object")
        text = canonical_json(data).decode("utf-8")
        with self.transaction():
            if self._index.row(object_id) is None:
                raise IntegrityError(f"object {object_id} is not in the store")
            self._index.put_telemetry(object_id, text)

    def telemetry(self, object_id: str) -> dict[str, Any] | None:
        split_id(object_id)
        with self.transaction():
            text = self._index.telemetry(object_id)
        return None if text is None else parse_json(text.encode("utf-8"))

    # -- graph walks -----------------------------------------------------------------------------------------

    def _walk(self, roots: Iterable[str], *, verify: bool, damaged: dict[str, str] | None = None,
              force: bool = False, cached: bool = False) -> set[str]:
        """Every object reachable from ``roots``, each checked to exist (and, when ``verify`` applies, read and
        hashed). ``damaged``: record failures and keep walking instead of raising. ``cached`` (reference
        updates): an object whose subtree an earlier cached walk checked is only checked to exist and is not
        descended into -- GC never removes a child an existing manifest references -- so publishing a node
        costs its new objects, not the history below it (the result is then not the full reachable set)."""
        deep = verify and (self.verify_references or force)
        visited: set[str] = set()
        pending = list(roots)
        while pending:
            object_id = pending.pop()
            if object_id in visited:
                continue
            visited.add(object_id)
            if cached and object_id in self._checked:
                self._present(object_id)
                continue
            try:
                kind, _ = split_id(object_id)
                if kind == "manifest":
                    if deep:
                        pending.extend(self._manifest(object_id)[1])
                    else:
                        self._present(object_id)
                        pending.extend(self._index.children(object_id))
                elif deep and object_id not in self._evicted:
                    self._get(object_id, verify=True)
                else:
                    self._present(object_id)
            except IntegrityError as exc:
                if damaged is None:
                    raise
                damaged[object_id] = str(exc)
                pending.extend(self._index.children(object_id))
        if cached:
            self._checked |= visited
        return visited

    def verify(self, object_id: str, *, recursive: bool = True) -> None:
        """Read and hash ``object_id`` (and, recursively, everything it reaches)."""
        with self.transaction():
            if recursive:
                self._walk([object_id], verify=True, force=True)
            else:
                self._get(object_id, verify=True)

    def check(self, object_id: str) -> None:
        """Existence check of everything ``object_id`` reaches (index and files; no hashing)."""
        with self.transaction():
            self._walk([object_id], verify=False)

    @property
    def damaged(self) -> dict[str, str]:
        return dict(self._damaged)

    # -- refs ------------------------------------------------------------------------------------------------

    @staticmethod
    def _check_name(name: Any) -> None:
        if not isinstance(name, str) or name == "" or "\x00" in name:
            raise ConfigurationError(f"ref name {name!r} must be a nonempty string without NUL")

    def get_ref(self, name: str) -> str | None:
        self._check_name(name)
        with self.transaction():
            return self._index.ref(name)

    def _expect(self, name: str, expected: Any) -> str | None:
        current = self._index.ref(name)
        if expected is not _UNSET and current != expected:
            raise StateError(f"ref {name!r} moved to {current!r} while {expected!r} was expected")
        return current

    def set_ref(self, name: str, object_id: str, *, expected: Any = _UNSET) -> None:
        """Point ``name`` at ``object_id`` -- compare-and-swap when ``expected`` is given (None: the ref must not
        exist yet); the target graph is checked first."""
        self._check_name(name)
        with self.transaction():
            self._expect(name, expected)
            self._walk([object_id], verify=True, cached=True)
            self._index.put_ref(name, object_id)

    def delete_ref(self, name: str, *, expected: Any = _UNSET) -> None:
        self._check_name(name)
        with self.transaction():
            if self._expect(name, expected) is None:
                raise StateError(f"ref {name!r} does not exist")
            self._index.remove_ref(name)

    def list_refs(self, prefix: str = "") -> dict[str, str]:
        with self.transaction():
            return {name: object_id for name, object_id in self._index.refs() if name.startswith(prefix)}

    # -- leases and owners -----------------------------------------------------------------------------------

    def lease(self, object_ids: str | Iterable[str], *, purpose: str = "read", verify: bool = True) -> ObjectLease:
        """Pin a graph for this process. ``purpose="staging"`` marks a pending publication: if its owner dies,
        the next open collects it."""
        if purpose not in ("read", "staging"):
            raise ConfigurationError(f"lease purpose {purpose!r} is neither 'read' nor 'staging'")
        if type(verify) is not bool:
            raise ConfigurationError("lease verification is a boolean")
        ids = tuple(sorted({object_ids} if isinstance(object_ids, str) else set(object_ids)))
        if not ids:
            raise ConfigurationError("a lease pins at least one object")
        with self.transaction():
            self._walk(ids, verify=verify)
            lease_id = ("staging-" if purpose == "staging" else "") + uuid.uuid4().hex
            for object_id in ids:
                self._index.add_lease(lease_id, self._owner, object_id)
            lease = ObjectLease(self, lease_id, ids)
            self._leases.add(lease)
            return lease

    def _release_lease(self, lease_id: str) -> None:
        with self.transaction():
            self._index.drop_lease(lease_id, self._owner)

    def _reap_dead_owners(self) -> None:
        """Drop owners whose process is gone; the graphs of their staging leases become GC candidates."""
        for owner, pid, stamp in self._index.owners():
            if _owner_alive(pid, stamp):
                continue
            frontier = [object_id for lease_id, object_id in self._index.leases_of(owner)
                        if lease_id.startswith("staging-")]
            while frontier:
                object_id = frontier.pop()
                if object_id not in self._recovered:
                    self._recovered.add(object_id)
                    frontier.extend(self._index.children(object_id))
            self._index.drop_owner(owner)

    def _sweep_files(self) -> tuple[int, int]:
        indexed = self._index.ids() - (self._evicted - set(self._restored))
        return self._files.sweep(indexed)

    # -- garbage collection and eviction ---------------------------------------------------------------------

    def collect_garbage(self, *, candidates: Iterable[str] | None = None) -> dict[str, int]:
        """Delete every object no ref or lease reaches (only among ``candidates`` when given). Index rows go
        in the transaction; files are removed after it commits, so a crash leaves only unindexed files, which
        the next open sweeps."""
        limit = None if candidates is None else set(candidates)
        for object_id in limit or ():
            split_id(object_id)
        damaged = None
        with self.transaction():
            self._reap_dead_owners()
            recovered = set(self._recovered)
            if limit is not None:
                limit |= recovered
            roots = [object_id for _, object_id in self._index.refs()] + self._index.leased()
            damaged = {} if self.on_damage == "keep" else None
            live = self._walk(roots, verify=True, damaged=damaged)
            if damaged is not None:
                self._damaged = damaged
            dead = set(self._index.all_sizes()) - live
            if limit is not None:
                dead &= limit
                edges = self._index.all_edges()
                while True:   # a candidate still referenced by a surviving object survives too
                    kept = {child for parent, child in edges if child in dead and parent not in dead}
                    if not kept:
                        break
                    dead -= kept
            self._index.drop_objects(dead, evicted=self._evicted)
            self._events.extend(("deleted", object_id) for object_id in dead)
            self._evicted -= dead
            self._checked -= dead
        with self.transaction():
            removed, freed = self._sweep_files()
            self._recovered -= recovered
        report = {"objects_removed": removed, "bytes_reclaimed": freed, "live_objects": len(live)}
        if damaged:
            report["damaged_objects"] = len(damaged)
        return report

    gc = collect_garbage

    def _leased_among(self, object_ids: Iterable[str]) -> set[str]:
        direct = set(self._index.leased())
        staged = self._index.leased(staging_only=True)
        reach = self._walk(staged, verify=False) if staged else set()
        return set(object_ids) & (direct | reach)

    def evict(self, object_ids: Iterable[str]) -> dict[str, Any]:
        """Remove payload files (blob / basis) all or nothing: index rows and edges stay, reads raise
        :class:`EvictedObjectError`. If any of them is leased, nothing is evicted."""
        ids = sorted({i for i in object_ids if not i.startswith("manifest:")})
        for object_id in ids:
            split_id(object_id)
        with self.transaction():
            leased = self._leased_among(ids)
            if leased:
                return {"evicted": 0, "bytes": 0, "leased": sorted(leased)}
            sizes = {i: row[1] for i in ids if (row := self._index.row(i)) is not None}
            fresh = [i for i in ids if i in sizes and i not in self._evicted]
            self._index.mark_evicted(fresh)
            self._evicted.update(fresh)
        freed = 0
        for object_id in fresh:
            with contextlib.suppress(FileNotFoundError):
                self.path_for(object_id).unlink()
                freed += sizes[object_id]
        return {"evicted": len(fresh), "bytes": freed, "leased": []}

    def evicted_ids(self, object_ids: Iterable[str] | None = None) -> set[str]:
        return set(self._evicted) if object_ids is None else set(object_ids) & self._evicted

    # -- accounting and lifetime -----------------------------------------------------------------------------

    def stats(self) -> dict[str, int]:
        with self.transaction():
            count, size, refs, leases, kinds = self._index.summary()
        return {"objects": count, "bytes": size, "refs": refs, "leases": leases,
                "blob_bytes": kinds.get("blob", 0), "basis_bytes": kinds.get("basis", 0),
                "manifest_bytes": kinds.get("manifest", 0), "evicted": len(self._evicted)}

    def close(self) -> None:
        with self._lock:
            if self._closed:
                return
            for lease in list(self._leases):
                lease._active = False
            with contextlib.suppress(StateError, IntegrityError):
                with self.transaction():
                    self._index.drop_owner(self._owner)
            self._shut()
        for pool in (self._readers, self._ahead):
            if pool is not None:
                pool.shutdown(wait=False)

    def __enter__(self) -> "ObjectStore":
        return self

    def __exit__(self, *args: Any) -> None:
        self.close()


__all__ = ["FORMAT", "IO_POLICIES", "MANIFEST_FORMAT", "EvictedObjectError", "ObjectLease", "ObjectStore",
           "ReadAhead", "split_id"]
