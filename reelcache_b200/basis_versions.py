"""Immutable FP16 basis row blocks and the version chains built from them.

Storage (shared with the reference implementation, reelcache/basis_versions.py, so that either can read the
other's store): every version is a manifest ``{"type": "basis_version", "version": 1, "record":
<reelcache.basis_version.v1>}`` that references exactly its own row block (a ``basis:`` object of FP16
little-endian rows) and, unless it is a root, its parent version. A version's view is its ancestors' rows
followed by its own block -- appended, never rewritten -- so chunks that share or extend a basis share these
objects and garbage collection follows the whole chain.

Lossy packets name the exact prefix view they were encoded against with a ``basis`` descriptor (shape, view
rank, byte count, SHA-256); :func:`attach_basis` puts an assembled prefix back only when it matches.
"""

from __future__ import annotations

import hashlib
import sys
from collections import OrderedDict
from dataclasses import dataclass
from typing import Any, Iterable, Mapping

import numpy as np
import torch

from .errors import CapacityError, ConfigurationError, IntegrityError
from .store import ObjectStore
from .types import BasisVersion, EncodedTensor, MatrixKey, ModelIdentity, json_copy, object_ref

MANIFEST_TYPE = "basis_version"
MANIFEST_VERSION = 1
_EXPONENT_MASK = np.uint16(0x7C00)   # an FP16 value with every exponent bit set is an infinity or a NaN


def finite_fp16(data) -> bool:
    """True when no FP16 value in ``data`` is an infinity or a NaN."""
    halves = np.frombuffer(data, dtype=np.uint16)
    return not bool(((halves & _EXPONENT_MASK) == _EXPONENT_MASK).any())


def rows_to_bytes(rows: torch.Tensor) -> bytes:
    """Little-endian bytes of a finite, nonempty FP16 ``[rows, channels]`` block."""
    ok = isinstance(rows, torch.Tensor) and rows.dtype == torch.float16 and rows.dim() == 2 and rows.numel() > 0
    if not ok:
        raise ConfigurationError("a basis block is a nonempty FP16 [rows, channels] tensor")
    if sys.byteorder != "little":
        raise ConfigurationError("basis blocks are stored little-endian; this host is not")
    data = rows.detach().cpu().contiguous().numpy().tobytes()
    if not finite_fp16(data):
        raise ConfigurationError("a basis block holds an infinity or a NaN")
    return data


def rows_from_bytes(data: bytes, rows: int, channels: int) -> torch.Tensor:
    if not isinstance(data, (bytes, bytearray)) or len(data) != 2 * rows * channels:
        raise IntegrityError(f"a basis block of {rows} x {channels} needs {2 * rows * channels} bytes")
    return torch.from_numpy(np.frombuffer(data, dtype=np.float16).reshape(rows, channels).copy())


@dataclass(frozen=True)
class _Link:
    """One version of a chain: its block and how many rows it adds."""

    ref: str
    block: str
    rows: int


class BasisVersionStore:
    """Basis versions of one model in one object store (the caller owns transactions)."""

    DIGEST_CACHE = 16384

    def __init__(self, store: ObjectStore, model: ModelIdentity):
        if not isinstance(store, ObjectStore):
            raise ConfigurationError("basis versions live in an ObjectStore")
        if not isinstance(model, ModelIdentity):
            raise ConfigurationError("basis versions belong to a ModelIdentity")
        self.store, self.model = store, model
        self._versions: dict[str, BasisVersion] = {}      # validated versions (their chains too)
        self._finite: set[str] = set()                     # blocks already checked to be finite
        self._running: OrderedDict[str, Any] = OrderedDict()  # version -> sha256 state of its full view
        self.verify_blocks = True   # hash blocks (and whole views) on assembly unless the store verifies reads

    # -- caches --------------------------------------------------------------------------------------------

    def drop_caches(self) -> None:
        self._versions.clear()
        self._finite.clear()
        self._running.clear()

    def cached_ids(self) -> list[str]:
        return list(self._versions) + list(self._finite) + list(self._running)

    def forget_unstored(self, present: set[str]) -> dict[str, int]:
        """Drop cache entries of objects no longer in the store (after eviction or GC)."""
        dropped = {"basis_versions": 0, "finite_blocks": 0, "view_digests": 0}
        for ref in [r for r in self._versions if r not in present]:
            del self._versions[ref]
            dropped["basis_versions"] += 1
        gone = {b for b in self._finite if b not in present}
        self._finite -= gone
        dropped["finite_blocks"] = len(gone)
        for ref in [r for r in self._running if r not in present]:
            del self._running[ref]
            dropped["view_digests"] += 1
        return dropped

    def missing(self, refs: Iterable[str]) -> list[str]:
        return [ref for ref in dict.fromkeys(refs) if ref not in self._versions]

    def _keep_running(self, ref: str, state) -> None:
        self._running[ref] = state
        self._running.move_to_end(ref)
        if len(self._running) > self.DIGEST_CACHE:
            self._running.popitem(last=False)

    # -- writing -------------------------------------------------------------------------------------------

    def _validate_rows(self, key: MatrixKey, rows: torch.Tensor) -> None:
        if not isinstance(key, MatrixKey) or key.layer >= self.model.layers:
            raise ConfigurationError(f"matrix {key!r} is not a matrix of the model")
        if rows.dim() != 2 or rows.shape[1] != self.model.channels_for(key):
            raise ConfigurationError(f"basis rows of {key!r} need {self.model.channels_for(key)} channels")

    def _write(self, version: BasisVersion, running) -> str:
        refs = [version.added_rows_ref]
        if version.parent_ref is not None:
            refs.append(version.parent_ref)
        ref = self.store.put_manifest({"type": MANIFEST_TYPE, "version": MANIFEST_VERSION,
                                       "record": version.to_dict()}, references=refs)
        self._versions[ref] = version
        self._keep_running(ref, running)
        return ref

    def put_root(self, key: MatrixKey, rows: torch.Tensor) -> tuple[str, BasisVersion]:
        """The first block of a new basis group, as a depth-zero version."""
        self._validate_rows(key, rows)
        data = rows_to_bytes(rows)
        block = self.store.put(data, kind="basis")
        running = hashlib.sha256(data)
        count = int(rows.shape[0])
        version = BasisVersion(None, block, count, count, int(rows.shape[1]),
                               BasisVersion.root_group_id(self.model.fingerprint, key, block), key,
                               self.model.fingerprint, 0, running.hexdigest())
        return self._write(version, running), version

    def put_extension(self, parent_ref: str, rows: torch.Tensor) -> tuple[str, BasisVersion]:
        """A new version appending ``rows`` to ``parent_ref``'s view (the parent stays as it is)."""
        parent = self.load(parent_ref)
        self._validate_rows(parent.key, rows)
        if parent.total_rank + rows.shape[0] > parent.channels:
            raise ConfigurationError(f"the extension would give {parent.key!r} more rows than channels")
        data = rows_to_bytes(rows)
        cached = self._running.get(parent_ref)
        running = cached.copy() if cached is not None else self._digest_of(parent_ref)
        running.update(data)
        block = self.store.put(data, kind="basis")
        count = int(rows.shape[0])
        version = BasisVersion(parent_ref, block, count, parent.total_rank + count, parent.channels,
                               parent.group_id, parent.key, parent.model_fingerprint, parent.depth + 1,
                               running.hexdigest())
        return self._write(version, running), version

    def _digest_of(self, ref: str):
        running = hashlib.sha256()
        for link in self._links(ref):
            running.update(self.store.get(link.block))
        return running

    # -- reading and validation ----------------------------------------------------------------------------

    def _decode(self, ref: str) -> BasisVersion:
        data, references = self.store.get_manifest_with_references(ref)
        if not isinstance(data, Mapping) or set(data) != {"type", "version", "record"} or \
                data.get("type") != MANIFEST_TYPE or data.get("version") != MANIFEST_VERSION:
            raise IntegrityError(f"{ref} is not a basis version manifest")
        try:
            version = BasisVersion.from_dict(data["record"])
        except (ConfigurationError, TypeError, AttributeError) as exc:
            raise IntegrityError(f"{ref} holds an invalid basis version record: {exc}") from exc
        wanted = {version.added_rows_ref} | ({version.parent_ref} if version.parent_ref else set())
        if sorted(wanted) != list(references):
            raise IntegrityError(f"{ref} references other objects than its block and parent")
        if version.model_fingerprint != self.model.fingerprint or version.key.layer >= self.model.layers:
            raise IntegrityError(f"{ref} belongs to another model")
        if version.channels != self.model.channels_for(version.key):
            raise IntegrityError(f"{ref} has another channel width than the model's {version.key!r}")
        if self.store.object_size(version.added_rows_ref) != version.added_bytes:
            raise IntegrityError(f"{ref}: its block's size disagrees with the rows it declares")
        return version

    def _check_link(self, version: BasisVersion) -> None:
        if version.parent_ref is None:
            bound = BasisVersion.root_group_id(version.model_fingerprint, version.key, version.added_rows_ref)
            if version.group_id != bound:
                raise IntegrityError("a root version's group id must derive from its first block")
            return
        parent = self._versions[version.parent_ref]
        consistent = (parent.total_rank + version.added_rank == version.total_rank
                      and (parent.channels, parent.key, parent.group_id, parent.model_fingerprint)
                      == (version.channels, version.key, version.group_id, version.model_fingerprint)
                      and parent.depth + 1 == version.depth)
        if not consistent:
            raise IntegrityError("an extension disagrees with its parent version")

    def load(self, ref: str) -> BasisVersion:
        """A validated version (its whole parent chain validated first, iteratively; cached)."""
        object_ref(ref, "basis version")
        pending = []
        cursor: str | None = ref
        while cursor is not None and cursor not in self._versions:
            version = self._decode(cursor)
            pending.append((cursor, version))
            cursor = version.parent_ref
        for current, version in reversed(pending):   # root side first: every parent is known
            self._check_link(version)
            self._versions[current] = version
        return self._versions[ref]

    def load_many(self, refs: Iterable[str]) -> list[BasisVersion]:
        return [self.load(ref) for ref in list(refs)]

    def chain(self, ref: str) -> list[tuple[str, BasisVersion]]:
        """``(ref, version)`` from the group's root to ``ref``."""
        out = []
        cursor: str | None = ref
        while cursor is not None:
            version = self.load(cursor)
            out.append((cursor, version))
            cursor = version.parent_ref
        out.reverse()
        return out

    def _links(self, ref: str) -> list[_Link]:
        return [_Link(r, v.added_rows_ref, v.added_rank) for r, v in self.chain(ref)]

    def blocks(self, ref: str) -> tuple[str, ...]:
        return tuple(link.block for link in self._links(ref))

    def prefetch_blocks(self, requests: Iterable[tuple[str, int]], block_cache: dict[str, bytes]) -> int:
        """Read every block the ``(version ref, rows)`` prefixes need into ``block_cache`` (parallel reads,
        hash-checked); returns the number of blocks read."""
        wanted: dict[str, None] = {}
        for ref, rows in requests:
            covered = 0
            for link in self._links(ref):
                if covered >= rows:
                    break
                if link.block not in block_cache:
                    wanted[link.block] = None
                covered += link.rows
        block_cache.update(self.store.get_many(list(wanted), verify=True))
        return len(wanted)

    def _prefix_parts(self, ref, rows, max_bytes, block_cache):
        """The blocks (and byte counts) of the first ``rows`` rows of ``ref``'s view, each block checked
        against its content address (or by the store), and the full view against the version digest."""
        version = self.load(ref)
        rows = version.total_rank if rows is None else rows
        if type(rows) is not int or rows < 1 or rows > version.total_rank:
            raise ConfigurationError(f"a view of {ref} takes 1..{version.total_rank} rows, not {rows!r}")
        row_bytes = 2 * version.channels
        if max_bytes is not None and rows * row_bytes > max_bytes:
            raise CapacityError(f"the view needs {rows * row_bytes} bytes, above the {max_bytes}-byte bound")
        trusted = self.store.verify_reads or not self.verify_blocks
        whole = hashlib.sha256() if rows == version.total_rank and not trusted else None
        parts = []
        left = rows
        for link in self._links(ref):
            if left == 0:
                break
            data = block_cache.get(link.block) if block_cache is not None else None
            if data is None:
                data = self.store.get(link.block)
                if not trusted and hashlib.sha256(data).hexdigest() != link.block.partition(":")[2]:
                    raise IntegrityError(f"block {link.block} does not hash to its address")
                if block_cache is not None:
                    block_cache[link.block] = data
            take = min(link.rows, left)
            size = take * row_bytes
            if len(data) < size:
                raise IntegrityError(f"block {link.block} is shorter than its rows")
            if whole is not None:
                whole.update(memoryview(data)[:size])
            parts.append((link.block, data, size))
            left -= take
        if whole is not None and whole.hexdigest() != version.view_sha256:
            raise IntegrityError(f"the assembled view of {ref} differs from its recorded digest")
        return version, rows, parts

    def assemble(self, ref: str, rows: int | None = None, *, max_bytes: int | None = None,
                 block_cache: dict[str, bytes] | None = None) -> torch.Tensor:
        """FP16 ``[rows, channels]`` prefix view (default: the whole version), contiguous."""
        version, rows, parts = self._prefix_parts(ref, rows, max_bytes, block_cache)
        out = np.empty(rows * version.channels, dtype=np.float16)
        raw = out.view(np.uint8)
        at = 0
        for _, data, size in parts:
            raw[at:at + size] = np.frombuffer(data, dtype=np.uint8, count=size)
            at += size
        return torch.from_numpy(out.reshape(rows, version.channels))

    def view_bytes(self, ref: str, rows: int, *, max_bytes: int | None = None,
                   block_cache: dict[str, bytes] | None = None) -> bytes:
        """The prefix view's bytes (every block checked to be finite once)."""
        _, _, parts = self._prefix_parts(ref, rows, max_bytes, block_cache)
        out = []
        for block, data, size in parts:
            piece = memoryview(data)[:size]
            if block not in self._finite:
                if finite_fp16(data):
                    self._finite.add(block)
                elif not finite_fp16(piece):
                    raise ConfigurationError(f"block {block} holds an infinity or a NaN")
            out.append(piece)
        return b"".join(out)

    def unique_block_bytes(self, refs: Iterable[str]) -> dict[str, int]:
        """Bytes of every distinct block the versions ``refs`` reach (storage accounting)."""
        sizes: dict[str, int] = {}
        for ref in refs:
            if ref is not None:
                for _, version in self.chain(ref):
                    sizes.setdefault(version.added_rows_ref, version.added_bytes)
        return sizes


def _descriptor(metadata) -> Mapping[str, Any] | None:
    value = metadata.get("basis") if isinstance(metadata, Mapping) else None
    return value if isinstance(value, Mapping) else None


def detach_basis(encoded: EncodedTensor):
    """``(metadata, payloads, metrics)`` of a lossy packet without its basis bytes; the descriptor stays."""
    if not isinstance(encoded, EncodedTensor) or encoded.basis is None:
        raise ConfigurationError("only a lossy single-matrix packet carries a basis to detach")
    descriptor = _descriptor(encoded.metadata)
    if descriptor is None or descriptor.get("sha256") != hashlib.sha256(encoded.basis).hexdigest():
        raise IntegrityError("the packet's basis bytes do not match its descriptor")
    metrics = None if encoded.metrics is None else json_copy(encoded.metrics)
    return json_copy(encoded.metadata), dict(encoded.payloads), metrics


def attach_basis(metadata: Mapping[str, Any], payloads: Mapping[str, bytes], basis: bytes, *, rank_view: int,
                 channels: int, check_digest: bool = True) -> EncodedTensor:
    """The packet with an assembled prefix view attached, once the view matches the bound descriptor."""
    descriptor = _descriptor(metadata)
    expected = {"shape": [rank_view, channels], "view_rank": rank_view, "dtype": "float16", "bytes": len(basis)}
    if descriptor is None or any(descriptor.get(name) != value for name, value in expected.items()):
        raise IntegrityError("the assembled view's geometry differs from the packet's basis descriptor")
    if check_digest and descriptor.get("sha256") != hashlib.sha256(basis).hexdigest():
        raise IntegrityError("the assembled view's digest differs from the packet's basis descriptor")
    return EncodedTensor(metadata, payloads, basis=basis)


__all__ = ["MANIFEST_TYPE", "BasisVersionStore", "attach_basis", "detach_basis", "finite_fp16", "rows_from_bytes",
           "rows_to_bytes"]
