"""Immutable FP16 basis row blocks and their version manifests (reference:
reelcache/basis_versions.py:73-432; same manifest form ``{"type": "basis_version", "version": 1,
"record": <reelcache.basis_version.v1>}`` referencing its parent version and its one row block).

A version's canonical view is its ancestors' rows followed by its own block, never reordered or
copied, so sharing a basis between chunks shares these objects and store GC sees the whole chain.
Lossy packets bind the exact prefix view they were encoded with by a ``basis`` descriptor (shape,
view rank, SHA-256); :func:`attach_basis` re-attaches an assembled prefix only after that check.
"""

from __future__ import annotations

import hashlib
import sys
from collections import OrderedDict
from typing import Any, Iterable, Mapping

import numpy as np
import torch

from .errors import CapacityError, ConfigurationError, IntegrityError
from .store import ObjectStore
from .types import BasisVersion, EncodedTensor, MatrixKey, ModelIdentity, json_copy, object_ref

MANIFEST_TYPE = "basis_version"
_FP16_EXPONENT = 0x7C00


def finite_fp16(data) -> bool:
    bits = np.frombuffer(data, dtype=np.uint16)
    return not bool(np.any((bits & _FP16_EXPONENT) == _FP16_EXPONENT))


def rows_to_bytes(rows: torch.Tensor) -> bytes:
    if not isinstance(rows, torch.Tensor) or rows.dtype != torch.float16 or rows.ndim != 2 or min(rows.shape) < 1:
        raise ConfigurationError("basis row blocks are nonempty FP16 [rows, channels] tensors")
    if sys.byteorder != "little":
        raise ConfigurationError("basis row serialization requires a little-endian host")
    data = rows.detach().to("cpu").contiguous().numpy().tobytes()
    if not finite_fp16(data):
        raise ConfigurationError("basis row blocks must be finite")
    return data


def rows_from_bytes(data: bytes, rows: int, channels: int) -> torch.Tensor:
    if not isinstance(data, (bytes, bytearray)) or len(data) != rows * channels * 2:
        raise IntegrityError("basis row block length disagrees with its declared geometry")
    return torch.from_numpy(np.frombuffer(data, dtype=np.float16).reshape(rows, channels).copy())


class BasisVersionStore:
    """Validated basis-version operations over one runtime's store (callers own transactions)."""

    VIEW_DIGESTS = 16384

    def __init__(self, store: ObjectStore, model: ModelIdentity):
        if not isinstance(store, ObjectStore) or not isinstance(model, ModelIdentity):
            raise ConfigurationError("basis versions require an ObjectStore and ModelIdentity")
        self.store, self.model = store, model
        self._cache: dict[str, BasisVersion] = {}
        self._finite_blocks: set[str] = set()
        self._view_digests: OrderedDict[str, Any] = OrderedDict()

    def drop_caches(self) -> None:
        self._cache.clear()
        self._finite_blocks.clear()
        self._view_digests.clear()

    def cached_ids(self) -> list[str]:
        return [*self._cache, *self._finite_blocks, *self._view_digests]

    def forget_unstored(self, present: set[str]) -> dict[str, int]:
        versions = [ref for ref in self._cache if ref not in present]
        for ref in versions:
            del self._cache[ref]
        blocks = [b for b in self._finite_blocks if b not in present]
        self._finite_blocks.difference_update(blocks)
        digests = [ref for ref in self._view_digests if ref not in present]
        for ref in digests:
            del self._view_digests[ref]
        return {"basis_versions": len(versions), "finite_blocks": len(blocks), "view_digests": len(digests)}

    def missing(self, refs: Iterable[str]) -> list[str]:
        return [ref for ref in dict.fromkeys(refs) if ref not in self._cache]

    # -- creation ------------------------------------------------------------------------------------------------

    def _check_rows(self, key: MatrixKey, rows: torch.Tensor) -> None:
        if not isinstance(key, MatrixKey) or key.layer >= self.model.layers:
            raise ConfigurationError("basis key is outside the model")
        if rows.ndim != 2 or rows.shape[1] != self.model.channels_for(key):
            raise ConfigurationError("basis rows do not match the model's channel width")

    def put_root(self, key: MatrixKey, rows: torch.Tensor) -> tuple[str, BasisVersion]:
        """Store a new group's first block and its depth-zero version."""
        self._check_rows(key, rows)
        data = rows_to_bytes(rows)
        block = self.store.put(data, kind="basis")
        digest = hashlib.sha256(data)
        version = BasisVersion(None, block, int(rows.shape[0]), int(rows.shape[0]), int(rows.shape[1]),
                               BasisVersion.root_group_id(self.model.fingerprint, key, block), key,
                               self.model.fingerprint, 0, digest.hexdigest())
        ref = self._put_version(version)
        self._remember_digest(ref, digest)
        return ref, version

    def put_extension(self, parent_ref: str, rows: torch.Tensor) -> tuple[str, BasisVersion]:
        """Append an immutable row block to ``parent_ref`` (the parent is unchanged)."""
        parent = self.load(parent_ref)
        self._check_rows(parent.key, rows)
        if parent.total_rank + rows.shape[0] > parent.channels:
            raise ConfigurationError("an extension cannot exceed the channel count")
        data = rows_to_bytes(rows)
        known = self._view_digests.get(parent_ref)
        if known is not None:
            digest = known.copy()
        else:
            digest = hashlib.sha256()
            for block, _ in self._blocks(parent_ref):
                digest.update(self.store.get(block))
        digest.update(data)
        block = self.store.put(data, kind="basis")
        version = BasisVersion(parent_ref, block, int(rows.shape[0]), parent.total_rank + int(rows.shape[0]),
                               parent.channels, parent.group_id, parent.key, parent.model_fingerprint,
                               parent.depth + 1, digest.hexdigest())
        ref = self._put_version(version)
        self._remember_digest(ref, digest)
        return ref, version

    def _remember_digest(self, ref: str, digest) -> None:
        self._view_digests[ref] = digest
        self._view_digests.move_to_end(ref)
        while len(self._view_digests) > self.VIEW_DIGESTS:
            self._view_digests.popitem(last=False)

    def _put_version(self, version: BasisVersion) -> str:
        references = [version.added_rows_ref] + ([] if version.parent_ref is None else [version.parent_ref])
        ref = self.store.put_manifest({"type": MANIFEST_TYPE, "version": 1, "record": version.to_dict()},
                                      references=references)
        self._cache[ref] = version
        return ref

    # -- validation and reads ------------------------------------------------------------------------------------

    def load(self, ref: str) -> BasisVersion:
        """Validate one version and (recursively, cached) its whole parent chain."""
        object_ref(ref, "basis version")
        cached = self._cache.get(ref)
        if cached is not None:
            return cached
        version = self._parse(*self.store.get_manifest_with_references(ref))
        if self.store.object_size(version.added_rows_ref) != version.added_bytes:
            raise IntegrityError("basis row block size disagrees with its version")
        if version.parent_ref is not None:
            self.load(version.parent_ref)
        self._link(version)
        self._cache[ref] = version
        return version

    def load_many(self, refs: Iterable[str]) -> list[BasisVersion]:
        refs = list(refs)
        for ref in refs:
            self.load(ref)
        return [self._cache[ref] for ref in refs]

    def _parse(self, data, references) -> BasisVersion:
        try:
            if data.get("type") != MANIFEST_TYPE or data.get("version") != 1 or set(data) != {"type", "version",
                                                                                               "record"}:
                raise IntegrityError("unsupported basis version manifest")
            version = BasisVersion.from_dict(data["record"])
        except (ConfigurationError, TypeError, AttributeError) as exc:
            raise IntegrityError("invalid basis version manifest") from exc
        expected = sorted({version.added_rows_ref} | ({version.parent_ref} if version.parent_ref else set()))
        if list(references) != expected:
            raise IntegrityError("basis version references disagree with its parent/block")
        if version.model_fingerprint != self.model.fingerprint or version.key.layer >= self.model.layers:
            raise IntegrityError("basis version belongs to another model")
        if version.channels != self.model.channels_for(version.key):
            raise IntegrityError("basis version channel width disagrees with the model")
        return version

    def _link(self, version: BasisVersion) -> None:
        if version.parent_ref is None:
            if version.group_id != BasisVersion.root_group_id(version.model_fingerprint, version.key,
                                                              version.added_rows_ref):
                raise IntegrityError("root basis group identity is not bound to its first block")
            return
        parent = self._cache[version.parent_ref]
        if (parent.total_rank + version.added_rank != version.total_rank or parent.channels != version.channels
                or parent.key != version.key or parent.group_id != version.group_id
                or parent.depth + 1 != version.depth or parent.model_fingerprint != version.model_fingerprint):
            raise IntegrityError("basis extension is inconsistent with its parent version")

    def chain(self, ref: str) -> list[tuple[str, BasisVersion]]:
        """Versions from the group root to ``ref`` (inclusive)."""
        result = []
        current: str | None = ref
        while current is not None:
            version = self.load(current)
            result.append((current, version))
            current = version.parent_ref
        return result[::-1]

    def _blocks(self, ref: str) -> list[tuple[str, int]]:
        return [(v.added_rows_ref, v.added_rank) for _, v in self.chain(ref)]

    def blocks(self, ref: str) -> tuple[str, ...]:
        return tuple(block for block, _ in self._blocks(ref))

    def prefetch_blocks(self, requests: Iterable[tuple[str, int]], block_cache: dict[str, bytes]) -> int:
        """Read (hash-checked, in parallel) every block the ``(version_ref, rows)`` prefixes need."""
        needed = []
        for ref, rows in requests:
            remaining = rows
            for block, count in self._blocks(ref):
                if remaining <= 0:
                    break
                if block not in block_cache:
                    needed.append(block)
                remaining -= count
        needed = list(dict.fromkeys(needed))
        block_cache.update(self.store.get_many(needed, verify=True))
        return len(needed)

    def _prefix(self, ref, rows, max_bytes, block_cache):
        version = self.load(ref)
        rows = version.total_rank if rows is None else rows
        if type(rows) is not int or not 1 <= rows <= version.total_rank:
            raise ConfigurationError("a basis view must be a nonempty legal prefix of its version")
        nbytes = rows * version.channels * 2
        if max_bytes is not None and nbytes > max_bytes:
            raise CapacityError(f"basis view needs {nbytes} bytes; workspace bound is {max_bytes}")
        parts, remaining = [], rows
        verified = self.store.verify_reads
        digest = hashlib.sha256() if rows == version.total_rank and not verified else None
        for block, count in self._blocks(ref):
            if remaining <= 0:
                break
            data = None if block_cache is None else block_cache.get(block)
            if data is None:
                data = self.store.get(block)
                if not verified and hashlib.sha256(data).hexdigest() != block.split(":", 1)[1]:
                    raise IntegrityError("basis row block bytes differ from their content address")
                if block_cache is not None:
                    block_cache[block] = data
            take = min(count, remaining)
            size = take * version.channels * 2
            if len(data) < size:
                raise IntegrityError("basis row block length disagrees with its declared geometry")
            if digest is not None:
                digest.update(memoryview(data)[:size])
            parts.append((block, data, size))
            remaining -= take
        if digest is not None and digest.hexdigest() != version.view_sha256:
            raise IntegrityError("assembled basis view differs from its version digest")
        return version, rows, parts

    def assemble(self, ref: str, rows: int | None = None, *, max_bytes: int | None = None,
                 block_cache: dict[str, bytes] | None = None) -> torch.Tensor:
        """Contiguous FP16 prefix view ``[rows, channels]`` from the version's ordered blocks."""
        version, rows, parts = self._prefix(ref, rows, max_bytes, block_cache)
        view = np.empty(rows * version.channels * 2, dtype=np.uint8)
        position = 0
        for _, data, size in parts:
            view[position:position + size] = np.frombuffer(data, dtype=np.uint8, count=size)
            position += size
        return torch.from_numpy(view.view(np.float16).reshape(rows, version.channels))

    def view_bytes(self, ref: str, rows: int, *, max_bytes: int | None = None,
                   block_cache: dict[str, bytes] | None = None) -> bytes:
        _, _, parts = self._prefix(ref, rows, max_bytes, block_cache)
        chunks = []
        for block, data, size in parts:
            chunk = memoryview(data)[:size]
            if block not in self._finite_blocks:
                if finite_fp16(data):
                    self._finite_blocks.add(block)
                elif not finite_fp16(chunk):
                    raise ConfigurationError("basis row blocks must be finite")
            chunks.append(chunk)
        return b"".join(chunks)

    def unique_block_bytes(self, refs: Iterable[str]) -> dict[str, int]:
        result: dict[str, int] = {}
        for ref in refs:
            if ref is None:
                continue
            for _, version in self.chain(ref):
                result.setdefault(version.added_rows_ref, version.added_bytes)
        return result


def detach_basis(encoded: EncodedTensor):
    """``(metadata, payloads, metrics)`` of a lossy packet without its basis bytes (the descriptor stays)."""
    if not isinstance(encoded, EncodedTensor) or encoded.basis is None:
        raise ConfigurationError("only lossy single-matrix packets carry a detachable basis")
    descriptor = encoded.metadata.get("basis") if isinstance(encoded.metadata, Mapping) else None
    if not isinstance(descriptor, Mapping) or hashlib.sha256(encoded.basis).hexdigest() != descriptor.get("sha256"):
        raise IntegrityError("packet basis bytes disagree with their descriptor")
    return (json_copy(encoded.metadata), dict(encoded.payloads),
            None if encoded.metrics is None else json_copy(encoded.metrics))


def attach_basis(metadata: Mapping[str, Any], payloads: Mapping[str, bytes], basis: bytes, *, rank_view: int,
                 channels: int, check_digest: bool = True) -> EncodedTensor:
    """Re-attach an assembled prefix view after checking it against the packet's basis descriptor."""
    descriptor = metadata.get("basis") if isinstance(metadata, Mapping) else None
    if (not isinstance(descriptor, Mapping) or descriptor.get("shape") != [rank_view, channels]
            or descriptor.get("view_rank") != rank_view or descriptor.get("dtype") != "float16"
            or descriptor.get("bytes") != len(basis)
            or (check_digest and hashlib.sha256(basis).hexdigest() != descriptor.get("sha256"))):
        raise IntegrityError("assembled basis view differs from the packet's bound prefix")
    return EncodedTensor(metadata, payloads, basis=basis)
