"""Cache epochs and newest-version-on-path history resolution (reference: reelcache/cache_epochs.py).

Chunk nodes publish the KV of their own new frames. A ``recache`` node adds no frames and publishes
a ``kv_recache`` epoch with new KV for earlier frames; a ``segment`` node publishes a
``longcat_segment`` epoch whose single segment-local range replaces the previous segment's. Restore
resolves each attended sub-range to the newest node on the ancestor path that covers it, so nodes
published before an epoch keep resolving to the versions they had.
"""

from __future__ import annotations

from dataclasses import dataclass
from typing import Iterable, Sequence

from .errors import ConfigurationError, StateError
from .types import CacheEpoch, ChunkNode, MatrixKey


@dataclass(frozen=True)
class CoverageEntry:
    token_start: int
    token_end: int
    chunk_id: str
    records: tuple[tuple[object, str], ...]
    source: str
    node_ref: str
    epoch_id: str
    packet_ref: str | None = None


@dataclass(frozen=True)
class ResolvedPiece:
    """One attended sub-range and the record set (and entry span) that backs it."""

    token_start: int
    token_end: int
    entry: CoverageEntry

    @property
    def offset(self) -> int:
        return self.token_start - self.entry.token_start

    def record(self, key: MatrixKey, stream: str | None = None) -> str:
        wanted = key if stream is None else (key, stream)
        for candidate, ref in self.entry.records:
            if candidate == wanted:
                return ref
        raise StateError(f"resolved range lacks a record for {wanted}")

    def to_dict(self) -> dict:
        return {"token_start": self.token_start, "token_end": self.token_end, "entry_start": self.entry.token_start,
                "entry_end": self.entry.token_end, "chunk_id": self.entry.chunk_id, "source": self.entry.source,
                "node": self.entry.node_ref, "epoch_id": self.entry.epoch_id}


def coverage(node_ref: str, node: ChunkNode, epoch: CacheEpoch) -> list[CoverageEntry]:
    """The KV ranges a node itself publishes (none for roots)."""
    if node.node_kind == "chunk":
        return [CoverageEntry(node.token_start, node.token_end, node.chunk_id, node.matrix_records, "chunk",
                              node_ref, node.cache_epoch_id, node.packet_ref)]
    if node.node_kind in ("recache", "segment"):
        return [CoverageEntry(r.token_start, r.token_end, r.chunk_id, r.records, "epoch", node_ref, epoch.epoch_id,
                              r.packet_ref) for r in epoch.ranges]
    return []


def resolve(path: Sequence[tuple[str, ChunkNode, CacheEpoch]], ranges: Iterable[tuple[int, int]]) -> list[ResolvedPiece]:
    """Resolve each attended ``[start, end)`` to the newest covering entry on ``path`` (root first).

    Uncovered history raises :class:`StateError` (never zero-filled); overlapping requests raise
    :class:`ConfigurationError`.
    """
    per_node = [coverage(ref, node, epoch) for ref, node, epoch in path]
    pieces: list[ResolvedPiece] = []
    for start, end in ranges:
        if type(start) is not int or type(end) is not int or not 0 <= start < end:
            raise ConfigurationError("attended ranges must be nonempty nonnegative integer intervals")
        open_spans = [(start, end)]
        for entries in reversed(per_node):
            if not open_spans:
                break
            still_open = []
            for low, high in open_spans:
                hits = sorted(((max(low, e.token_start), min(high, e.token_end), e) for e in entries
                               if max(low, e.token_start) < min(high, e.token_end)), key=lambda item: item[0])
                cursor = low
                for left, right, entry in hits:
                    if left > cursor:
                        still_open.append((cursor, left))
                    pieces.append(ResolvedPiece(left, right, entry))
                    cursor = max(cursor, right)
                if cursor < high:
                    still_open.append((cursor, high))
            open_spans = still_open
        if open_spans:
            raise StateError(f"attended history {open_spans} is not covered by the node's ancestor path")
    pieces.sort(key=lambda piece: piece.token_start)
    for left, right in zip(pieces, pieces[1:]):
        if left.token_end > right.token_start:
            raise ConfigurationError("attended ranges overlap; request each token once")
    return pieces
