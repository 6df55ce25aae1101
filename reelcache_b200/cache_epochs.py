"""Cache epochs and newest-version-on-path history resolution (the behaviour of reference
reelcache/cache_epochs.py:60-110).

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
        found = dict(self.entry.records).get(wanted)
        if found is None:
            raise StateError(f"the range backing tokens {self.token_start}..{self.token_end} has no {wanted}")
        return found

    def to_dict(self) -> dict:
        return {"token_start": self.token_start, "token_end": self.token_end, "entry_start": self.entry.token_start,
                "entry_end": self.entry.token_end, "chunk_id": self.entry.chunk_id, "source": self.entry.source,
                "node": self.entry.node_ref, "epoch_id": self.entry.epoch_id}


def coverage(node_ref: str, node: ChunkNode, epoch: CacheEpoch) -> list[CoverageEntry]:
    """The KV ranges a node itself publishes: a chunk node its own frames, a recache or segment node every
    range of its epoch, a root nothing."""
    kind = node.node_kind
    if kind == "chunk":
        return [CoverageEntry(node.token_start, node.token_end, node.chunk_id, node.matrix_records, "chunk",
                              node_ref, node.cache_epoch_id, node.packet_ref)]
    if kind not in ("recache", "segment"):
        return []
    return [CoverageEntry(span.token_start, span.token_end, span.chunk_id, span.records, "epoch", node_ref,
                          epoch.epoch_id, span.packet_ref) for span in epoch.ranges]


def _newest(layers: Sequence[list[CoverageEntry]], token: int) -> CoverageEntry | None:
    """The entry of the deepest node (the newest on the path) whose range contains ``token``."""
    for entries in reversed(layers):
        for entry in entries:
            if entry.token_start <= token < entry.token_end:
                return entry
    return None


def resolve(path: Sequence[tuple[str, ChunkNode, CacheEpoch]], ranges: Iterable[tuple[int, int]]) -> list[ResolvedPiece]:
    """Back every attended ``[start, end)`` by the newest covering entry on ``path`` (root first).

    Sweep: the range is cut at every entry boundary inside it; each elementary interval takes the newest
    entry covering it, and neighbouring intervals backed by the same entry merge into one piece. History no
    entry covers raises :class:`StateError` (it is never zero-filled); requested ranges that overlap raise
    :class:`ConfigurationError`."""
    layers = [coverage(ref, node, epoch) for ref, node, epoch in path]
    pieces: list[ResolvedPiece] = []
    for start, end in ranges:
        if type(start) is not int or type(end) is not int or start < 0 or end <= start:
            raise ConfigurationError(f"attended range ({start!r}, {end!r}) is not a nonempty interval of tokens")
        cuts = {start, end}
        for entries in layers:
            for entry in entries:
                if entry.token_start < end and entry.token_end > start:
                    cuts.update((max(start, entry.token_start), min(end, entry.token_end)))
        points = sorted(cuts)
        run: list[ResolvedPiece] = []
        missing = []
        for left, right in zip(points, points[1:]):
            entry = _newest(layers, left)
            if entry is None:
                missing.append((left, right))
                continue
            if run and run[-1].entry is entry and run[-1].token_end == left:
                run[-1] = ResolvedPiece(run[-1].token_start, right, entry)
            else:
                run.append(ResolvedPiece(left, right, entry))
        if missing:
            raise StateError(f"no node on the ancestor path covers the attended tokens {missing}")
        pieces.extend(run)
    pieces.sort(key=lambda piece: piece.token_start)
    for first, second in zip(pieces, pieces[1:]):
        if first.token_end > second.token_start:
            raise ConfigurationError("the attended ranges overlap; name every token once")
    return pieces
