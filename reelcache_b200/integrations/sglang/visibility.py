"""Visibility plans: which archived token ranges the next chunk attends to and where they sit in the
native KV cache (the counterpart of reference reelcache/integrations/sglang/visibility.py:22-151).

``full_history`` attends to every earlier chunk; ``sink_window`` to the first ``sink_frames`` latent
frames plus the most recent frames that fill ``window_frames``. A plan's spans name, per archived
node, the node-relative token offset, the length and the cache slot they are installed at.
"""

from __future__ import annotations

from dataclasses import dataclass
from typing import Sequence

from .profiles import ModelProfile


@dataclass(frozen=True)
class TokenSpan:
    node_ref: str
    chunk_index: int
    node_offset: int
    length: int
    slot_start: int
    token_start: int
    role: str  # "sink" | "window" | "history"

    def to_dict(self) -> dict:
        return {"node": self.node_ref, "chunk": self.chunk_index, "node_offset": self.node_offset,
                "length": self.length, "slot_start": self.slot_start, "token_start": self.token_start,
                "role": self.role}


@dataclass(frozen=True)
class VisibilityPlan:
    next_chunk: int
    spans: tuple[TokenSpan, ...]

    @property
    def attended_tokens(self) -> int:
        return sum(span.length for span in self.spans)

    def nodes(self) -> list[str]:
        seen = []
        for span in self.spans:
            if span.node_ref not in seen:
                seen.append(span.node_ref)
        return seen

    def ranges(self) -> list[tuple[int, int]]:
        """Global token ranges attended (for the restorer's ``ranges``)."""
        return [(span.token_start, span.token_start + span.length) for span in self.spans]

    def to_dict(self) -> dict:
        return {"next_chunk": self.next_chunk, "spans": [s.to_dict() for s in self.spans],
                "attended_tokens": self.attended_tokens}


def build_visibility_plan(profile: ModelProfile, chunk_nodes: Sequence[str], next_chunk: int) -> VisibilityPlan:
    """``chunk_nodes[i]`` is the node holding chunk ``i`` of the path (its own token range)."""
    per_chunk = profile.chunk_tokens
    frame = profile.tokens_per_frame
    spans: list[TokenSpan] = []
    if profile.visibility == "full_history":
        for index in range(next_chunk):
            spans.append(TokenSpan(chunk_nodes[index], index, 0, per_chunk, index * per_chunk, index * per_chunk,
                                   "history"))
        return VisibilityPlan(next_chunk, tuple(spans))
    sink_tokens = profile.sink_frames * frame
    window_tokens = profile.window_frames * frame - sink_tokens - per_chunk  # room left for history
    end = next_chunk * per_chunk
    keep: list[tuple[int, int, str]] = []
    sink_end = min(sink_tokens, end)
    if sink_end > 0:
        keep.append((0, sink_end, "sink"))
    window_start = max(sink_end, end - max(window_tokens, 0))
    if window_start < end:
        keep.append((window_start, end, "window"))
    slot = 0
    for start, stop, role in keep:
        cursor = start
        while cursor < stop:
            index = cursor // per_chunk
            chunk_end = min(stop, (index + 1) * per_chunk)
            spans.append(TokenSpan(chunk_nodes[index], index, cursor - index * per_chunk, chunk_end - cursor, slot,
                                   cursor, role))
            slot += chunk_end - cursor
            cursor = chunk_end
    return VisibilityPlan(next_chunk, tuple(spans))


def resolve_plan(runtime, head_ref: str, plan: VisibilityPlan) -> VisibilityPlan:
    """The plan with every span cut at KV-version boundaries: each piece names the holder of the newest version on
    the head's path (a chunk node ref, or ``node#range`` of a recache epoch range, the raw tier's keys) and its
    offset inside that holder's range. Spans keep their chunk index (RoPE rows) and cache slots."""
    from ...archive_pipeline import range_holder
    if not plan.spans:
        return plan
    pieces = runtime.resolve_history(head_ref, plan.ranges())
    spans: list[TokenSpan] = []
    for span in plan.spans:
        end = span.token_start + span.length
        for piece in pieces:
            left, right = max(piece.token_start, span.token_start), min(piece.token_end, end)
            if left >= right:
                continue
            entry = piece.entry
            holder = entry.node_ref if entry.source == "chunk" else range_holder(entry.node_ref, entry.chunk_id)
            spans.append(TokenSpan(holder, span.chunk_index, left - entry.token_start, right - left,
                                   span.slot_start + left - span.token_start, left, span.role))
    return VisibilityPlan(plan.next_chunk, tuple(spans))
