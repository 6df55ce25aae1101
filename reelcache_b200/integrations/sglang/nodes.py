"""Plain-data tree nodes of a serving session (the counterpart of reference
reelcache/integrations/sglang/nodes.py:29-247): one :class:`BridgeNode` per published lineage node,
with its chunk index, token coverage and kind."""

from __future__ import annotations

from dataclasses import dataclass
from typing import Any


@dataclass(frozen=True)
class BridgeNode:
    node_ref: str
    kind: str            # root | chunk | recache | segment
    chunk_index: int     # -1 for the root
    token_start: int
    token_end: int
    parent_ref: str | None

    def to_dict(self) -> dict[str, Any]:
        return {"node": self.node_ref, "kind": self.kind, "chunk": self.chunk_index, "token_start": self.token_start,
                "token_end": self.token_end, "parent": self.parent_ref}


def path_nodes(runtime, head_ref: str) -> list[BridgeNode]:
    """The root-to-head path of a lineage node as :class:`BridgeNode` records."""
    out = []
    chunk = -1
    for ref, node, _epoch in runtime.node_path(head_ref):
        if node.node_kind == "chunk":
            chunk += 1
        out.append(BridgeNode(ref, node.node_kind, chunk if node.node_kind == "chunk" else -1, node.token_start,
                              node.token_end, node.parent_ref))
    return out


def chunk_nodes(runtime, head_ref: str) -> list[str]:
    """Chunk node refs in chunk order (index i -> node holding chunk i)."""
    return [n.node_ref for n in path_nodes(runtime, head_ref) if n.kind == "chunk"]
