"""Tiered KV history under Ulysses sequence parallelism (the counterpart of reference
reelcache/sp_kv.py:1-772; design from its lines 1-30).

Under Ulysses every rank owns a **head slice** of every chunk's K and V.

1. **Capture**: each clean chunk's head slices are gathered to the storage owner
   (:meth:`DistributedOwner.gather_matrix`, ``heads`` layout), which archives the canonical matrices
   as one lineage node; every rank keeps its own slices in its **hot tier**.
2. **Hot tier**: a per-rank byte budget; the oldest chunks leave first, and the membership is agreed
   collectively (every rank evicts the same chunks, so a chunk is hot on all ranks or on none).
3. **Cold tier**: a chunk that is not hot is decoded on exactly one rank -- round robin by chunk,
   rotated by layer (``(chunk + layer) % world``) -- from the shared store of the node, and its head
   columns are scattered to their ranks (:meth:`SPTieredHistory.load_layer`: point-to-point transfers of the
   dense slices). On CUDA, :meth:`SPTieredHistory.prepare_fused` instead keeps the decoder's 8-bit
   coefficients and basis in its symmetric arena and every rank's fused restore reads its heads from there
   over NVLink (parallel/sp_restore.py): the scatter disappears into the restore kernels.
"""

from __future__ import annotations

from collections import OrderedDict
from typing import Any

import torch

from ..errors import ConfigurationError, StateError
from ..types import MatrixKey, TensorContext
from .distributed import DistributedOwner, KVLayout


class SPTieredHistory:
    def __init__(self, transport: DistributedOwner, runtime, lineage: str, *, layers: int, kv_heads: int,
                 head_dim: int, chunk_tokens: int, grid: tuple[int, int, int], hot_budget_bytes: int, method=None,
                 device="cpu"):
        self.t = transport
        self.runtime = runtime          # every rank: a LineageRuntime over the shared store
        self.lineage = lineage
        self.layers = layers
        self.layout = KVLayout(chunk_tokens, kv_heads, head_dim, transport.world_size)
        self.grid = grid
        self.hot_budget = hot_budget_bytes
        self.method = method
        self.device = torch.device(device)
        self.hot: "OrderedDict[int, dict]" = OrderedDict()   # chunk -> {(layer, target): local slice}
        self.nodes: list[str] = []                             # node ref of every captured chunk
        self.stats = {"captured": 0, "hot_hits": 0, "cold_decodes": 0, "cold_received": 0, "evicted": 0}

    def _slice_bytes(self, slices: dict) -> int:
        return sum(t.numel() * t.element_size() for t in slices.values())

    def capture(self, chunk: int, local: dict[tuple[int, str], torch.Tensor]) -> str:
        """Archive chunk ``chunk`` from every rank's head slices; returns the published node (all ranks)."""
        if chunk != len(self.nodes):
            raise ConfigurationError("chunks are captured in order")
        canonical = {}
        for layer in range(self.layers):
            for target in ("K", "V"):
                full = self.t.gather_matrix(local[(layer, target)], self.layout, source_layout="heads",
                                            operation=f"capture:{chunk}:{layer}:{target}")
                if self.t.is_owner:
                    canonical[MatrixKey(layer, target)] = full

        def commit():
            frames, h, w = self.grid
            contexts = {key: TensorContext(self.runtime.model, key, chunk * self.layout.tokens, frames, h, w,
                                           "pre_rope" if key.target == "K" else "none") for key in canonical}
            return self.runtime.commit_node(self.lineage, f"chunk-{chunk}", canonical, contexts, method=self.method,
                                            device=self.device).node_ref

        node = self.t.owner_call(f"capture:{chunk}:commit", commit)
        node = self.t.broadcast_json(node, operation=f"capture:{chunk}:node")
        self.nodes.append(node)
        self.runtime.drop_manifest_caches()
        self.hot[chunk] = {key: value.detach().clone() for key, value in local.items()}
        self._agree_budget()
        self.stats["captured"] += 1
        return node

    def _agree_budget(self) -> None:
        """Evict the oldest hot chunks until every rank's hot tier fits its budget (same set everywhere)."""
        mine = sum(self._slice_bytes(s) for s in self.hot.values())
        wanted = []
        order = list(self.hot)
        used = mine
        for chunk in order:
            if used <= self.hot_budget:
                break
            wanted.append(chunk)
            used -= self._slice_bytes(self.hot[chunk])
        proposals = self.t.checkpoint("hot:agree", details=wanted)
        evict = sorted({c for p in proposals for c in p})
        for chunk in evict:
            self.hot.pop(chunk, None)
            self.stats["evicted"] += 1

    def hot_chunks(self) -> list[int]:
        return list(self.hot)

    def load_layer(self, layer: int, chunks: int | None = None) -> dict[str, torch.Tensor]:
        """This rank's ``[history_tokens, local_channels]`` K and V of ``layer`` for chunks ``0..chunks-1``."""
        chunks = len(self.nodes) if chunks is None else chunks
        out = {}
        for target in ("K", "V"):
            parts = []
            for chunk in range(chunks):
                if chunk in self.hot:
                    parts.append(self.hot[chunk][(layer, target)])
                    self.stats["hot_hits"] += 1
                    continue
                parts.append(self._cold(chunk, layer, target))
            out[target] = torch.cat(parts) if parts else torch.empty(0, self.layout.local_channels)
        return out

    def prepare_fused(self, destination, *, chunks: int | None = None, rope=None, stream=None):
        """Stage the cold history for fused restores (CUDA, one process per GPU): the decoder rank of every
        (chunk, layer) -- ``(chunk + layer) % world``, as for :meth:`load_layer` -- loads the stored 8-bit
        coefficients and basis into its symmetric arena, and every rank's restore kernels read its own head
        columns from there over NVLink (no scatter collective). Returns a
        :class:`~.sp_restore.FusedHistoryRestore`; each ``restore()`` writes ``destination(layer, target)``
        (``[1, chunks * chunk_tokens, local_heads, head_dim]``). ``rope(chunk)`` gives the ``RopePositions`` of
        a chunk's K (None: no rotation). Collective."""
        from ..archive_restore import LineageRestorer
        from .sp_restore import FusedHistoryRestore, HistoryLayout, plan_history

        chunks = len(self.nodes) if chunks is None else chunks
        world = self.t.world_size
        tokens = self.layout.tokens
        shapes, owners, keys = [], [], []
        ranks = {}
        error = None
        mine = {}
        try:
            restorer = LineageRestorer(self.runtime, self.t.device)
            for chunk in range(chunks):
                span = [(chunk * tokens, (chunk + 1) * tokens)]
                wanted = [MatrixKey(layer, target) for layer in range(self.layers) for target in ("K", "V")
                          if (chunk + layer) % world == self.t.rank]
                if wanted:
                    factors = restorer.node_factors(self.nodes[chunk], wanted, ranges=span, stream=stream)
                    for (start, key), value in factors.items():
                        mine[(chunk, key.layer, key.target)] = value
                        ranks[f"{chunk}:{key.layer}:{key.target}"] = int(value[0].shape[1])
        except Exception as exc:  # noqa: BLE001 - agreed before any payload moves
            error = exc
        reported = self.t.checkpoint("fused:ranks", error=error, details=ranks)
        every = {k: v for rows in reported for k, v in rows.items()}
        for chunk in range(chunks):
            for layer in range(self.layers):
                for target in ("K", "V"):
                    shapes.append((chunk, layer, target, tokens, every[f"{chunk}:{layer}:{target}"]))
                    owners.append((chunk + layer) % world)
        plan = plan_history(shapes, world, self.layout.channels, owners=owners)
        layout = HistoryLayout("heads", world, chunks=chunks, tokens=tokens, heads=self.layout.kv_heads,
                               head_dim=self.layout.head_dim)
        fused = FusedHistoryRestore.create(plan, layout, self.grid, self.t.device,
                                           group=self.t.group if world > 1 else None)
        fused.stage({tile.index: mine[(tile.chunk, tile.layer, tile.target)] for tile in plan.owned(self.t.rank)})
        fused.build(destination, None if rope is None else (lambda tile: rope(tile.chunk)), stream=stream)
        self.stats["fused_prepared"] = self.stats.get("fused_prepared", 0) + 1
        return fused

    def _cold(self, chunk: int, layer: int, target: str) -> torch.Tensor:
        decoder = (chunk + layer) % self.t.world_size
        key = MatrixKey(layer, target)
        full = None
        error = None
        if self.t.rank == decoder:
            try:
                start = chunk * self.layout.tokens
                full = self.runtime.acquire_node_history(self.nodes[chunk], key,
                                                         ranges=[(start, start + self.layout.tokens)],
                                                         device=self.t.device).contiguous()
                self.stats["cold_decodes"] += 1
            except BaseException as exc:  # noqa: BLE001 - raised on every rank by the checkpoint
                error = exc
        self.t.checkpoint(f"cold:{chunk}:{layer}:{target}", error=error)
        mine = None
        for destination in range(self.t.world_size):
            columns = self.layout.columns(destination)
            piece = full[:, columns].contiguous() if full is not None else None
            if destination == decoder:
                if self.t.rank == decoder:
                    mine = piece
                continue
            got = self.t.transfer_tensor(piece, source=decoder, destination=destination,
                                         operation=f"cold:{chunk}:{layer}:{target}:{destination}")
            if self.t.rank == destination:
                mine = got
                self.stats["cold_received"] += 1
        if mine is None:
            raise StateError("cold history slice missing")
        return mine
