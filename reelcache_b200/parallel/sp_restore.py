"""Sequence-parallel restore of an archived history with the coefficient all-gather fused into the
restore pipeline's kernels over NVLink peer memory.

The counterpart of reference reelcache/factor_sharding.py:1893-2205 (``FactorShardDomain.reconstruct``:
one batched NCCL point-to-point round per matrix ships coefficient rows and basis columns to every
native owner, which then runs FP32 GEMMs) and reelcache/sp_kv.py:639-766 (``load_layer``: cold chunks
decoded on one rank, head slices scattered with ``batch_isend_irecv``).

Ownership. Every archived matrix (one chunk's K or V of one layer) has one **factor owner**, by default
``(layer + [target == "V"]) % world`` (the reference's whole-matrix rotation, factor_sharding.py:158). The
owner holds the matrix's 8-bit coefficients ``[tokens, k_pad]`` and its FP16 basis ``[rank, channels]`` in
its symmetric arena (:mod:`.symmetric`), so every peer can read them.

Native layouts (:class:`HistoryLayout`) say which part of the restored KV each rank keeps:

* ``"sequence"`` (default): the history's tokens are cut into ``world`` contiguous ranges of whole
  chunks; a rank restores every matrix of its own chunks (all heads). Each coefficient byte crosses
  NVLink at most once and no rank restores anything twice.
* ``"heads"``: Ulysses head slices -- every rank restores all tokens of every matrix for its heads
  (uneven splits allowed).
* ``"rows"``: the reference's row layout -- every rank restores its contiguous row slice of every chunk.

Fusion. There is no separate gather: the restore pipeline's unpack kernel loads the owner's coefficient
rows straight from the owner's memory (8-byte peer loads, each remote byte read once) into this rank's
FP16 A operand, the basis-preparation kernel reads the owner's basis rows the same way, and the tcgen05
restore GEMM (bias, RoPE, cast, TMA store into this rank's KV) then runs on local operands. No load uses
TMA multicast.

Synchronization. Staging writes the arenas once (host barrier at set-up). A device-timed restore of
resident factors then needs no barrier at all. The end-to-end path (:meth:`FusedHistoryRestore.restore`
with ``from_host=True``) uploads each owner's coefficients from pinned host memory into one of two
coefficient regions (by call parity) and runs one bounded device barrier before the peers' unpack reads
them; with two regions that single barrier per call also keeps the next-but-one upload behind every
peer's reads of the region it overwrites. No host synchronization runs inside a restore.
"""

from __future__ import annotations

from dataclasses import dataclass
from typing import Any, Callable, Mapping, Sequence

import numpy as np
import torch

from ..errors import CapacityError, ConfigurationError, StateError
from .symmetric import align

LAYOUT_KINDS = ("sequence", "heads", "rows")


def default_owner(layer: int, target: str, world: int) -> int:
    """Whole-matrix factor owner: alternating over layers, V one rank after K."""
    return (layer + (1 if target == "V" else 0)) % world


def k_pad_of(rank: int) -> int:
    return (rank + 63) // 64 * 64


@dataclass(frozen=True)
class HistoryTile:
    """One archived matrix of the history and where its factors live in the owner's arena."""

    index: int
    chunk: int
    layer: int
    target: str
    tokens: int
    rank: int
    channels: int
    owner: int
    coeff_offset: int      # uint8 [tokens, k_pad] (row stride k_pad) in coefficient region 0
    basis_offset: int      # float16 [rank, channels]

    @property
    def k_pad(self) -> int:
        return k_pad_of(self.rank)

    @property
    def coeff_bytes(self) -> int:
        return self.tokens * self.k_pad

    @property
    def basis_bytes(self) -> int:
        return self.rank * self.channels * 2


@dataclass(frozen=True)
class Piece:
    """The part of one tile a rank restores: rows ``[row0, row0 + rows)`` and channels
    ``[col0, col0 + cols)`` of the matrix, written at row ``dest_row`` of the rank's local KV."""

    row0: int
    rows: int
    col0: int
    cols: int
    dest_row: int


class HistoryLayout:
    """Native ownership of a restored history of ``chunks`` chunks of ``tokens`` tokens each."""

    def __init__(self, kind: str, world: int, *, chunks: int, tokens: int, heads: int, head_dim: int):
        if kind not in LAYOUT_KINDS:
            raise ConfigurationError(f"layout kind must be one of {LAYOUT_KINDS}")
        for name, value in (("world", world), ("chunks", chunks), ("tokens", tokens), ("heads", heads),
                            ("head_dim", head_dim)):
            if type(value) is not int or value < 1:
                raise ConfigurationError(f"{name} must be a positive integer")
        if kind == "sequence" and chunks < world:
            raise ConfigurationError("a sequence layout needs at least one chunk per rank")
        if kind == "heads" and heads < world:
            raise ConfigurationError("a head layout needs at least one head per rank")
        if kind == "rows" and tokens < world:
            raise ConfigurationError("a row layout needs at least one token per rank and chunk")
        self.kind, self.world = kind, world
        self.chunks, self.tokens, self.heads, self.head_dim = chunks, tokens, heads, head_dim

    @property
    def channels(self) -> int:
        return self.heads * self.head_dim

    def chunk_range(self, rank: int) -> range:
        """``sequence``: the chunks of ``rank`` (contiguous; earlier ranks take the remainder first)."""
        base, extra = divmod(self.chunks, self.world)
        start = rank * base + min(rank, extra)
        return range(start, start + base + (1 if rank < extra else 0))

    def native_of(self, chunk: int) -> int:
        for rank in range(self.world):
            if chunk in self.chunk_range(rank):
                return rank
        raise ConfigurationError("chunk outside the history")

    def head_range(self, rank: int) -> range:
        return range(rank * self.heads // self.world, (rank + 1) * self.heads // self.world)

    def row_range(self, rank: int) -> range:
        base, extra = divmod(self.tokens, self.world)
        start = rank * base + min(rank, extra)
        return range(start, start + base + (1 if rank < extra else 0))

    def local_tokens(self, rank: int) -> int:
        if self.kind == "sequence":
            return len(self.chunk_range(rank)) * self.tokens
        if self.kind == "rows":
            return self.chunks * len(self.row_range(rank))
        return self.chunks * self.tokens

    def local_heads(self, rank: int) -> int:
        return len(self.head_range(rank)) if self.kind == "heads" else self.heads

    def pieces(self, rank: int, tile: HistoryTile) -> list[Piece]:
        if self.kind == "sequence":
            chunks = self.chunk_range(rank)
            if tile.chunk not in chunks:
                return []
            return [Piece(0, tile.tokens, 0, self.channels, (tile.chunk - chunks.start) * self.tokens)]
        if self.kind == "heads":
            heads = self.head_range(rank)
            return [Piece(0, tile.tokens, heads.start * self.head_dim, len(heads) * self.head_dim,
                          tile.chunk * self.tokens)]
        rows = self.row_range(rank)
        return [Piece(rows.start, len(rows), 0, self.channels, tile.chunk * len(rows))]

    def to_dict(self) -> dict[str, Any]:
        return {"kind": self.kind, "world": self.world, "chunks": self.chunks, "tokens": self.tokens,
                "heads": self.heads, "head_dim": self.head_dim}


@dataclass(frozen=True)
class HistoryPlan:
    """Every tile's owner and arena offsets, identical on every rank. Per owner the arena holds its
    bases, then coefficient region 0, then (double-buffered plans) coefficient region 1."""

    tiles: tuple[HistoryTile, ...]
    world: int
    basis_bytes: tuple[int, ...]       # per owner
    coeff_bytes: tuple[int, ...]       # per owner and region
    regions: int

    @property
    def capacity(self) -> int:
        return max(align(b) + self.regions * align(c) for b, c in zip(self.basis_bytes, self.coeff_bytes))

    def region_shift(self, owner: int) -> int:
        """Byte distance between coefficient regions 0 and 1 of ``owner``."""
        return align(self.coeff_bytes[owner])

    def owned(self, rank: int) -> list[HistoryTile]:
        return [t for t in self.tiles if t.owner == rank]


def plan_history(shapes: Sequence[tuple[int, int, str, int, int]], world: int, channels: int, *,
                 owner: Callable[[int, str, int], int] = default_owner, owners: Sequence[int] | None = None,
                 regions: int = 2) -> HistoryPlan:
    """``shapes``: ``(chunk, layer, target, tokens, rank)`` of every matrix of the history; ``owners`` (one per
    shape) overrides the ``owner`` rule. Offsets are 256-byte aligned (TMA and vector loads), bases first so
    that they stay put across regions."""
    if owners is not None and len(owners) != len(shapes):
        raise ConfigurationError("one owner per matrix")
    if regions not in (1, 2):
        raise ConfigurationError("one or two coefficient regions")
    basis_cursor = [0] * world
    coeff_cursor = [0] * world
    staged: list = [None] * len(shapes)
    # coefficients layer-major in every owner's region: a stage of consecutive layers is one contiguous upload
    order = sorted(range(len(shapes)), key=lambda i: (shapes[i][1], shapes[i][2], shapes[i][0]))
    for index in order:
        chunk, layer, target, tokens, rank = shapes[index]
        if rank < 1 or rank > channels or tokens < 1:
            raise ConfigurationError("tile rank must be in [1, channels] and tokens positive")
        o = owner(layer, target, world) if owners is None else owners[index]
        if not 0 <= o < world:
            raise ConfigurationError("matrix owner outside the group")
        staged[index] = (chunk, layer, target, tokens, rank, o, coeff_cursor[o], basis_cursor[o])
        basis_cursor[o] += align(rank * channels * 2)
        coeff_cursor[o] += align(tokens * k_pad_of(rank))
    tiles = tuple(HistoryTile(i, c, l, t, n, r, channels, o, align(basis_cursor[o]) + co, bo)
                  for i, (c, l, t, n, r, o, co, bo) in enumerate(staged))
    return HistoryPlan(tiles, world, tuple(basis_cursor), tuple(coeff_cursor), regions)


class LocalArena:
    """The single-process stand-in of :class:`~.symmetric.SymmetricArena`: ``world`` buffers on one
    device, one per emulated rank (``world = 1``: the plain single-GPU restore). Barriers are no-ops:
    every emulated rank's work runs in stream order on one GPU, so nothing ever waits on a peer."""

    def __init__(self, device, capacity: int, world: int = 1, rank: int = 0):
        self.device = torch.device(device)
        self.world, self.rank = world, rank
        self.capacity = align(max(int(capacity), 256))
        self.buffers = [torch.empty(self.capacity, dtype=torch.uint8, device=self.device) for _ in range(world)]
        self.epoch = 0

    def for_rank(self, rank: int) -> "LocalArena":
        other = LocalArena.__new__(LocalArena)
        other.__dict__.update(self.__dict__)
        other.rank = rank
        return other

    def view(self, peer: int, offset: int, shape, dtype) -> torch.Tensor:
        itemsize = torch.empty((), dtype=dtype).element_size()
        count = int(np.prod(shape)) if len(shape) else 1
        if offset < 0 or offset + count * itemsize > self.capacity or offset % itemsize:
            raise CapacityError("region lies outside the arena")
        return self.buffers[peer][offset:offset + count * itemsize].view(dtype).view(tuple(shape))

    def barrier(self, stream=None) -> None:
        self.epoch += 1

    def check(self) -> None:
        from ..ops._ext import check_status
        check_status(self.device)

    def close(self) -> None:
        self.buffers = []


class FusedHistoryRestore:
    """Collective restore of a history whose factors are spread over the ranks' arenas.

    ``stage`` once (owners write their factors; every rank learns every tile's affine), ``build`` once per
    destination (the restore program of this rank's pieces, operands pointing into the owners' arenas),
    then ``restore`` any number of times on a stream. ``arena``: a :class:`~.symmetric.SymmetricArena` of
    the group (one process per GPU) or a :class:`LocalArena` (one GPU; ``world > 1`` emulates every rank
    on it, for tests of the plan on one device)."""

    def __init__(self, plan: HistoryPlan, layout: HistoryLayout, grid: tuple[int, int, int], arena, *,
                 group=None, precision: str = "fp16x2"):
        if plan.world != layout.world or arena.world != plan.world:
            raise ConfigurationError("plan, layout and arena describe different groups")
        if grid[0] * grid[1] * grid[2] != layout.tokens:
            raise ConfigurationError("the grid must cover one chunk's tokens")
        self.plan, self.layout, self.grid, self.arena = plan, layout, tuple(grid), arena
        self.group = group
        self.device = arena.device
        self.precision = precision
        self.emulated = isinstance(arena, LocalArena) and arena.world > 1
        self.affine: list[tuple[np.ndarray, np.ndarray, float]] | None = None
        self.programs: dict[tuple[int, int], Any] = {}
        self.current = 0          # coefficient region written by the latest upload
        self.mirror = None        # pinned host copy of this owner's coefficient region
        self.stages = 4           # upload / barrier / restore stages of an end-to-end restore
        self._copies = None       # copy stream of the staged uploads
        self.stats = {"restores": 0, "uploads": 0, "remote_coeff_bytes": 0, "local_coeff_bytes": 0,
                      "remote_basis_bytes": 0}

    @classmethod
    def create(cls, plan: HistoryPlan, layout: HistoryLayout, grid, device, *, group=None,
               precision: str = "fp16x2") -> "FusedHistoryRestore":
        """With one rank: a local arena; else the group's symmetric arena (collective)."""
        if plan.world == 1:
            arena = LocalArena(device, plan.capacity)
        else:
            from .symmetric import SymmetricArena
            arena = SymmetricArena(group, device, plan.capacity)
        return cls(plan, layout, grid, arena, group=group, precision=precision)

    @property
    def rank(self) -> int:
        return self.arena.rank

    def _owners(self) -> list[int]:
        return list(range(self.plan.world)) if self.emulated else [self.arena.rank]

    def _coeff_view(self, tile: HistoryTile, region: int, row0: int = 0, rows: int | None = None):
        rows = tile.tokens - row0 if rows is None else rows
        offset = tile.coeff_offset + region * self.plan.region_shift(tile.owner) + row0 * tile.k_pad
        return self.arena.view(tile.owner, offset, (rows, tile.k_pad), torch.uint8)

    def _basis_view(self, tile: HistoryTile):
        return self.arena.view(tile.owner, tile.basis_offset, (tile.rank, tile.channels), torch.float16)

    # -- staging --------------------------------------------------------------------------------------------

    def stage(self, factors: Mapping[int, tuple[torch.Tensor, torch.Tensor, Any, Any]]) -> None:
        """Owners write their tiles' factors into their arena; ``factors[tile.index]`` = (uint8 coefficients
        ``[tokens, >= rank]`` on this device, FP16 basis ``[>= rank, channels]``, scale ``[rank]``, offset
        ``[rank]``) for every tile this rank owns (every tile when emulated). Collective: one all-reduce of the
        affines and basis bounds, then a host barrier (set-up only)."""
        import torch.distributed as dist

        plan = self.plan
        slots, cursor = [], 0
        for tile in plan.tiles:
            slots.append(cursor)
            cursor += 1 + 2 * tile.rank
        meta = np.zeros(max(cursor, 1), dtype=np.float64)
        owners = set(self._owners())
        bounds = {}
        for tile in plan.tiles:
            if tile.owner not in owners:
                continue
            if tile.index not in factors:
                raise ConfigurationError(f"owner {tile.owner} has no factors for tile {tile.index}")
            coeff, basis, scale, offset = factors[tile.index]
            if coeff.dtype != torch.uint8 or coeff.dim() != 2 or coeff.shape[0] != tile.tokens or \
                    coeff.shape[1] < tile.rank:
                raise ConfigurationError("coefficients must be uint8 [tokens, >= rank]")
            if basis.dtype != torch.float16 or basis.shape[0] < tile.rank or basis.shape[1] != tile.channels:
                raise ConfigurationError("basis must be float16 [>= rank, channels]")
            for region in range(plan.regions):
                self._coeff_view(tile, region)[:, :tile.rank].copy_(coeff[:, :tile.rank])
            self._basis_view(tile).copy_(basis[:tile.rank])
            s = slots[tile.index]
            bounds[s] = basis[:tile.rank].abs().amax()
            meta[s + 1:s + 1 + tile.rank] = np.asarray(scale, dtype=np.float64)[:tile.rank]
            meta[s + 1 + tile.rank:s + 1 + 2 * tile.rank] = np.asarray(offset, dtype=np.float64)[:tile.rank]
        if bounds:  # one device-to-host read for every owned basis bound
            values = torch.stack(list(bounds.values())).double().cpu().numpy()
            for s, value in zip(bounds, values):
                meta[s] = value
        meta_t = torch.from_numpy(meta).to(self.device)
        if not self.emulated and plan.world > 1:
            dist.all_reduce(meta_t, op=dist.ReduceOp.SUM, group=self.group)
        host = meta_t.cpu().numpy()
        self.affine = []
        for tile, s in zip(plan.tiles, slots):
            self.affine.append((host[s + 1:s + 1 + tile.rank].astype(np.float32),
                                host[s + 1 + tile.rank:s + 1 + 2 * tile.rank].astype(np.float32), float(host[s])))
        torch.cuda.synchronize(self.device)
        if not self.emulated and plan.world > 1:
            dist.barrier(group=self.group)
        self.current = 0

    # -- programs -------------------------------------------------------------------------------------------

    def build(self, destination: Callable[[int, str], torch.Tensor], rope: Callable[[HistoryTile], Any] | None = None,
              *, stream=None, rank: int | None = None) -> int:
        """Plan this rank's restore (``rank``: the emulated rank on a local arena). ``destination(layer,
        target)`` is the rank's local KV ``[1, local_tokens, local_heads, head_dim]``; ``rope(tile)`` gives the
        ``RopePositions`` of a K tile (None: no rotation). Returns the number of restore jobs."""
        from ..ops.restore import RestoreProgram
        from ..restore_kernels import restore_rope_item

        if self.affine is None:
            raise StateError("stage() the factors before building the restore")
        rank = self.arena.rank if rank is None else rank
        if not self.emulated and rank != self.arena.rank:
            raise ConfigurationError("only an emulated arena builds another rank's program")
        stream = stream or torch.cuda.current_stream(self.device)
        layout, head_dim = self.layout, self.layout.head_dim
        jobs = 0
        for region in range(self.plan.regions):
            program = RestoreProgram(self.device, stream, precision=self.precision)
            for tile in self.plan.tiles:
                scale, offset, qmax = self.affine[tile.index]
                for piece in layout.pieces(rank, tile):
                    values = self._coeff_view(tile, region, piece.row0, piece.rows)
                    basis = self._basis_view(tile)[:, piece.col0:piece.col0 + piece.cols]
                    cache = destination(tile.layer, tile.target)
                    rows = cache[0] if cache.dim() == 4 else cache
                    dest = rows[piece.dest_row:piece.dest_row + piece.rows]
                    if dest.shape[0] != piece.rows or dest.shape[1] * dest.shape[2] != piece.cols:
                        raise ConfigurationError("destination does not hold this rank's native piece")
                    positions = rope(tile) if (rope is not None and tile.target == "K") else None
                    whole = piece.rows == tile.tokens
                    grid = self.grid if whole else (1, 1, piece.rows)
                    if positions is None:
                        item = None
                    elif whole:
                        item = restore_rope_item(positions, self.grid, self.device, stream, program.keepalive)
                    else:  # a row slice: per-token tables of the whole chunk, read from the slice's first row
                        cos, sin = positions.table.token_tables(positions.rows, self.grid, self.device, stream)
                        program.keepalive.extend((cos, sin))
                        pairs = positions.table.pairs
                        step = piece.row0 * pairs * 4
                        item = ("tokens", cos.data_ptr() + step, sin.data_ptr() + step, pairs)
                    program.add({"kind": "u8", "values": values, "tokens": piece.rows, "rank": tile.rank,
                                 "grid": grid, "basis": basis, "qmax": qmax, "scale": scale, "offset": offset,
                                 "rope": item,
                                 "dest": (dest.data_ptr(), (dest.stride(0), dest.stride(1), dest.stride(2)),
                                          dest.dtype, piece.cols, head_dim)}, group=tile.layer)
                    if region == 0:
                        jobs += 1
                        remote = tile.owner != rank
                        key = "remote_coeff_bytes" if remote else "local_coeff_bytes"
                        self.stats.setdefault("plan_" + key, 0)
                        self.stats["plan_" + key] += piece.rows * tile.k_pad
                        if remote:
                            self.stats.setdefault("plan_remote_basis_bytes", 0)
                            self.stats["plan_remote_basis_bytes"] += tile.rank * piece.cols * 2
            if program.jobs:
                program.prepare(run_aux=False)
            self.programs[(rank, region)] = program
        return jobs

    def launch_count(self, rank: int | None = None) -> int:
        program = self.programs.get((self.arena.rank if rank is None else rank, 0))
        return 0 if program is None or not program.jobs else program.batch_launch_count(aux=True)

    def launch(self, stream=None, *, rank: int | None = None, region: int | None = None) -> int:
        """Enqueue this rank's restore (unpack from the owners' coefficients, basis preparation from their
        bases, tcgen05 restore) on ``stream``; no host synchronization, no barrier."""
        rank = self.arena.rank if rank is None else rank
        program = self.programs[(rank, self.current if region is None else region)]
        if not program.jobs:
            return 0
        stream = stream or torch.cuda.current_stream(self.device)
        launches = 0
        for batch in program.batches():
            launches += program.launch_batch(batch, stream, aux=True)
        return launches

    def host_mirror(self) -> torch.Tensor:
        """Pinned host copy of this owner's coefficient region (the bytes an end-to-end restore uploads)."""
        if self.mirror is None:
            owner = self.arena.rank
            base = align(self.plan.basis_bytes[owner])
            nbytes = max(self.plan.coeff_bytes[owner], 16)
            region = self.arena.view(owner, base, (nbytes,), torch.uint8)
            self.mirror = torch.empty(nbytes, dtype=torch.uint8, pin_memory=True)
            self.mirror.copy_(region)
        return self.mirror

    def restore(self, stream=None, *, from_host: bool = False) -> int:
        """One restore of the whole history into every rank's native KV.

        ``from_host``: upload this owner's coefficients from pinned host memory into the region the previous
        upload did not write, in stages of consecutive layers, each followed by a bounded device barrier before
        that stage's restore launches (every owner's upload of the stage done before any peer's unpack reads it;
        the region written here was last read before the previous upload's barriers), so a stage restores
        while the next one uploads. Without it the resident coefficients of the latest upload are restored
        again. Collective only with ``from_host`` (the barriers); returns the kernels this rank launched."""
        stream = stream or torch.cuda.current_stream(self.device)
        if self.emulated and from_host:
            raise ConfigurationError("an emulated arena restores resident factors only")
        if from_host:
            launches = self._pipelined_upload_and_launch(stream)
        else:
            launches = self.launch(stream)
        self.stats["restores"] += 1
        for key in ("remote_coeff_bytes", "local_coeff_bytes", "remote_basis_bytes"):
            self.stats[key] += self.stats.get("plan_" + key, 0)
        return launches

    def _stages(self) -> list[list[int]]:
        """The history's layers in ``self.stages`` contiguous groups (the same on every rank)."""
        layers = sorted({tile.layer for tile in self.plan.tiles})
        count = max(1, min(self.stages, len(layers)))
        size = -(-len(layers) // count)
        return [layers[i:i + size] for i in range(0, len(layers), size)]

    def _pipelined_upload_and_launch(self, stream) -> int:
        """Upload this owner's coefficients stage by stage (consecutive layers, contiguous bytes) on a copy
        stream into the region the previous upload did not write; before a stage's restore launches, a bounded
        device barrier (every owner's upload of that stage has landed). Stage s's restore runs while stage s + 1
        crosses PCIe."""
        mirror = self.host_mirror()
        owner = self.arena.rank
        region = 1 - self.current if self.plan.regions == 2 else 0
        base0 = align(self.plan.basis_bytes[owner])
        shift = region * self.plan.region_shift(owner)
        if self._copies is None:
            self._copies = torch.cuda.Stream(self.device)
        copies = self._copies
        copies.wait_stream(stream)   # the region was last read before the previous upload's barriers
        stages = self._stages()
        events = []
        with torch.cuda.stream(copies):
            for layers in stages:
                wanted = set(layers)
                mine = [t for t in self.plan.tiles if t.owner == owner and t.layer in wanted]
                if mine:
                    lo = min(t.coeff_offset for t in mine)
                    hi = max(t.coeff_offset + align(t.tokens * t.k_pad) for t in mine)
                    hi = min(hi, base0 + mirror.numel())
                    self.arena.view(owner, lo + shift, (hi - lo,), torch.uint8).copy_(
                        mirror[lo - base0:hi - base0], non_blocking=True)
                event = torch.cuda.Event()
                event.record(copies)
                events.append(event)
        self.current = region
        self.stats["uploads"] += 1
        program = self.programs[(owner, region)]
        launches = 0
        for layers, event in zip(stages, events):
            stream.wait_event(event)
            self.arena.barrier(stream)
            launches += 1
            present = [layer for layer in layers if layer in program.groups]
            for batch in (program.batches(present) if present else ()):
                launches += program.launch_batch(batch, stream, aux=True)
        return launches

    def check(self) -> None:
        self.arena.check()

    def close(self) -> None:
        self.programs.clear()
        self.arena.close()


__all__ = ["LAYOUT_KINDS", "FusedHistoryRestore", "HistoryLayout", "HistoryPlan", "HistoryTile", "LocalArena",
           "Piece", "default_owner", "plan_history"]
