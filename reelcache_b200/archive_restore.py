"""Restore of a lineage node's attended history into native KV caches (reference:
reelcache/archive_restore.py:72-1479).

:class:`LineageRestorer` resolves a node's history (newest version of every attended range on its
ancestor path), keeps decoded node packs in pinned host memory (the prepared-packet cache / decoded
tier: restores skip entropy decoding) and FP16 basis prefixes on the device (:class:`DeviceBasisCache`),
copies the history's 8-bit coefficient tiles to the device with one asynchronous copy per pack, and
reconstructs every layer with the fused sm_100a kernels (ops/restore.py): unpack + basis preparation
for all jobs, then one tcgen05 GEMM launch per layer that writes ``RoPE(dequant(P) @ Q)`` into the
cache. Layers are marked on a :class:`~reelcache_b200.overlapped_restore.LayerReadiness` so the first
forward of the next chunk waits only for the layer it is about to attend over.
"""

from __future__ import annotations

import threading
import time
from collections import OrderedDict
from dataclasses import dataclass, field
from typing import Any, Callable, Mapping, Sequence

import numpy as np
import torch

from .cache_epochs import ResolvedPiece
from .errors import CapacityError, ConfigurationError, IntegrityError, UnsupportedError
from .lineage import LineageRuntime
from .ops.restore import RestoreProgram
from .overlapped_restore import LayerReadiness, OverlappedRestore, start_overlapped_restore
from .restore_kernels import DEFAULT_PRECISION, RopePositions, RopeTable, restore_rope_item
from .types import MatrixKey, entry_parts


class DeviceBasisCache:
    """FP16 basis prefixes ``[rank, C]`` on one device by (version ref, rank), LRU under a byte budget
    (plus max |Q| of each, for the restore's exact prescale)."""

    def __init__(self, runtime: LineageRuntime, device, *, budget_bytes: int = 4 << 30):
        self.runtime = runtime
        self.device = torch.device(device)
        self.budget = budget_bytes
        self._lock = threading.Lock()
        self._entries: OrderedDict = OrderedDict()
        self.bytes = 0
        self.hits = 0
        self.misses = 0

    def get(self, version_ref: str, rank: int, stream=None) -> tuple[torch.Tensor, float]:
        key = (version_ref, rank)
        with self._lock:
            hit = self._entries.get(key)
            if hit is not None:
                self._entries.move_to_end(key)
                self.hits += 1
                return hit
        rows = self.runtime.basis.assemble(version_ref, rank)
        qmax = float(np.abs(rows.numpy().astype(np.float32)).max(initial=0.0))
        ctx = torch.cuda.stream(stream) if stream is not None else _Null()
        with ctx:
            device_rows = rows.pin_memory().to(self.device, non_blocking=True) if self.device.type == "cuda" \
                else rows.to(self.device)
        entry = (device_rows, qmax)
        with self._lock:
            self.misses += 1
            self._entries[key] = entry
            self.bytes += device_rows.numel() * 2
            while self.bytes > self.budget and len(self._entries) > 1:
                _, (old, _) = self._entries.popitem(last=False)
                self.bytes -= old.numel() * 2
        return entry

    def stats(self) -> dict[str, int]:
        return {"entries": len(self._entries), "bytes": self.bytes, "hits": self.hits, "misses": self.misses}


@dataclass
class PreparedPack:
    """A node pack's decoded coefficient tiles in (pinned) host memory, and its affines."""

    packet_ref: str
    raw: torch.Tensor              # uint8 [raw_bytes] (pinned when possible)
    tiles: list
    scales: list
    offsets: list
    nbytes: int

    def tile_view(self, device_raw: torch.Tensor, index: int) -> torch.Tensor:
        coeff = self.tiles[index]["coefficients"]
        tokens, rank = coeff["shape"]
        return device_raw[coeff["offset"]:coeff["offset"] + coeff["bytes"]].view(tokens, rank)


@dataclass
class _RestorePlan:
    program: RestoreProgram
    device_raw: dict
    copies: list
    nbytes: int
    done: Any = None  # event after the plan's last launch


@dataclass
class HistoryEntry:
    piece: ResolvedPiece
    packet_ref: str
    tiles: dict  # entry -> (tile index, record)


@dataclass
class RestoreResult:
    node_ref: str
    readiness: LayerReadiness
    handle: OverlappedRestore | None
    stats: dict = field(default_factory=dict)

    def wait(self, layer: int, stream=None) -> None:
        self.readiness.wait(layer, stream)

    def join(self):
        if self.handle is not None:
            self.handle.join()
        return self.stats


class LineageRestorer:
    """Restores lineage nodes into caches with the fused sm_100a path."""

    def __init__(self, runtime: LineageRuntime, device, *, precision: str = "auto",
                 prepared_budget_bytes: int = 4 << 30, basis_budget_bytes: int = 4 << 30, pin_memory: bool = True,
                 plan_budget_bytes: int = 2 << 30, staging=None, verify_packs: bool = True):
        """``staging``: a :class:`~reelcache_b200.restore_staging.StagingEngine` that reads cold packs with
        parallel native ``pread`` into its pinned ring (default: the store's reads). ``verify_packs``: check
        every tile of a decoded pack against its digest."""
        self.staging = staging
        self.verify_packs = verify_packs
        self.runtime = runtime
        self.device = torch.device(device)
        self.precision = precision
        self.bases = DeviceBasisCache(runtime, self.device, budget_bytes=basis_budget_bytes)
        self.prepared_budget = prepared_budget_bytes
        self.pin_memory = pin_memory and self.device.type == "cuda"
        self._prepared: OrderedDict = OrderedDict()
        self._prepared_bytes = 0
        self._lock = threading.Lock()
        self._histories: dict = {}
        self._plans: OrderedDict = OrderedDict()
        self._plan_bytes = 0
        self.plan_budget = plan_budget_bytes
        self._copies = None
        self.stats_ = {"restores": 0, "packs_prepared": 0, "h2d_bytes": 0, "plans_built": 0, "plan_hits": 0}

    # -- preparation ---------------------------------------------------------------------------------------------

    def prepared_pack(self, packet_ref: str) -> PreparedPack:
        """Decoded pack in pinned host memory (cached, LRU under the prepared budget)."""
        with self._lock:
            hit = self._prepared.get(packet_ref)
            if hit is not None:
                self._prepared.move_to_end(packet_ref)
                return hit
        reader = None
        if self.staging is not None:
            def reader(ids):
                staged = self.staging.stage(ids)
                try:
                    return {object_id: staged.bytes(object_id) for object_id in ids}
                finally:
                    staged.release()
        _, pack = self.runtime.node_pack(packet_ref, verify=self.verify_packs, reader=reader)
        raw = torch.from_numpy(np.array(pack.raw, dtype=np.uint8, copy=True))
        if self.pin_memory:
            raw = raw.pin_memory()
        scales, offsets = [], []
        for index in range(len(pack.tiles)):
            s, o = pack.scale_offset(index)
            scales.append(s)
            offsets.append(o)
        prepared = PreparedPack(packet_ref, raw, list(pack.tiles), scales, offsets, raw.numel())
        with self._lock:
            self._prepared[packet_ref] = prepared
            self._prepared_bytes += prepared.nbytes
            self.stats_["packs_prepared"] += 1
            while self._prepared_bytes > self.prepared_budget and len(self._prepared) > 1:
                _, old = self._prepared.popitem(last=False)
                self._prepared_bytes -= old.nbytes
        return prepared

    def history(self, node_ref: str, ranges: Sequence[tuple[int, int]] | None = None) -> list[HistoryEntry]:
        """Resolved history of a node: per attended piece its pack and tile of every matrix entry."""
        key = (node_ref, None if ranges is None else tuple(map(tuple, ranges)))
        hit = self._histories.get(key)
        if hit is not None:
            return hit
        entries = []
        for piece in self.runtime.resolve_history(node_ref, ranges):
            tiles = {}
            packet_ref = None
            for entry, record_ref in piece.entry.records:
                record = self.runtime.load_record(record_ref)
                if record.codec.kind == "raw":
                    raise UnsupportedError("RAW history restores through RawLineageRestorer")
                if record.codec.kind == "svd":
                    raise UnsupportedError("SVD-only (factor pack) history restores through FactorLineageRestorer")
                packet_ref = record.packet_ref
                tiles[entry] = (record.decision["packet"]["tile"], record)
            entries.append(HistoryEntry(piece, packet_ref, tiles))
        self._histories[key] = entries
        return entries

    def prewarm(self, node_ref: str, ranges=None) -> int:
        entries = self.history(node_ref, ranges)
        for item in entries:
            self.prepared_pack(item.packet_ref)
        for item in entries:
            for _, record in item.tiles.values():
                self.bases.get(record.basis_version_ref, record.rank_view)
        return len(entries)

    # -- restore -------------------------------------------------------------------------------------------------

    def build_program(self, node_ref: str, destination: Callable[[int, str], torch.Tensor],
                      rope: Callable[[ResolvedPiece], tuple[RopeTable, tuple]], *, stream=None, ranges=None,
                      stream_label: str | None = None, layers: Sequence[int] | None = None,
                      device_raw: dict | None = None, slot_of: Callable[[ResolvedPiece], int] | None = None
                      ) -> RestoreProgram:
        """Plan the restore of ``node_ref``: one job per (layer, K/V, piece) reading the history's packs
        from ``device_raw`` (packet ref -> device uint8 copy of the pack; default: copied now on
        ``stream``). ``destination(layer, "K"|"V")`` returns the native BTHD cache tensor
        ``[1, capacity, heads, head_dim]``; ``rope(piece)`` returns the (table, (t_row, h_row, w_row)) of its positions
        (``rope=None``: the destination receives pre-RoPE K, and ranges may cut frames); ``slot_of(piece)`` the first
        cache row of the piece (default: its global token index)."""
        stream = stream or torch.cuda.current_stream(self.device)
        entries = self.history(node_ref, ranges)
        model = self.runtime.model
        layers = range(model.layers) if layers is None else layers
        precision = self.precision
        if device_raw is None:
            device_raw = {}
            with torch.cuda.stream(stream):
                for item in entries:
                    if item.packet_ref in device_raw:
                        continue
                    prepared = self.prepared_pack(item.packet_ref)
                    device_raw[item.packet_ref] = prepared.raw.to(self.device, non_blocking=True)
                    self.stats_["h2d_bytes"] += prepared.nbytes
        program = None
        for layer in layers:
            for target in ("K", "V"):
                cache = destination(layer, target)  # native BTHD cache [1, capacity, heads, head_dim]
                head_dim = cache.shape[-1]
                rows = cache[0]
                if program is None:
                    if precision == "auto":
                        precision = DEFAULT_PRECISION
                    program = RestoreProgram(self.device, stream, precision=precision)
                    program.keepalive.extend(device_raw.values())
                key = MatrixKey(layer, target)
                entry_key = key if stream_label is None else (key, stream_label)
                for item in entries:
                    piece = item.piece
                    tile_index, record = item.tiles[entry_key]
                    prepared = self.prepared_pack(item.packet_ref)
                    values = prepared.tile_view(device_raw[item.packet_ref], tile_index)
                    tokens = piece.token_end - piece.token_start
                    context = record.context
                    if piece.offset or tokens != context.token_count:
                        values = values[piece.offset:piece.offset + tokens]
                        if tokens % (context.height * context.width) and rope is not None:
                            raise UnsupportedError("partial-frame history ranges are not restorable with RoPE")
                    if tokens % (context.height * context.width):
                        grid = (1, 1, tokens)  # rows of frames (no RoPE: the grid only shapes the job)
                    else:
                        grid = (tokens // (context.height * context.width), context.height, context.width)
                    basis, qmax = self.bases.get(record.basis_version_ref, record.rank_view, stream)
                    first_row = piece.token_start if slot_of is None else slot_of(piece)
                    slot = rows[first_row:first_row + tokens]  # [tokens, heads, head_dim]
                    job = {"kind": "u8", "values": values, "tokens": tokens, "rank": record.rank_view,
                           "grid": grid, "basis": basis, "qmax": qmax, "scale": prepared.scales[tile_index],
                           "offset": prepared.offsets[tile_index],
                           "dest": (slot.data_ptr(), (slot.stride(0), slot.stride(1), slot.stride(2)), slot.dtype,
                                    slot.shape[1] * slot.shape[2], head_dim),
                           "rope": None}
                    if target == "K" and context.key_space == "pre_rope" and rope is not None:
                        table, rope_rows = rope(piece)
                        first = piece.offset // (context.height * context.width)
                        rope_rows = (rope_rows[0] + first, rope_rows[1], rope_rows[2])
                        job["rope"] = restore_rope_item(RopePositions(table, rope_rows), grid, self.device, stream,
                                                        program.keepalive)
                    program.add(job, group=layer)
        return program

    def gather_program(self, node_ref: str, destination: Callable[[int, str], torch.Tensor],
                       gathers: Sequence[tuple[int, int, int, int, int]], *, stream=None) -> RestoreProgram:
        """Restore a rank's token subset of a single-range history (a LongCat segment) without RoPE:
        ``gathers`` = ``(dest_row, tokens, run_len, run_stride, run_offset)`` jobs per matrix, each reading
        coefficient rows ``(t // run_len) * run_stride + run_offset + t % run_len`` of the range and writing
        ``tokens`` compact rows from ``dest_row`` of ``destination(layer, "K"|"V")`` ([1, rows, heads, head_dim])."""
        stream = stream or torch.cuda.current_stream(self.device)
        entries = self.history(node_ref)
        if len(entries) != 1 or entries[0].piece.offset:
            raise UnsupportedError("gathered restores read one whole history range (a segment)")
        item = entries[0]
        prepared = self.prepared_pack(item.packet_ref)
        with torch.cuda.stream(stream):
            device_raw = prepared.raw.to(self.device, non_blocking=True)
        self.stats_["h2d_bytes"] += prepared.nbytes
        program = RestoreProgram(self.device, stream, precision=DEFAULT_PRECISION if self.precision == "auto"
                                 else self.precision)
        program.keepalive.append(device_raw)
        for layer in range(self.runtime.model.layers):
            for target in ("K", "V"):
                rows = destination(layer, target)[0]
                tile_index, record = item.tiles[MatrixKey(layer, target)]
                values = prepared.tile_view(device_raw, tile_index)
                basis, qmax = self.bases.get(record.basis_version_ref, record.rank_view, stream)
                for dest_row, tokens, run_len, run_stride, run_offset in gathers:
                    slot = rows[dest_row:dest_row + tokens]
                    program.add({"kind": "u8", "values": values, "tokens": tokens, "rank": record.rank_view,
                                 "grid": (1, 1, tokens), "basis": basis, "qmax": qmax,
                                 "scale": prepared.scales[tile_index], "offset": prepared.offsets[tile_index],
                                 "runs": (run_len, run_stride, run_offset),
                                 "dest": (slot.data_ptr(), (slot.stride(0), slot.stride(1), slot.stride(2)),
                                          slot.dtype, slot.shape[1] * slot.shape[2], slot.shape[2]),
                                 "rope": None}, group=layer)
        return program

    def node_factors(self, node_ref: str, keys: Sequence[MatrixKey], *, ranges=None, stream=None,
                     stream_label: str | None = None) -> dict:
        """The stored factors of ``keys`` for every history piece of ``node_ref`` (within ``ranges``):
        ``{(token_start, key): (uint8 coefficients [tokens, rank] on the device, FP16 basis [rank, C], scale,
        offset)}`` -- what a sequence-parallel owner stages for its peers' fused restores."""
        stream = stream or torch.cuda.current_stream(self.device)
        out, device_raw = {}, {}
        for item in self.history(node_ref, ranges):
            if item.packet_ref not in device_raw:
                prepared = self.prepared_pack(item.packet_ref)
                with torch.cuda.stream(stream):
                    device_raw[item.packet_ref] = prepared.raw.to(self.device, non_blocking=True)
                self.stats_["h2d_bytes"] += prepared.nbytes
            prepared = self.prepared_pack(item.packet_ref)
            piece = item.piece
            tokens = piece.token_end - piece.token_start
            for key in keys:
                entry = key if stream_label is None else (key, stream_label)
                tile_index, record = item.tiles[entry]
                values = prepared.tile_view(device_raw[item.packet_ref], tile_index)[piece.offset:piece.offset + tokens]
                basis, _ = self.bases.get(record.basis_version_ref, record.rank_view, stream)
                out[(piece.token_start, key)] = (values, basis[:record.rank_view], prepared.scales[tile_index],
                                                 prepared.offsets[tile_index])
        return out

    def _plan_key(self, node_ref, destination, rope, ranges, slot_of=None):
        """Identity of a restore plan: the node, its ranges, every destination tensor (address, shape,
        strides, dtype) and every piece's RoPE table and positions."""
        model = self.runtime.model
        dests = []
        for layer in range(model.layers):
            for target in ("K", "V"):
                t = destination(layer, target)
                dests.append((t.data_ptr(), tuple(t.shape), t.stride(), t.dtype))
        ropes = []
        for item in self.history(node_ref, ranges):
            slot = None if slot_of is None else slot_of(item.piece)
            if rope is None:
                ropes.append((None, slot))
                continue
            table, rows = rope(item.piece)
            ropes.append((id(table), table._stamp(), tuple(rows), slot))
        return (node_ref, None if ranges is None else tuple(map(tuple, ranges)), tuple(dests), tuple(ropes))

    def _layer_copies(self, entries, layer_count):
        """Per layer, the (packet ref, byte range) covering that layer's tiles in each pack."""
        copies = []
        for layer in range(layer_count):
            spans = {}
            for item in entries:
                prepared = self.prepared_pack(item.packet_ref)
                for target in ("K", "V"):
                    found = [v for k, v in item.tiles.items() if entry_parts(k)[0] == MatrixKey(layer, target)]
                    for tile_index, _ in found:
                        coeff = prepared.tiles[tile_index]["coefficients"]
                        lo, hi = coeff["offset"], coeff["offset"] + coeff["bytes"]
                        old = spans.get(item.packet_ref)
                        spans[item.packet_ref] = (lo, hi) if old is None else (min(old[0], lo), max(old[1], hi))
            copies.append(sorted(spans.items()))
        return copies

    def _plan(self, node_ref, destination, rope, stream, ranges, slot_of=None):
        key = self._plan_key(node_ref, destination, rope, ranges, slot_of)
        with self._lock:
            plan = self._plans.get(key)
            if plan is not None:
                self._plans.move_to_end(key)
                self.stats_["plan_hits"] += 1
                return plan
        entries = self.history(node_ref, ranges)
        device_raw = {}
        for item in entries:
            if item.packet_ref not in device_raw:
                prepared = self.prepared_pack(item.packet_ref)
                device_raw[item.packet_ref] = torch.empty(prepared.nbytes, dtype=torch.uint8, device=self.device)
        program = self.build_program(node_ref, destination, rope, stream=stream, ranges=ranges, device_raw=device_raw,
                                     slot_of=slot_of)
        with torch.cuda.stream(stream):
            program.prepare(run_aux=False)
        plan = _RestorePlan(program, device_raw, self._layer_copies(entries, self.runtime.model.layers),
                            sum(t.numel() for t in device_raw.values()) + program.scratch_bytes)
        with self._lock:
            self._plans[key] = plan
            self._plan_bytes += plan.nbytes
            self.stats_["plans_built"] += 1
            while self._plan_bytes > self.plan_budget and len(self._plans) > 1:
                _, old = self._plans.popitem(last=False)
                self._plan_bytes -= old.nbytes
        return plan

    def restore(self, node_ref: str, destination, rope, *, stream=None, overlapped: bool = True, ranges=None,
                readiness: LayerReadiness | None = None, thread: bool = False,
                slot_of: Callable[[ResolvedPiece], int] | None = None) -> RestoreResult:
        """Restore ``node_ref``'s history; returns a :class:`RestoreResult` whose readiness marks each layer
        (the caller's forward waits per layer). All GPU work runs on ``stream`` (default: a side stream).

        Per layer, the pack bytes of that layer's tiles are copied host->device on a copy stream while
        the previous layer restores; the layer's unpack, basis preparation and fused GEMM then run on
        ``stream``. Plans (job tables, tensor maps, device staging of the packs) are built once per
        (node, destinations, RoPE positions) and relaunched; a relaunch first waits for the previous
        use of its staging to finish."""
        started = time.perf_counter()
        model = self.runtime.model
        stream = stream or torch.cuda.Stream(self.device)
        readiness = readiness or LayerReadiness(model.layers)
        plan = self._plan(node_ref, destination, rope, stream, ranges, slot_of)
        program = plan.program
        copy_stream = self._copy_stream()
        if plan.done is not None:
            copy_stream.wait_event(plan.done)
        # Overlapped: one launch per layer, so the forward's layer L waits for layer L only. Otherwise
        # consecutive layers share a launch (up to 48 jobs) and their pack bytes one copy per pack: fewer,
        # fuller launches and copies (the host issues a handful of copies instead of one per layer and pack).
        units = [(layer,) for layer in range(model.layers)] if overlapped else program.batches()
        events = {}
        with torch.cuda.stream(copy_stream):
            for unit in units:
                spans: dict[str, tuple[int, int]] = {}
                for layer in unit:
                    for packet_ref, (lo, hi) in plan.copies[layer]:
                        old = spans.get(packet_ref)
                        spans[packet_ref] = (lo, hi) if old is None else (min(old[0], lo), max(old[1], hi))
                for packet_ref, (lo, hi) in spans.items():
                    host = self.prepared_pack(packet_ref).raw
                    plan.device_raw[packet_ref][lo:hi].copy_(host[lo:hi], non_blocking=True)
                    self.stats_["h2d_bytes"] += hi - lo
                event = torch.cuda.Event()
                event.record(copy_stream)
                for layer in unit:
                    events[layer] = event
        self.stats_["restores"] += 1
        batch_of = {unit[0]: unit for unit in units}

        def issue(layer):
            if overlapped:
                stream.wait_event(events[layer])
                program.launch(layer, stream, aux=True)
            elif layer in batch_of:
                stream.wait_event(events[layer])
                program.launch_batch(batch_of[layer], stream, aux=True)

        def finish():
            done = torch.cuda.Event()
            done.record(stream)
            plan.done = done

        handle = start_overlapped_restore(issue, model.layers, stream=stream, thread=thread and overlapped,
                                          readiness=readiness, finish=finish)
        stats = {"jobs": len(program.jobs), "launches": program.launches, "prepare_seconds": time.perf_counter() - started}
        result = RestoreResult(node_ref, readiness, handle, stats)
        result.program = program
        return result

    def _copy_stream(self):
        if self._copies is None:
            self._copies = torch.cuda.Stream(self.device)
        return self._copies

    def stats(self) -> dict[str, Any]:
        return {**self.stats_, "prepared_packs": len(self._prepared), "prepared_bytes": self._prepared_bytes,
                "bases": self.bases.stats()}


class _Null:
    def __enter__(self):
        return self

    def __exit__(self, *args):
        return False


# ---------------------------------------------------------------------------------------------------------
# Restorers of the other representations (reference reelcache/archive_restore.py:1325 SoftwareLineageRestorer,
# :1396 RawLineageRestorer; reelcache/factor_packs.py:673 FactorLineageRestorer): the same ``restore`` contract
# as LineageRestorer, built from per-layer ReconstructionJobs run by restore_kernels.reconstruct (the fused
# sm_100a kernels on CUDA, the reference path on the host).
# ---------------------------------------------------------------------------------------------------------


class JobLineageRestorer:
    """Base of the per-layer job restorers: ``_prepare(pieces)`` loads what the history needs once, ``_source``
    gives the (source, basis) of one piece's matrix."""

    kinds: tuple = ()

    def __init__(self, runtime: LineageRuntime, device, *, pin_memory: bool = True):
        self.runtime = runtime
        self.device = torch.device(device)
        self.pin_memory = pin_memory and self.device.type == "cuda"
        self._bases: dict = {}
        self.stats_ = {"restores": 0, "jobs": 0, "h2d_bytes": 0}

    def _basis(self, record) -> torch.Tensor:
        key = (record.basis_version_ref, record.rank_view)
        hit = self._bases.get(key)
        if hit is None:
            hit = self.runtime.basis.assemble(record.basis_version_ref, record.rank_view).to(self.device)
            self._bases[key] = hit
        return hit

    def _check(self, record) -> None:
        if record.codec.kind not in self.kinds:
            raise UnsupportedError(f"{type(self).__name__} restores {self.kinds} histories, not {record.codec.kind}")

    def _prepare(self, pieces) -> None:
        return None

    def _source(self, piece, record, rows: slice):
        raise NotImplementedError

    def jobs(self, pieces, layer: int, destination, rope, *, stream_label: str | None = None,
             slot_of: Callable[[ResolvedPiece], int] | None = None) -> list:
        from . import restore_kernels as rk
        jobs = []
        for piece in pieces:
            tokens = piece.token_end - piece.token_start
            for target in ("K", "V"):
                record = self.runtime.load_record(piece.record(MatrixKey(layer, target), stream_label))
                self._check(record)
                context = record.context
                plane = context.height * context.width
                if piece.offset % plane or tokens % plane:
                    raise UnsupportedError("partial-frame history ranges are not restorable")
                source, basis = self._source(piece, record, slice(piece.offset, piece.offset + tokens))
                first_row = piece.token_start if slot_of is None else slot_of(piece)
                view = rk.NativeView(destination(layer, target), "BTHD", first_row)
                positions = None
                if target == "K" and context.key_space == "pre_rope":
                    table, rows = rope(piece)
                    first = piece.offset // plane
                    positions = rk.RopePositions(table, (rows[0] + first, rows[1], rows[2]))
                jobs.append(rk.ReconstructionJob(source, view, (tokens // plane, context.height, context.width),
                                                 basis, rope=positions))
        return jobs

    def restore(self, node_ref: str, destination, rope, *, stream=None, overlapped: bool = True, ranges=None,
                readiness: LayerReadiness | None = None, thread: bool = False,
                stream_label: str | None = None, slot_of: Callable[[ResolvedPiece], int] | None = None
                ) -> RestoreResult:
        """Restore ``node_ref``'s attended history layer by layer (marking ``readiness``)."""
        from . import restore_kernels as rk
        started = time.perf_counter()
        model = self.runtime.model
        cuda = self.device.type == "cuda"
        if cuda and stream is None:
            stream = torch.cuda.Stream(self.device)
        readiness = readiness or LayerReadiness(model.layers)
        pieces = self.runtime.resolve_history(node_ref, ranges)
        for piece in pieces:  # refuse other representations before any work is issued
            for _, record_ref in piece.entry.records:
                self._check(self.runtime.load_record(record_ref))
        self._prepare(pieces)
        handles = []

        def issue(layer):
            jobs = self.jobs(pieces, layer, destination, rope, stream_label=stream_label, slot_of=slot_of)
            if jobs:
                handles.append(rk.reconstruct(jobs, stream=stream))
                self.stats_["jobs"] += len(jobs)

        self.stats_["restores"] += 1
        handle = start_overlapped_restore(issue, model.layers, stream=stream if cuda else None,
                                          thread=thread and overlapped, readiness=readiness)
        result = RestoreResult(node_ref, readiness, handle, {"pieces": len(pieces),
                                                             "prepare_seconds": time.perf_counter() - started})
        result.handles = handles
        return result

    def stats(self) -> dict[str, Any]:
        return dict(self.stats_)


class RawLineageRestorer(JobLineageRestorer):
    """Exact RAW histories: each record's dense pre-RoPE matrix is read once from its RAW packet into (pinned)
    host memory, copied to the device and installed with RoPE by the dense restore kernel (bitwise the stored
    values, up to the cache dtype)."""

    kinds = ("raw",)

    def __init__(self, runtime: LineageRuntime, device, *, budget_bytes: int = 8 << 30, pin_memory: bool = True):
        super().__init__(runtime, device, pin_memory=pin_memory)
        self.budget = budget_bytes
        self._dense: OrderedDict = OrderedDict()
        self._bytes = 0

    def dense(self, record) -> torch.Tensor:
        from . import codecs
        from .types import EncodedTensor
        hit = self._dense.get(record.packet_ref)
        if hit is not None:
            self._dense.move_to_end(record.packet_ref)
            return hit
        packet = self.runtime.load_packet(record.packet_ref)
        blobs = self.runtime.store.get_many(list(packet["payloads"].values()))
        payloads = {name: blobs[ref] for name, ref in packet["payloads"].items()}
        values = codecs.decode_tensor(EncodedTensor(packet["metadata"], payloads), device="cpu")
        values = values.reshape(record.context.token_count, record.context.channels).contiguous()
        if self.pin_memory:
            values = values.pin_memory()
        self._dense[record.packet_ref] = values
        self._bytes += values.numel() * values.element_size()
        while self._bytes > self.budget and len(self._dense) > 1:
            _, old = self._dense.popitem(last=False)
            self._bytes -= old.numel() * old.element_size()
        return values

    def _source(self, piece, record, rows: slice):
        from . import restore_kernels as rk
        values = self.dense(record)[rows]
        if values.dtype not in (torch.float32, torch.float16, torch.bfloat16):
            values = values.float()
        if self.device.type == "cuda":
            values = values.to(self.device, non_blocking=self.pin_memory)
            self.stats_["h2d_bytes"] += values.numel() * values.element_size()
        return rk.DenseSource(values), None


class SoftwareLineageRestorer(JobLineageRestorer):
    """Node-pack (``svd_hevc``) histories decoded in software on the host (the stream codec's CPU decoder; no
    prepared-pack cache, decoder pool or staging): the uint8 coefficient tiles and their affines feed the same
    reconstruction jobs. The portable path (any device) and the oracle of the GPU restorer."""

    kinds = ("svd_hevc",)

    def __init__(self, runtime: LineageRuntime, device, *, pin_memory: bool = False):
        super().__init__(runtime, device, pin_memory=pin_memory)
        self._packs: dict = {}

    def _prepare(self, pieces) -> None:
        self._packs = {}
        for piece in pieces:
            for _, record_ref in piece.entry.records:
                record = self.runtime.load_record(record_ref)
                if record.codec.kind == "svd_hevc" and record.packet_ref not in self._packs:
                    self._packs[record.packet_ref] = self.runtime.node_pack(record.packet_ref)[1]

    def _source(self, piece, record, rows: slice):
        from . import restore_kernels as rk
        pack = self._packs[record.packet_ref]
        index = record.decision["packet"]["tile"]
        pixels = torch.from_numpy(np.array(pack.pixels(index)[rows], copy=True))
        scale, offset = pack.scale_offset(index)
        if self.device.type == "cuda":
            pixels = pixels.to(self.device)
            self.stats_["h2d_bytes"] += pixels.numel()
        return rk.CoefficientSource(pixels, scale, offset), self._basis(record)
