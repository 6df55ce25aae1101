"""Packed decode: prepared node packets and the layer-ahead decode-then-reconstruct restore path (the
counterpart of reference reelcache/packed_decode.py:82-736).

:func:`prepare_packet` reads a node pack once (tile map, per-tile affines, basis references, stream
digest); :class:`PackedRestorer` plans a node's history (``plan``), submits the coefficient-stream
decodes to a :class:`DecoderPool` per layer (``submit`` -> :class:`RestoreBatch`, lazily layer by
layer with ``submit_through(layer)``), takes packs the :class:`DecodedTier` routes past the decoder,
and reconstructs each layer's jobs into the native slots with the restore kernels
(``restore_kernels.reconstruct``, uint8 :class:`CoefficientSource` jobs).
"""

from __future__ import annotations

import hashlib
from dataclasses import dataclass, field
from typing import Any, Callable

import numpy as np
import torch

from . import restore_kernels as rk
from .errors import IntegrityError
from .types import MatrixKey, entry_parts


@dataclass
class PreparedPacket:
    packet_ref: str
    stream: bytes
    stream_codec: str
    digest: str
    tiles: list                        # per tile: {"entry", "coefficients": {offset, bytes, shape}, ...}
    affines: list                      # per tile: (scale, offset) float32 host arrays
    raw_shape: tuple[int, int]


def prepare_packet(runtime, packet_ref: str) -> PreparedPacket:
    packet, pack = runtime.node_pack(packet_ref)
    stream = runtime.store.get(packet["payloads"]["stream"])
    meta = packet["metadata"]
    tiles = list(pack.tiles)
    affines = [pack.scale_offset(i) for i in range(len(tiles))]
    return PreparedPacket(packet_ref, stream, meta.get("stream_codec", "raw8"), hashlib.sha256(stream).hexdigest(),
                          tiles, affines, (1, pack.raw.size))


@dataclass
class RestoreBatch:
    """Decode tickets of one restore, layer by layer."""

    layers: int
    submitted: int = 0
    tickets: dict = field(default_factory=dict)     # packet ref -> DecodeTicket (whole-pack decode)
    routed: list = field(default_factory=list)

    def ready(self, packet_ref: str) -> np.ndarray:
        return self.tickets[packet_ref].wait()


class PackedRestorer:
    def __init__(self, runtime, decoder_pool, *, decoded_tier=None, device="cuda"):
        self.runtime = runtime
        self.pool = decoder_pool
        self.tier = decoded_tier
        self.device = torch.device(device)
        self._prepared: dict[str, PreparedPacket] = {}

    def prepared(self, packet_ref: str) -> PreparedPacket:
        hit = self._prepared.get(packet_ref)
        if hit is None:
            hit = prepare_packet(self.runtime, packet_ref)
            self._prepared[packet_ref] = hit
            if self.tier is not None:
                self.tier.bind(packet_ref, hit.digest)
        return hit

    def plan(self, node_ref: str, ranges=None) -> list:
        """Resolved history pieces with their prepared packets."""
        pieces = self.runtime.resolve_history(node_ref, ranges)
        for piece in pieces:
            _, record_ref = piece.entry.records[0]
            self.prepared(self.runtime.load_record(record_ref).packet_ref)
        return pieces

    def submit(self, pieces, layers: int) -> RestoreBatch:
        batch = RestoreBatch(layers)
        refs = []
        for piece in pieces:
            _, record_ref = piece.entry.records[0]
            refs.append(self.runtime.load_record(record_ref).packet_ref)
        refs = list(dict.fromkeys(refs))
        if self.tier is not None:
            batch.routed = self.tier.route([(r, len(self.prepared(r).stream)) for r in refs], layers)
        for ref in refs:
            if ref in batch.routed:
                continue
            prep = self.prepared(ref)
            batch.tickets[ref] = self.pool.decode_stream(prep.stream, prep.stream_codec, prep.raw_shape)
        batch.submitted = layers
        return batch

    def submit_through(self, batch: RestoreBatch, layer: int) -> None:
        """Whole-pack decodes cover every layer at once; nothing more to submit per layer."""
        return None

    def _tile(self, batch: RestoreBatch, packet_ref: str, index: int) -> torch.Tensor:
        prep = self.prepared(packet_ref)
        coeff = prep.tiles[index]["coefficients"]
        tokens, rank = coeff["shape"]
        if packet_ref in batch.routed:
            raw = self.tier.tiles(packet_ref)[0].reshape(-1)
        else:
            raw = torch.from_numpy(np.array(batch.ready(packet_ref), copy=True).reshape(-1))
        return raw[coeff["offset"]:coeff["offset"] + coeff["bytes"]].view(tokens, rank)

    def reconstruct(self, batch: RestoreBatch, pieces, layer: int, destination: Callable, rope: Callable,
                    *, stream=None) -> Any:
        """Restore one layer's K and V of every piece into ``destination(layer, which)`` (BTHD slots)."""
        jobs = []
        bases = {}
        for piece in pieces:
            entries = {entry_parts(e)[0]: ref for e, ref in piece.entry.records}
            for target in ("K", "V"):
                record = self.runtime.load_record(entries[MatrixKey(layer, target)])
                prep = self.prepared(record.packet_ref)
                tile_index = record.decision["packet"]["tile"]
                values = self._tile(batch, record.packet_ref, tile_index)
                tokens = piece.token_end - piece.token_start
                values = values[piece.offset:piece.offset + tokens]
                scale, offset = prep.affines[tile_index]
                key = (record.basis_version_ref, record.rank_view)
                if key not in bases:
                    bases[key] = self.runtime.basis.assemble(record.basis_version_ref, record.rank_view).to(self.device)
                ctx = record.context
                frames = tokens // (ctx.height * ctx.width)
                cache = destination(layer, target)
                view = rk.NativeView(cache, "BTHD", piece.token_start)
                positions = None
                if target == "K" and ctx.key_space == "pre_rope":
                    table, rows = rope(piece)
                    first = piece.offset // (ctx.height * ctx.width)
                    positions = rk.RopePositions(table, (rows[0] + first, rows[1], rows[2]))
                jobs.append(rk.ReconstructionJob(rk.CoefficientSource(values.to(self.device), scale, offset), view,
                                                 (frames, ctx.height, ctx.width), bases[key], rope=positions))
        if not jobs:
            return None
        return rk.reconstruct(jobs, backend="auto", stream=stream)

    def release(self, batch: RestoreBatch) -> None:
        if self.tier is not None and batch.routed:
            self.tier.release(batch.routed)
