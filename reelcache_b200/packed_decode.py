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

from . import _hevc
from . import restore_kernels as rk
from .errors import ConfigurationError, IntegrityError
from .types import MatrixKey, entry_parts


@dataclass(frozen=True, eq=False)
class PreparedTile:
    """One matrix of a prepared node pack: where its 8-bit coefficients sit in the pack (``offset``, ``nbytes``,
    ``shape`` = ``[tokens, rank]``), their per-column affine and the basis the record binds (the version ref and
    rank view; resolved by the restorer's basis cache). ``grid`` and ``token_start`` place it in the history."""

    key: Any
    layer: int
    target: str
    index: int
    offset: int
    nbytes: int
    shape: tuple[int, int]
    scale: np.ndarray
    bias: np.ndarray
    basis_version_ref: str | None
    rank: int
    grid: tuple[int, int, int]
    token_start: int

    def pixels(self, raw) -> Any:
        """This tile's ``[tokens, rank]`` uint8 view of a pack's decoded bytes (host array or device tensor)."""
        flat = raw.reshape(-1)
        return flat[self.offset:self.offset + self.nbytes].reshape(self.shape)


@dataclass
class PreparedPacket:
    packet_ref: str
    stream: bytes
    stream_codec: str
    digest: str
    tiles: list                        # per tile: {"entry", "coefficients": {offset, bytes, shape}, ...}
    affines: list                      # per tile: (scale, offset) float32 host arrays
    raw_shape: tuple[int, int]

    def tile(self, index: int) -> dict:
        """The pack's tile entry ``index`` (coefficient placement and its matrix entry)."""
        if not 0 <= index < len(self.tiles):
            raise ConfigurationError(f"pack {self.packet_ref} has {len(self.tiles)} tiles, not {index + 1}")
        return self.tiles[index]


def prepared_tiles(runtime, prepared: "PreparedPacket", records) -> list[PreparedTile]:
    """The :class:`PreparedTile` of every ``(entry, record ref)`` of a history piece that lives in ``prepared``."""
    out = []
    for entry, record_ref in records:
        record = runtime.load_record(record_ref)
        if record.packet_ref != prepared.packet_ref:
            continue
        key, _ = entry_parts(entry)
        index = record.decision["packet"]["tile"]
        coeff = prepared.tiles[index]["coefficients"]
        scale, bias = prepared.affines[index]
        ctx = record.context
        out.append(PreparedTile(entry, key.layer, key.target, index, int(coeff["offset"]), int(coeff["bytes"]),
                                tuple(coeff["shape"]), scale, bias, record.basis_version_ref, int(record.rank_view),
                                (ctx.frames, ctx.height, ctx.width), ctx.token_start))
    return out


def canonical_canvas_shapes(frames: int, height: int, width: int, pix_fmt: str = "yuv444p", *, channels: int,
                            max_rank: int | None = None) -> list[tuple[int, int, str]]:
    """``(width, height, pix_fmt)`` of every canonical node canvas of one tile geometry, smallest first: one per
    rank step of the canvas ladder up to ``max_rank`` (default ``channels``), leaving out canvases beyond the
    largest HEVC picture. Warming a decoder for each covers every pack of the geometry."""
    from .node_packets import CANVAS_RANK_LADDER, canvas_layout

    if not (type(channels) is int and channels > 0):
        raise ConfigurationError(f"channels={channels!r}: expected an int >= 1")
    limit = channels if max_rank is None else max_rank
    if not (type(limit) is int and 1 <= limit <= channels):
        raise ConfigurationError(f"max_rank={max_rank!r}: expected an int in [1, {channels}]")
    _hevc.validate_parameters(pix_fmt)
    shapes: list[tuple[int, int, str]] = []
    for step in CANVAS_RANK_LADDER:
        try:
            layout = canvas_layout(frames, height, width, min(step, channels), pix_fmt)
        except Exception:  # noqa: BLE001 -- a mosaic larger than the HEVC maximum picture: no pack uses it
            break
        shape = (layout["image_width"], layout["image_height"], pix_fmt)
        if shape not in shapes:
            shapes.append(shape)
        if step >= limit:
            break
    return shapes


def device_tile_pixels(canvas: torch.Tensor, first: int, layout, rank: int | None = None) -> torch.Tensor:
    """One tile's ``[tokens, rank]`` uint8 coefficients gathered on the device from its decoded canvas pictures
    (``canvas[first:first + segments * frames]`` of ``[pictures, planes, image_h, image_w]``; ``layout`` the
    tile's ``reelcache.channel_tiles.v1`` layout). The inverse of the mosaic kernel, for diagnostics and for
    decoders that leave pictures on the device."""
    frames, height, width = layout["frames"], layout["height"], layout["width"]
    planes, (columns, _) = layout["planes"], layout["grid"]
    slots, segments = layout["channels_per_segment"], layout["segments"]
    rank = layout.get("tile_rank", layout["rank"]) if rank is None else rank
    if canvas.dim() != 4 or canvas.dtype != torch.uint8:
        raise ConfigurationError(f"canvas must be uint8 [pictures, planes, H, W], got {canvas.dtype} "
                                 f"{tuple(canvas.shape)}")
    if canvas.shape[0] < first + segments * frames or canvas.shape[1] < planes or \
            canvas.shape[2] < layout["image_height"] or canvas.shape[3] < layout["image_width"]:
        raise IntegrityError(f"canvas {tuple(canvas.shape)} is smaller than the tile's layout")
    out = torch.empty((frames, height, width, rank), dtype=torch.uint8, device=canvas.device)
    for channel in range(rank):
        segment, cell = divmod(channel, slots)
        plane = cell % planes
        row, column = divmod(cell // planes, columns)
        pictures = canvas[first + segment * frames:first + (segment + 1) * frames, plane]
        out[..., channel] = pictures[:, row * height:(row + 1) * height, column * width:(column + 1) * width]
    return out.reshape(frames * height * width, rank)


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


__all__ = ["PackedRestorer", "PreparedPacket", "PreparedTile", "RestoreBatch", "canonical_canvas_shapes",
           "device_tile_pixels", "prepare_packet", "prepared_tiles"]
