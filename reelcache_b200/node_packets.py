"""Node packets: canonical canvases and device finalization of coefficient tiles (the counterpart of reference
reelcache/node_packets.py:1-31; ladder :57-115, ``quantize_device`` :156, ``mosaic_device`` :176, ``NodeCanvas``
:222, ``finalize_tile`` :290, ``finalize_tiles`` :382, ``assemble_canvas`` :451, ``detach/attach_pack_bases``
:771-791).

* **Canvas ladder.** A tile of rank ``r`` is laid out on the canvas of the smallest ladder rank ``>= r``
  (:data:`CANVAS_RANK_LADDER`, 32 ... 8192), so canvases of one geometry come in a few canonical sizes and a
  video decoder session per size is reused; the unused slots are zero.
* **Device finalization.** :func:`finalize_tile` re-measures the FP32 coefficients on the device (per-column
  extrema, the covering FP32 affine on the host from those few bytes, FP64 ``rint`` quantization bitwise equal
  to the host path: ``csrc/fit/quantize.cu``), mosaics the uint8 pixels into the channel-tile canvas on the
  device (``csrc/fit/mosaic.cu``) and copies only the uint8 canvas and the affine to the host
  (:meth:`NodeCanvas.to_host`, pinned).
* **Pack bases.** :func:`detach_pack_bases` splits the inline basis descriptors out of a pack's metadata (the
  pack then references external basis versions); :func:`attach_pack_bases` restores them.
"""

from __future__ import annotations

from dataclasses import dataclass
from typing import Any, Mapping, Sequence

import numpy as np
import torch

from . import _hevc
from .errors import ConfigurationError

CANVAS_RANK_LADDER = (32, 48, 64, 96, 128, 192, 256, 384, 512, 768, 1024, 1536, 2048, 3072, 4096, 6144, 8192)


def canvas_rank(rank: int) -> int:
    """The ladder rank whose canvas holds a tile of ``rank`` columns."""
    for ladder in CANVAS_RANK_LADDER:
        if ladder >= rank:
            return ladder
    raise ConfigurationError(f"rank {rank} exceeds the canvas ladder ({CANVAS_RANK_LADDER[-1]})")


def canvas_layout(frames: int, height: int, width: int, rank: int, pix_fmt: str = "yuv444p") -> dict:
    """The channel-tile layout of the tile's ladder canvas, with the tile's own rank recorded."""
    layout = _hevc.video_layout(frames, height, width, canvas_rank(rank), pix_fmt)
    layout = dict(layout)
    layout["tile_rank"] = int(rank)
    return layout


def _geometry(layout: Mapping[str, Any], rank: int) -> list[int]:
    columns, rows = layout["grid"]
    return [layout["frames"], layout["height"], layout["width"], int(rank), layout["planes"], columns, rows,
            layout["image_height"], layout["image_width"], layout["channels_per_segment"], layout["segments"]]


def mosaic_device(pixels: torch.Tensor, layout: Mapping[str, Any], rank: int | None = None) -> torch.Tensor:
    """u8 ``[N, >= rank]`` (CUDA) -> canvas ``[segments * frames, planes, image_h, image_w]`` (CUDA); channels
    beyond ``rank`` (the ladder's spare slots) are zero."""
    from .ops._ext import ext
    rank = pixels.shape[1] if rank is None else rank
    canvas = torch.empty((layout["segments"] * layout["frames"], layout["planes"], layout["image_height"],
                          layout["image_width"]), dtype=torch.uint8, device=pixels.device)
    ext().mosaic_u8(pixels, canvas, _geometry(layout, rank))
    return canvas


def mosaic_host(pixels: np.ndarray, layout: Mapping[str, Any], rank: int | None = None) -> np.ndarray:
    """The host reference of :func:`mosaic_device` (zero-filled spare ladder slots)."""
    rank = pixels.shape[1] if rank is None else rank
    padded = np.zeros((pixels.shape[0], layout["rank"]), dtype=np.uint8)
    padded[:, :rank] = pixels[:, :rank]
    return _hevc.mosaic_all(padded, layout)


@dataclass
class NodeCanvas:
    """One finalized tile: its canvas (device or host), affine records and layouts."""

    canvas: Any
    affine: np.ndarray
    normalization: Mapping[str, Any]
    layout: Mapping[str, Any]
    rank: int

    @property
    def nbytes(self) -> int:
        return int(self.canvas.numel() if isinstance(self.canvas, torch.Tensor) else self.canvas.size)

    def to_host(self, *, pin: bool = True) -> "NodeCanvas":
        if not isinstance(self.canvas, torch.Tensor) or not self.canvas.is_cuda:
            return self
        host = torch.empty(self.canvas.shape, dtype=torch.uint8, pin_memory=pin and torch.cuda.is_available())
        host.copy_(self.canvas, non_blocking=pin)
        if pin:
            torch.cuda.current_stream(self.canvas.device).synchronize()
        return NodeCanvas(host.numpy(), self.affine, self.normalization, self.layout, self.rank)

    def pixels(self) -> np.ndarray:
        """The tile's u8 coefficients ``[N, rank]`` back from the canvas (host)."""
        canvas = self.canvas.cpu().numpy() if isinstance(self.canvas, torch.Tensor) else self.canvas
        return _hevc.unmosaic_all(canvas, self.layout)[:, :self.rank]


def finalize_tile(coefficients: torch.Tensor, grid: tuple[int, int, int], *, normalization: str = "per_channel",
                  protected_fraction: float = 1.0, pix_fmt: str = "yuv444p") -> NodeCanvas:
    """Quantize and mosaic one tile's FP32 coefficients ``[N, rank]`` (device path on CUDA, host otherwise)."""
    frames, height, width = grid
    if coefficients.ndim != 2 or coefficients.shape[0] != frames * height * width:
        raise ConfigurationError("coefficients must be [frames * height * width, rank]")
    rank = int(coefficients.shape[1])
    layout = canvas_layout(frames, height, width, rank, pix_fmt)
    if coefficients.is_cuda:
        from .ops.quant import quantize_device
        pixels, affine, norm = quantize_device(coefficients, normalization, protected_fraction, as_numpy=False)
        return NodeCanvas(mosaic_device(pixels, layout, rank), affine, norm, layout, rank)
    pixels, affine, norm = _hevc.quantize_coefficients(coefficients.detach().float().numpy(), normalization,
                                                       protected_fraction)
    return NodeCanvas(mosaic_host(pixels, layout, rank), affine, norm, layout, rank)


def finalize_tiles(tiles: Sequence[tuple[torch.Tensor, tuple[int, int, int]]], **options) -> list[NodeCanvas]:
    return [finalize_tile(coefficients, grid, **options) for coefficients, grid in tiles]


def assemble_canvas(canvases: Sequence[NodeCanvas]) -> tuple[np.ndarray, list[dict]]:
    """One node's pictures (tiles of one canvas geometry concatenated picture-major) and the per-tile picture
    ranges."""
    if not canvases:
        raise ConfigurationError("a node canvas needs tiles")
    shapes = {tuple(c.canvas.shape[1:]) for c in canvases}
    if len(shapes) != 1:
        raise ConfigurationError("one node canvas holds tiles of one canvas geometry")
    host = [c.to_host(pin=False).canvas for c in canvases]
    ranges, start = [], 0
    for c, pictures in zip(canvases, host):
        ranges.append({"first_picture": start, "pictures": int(pictures.shape[0]), "rank": c.rank,
                       "ladder_rank": c.layout["rank"]})
        start += pictures.shape[0]
    return np.concatenate(host, axis=0), ranges


def detach_pack_bases(metadata: Mapping[str, Any]) -> tuple[dict, list]:
    """(metadata without inline basis descriptors, the descriptors in tile order)."""
    out = dict(metadata)
    tiles, bases = [], []
    for tile in metadata.get("tiles", []):
        tile = dict(tile)
        bases.append(tile.pop("basis", None))
        tiles.append(tile)
    out["tiles"] = tiles
    out["bases"] = "external"
    return out, bases


def attach_pack_bases(metadata: Mapping[str, Any], bases: Sequence[Any]) -> dict:
    tiles = list(metadata.get("tiles", []))
    if len(tiles) != len(bases):
        raise ConfigurationError("one basis descriptor per tile")
    out = dict(metadata)
    out["tiles"] = [{**tile, "basis": basis} for tile, basis in zip(tiles, bases)]
    out.pop("bases", None)
    return out


__all__ = ["CANVAS_RANK_LADDER", "NodeCanvas", "assemble_canvas", "attach_pack_bases", "canvas_layout", "canvas_rank",
           "detach_pack_bases", "finalize_tile", "finalize_tiles", "mosaic_device", "mosaic_host"]
