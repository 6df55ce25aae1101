"""Restore jobs: where a restored matrix comes from (sources), where it goes (native views) and how its
keys are rotated (RoPE positions). The public names and their meaning follow the reference's restore-kernel
API (reelcache/restore_kernels.py: ``NativeView``, ``PictureSource``, ``CoefficientSource``,
``ReconstructionJob``, ``RopePositions``); the classes here are this package's own.

A job reconstructs one canonical ``[N, C]`` matrix -- ``N = frames * height * width`` tokens in (frame, row,
column) order, ``C = heads * head_dim`` -- as ``coefficients[:, :rank] @ basis[:rank]`` (or copies a dense
matrix), optionally rotates K by RoPE at its original positions, and writes the result into a slot of a native
cache tensor.
"""

from __future__ import annotations

import math
from collections.abc import Mapping
from dataclasses import dataclass
from typing import Any

import numpy as np
import torch

from .errors import ConfigurationError

OUTPUT_DTYPES = (torch.bfloat16, torch.float16, torch.float32)
COEFFICIENT_DTYPES = (torch.float32, torch.float16, torch.bfloat16)


def _bad(message: str):
    raise ConfigurationError(message)


def _count(value, what: str, *, at_least: int = 0) -> int:
    if type(value) is not int or value < at_least:
        _bad(f"{what}: expected an integer >= {at_least}, got {value!r}")
    return value


def _tensor(value, what: str) -> torch.Tensor:
    if not isinstance(value, torch.Tensor) or value.layout != torch.strided or value.device.type == "meta":
        _bad(f"{what}: expected a materialized strided tensor")
    return value


def host_affine(value, columns: int, what: str) -> np.ndarray:
    """A finite host float32 vector of one entry per coefficient column (a packet's affine payload)."""
    if isinstance(value, torch.Tensor):
        if value.device.type != "cpu":
            _bad(f"{what} stays on the host (it comes from the packet's affine payload)")
        value = value.detach().numpy()
    array = np.asarray(value)
    if array.dtype != np.float32 or array.shape != (columns,):
        _bad(f"{what}: expected float32 [{columns}], got {array.dtype} {array.shape}")
    if not np.isfinite(array).all():
        _bad(f"{what} holds a non-finite value")
    return np.ascontiguousarray(array)


def expand_affine(affine, normalization, rank):
    """Per-column ``(scale, offset)`` of a packet's ``[2, records]`` affine. ``per_channel`` has one record
    per column; the shared layouts (``global`` / ``leading_columns``) have a shared record 0 followed by one
    record for each of the ``protected_count`` leading columns."""
    table = np.asarray(affine)
    if table.dtype != np.dtype("<f4") or table.ndim != 2 or table.shape[0] != 2:
        _bad("affine: expected a little-endian float32 [2, records] array")
    if not isinstance(normalization, Mapping) or "mode" not in normalization:
        _bad("normalization: expected the packet's normalization layout")
    _count(rank, "rank", at_least=1)
    if normalization["mode"] == "per_channel":
        if table.shape[1] != rank:
            _bad(f"a per-channel affine has {rank} records, not {table.shape[1]}")
        return table[0].copy(), table[1].copy()
    leading = normalization.get("protected_count")
    if type(leading) is not int or leading < 0 or leading > rank or table.shape[1] != leading + 1:
        _bad(f"a shared affine with {leading!r} protected columns has {table.shape[1]} records")
    scale = np.full(rank, table[0, 0], dtype=np.float32)
    offset = np.full(rank, table[1, 0], dtype=np.float32)
    scale[:leading] = table[0, 1:]
    offset[:leading] = table[1, 1:]
    return scale, offset


def wan_sections(pairs):
    """The (frame, row, column) split of ``head_dim // 2`` rotation pairs used by Wan and LongCat."""
    _count(pairs, "pairs", at_least=1)
    third = pairs // 3
    return (pairs - 2 * third, third, third)


# -------------------------------------------------------------------------------------------------------------
# Native destinations
# -------------------------------------------------------------------------------------------------------------

@dataclass(frozen=True)
class _Axes:
    rank: int              # tensor dimensions
    batch: int | None      # batch axis (None: packed)
    token: int
    head: int
    dim: int


_LAYOUT_AXES = {"BTHD": _Axes(4, 0, 1, 2, 3), "THD": _Axes(3, None, 0, 1, 2), "BHTD": _Axes(4, 0, 2, 1, 3)}
LAYOUTS = tuple(_LAYOUT_AXES)


@dataclass(frozen=True, eq=False)
class NativeView:
    """A native KV cache tensor, its layout (``BTHD``, ``THD`` or ``BHTD``, any strides) and the slot's
    first token (and batch row)."""

    tensor: torch.Tensor
    layout: str = "BTHD"
    token_offset: int = 0
    batch_index: int = 0

    def __post_init__(self):
        tensor = _tensor(self.tensor, "destination")
        axes = _LAYOUT_AXES.get(self.layout)
        if axes is None:
            _bad(f"layout {self.layout!r} is not one of {LAYOUTS}")
        if tensor.dim() != axes.rank:
            _bad(f"a {self.layout} destination has {axes.rank} dimensions, not {tensor.dim()}")
        if tensor.dtype not in OUTPUT_DTYPES:
            _bad(f"destination dtype {tensor.dtype} is not bfloat16, float16 or float32")
        _count(self.token_offset, "token_offset")
        _count(self.batch_index, "batch_index")
        if axes.batch is None and self.batch_index:
            _bad("a packed THD destination has no batch rows")
        if axes.batch is not None and self.batch_index >= tensor.shape[axes.batch]:
            _bad(f"batch row {self.batch_index} is outside the destination")
        if tensor.shape[axes.dim] % 2:
            _bad("RoPE pairs need an even head_dim")
        if any(size > 1 and stride == 0 for size, stride in zip(tensor.shape, tensor.stride())):
            _bad("the destination broadcasts (a zero stride): its slots would alias")

    @property
    def _axes(self) -> _Axes:
        return _LAYOUT_AXES[self.layout]

    @property
    def heads(self):
        return self.tensor.shape[self._axes.head]

    @property
    def head_dim(self):
        return self.tensor.shape[self._axes.dim]

    @property
    def channels(self):
        return self.heads * self.head_dim

    @property
    def capacity(self):
        return self.tensor.shape[self._axes.token]

    def strides(self):
        """Element strides of (token, head, dim)."""
        s, a = self.tensor.stride(), self._axes
        return s[a.token], s[a.head], s[a.dim]

    def element_offset(self):
        """Elements from the data pointer to (batch_index, token_offset, head 0, dim 0)."""
        a = self._axes
        batch = 0 if a.batch is None else self.batch_index * self.tensor.stride(a.batch)
        return batch + self.token_offset * self.tensor.stride(a.token)

    def address(self):
        return self.tensor.data_ptr() + self.element_offset() * self.tensor.element_size()

    def slot(self, tokens):
        """The slot as a ``[tokens, heads, head_dim]`` view."""
        a = self._axes
        view = self.tensor if a.batch is None else self.tensor.select(a.batch, self.batch_index)
        view = view.narrow(a.token - (0 if a.batch is None else 1), self.token_offset, tokens)
        return view if self.layout != "BHTD" else view.transpose(0, 1)


# -------------------------------------------------------------------------------------------------------------
# RoPE positions
# -------------------------------------------------------------------------------------------------------------

@dataclass(frozen=True, eq=False)
class RopePositions:
    """Where a chunk's tokens sit in a rotation table: ``(t_row, h_row, w_row)`` of its first frame / row /
    column for separable tables (an int is the frame row), one first row for dense tables."""

    table: Any
    rows: Any = 0

    def __post_init__(self):
        from .restore_kernels import RopeTable
        if not isinstance(self.table, RopeTable):
            _bad("RoPE positions point into a RopeTable")
        if self.table.sections is None:
            _count(self.rows, "dense RoPE row")
            return
        rows = (self.rows, 0, 0) if type(self.rows) is int else tuple(self.rows)
        if len(rows) != 3:
            _bad(f"separable RoPE positions are (t_row, h_row, w_row), not {self.rows!r}")
        for value in rows:
            _count(value, "RoPE row")
        object.__setattr__(self, "rows", rows)


# -------------------------------------------------------------------------------------------------------------
# Sources
# -------------------------------------------------------------------------------------------------------------

@dataclass(frozen=True, eq=False)
class CoefficientSource:
    """Coefficients ``[N, >= rank]`` already taken out of their pictures: 8-bit values with their per-column
    affine, or float values. ``bound`` optionally bounds ``|coefficients|`` (saves a reduction)."""

    values: torch.Tensor
    scale: Any = None
    offset: Any = None
    bound: float | None = None

    def __post_init__(self):
        values = _tensor(self.values, "coefficients")
        if values.dim() != 2:
            _bad(f"coefficients are a [tokens, rank] matrix, not {tuple(values.shape)}")
        b = self.bound
        if b is not None and (isinstance(b, bool) or not isinstance(b, (int, float)) or not math.isfinite(b) or b < 0):
            _bad(f"bound {b!r} is not a finite nonnegative number")
        has_affine = self.scale is not None or self.offset is not None
        if values.dtype == torch.uint8:
            if self.scale is None or self.offset is None:
                _bad("8-bit coefficients come with their scale and offset")
            columns = values.shape[1]
            object.__setattr__(self, "scale", host_affine(self.scale, columns, "scale"))
            object.__setattr__(self, "offset", host_affine(self.offset, columns, "offset"))
            if (self.scale < 0).any():
                _bad("affine scales are nonnegative")
        elif values.dtype in COEFFICIENT_DTYPES:
            if has_affine:
                _bad("float coefficients are already dequantized: no affine")
        else:
            _bad(f"coefficients are uint8 or float32/float16/bfloat16, not {values.dtype}")

    @property
    def quantized(self):
        return self.values.dtype == torch.uint8


@dataclass(frozen=True)
class _Mosaic:
    """The geometry of a ``reelcache.channel_tiles.v1`` layout."""

    frames: int
    height: int
    width: int
    rank: int
    planes: int
    columns: int
    rows: int
    slots: int
    segments: int

    @classmethod
    def of(cls, layout) -> "_Mosaic":
        names = ("frames", "height", "width", "rank", "planes", "grid", "channels_per_segment", "segments")
        if not isinstance(layout, Mapping) or not all(name in layout for name in names):
            _bad("pictures come with a reelcache.channel_tiles.v1 layout")
        columns, rows = layout["grid"]
        mosaic = cls(layout["frames"], layout["height"], layout["width"], layout["rank"], layout["planes"], columns,
                     rows, layout["channels_per_segment"], layout["segments"])
        for name, value in mosaic.__dict__.items():
            _count(value, f"layout {name}", at_least=1)
        if mosaic.slots != columns * rows * mosaic.planes:
            _bad("a segment holds grid columns x grid rows x planes channels")
        if mosaic.segments != -(-mosaic.rank // mosaic.slots):
            _bad("the segment count does not cover the rank")
        return mosaic


@dataclass(frozen=True, eq=False)
class PictureSource:
    """8-bit coefficients read in place from decoded pictures ``pictures[segment][frame]``: uint8 views
    ``[planes, rows, columns]`` whose origin is this matrix's rectangle, all with the same strides."""

    pictures: Any
    layout: Mapping
    scale: Any
    offset: Any

    def __post_init__(self):
        mosaic = _Mosaic.of(self.layout)
        grid = tuple(tuple(segment) for segment in self.pictures)
        if len(grid) != mosaic.segments or any(len(segment) != mosaic.frames for segment in grid):
            _bad(f"pictures are indexed [segment][frame]: {mosaic.segments} x {mosaic.frames} views")
        reach = (mosaic.planes, mosaic.rows * mosaic.height, mosaic.columns * mosaic.width)
        first = grid[0][0]
        for view in (v for segment in grid for v in segment):
            _tensor(view, "picture")
            if view.dtype != torch.uint8 or view.dim() != 3:
                _bad("pictures are uint8 [planes, rows, columns] views")
            if any(have < need for have, need in zip(view.shape, reach)):
                _bad(f"a picture view {tuple(view.shape)} does not cover the {reach} rectangle")
            if view.stride(2) != 1:
                _bad("picture rows must be contiguous")
            if view.stride()[:2] != first.stride()[:2] or view.device != first.device:
                _bad("the pictures of one matrix share their plane and row strides and their device")
        object.__setattr__(self, "pictures", grid)
        object.__setattr__(self, "scale", host_affine(self.scale, mosaic.rank, "scale"))
        object.__setattr__(self, "offset", host_affine(self.offset, mosaic.rank, "offset"))
        if (self.scale < 0).any():
            _bad("affine scales are nonnegative")

    @property
    def device(self):
        return self.pictures[0][0].device

    @property
    def rank(self):
        return self.layout["rank"]

    @property
    def plane_stride(self):
        return self.pictures[0][0].stride(0)

    @property
    def row_stride(self):
        return self.pictures[0][0].stride(1)

    @classmethod
    def from_canvases(cls, canvases, layout, picture_indices, origins, scale, offset):
        """Views on decoded canvases ``[pictures, planes, height, width]``. ``origins`` is one ``(y, x)`` for
        every picture, or a ``[segment][frame]`` table of them (tile maps of node-pack schema v2)."""
        canvases = _tensor(canvases, "canvases")
        if canvases.dim() != 4 or canvases.dtype != torch.uint8:
            _bad("canvases are uint8 [pictures, planes, height, width]")
        shared = len(origins) == 2 and all(type(v) is int for v in origins)
        views = []
        for s, segment in enumerate(picture_indices):
            row = []
            for f, index in enumerate(segment):
                y, x = origins if shared else origins[s][f]
                for value, what in ((index, "picture index"), (y, "rectangle y"), (x, "rectangle x")):
                    _count(value, what)
                if index >= canvases.shape[0]:
                    _bad(f"picture {index} is outside the {canvases.shape[0]} canvases")
                row.append(canvases[index, :, y:, x:])
            views.append(tuple(row))
        return cls(tuple(views), layout, scale, offset)


@dataclass(frozen=True, eq=False)
class DenseSource:
    """A whole canonical ``[N, C]`` matrix (RAW archive, raw tier)."""

    values: torch.Tensor

    def __post_init__(self):
        values = _tensor(self.values, "dense values")
        if values.dim() != 2 or values.dtype not in COEFFICIENT_DTYPES:
            _bad("dense values are a float32/float16/bfloat16 [tokens, channels] matrix")


# -------------------------------------------------------------------------------------------------------------
# Jobs
# -------------------------------------------------------------------------------------------------------------

@dataclass(frozen=True, eq=False)
class ReconstructionJob:
    """One restored matrix into one native slot. ``basis_t`` may supply the fused kernel's operand form of the
    same basis (transposed, zero-padded FP16 ``[C, ceil(R / 64) * 64]``), which saves a transpose per call."""

    source: Any
    destination: NativeView
    grid: tuple
    basis: torch.Tensor | None = None
    rank: int | None = None
    rope: RopePositions | None = None
    label: str | None = None
    basis_t: torch.Tensor | None = None

    def __post_init__(self):
        if not isinstance(self.source, (CoefficientSource, PictureSource, DenseSource)):
            _bad("a job reads a CoefficientSource, a PictureSource or a DenseSource")
        if not isinstance(self.destination, NativeView):
            _bad("a job writes into a NativeView")
        grid = tuple(self.grid)
        if len(grid) != 3:
            _bad(f"grid is (frames, height, width), not {self.grid!r}")
        for value in grid:
            _count(value, "grid size", at_least=1)
        object.__setattr__(self, "grid", grid)
        if self.destination.token_offset + self.tokens > self.destination.capacity:
            _bad(f"tokens {self.destination.token_offset}..{self.destination.token_offset + self.tokens} exceed the "
                 f"cache capacity {self.destination.capacity}")
        if isinstance(self.source, DenseSource):
            self._check_dense()
        else:
            self._check_factors()
        if self.rope is not None:
            self._check_rope()

    def _check_dense(self):
        if self.basis is not None or self.rank is not None:
            _bad("a dense source has no basis and no rank")
        if tuple(self.source.values.shape) != (self.tokens, self.channels):
            _bad(f"dense values are [{self.tokens}, {self.channels}], not {tuple(self.source.values.shape)}")

    def _check_factors(self):
        basis = _tensor(self.basis, "basis")
        if basis.dim() != 2 or basis.shape[1] != self.channels:
            _bad(f"the basis is [rows, {self.channels}], not {tuple(basis.shape)}")
        if basis.dtype not in (torch.float16, torch.float32):
            _bad("the basis is the stored float16 rows (float32 for reference use)")
        if isinstance(self.source, PictureSource):
            layout = self.source.layout
            if (layout["frames"], layout["height"], layout["width"]) != self.grid:
                _bad("the picture layout and the job grid disagree")
            columns = layout["rank"]
            exact = True
        else:
            if self.source.values.shape[0] != self.tokens:
                _bad(f"{self.source.values.shape[0]} coefficient rows for {self.tokens} tokens")
            columns = self.source.values.shape[1]
            exact = False
        rank = columns if self.rank is None else _count(self.rank, "rank", at_least=1)
        if rank > basis.shape[0]:
            _bad(f"rank {rank} exceeds the {basis.shape[0]} basis rows")
        if rank > columns or (exact and rank != columns):
            _bad(f"rank {rank} does not match the {columns} coefficient columns")
        object.__setattr__(self, "rank", rank)
        bt = self.basis_t
        if bt is not None and (bt.dtype != torch.float16 or bt.dim() != 2 or bt.shape[0] != self.channels
                               or bt.shape[1] % 64 or bt.shape[1] < rank or bt.stride(1) != 1):
            _bad("basis_t is float16 [channels, rank rounded up to 64] with unit column stride")

    def _check_rope(self):
        if not isinstance(self.rope, RopePositions):
            _bad("rope is given as RopePositions")
        table = self.rope.table
        if table.head_dim != self.destination.head_dim:
            _bad(f"the RoPE table rotates head_dim {table.head_dim}, the destination has {self.destination.head_dim}")
        if table.sections is None:
            if self.rope.rows + self.tokens > table.rows:
                _bad("the dense RoPE rows run past the table")
            return
        for first, count, limit, pairs in zip(self.rope.rows, self.grid, table.section_rows, table.sections):
            if pairs and first + count > limit:
                _bad("a separable RoPE section runs past its rows")

    @property
    def tokens(self):
        f, h, w = self.grid
        return f * h * w

    @property
    def channels(self):
        return self.destination.channels

    def tensors(self):
        """Every tensor the job reads or writes (kept alive until its work completes)."""
        out = [self.destination.tensor]
        if isinstance(self.source, PictureSource):
            out += [view for segment in self.source.pictures for view in segment]
        else:
            out.append(self.source.values)
        out += [t for t in (self.basis, self.basis_t) if t is not None]
        if self.rope is not None:
            out += [self.rope.table.cos, self.rope.table.sin]
        return out


__all__ = ["COEFFICIENT_DTYPES", "LAYOUTS", "OUTPUT_DTYPES", "CoefficientSource", "DenseSource", "NativeView",
           "PictureSource", "ReconstructionJob", "RopePositions", "expand_affine", "host_affine", "wan_sections"]
