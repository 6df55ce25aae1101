"""Batched, fused reconstruction of restored KV matrices into native caches.

Same contract as the reference's restore-kernel API (reelcache/restore_kernels.py:1-89, public
names at :2336-2447): one call reconstructs any number of restored matrices -- one layer's K or V
of one chunk each -- straight into native cache slots::

    pre-RoPE K or V  =  dequantize(unpack(pixels)) @ Q[:rank]
    native slot      <- cast(RoPE(K at its original positions))    (K)
    native slot      <- cast(V)                                    (V)

* A canonical matrix is ``[N, C]``: ``N = frames * height * width`` tokens in (frame, row,
  column) order and ``C = heads * head_dim`` channels.
* The basis is the immutable FP16 row matrix ``Q[R, C]``; a job uses the prefix view ``Q[:rank]``.
* Coefficients ``P[N, rank]``; 8-bit pixels carry them with an FP32 affine per rank column and are
  dequantized as ``float(pixel) * scale + offset`` with two roundings (no FMA).
* Pictures use the ``reelcache.channel_tiles.v1`` mosaic: rank column ``k`` lives in segment
  ``k // channels_per_segment``; inside a segment, cell ``i`` uses plane ``i % planes`` and grid cell
  ``divmod(i // planes, grid_columns)``; each frame is one picture per segment.
* RoPE rotates interleaved pairs ``(2j, 2j + 1)`` from FP32 cos/sin tables with separable
  (t, h, w) sections (Wan / LongCat) or a dense per-token table.
* Native layouts ``BTHD``, ``THD`` and ``BHTD`` with any strides.

Backends:

* ``fused`` (CUDA; the ``auto`` choice on CUDA): one persistent sm_100a kernel per launch group
  (csrc/restore/restore_sm100.cu) -- a gather producer unpacks and dequantizes the pixels into
  swizzled shared memory, TMA streams the transposed FP16 basis, ``tcgen05.mma`` accumulates in TMEM
  and the epilogue applies RoPE, casts and stores. Dense sources use csrc/restore/rope_store.cu.
* ``reference`` (plain torch, FP64 or FP32 math; CPU or GPU; the ``auto`` choice on CPU).

Precisions of the fused kernel: ``fp16x2`` (default; coefficients prescaled by an exact power of two
and split into FP16 hi + lo, two tensor-core products, FP32 accumulation) and ``fp16`` (hi only).
:func:`error_bound` gives the elementwise bound each mode satisfies (same first-order analysis as the
reference, :1176-1230). There is no silent fallback: CUDA jobs raise
:class:`~reelcache_b200.errors.UnsupportedError` when the native extension is missing.
"""

from __future__ import annotations

import math
import threading
from collections import OrderedDict
from collections.abc import Mapping, Sequence
from dataclasses import dataclass, field
from typing import Any

import numpy as np
import torch

from .errors import ConfigurationError, IntegrityError, UnsupportedError

LAYOUTS = ("BTHD", "THD", "BHTD")
PRECISIONS = ("fp32", "tf32", "tf32x3", "fp16", "fp16x2", "bf16")
KERNEL_PRECISIONS = ("fp16", "fp16x2")
BACKENDS = ("auto", "reference", "fused")
OUTPUT_DTYPES = (torch.bfloat16, torch.float16, torch.float32)
COEFFICIENT_DTYPES = (torch.float32, torch.float16, torch.bfloat16)
DEFAULT_PRECISION = "fp16x2"
MAX_JOBS_PER_LAUNCH = 16
MAX_DENSE_JOBS_PER_LAUNCH = 48
_OUT_CODE = {torch.bfloat16: 0, torch.float16: 1, torch.float32: 2}


def _int(value, name, *, minimum=0):
    if type(value) is not int or value < minimum:
        raise ConfigurationError(f"{name} must be an integer >= {minimum}")
    return value


def _require_tensor(value, name):
    if not isinstance(value, torch.Tensor) or value.layout != torch.strided:
        raise ConfigurationError(f"{name} must be a strided torch.Tensor")
    if value.device.type == "meta":
        raise ConfigurationError(f"{name} cannot be a meta tensor")
    return value


def _host_vector(value, length, name):
    if isinstance(value, torch.Tensor):
        if value.device.type != "cpu":
            raise ConfigurationError(f"{name} must be a host array (the packet's affine payload)")
        value = value.detach().numpy()
    array = np.asarray(value)
    if array.dtype != np.float32 or array.shape != (length,):
        raise ConfigurationError(f"{name} must be a float32 vector with one entry per rank column")
    if not np.isfinite(array).all():
        raise ConfigurationError(f"{name} must be finite")
    return np.ascontiguousarray(array)


def expand_affine(affine, normalization, rank):
    """Per-column ``(scale, offset)`` from a packet's ``[2, records]`` affine payload.

    ``per_channel``: one record per rank column. ``global`` / ``leading_columns``: record 0 is the
    shared affine and records 1.. cover the ``protected_count`` leading columns.
    """
    affine = np.asarray(affine)
    if affine.dtype != np.dtype("<f4") or affine.ndim != 2 or affine.shape[0] != 2:
        raise ConfigurationError("affine must be a little-endian float32 [2, records] array")
    if not isinstance(normalization, Mapping) or "mode" not in normalization:
        raise ConfigurationError("normalization must be the packet normalization layout")
    _int(rank, "rank", minimum=1)
    if normalization["mode"] == "per_channel":
        if affine.shape[1] != rank:
            raise ConfigurationError("per-channel affine must have one record per rank column")
        return affine[0].copy(), affine[1].copy()
    scale = np.full(rank, affine[0, 0], dtype=np.float32)
    offset = np.full(rank, affine[1, 0], dtype=np.float32)
    count = normalization.get("protected_count")
    if type(count) is not int or not 0 <= count <= rank or affine.shape[1] != count + 1:
        raise ConfigurationError("affine record count differs from the protected columns")
    if count:
        scale[:count], offset[:count] = affine[0, 1:], affine[1, 1:]
    return scale, offset


# (cos, sin) entries of one job's separable tables that the fused epilogue stages in shared memory
PACKED_ROPE_ENTRIES = 3072


def restore_rope_item(positions, grid, device, stream, keepalive):
    """RoPE description of one fused-restore job: ``("packed", address, pairs, sec_t, sec_h,
    entries)`` for separable tables that fit in shared memory, else ``("tokens", cos address, sin
    address, pairs)`` with per-token FP32 rows."""
    table = positions.table
    packed = table.packed_tables(positions.rows, grid, device, stream)
    if packed is not None:
        pack, (sec_t, sec_h, entries) = packed
        keepalive.append(pack)
        return ("packed", pack.data_ptr(), table.pairs, sec_t, sec_h, entries)
    cos, sin = table.token_tables(positions.rows, grid, device, stream)
    keepalive.extend((cos, sin))
    return ("tokens", cos.data_ptr(), sin.data_ptr(), table.pairs)


def wan_sections(pairs):
    """Wan / LongCat 3-D split of ``pairs = head_dim // 2`` into (t, h, w) pair counts."""
    _int(pairs, "pairs", minimum=1)
    return (pairs - 2 * (pairs // 3), pairs // 3, pairs // 3)


# ---------------------------------------------------------------------------------------------
# Destinations, RoPE tables and sources
# ---------------------------------------------------------------------------------------------


@dataclass(frozen=True, eq=False)
class NativeView:
    """A native cache tensor, its layout and the first destination token."""

    tensor: torch.Tensor
    layout: str = "BTHD"
    token_offset: int = 0
    batch_index: int = 0

    def __post_init__(self):
        tensor = _require_tensor(self.tensor, "destination tensor")
        if self.layout not in LAYOUTS:
            raise ConfigurationError(f"destination layout must be one of {LAYOUTS}")
        if tensor.ndim != (3 if self.layout == "THD" else 4):
            raise ConfigurationError(f"{self.layout} destination has the wrong number of dimensions")
        if tensor.dtype not in OUTPUT_DTYPES:
            raise ConfigurationError("destination dtype must be bfloat16, float16 or float32")
        _int(self.token_offset, "token_offset")
        _int(self.batch_index, "batch_index")
        if self.layout == "THD" and self.batch_index:
            raise ConfigurationError("a packed THD destination has no batch dimension")
        if self.layout != "THD" and self.batch_index >= tensor.shape[0]:
            raise ConfigurationError("batch_index is outside the destination")
        if self.head_dim % 2:
            raise ConfigurationError("head_dim must be even")
        if any(size > 1 and stride == 0 for size, stride in zip(tensor.shape, tensor.stride())):
            raise ConfigurationError("destination views with broadcast (zero) strides alias")

    @property
    def heads(self):
        return self.tensor.shape[1] if self.layout == "BHTD" else self.tensor.shape[-2]

    @property
    def head_dim(self):
        return self.tensor.shape[-1]

    @property
    def channels(self):
        return self.heads * self.head_dim

    @property
    def capacity(self):
        return self.tensor.shape[2] if self.layout == "BHTD" else self.tensor.shape[-3]

    def strides(self):
        """Element strides of (token, head, dim)."""
        stride = self.tensor.stride()
        if self.layout == "BHTD":
            return stride[2], stride[1], stride[3]
        return stride[-3], stride[-2], stride[-1]

    def element_offset(self):
        """Element offset (from the tensor's data pointer) of (batch_index, token_offset, 0, 0)."""
        base = 0
        if self.layout != "THD":
            base += self.batch_index * self.tensor.stride(0)
        return base + self.token_offset * self.strides()[0]

    def address(self):
        return self.tensor.data_ptr() + self.element_offset() * self.tensor.element_size()

    def slot(self, tokens):
        """A ``[tokens, H, D]`` view of the destination slot."""
        stop = self.token_offset + tokens
        if self.layout == "THD":
            return self.tensor[self.token_offset:stop]
        if self.layout == "BTHD":
            return self.tensor[self.batch_index, self.token_offset:stop]
        return self.tensor[self.batch_index, :, self.token_offset:stop].transpose(0, 1)


@dataclass(frozen=True, eq=False)
class RopeTable:
    """cos/sin rotation tables ``[rows, head_dim // 2]`` for interleaved pairs.

    ``sections=(t, h, w)`` makes the table separable: pair ``j`` of the token at (frame f, row y,
    column x) uses row ``t_row + f`` when ``j < t``, ``h_row + y`` when ``j < t + h`` and
    ``w_row + x`` otherwise. ``sections=None`` is a dense per-token table. FP32 device copies are
    cached per device (:meth:`kernel_tables`) and refreshed when the tables change in place.
    """

    cos: torch.Tensor
    sin: torch.Tensor
    sections: tuple | None = None
    section_rows: tuple | None = None
    _device_cache: dict = field(default_factory=dict, init=False, repr=False, compare=False)

    def __post_init__(self):
        cos, sin = _require_tensor(self.cos, "RoPE cos"), _require_tensor(self.sin, "RoPE sin")
        if (cos.ndim != 2 or cos.shape != sin.shape or cos.dtype != sin.dtype
                or cos.dtype not in (torch.float32, torch.float64) or cos.device != sin.device
                or min(cos.shape) < 1):
            raise ConfigurationError("RoPE cos/sin must be matching float32/float64 [rows, head_dim // 2] tensors")
        rows, pairs = cos.shape
        if self.sections is not None:
            sections = tuple(self.sections)
            if len(sections) != 3 or any(type(v) is not int or v < 0 for v in sections) or sum(sections) != pairs:
                raise ConfigurationError("RoPE sections must be three nonnegative pair counts summing to head_dim // 2")
            object.__setattr__(self, "sections", sections)
            limits = (rows, rows, rows) if self.section_rows is None else tuple(self.section_rows)
            if len(limits) != 3 or any(type(v) is not int or not 0 <= v <= rows for v in limits):
                raise ConfigurationError("section_rows must be three row counts within the table")
            object.__setattr__(self, "section_rows", limits)
        elif self.section_rows is not None:
            raise ConfigurationError("section_rows requires separable sections")

    @property
    def rows(self):
        return self.cos.shape[0]

    @property
    def pairs(self):
        return self.cos.shape[1]

    @property
    def head_dim(self):
        return 2 * self.pairs

    @classmethod
    def from_complex(cls, freqs, sections="wan"):
        freqs = _require_tensor(freqs, "freqs")
        if not freqs.is_complex() or freqs.ndim != 2:
            raise ConfigurationError("freqs must be a complex [rows, head_dim // 2] tensor")
        real = torch.view_as_real(freqs.resolve_conj())
        dtype = torch.float64 if freqs.dtype == torch.complex128 else torch.float32
        if sections == "wan":
            sections = wan_sections(freqs.shape[1])
        return cls(real[..., 0].to(dtype).contiguous(), real[..., 1].to(dtype).contiguous(), sections)

    @classmethod
    def from_axes(cls, temporal, height, width):
        """Separable table from per-axis complex tensors ``[positions, pairs]`` (unused cells NaN)."""
        axes = [_require_tensor(v, "axis freqs") for v in (temporal, height, width)]
        if any(not v.is_complex() or v.ndim != 2 for v in axes):
            raise ConfigurationError("axis frequencies must be complex [positions, pairs] tensors")
        dtype = torch.float64 if all(v.dtype == torch.complex128 for v in axes) else torch.float32
        rows = max(v.shape[0] for v in axes)
        pairs = sum(v.shape[1] for v in axes)
        cos = torch.full((rows, pairs), float("nan"), dtype=dtype, device=axes[0].device)
        sin = torch.full_like(cos, float("nan"))
        column = 0
        for v in axes:
            real = torch.view_as_real(v.resolve_conj()).to(dtype)
            cos[:v.shape[0], column:column + v.shape[1]] = real[..., 0]
            sin[:v.shape[0], column:column + v.shape[1]] = real[..., 1]
            column += v.shape[1]
        return cls(cos, sin, tuple(v.shape[1] for v in axes), tuple(v.shape[0] for v in axes))

    @classmethod
    def from_cos_sin(cls, cos, sin, sections=None):
        return cls(cos, sin, sections)

    @classmethod
    def wan(cls, head_dim, max_positions=1024, *, theta=10000.0, device="cpu"):
        """Wan / causal-Wan 3-axis tables: per-axis ``1 / theta ** (2j / dim_axis)`` frequencies with
        axis dims ``[d - 4 (d // 6), 2 (d // 6), 2 (d // 6)]`` (44/42/42 for d = 128), FP64."""
        _int(head_dim, "head_dim", minimum=8)
        dims = (head_dim - 4 * (head_dim // 6), 2 * (head_dim // 6), 2 * (head_dim // 6))
        positions = torch.arange(max_positions, dtype=torch.float64)
        parts = []
        for dim in dims:
            inv = 1.0 / (theta ** (torch.arange(0, dim, 2, dtype=torch.float64) / dim))
            parts.append(torch.outer(positions, inv))
        angles = torch.cat(parts, dim=1)
        return cls(torch.cos(angles).to(device), torch.sin(angles).to(device), tuple(d // 2 for d in dims))

    @classmethod
    def longcat(cls, head_dim, num_frames, height, width, *, base=10000.0, device="cpu"):
        """LongCat-Video ``rope_3d`` tables computed in float32 (per-axis grids and frequencies)."""
        _int(head_dim, "head_dim", minimum=8)
        if head_dim % 8:
            raise ConfigurationError("LongCat 3D RoPE requires head_dim divisible by 8")
        dims = (head_dim - 4 * (head_dim // 6), 2 * (head_dim // 6), 2 * (head_dim // 6))
        tables = []
        for dim, count in zip(dims, (num_frames, height, width)):
            _int(count, "axis length", minimum=1)
            inverse = 1.0 / (base ** (torch.arange(0, dim, 2)[: dim // 2].float() / dim))
            grid = torch.arange(count, dtype=torch.float32)
            tables.append(torch.outer(grid, inverse))
        rows = max(t.shape[0] for t in tables)
        pairs = sum(t.shape[1] for t in tables)
        cos = torch.full((rows, pairs), float("nan"), dtype=torch.float32)
        sin = torch.full_like(cos, float("nan"))
        column = 0
        for t in tables:
            cos[:t.shape[0], column:column + t.shape[1]] = t.cos()
            sin[:t.shape[0], column:column + t.shape[1]] = t.sin()
            column += t.shape[1]
        return cls(cos.to(device), sin.to(device), tuple(t.shape[1] for t in tables),
                   tuple(t.shape[0] for t in tables))

    def _stamp(self):
        if self.cos.is_inference() or self.sin.is_inference():
            return (self.cos.data_ptr(), self.sin.data_ptr())
        return (self.cos._version, self.sin._version, self.cos.data_ptr(), self.sin.data_ptr())

    def invalidate(self):
        self._device_cache.clear()

    def kernel_tables(self, device, stream=None):
        """Contiguous FP32 ``(cos, sin)`` on ``device``, ordered before work enqueued next on ``stream``."""
        device = torch.device(device)
        if device.type == "cuda" and device.index is None:
            device = torch.device("cuda", torch.cuda.current_device())
        stamp = self._stamp()
        entry = self._device_cache.get(device)
        if entry is None or entry[2] != stamp:
            with torch.inference_mode(False), torch.no_grad():
                if self.cos.device == device and self.cos.dtype == torch.float32 and self.cos.is_contiguous() \
                        and self.sin.is_contiguous():
                    cos, sin = self.cos, self.sin
                else:
                    ctx = torch.cuda.stream(stream) if (stream is not None and device.type == "cuda") else _null()
                    with ctx:
                        cos = self.cos.to(device=device, dtype=torch.float32).contiguous()
                        sin = self.sin.to(device=device, dtype=torch.float32).contiguous()
            entry = (cos, sin, stamp)
            self._device_cache[device] = entry
        return entry[0], entry[1]

    def token_tables(self, positions_rows, grid, device, stream=None):
        """Per-token FP32 ``(cos, sin)`` ``[tokens, pairs]`` of one chunk's positions (cached per
        positions, grid and device): the fused restore epilogue reads each token's 16-pair slices
        with 16-byte loads instead of resolving the three axis sections per pair."""
        device = torch.device(device)
        if device.type == "cuda" and device.index is None:
            device = torch.device("cuda", torch.cuda.current_device())
        stamp = self._stamp()
        key = ("tok", device, positions_rows if isinstance(positions_rows, int) else tuple(positions_rows),
               tuple(grid))
        entry = self._device_cache.get(key)
        if entry is None or entry[2] != stamp:
            cos, sin = self.kernel_tables(device, stream)
            frames, height, width = grid
            tokens = frames * height * width
            ctx = torch.cuda.stream(stream) if (stream is not None and device.type == "cuda") else _null()
            with torch.inference_mode(False), torch.no_grad(), ctx:
                if self.sections is None:
                    first = positions_rows
                    out_cos = cos[first:first + tokens].contiguous()
                    out_sin = sin[first:first + tokens].contiguous()
                else:
                    index = torch.arange(tokens, device=device)
                    coordinates = (index // (height * width), (index % (height * width)) // width, index % width)
                    out_cos = torch.empty((tokens, self.pairs), dtype=torch.float32, device=device)
                    out_sin = torch.empty_like(out_cos)
                    column = 0
                    for axis, pairs in enumerate(self.sections):
                        rows = positions_rows[axis] + coordinates[axis]
                        out_cos[:, column:column + pairs] = cos[rows, column:column + pairs]
                        out_sin[:, column:column + pairs] = sin[rows, column:column + pairs]
                        column += pairs
            entry = (out_cos, out_sin, stamp)
            if len(self._device_cache) > 256:
                for stale in [k for k in self._device_cache if isinstance(k, tuple) and k and k[0] == "tok"][:128]:
                    del self._device_cache[stale]
            self._device_cache[key] = entry
        return entry[0], entry[1]

    def packed_tables(self, positions_rows, grid, device, stream=None):
        """Separable tables of one chunk as FP32 ``(cos, sin)`` pairs ``[T*Pt + H*Ph + W*Pw, 2]``:
        frame section rows ``t_row .. t_row + T``, then the row section, then the column section
        (cached per positions, grid and device). The fused restore epilogue keeps these in shared
        memory; ``None`` for dense tables or more than ``PACKED_ROPE_ENTRIES`` entries."""
        if self.sections is None:
            return None
        frames, height, width = grid
        sec_t, sec_h, sec_w = self.sections
        entries = frames * sec_t + height * sec_h + width * sec_w
        if entries > PACKED_ROPE_ENTRIES:
            return None
        device = torch.device(device)
        if device.type == "cuda" and device.index is None:
            device = torch.device("cuda", torch.cuda.current_device())
        stamp = self._stamp()
        key = ("pack", device, tuple(positions_rows), tuple(grid))
        entry = self._device_cache.get(key)
        if entry is None or entry[1] != stamp:
            cos, sin = self.kernel_tables(device, stream)
            ctx = torch.cuda.stream(stream) if (stream is not None and device.type == "cuda") else _null()
            with torch.inference_mode(False), torch.no_grad(), ctx:
                parts, column = [], 0
                for axis, (count, pairs) in enumerate(zip(grid, self.sections)):
                    first = positions_rows[axis]
                    block = torch.stack((cos[first:first + count, column:column + pairs],
                                         sin[first:first + count, column:column + pairs]), dim=-1)
                    parts.append(block.reshape(-1, 2))
                    column += pairs
                if entries % 2:  # storage padded to whole 16-byte units (the kernel bulk-copies it)
                    parts.append(torch.zeros((1, 2), dtype=torch.float32, device=device))
                pack = torch.cat(parts).contiguous()
            entry = (pack, stamp)
            if len(self._device_cache) > 256:
                for stale in [k for k in self._device_cache if isinstance(k, tuple) and k and k[0] == "pack"][:128]:
                    del self._device_cache[stale]
            self._device_cache[key] = entry
        return entry[0], (sec_t, sec_h, entries)

    def kernel_tables_t(self, device, stream=None):
        """Transposed FP32 ``(cos, sin)`` ``[pairs, rows]`` for the sm_100a kernels: lanes of a warp
        hold consecutive tokens, so the rows they read for one pair are adjacent in memory."""
        device = torch.device(device)
        if device.type == "cuda" and device.index is None:
            device = torch.device("cuda", torch.cuda.current_device())
        stamp = self._stamp()
        key = ("t", device)
        entry = self._device_cache.get(key)
        if entry is None or entry[2] != stamp:
            cos, sin = self.kernel_tables(device, stream)
            ctx = torch.cuda.stream(stream) if (stream is not None and device.type == "cuda") else _null()
            with torch.inference_mode(False), torch.no_grad(), ctx:
                entry = (cos.t().contiguous(), sin.t().contiguous(), stamp)
            self._device_cache[key] = entry
        return entry[0], entry[1]


@dataclass(frozen=True, eq=False)
class RopePositions:
    """Original positions of one chunk in a :class:`RopeTable` (separable: ``(t_row, h_row, w_row)``)."""

    table: RopeTable
    rows: Any = 0

    def __post_init__(self):
        if not isinstance(self.table, RopeTable):
            raise ConfigurationError("RoPE positions require a RopeTable")
        if self.table.sections is None:
            _int(self.rows, "dense RoPE row")
        else:
            rows = self.rows
            if type(rows) is int:
                rows = (rows, 0, 0)
            rows = tuple(rows)
            if len(rows) != 3:
                raise ConfigurationError("separable RoPE positions are (t_row, h_row, w_row)")
            for value in rows:
                _int(value, "RoPE row")
            object.__setattr__(self, "rows", rows)


@dataclass(frozen=True, eq=False)
class CoefficientSource:
    """Coefficients ``[N, >= rank]`` already unpacked from their pictures (uint8 + affine or float)."""

    values: torch.Tensor
    scale: Any = None
    offset: Any = None
    bound: float | None = None

    def __post_init__(self):
        values = _require_tensor(self.values, "coefficients")
        if values.ndim != 2:
            raise ConfigurationError("coefficients must be a [tokens, rank] matrix")
        if self.bound is not None and (isinstance(self.bound, bool) or not isinstance(self.bound, (int, float))
                                       or not math.isfinite(self.bound) or self.bound < 0):
            raise ConfigurationError("bound must be a finite nonnegative upper bound on |coefficients|")
        if values.dtype == torch.uint8:
            if self.scale is None or self.offset is None:
                raise ConfigurationError("quantized coefficients require their affine scale and offset")
            object.__setattr__(self, "scale", _host_vector(self.scale, values.shape[1], "scale"))
            object.__setattr__(self, "offset", _host_vector(self.offset, values.shape[1], "offset"))
            if np.any(self.scale < 0):
                raise ConfigurationError("affine scales must be nonnegative")
        elif values.dtype in COEFFICIENT_DTYPES:
            if self.scale is not None or self.offset is not None:
                raise ConfigurationError("dequantized coefficients take no affine")
        else:
            raise ConfigurationError("coefficients must be uint8 pixels or float32/float16/bfloat16 values")

    @property
    def quantized(self):
        return self.values.dtype == torch.uint8


@dataclass(frozen=True, eq=False)
class PictureSource:
    """Quantized coefficients read in place from decoded pictures ``pictures[segment][frame]``
    (uint8 views ``[planes, rows, columns]`` whose origin is this matrix's rectangle)."""

    pictures: Any
    layout: Mapping
    scale: Any
    offset: Any

    def __post_init__(self):
        layout = self.layout
        required = ("frames", "height", "width", "rank", "planes", "grid", "channels_per_segment", "segments")
        if not isinstance(layout, Mapping) or any(name not in layout for name in required):
            raise ConfigurationError("picture layout must be a reelcache.channel_tiles.v1 layout")
        frames, height, width, rank = (layout[n] for n in ("frames", "height", "width", "rank"))
        planes, slots, segments = layout["planes"], layout["channels_per_segment"], layout["segments"]
        for value, name in ((frames, "frames"), (height, "height"), (width, "width"), (rank, "rank"),
                            (planes, "planes"), (slots, "channels_per_segment"), (segments, "segments")):
            _int(value, f"layout {name}", minimum=1)
        columns, rows = layout["grid"]
        _int(columns, "grid columns", minimum=1)
        _int(rows, "grid rows", minimum=1)
        if slots != columns * rows * planes or segments != math.ceil(rank / slots):
            raise ConfigurationError("picture layout slot/segment counts are inconsistent")
        pictures = tuple(tuple(segment) for segment in self.pictures)
        if len(pictures) != segments or any(len(segment) != frames for segment in pictures):
            raise ConfigurationError("pictures must be indexed [segment][frame] for every segment and frame")
        strides = None
        device = None
        for segment in pictures:
            for picture in segment:
                _require_tensor(picture, "picture")
                if picture.dtype != torch.uint8 or picture.ndim != 3:
                    raise ConfigurationError("pictures must be uint8 [planes, rows, columns] views")
                if picture.shape[0] < planes or picture.shape[1] < rows * height or picture.shape[2] < columns * width:
                    raise ConfigurationError("picture view does not cover the matrix rectangle")
                if picture.stride(2) != 1:
                    raise ConfigurationError("picture rows must be contiguous (unit column stride)")
                current = (picture.stride(0), picture.stride(1))
                if strides is None:
                    strides, device = current, picture.device
                elif current != strides or picture.device != device:
                    raise ConfigurationError("pictures of one matrix must share plane/row strides and device")
        object.__setattr__(self, "pictures", pictures)
        object.__setattr__(self, "scale", _host_vector(self.scale, rank, "scale"))
        object.__setattr__(self, "offset", _host_vector(self.offset, rank, "offset"))
        if np.any(self.scale < 0):
            raise ConfigurationError("affine scales must be nonnegative")

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
        """Views on decoded canvases ``[pictures, planes, height, width]``; ``origins`` is one
        ``(y, x)`` or a ``[segment][frame]`` table of origins (schema v2 tile map)."""
        canvases = _require_tensor(canvases, "canvases")
        if canvases.ndim != 4 or canvases.dtype != torch.uint8:
            raise ConfigurationError("canvases must be uint8 [pictures, planes, height, width]")
        single = len(origins) == 2 and all(type(v) is int for v in origins)
        pictures = []
        for s_index, segment in enumerate(picture_indices):
            row = []
            for f_index, picture in enumerate(segment):
                y, x = origins if single else origins[s_index][f_index]
                _int(picture, "picture index")
                _int(y, "rectangle y")
                _int(x, "rectangle x")
                if picture >= canvases.shape[0]:
                    raise ConfigurationError("picture index is outside the canvases")
                row.append(canvases[picture, :, y:, x:])
            pictures.append(tuple(row))
        return cls(tuple(pictures), layout, scale, offset)


@dataclass(frozen=True, eq=False)
class DenseSource:
    """An uncompressed canonical ``[N, C]`` matrix (RAW archive, raw tier)."""

    values: torch.Tensor

    def __post_init__(self):
        values = _require_tensor(self.values, "dense values")
        if values.ndim != 2 or values.dtype not in COEFFICIENT_DTYPES:
            raise ConfigurationError("dense values must be a float32/float16/bfloat16 [tokens, channels] matrix")


@dataclass(frozen=True, eq=False)
class ReconstructionJob:
    """Reconstruct one restored matrix into one native destination slot.

    ``basis_t`` optionally supplies the kernel's operand layout of the same basis: the transposed,
    zero-padded FP16 matrix ``[C, ceil(R / 64) * 64]`` (the device basis cache keeps it), saving the
    per-call transpose.
    """

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
            raise ConfigurationError("source must be a CoefficientSource, PictureSource or DenseSource")
        if not isinstance(self.destination, NativeView):
            raise ConfigurationError("destination must be a NativeView")
        grid = tuple(self.grid)
        if len(grid) != 3:
            raise ConfigurationError("grid must be (frames, height, width)")
        for value in grid:
            _int(value, "grid size", minimum=1)
        object.__setattr__(self, "grid", grid)
        tokens = self.tokens
        channels = self.destination.channels
        if self.destination.token_offset + tokens > self.destination.capacity:
            raise ConfigurationError("destination slot exceeds the native cache capacity")
        if isinstance(self.source, DenseSource):
            if self.basis is not None or self.rank is not None:
                raise ConfigurationError("dense sources take no basis or rank")
            if tuple(self.source.values.shape) != (tokens, channels):
                raise ConfigurationError("dense values must be [tokens, heads * head_dim]")
        else:
            basis = _require_tensor(self.basis, "basis")
            if basis.ndim != 2 or basis.shape[1] != channels:
                raise ConfigurationError("basis must be [rows, heads * head_dim] of the destination")
            if basis.dtype not in (torch.float16, torch.float32):
                raise ConfigurationError("basis must be the canonical float16 rows (float32 for reference use)")
            if isinstance(self.source, PictureSource):
                layout = self.source.layout
                if (layout["frames"], layout["height"], layout["width"]) != grid:
                    raise ConfigurationError("picture layout geometry differs from the job grid")
                columns = layout["rank"]
            else:
                if self.source.values.shape[0] != tokens:
                    raise ConfigurationError("coefficient rows differ from the job token count")
                columns = self.source.values.shape[1]
            rank = columns if self.rank is None else self.rank
            _int(rank, "rank", minimum=1)
            if rank > basis.shape[0]:
                raise ConfigurationError("rank view exceeds the basis rows")
            if rank > columns or (isinstance(self.source, PictureSource) and rank != columns):
                raise ConfigurationError("rank view exceeds the available coefficient columns")
            object.__setattr__(self, "rank", rank)
            if self.basis_t is not None:
                bt = self.basis_t
                if (bt.dtype != torch.float16 or bt.ndim != 2 or bt.shape[0] != channels or bt.shape[1] % 64
                        or bt.shape[1] < rank or bt.stride(1) != 1):
                    raise ConfigurationError("basis_t must be float16 [channels, rank_pad] (rank_pad % 64 == 0)")
        if self.rope is not None:
            if not isinstance(self.rope, RopePositions):
                raise ConfigurationError("rope must be RopePositions")
            table = self.rope.table
            if table.head_dim != self.destination.head_dim:
                raise ConfigurationError("RoPE table pairs differ from head_dim // 2")
            if table.sections is None:
                if self.rope.rows + tokens > table.rows:
                    raise ConfigurationError("dense RoPE rows exceed the table")
            else:
                limits = table.section_rows
                needed = (self.rope.rows[0] + grid[0], self.rope.rows[1] + grid[1], self.rope.rows[2] + grid[2])
                if any(need > limit for need, limit, pairs in zip(needed, limits, table.sections) if pairs):
                    raise ConfigurationError("separable RoPE rows exceed the table")

    @property
    def tokens(self):
        frames, height, width = self.grid
        return frames * height * width

    @property
    def channels(self):
        return self.destination.channels

    def tensors(self):
        result = [self.destination.tensor]
        source = self.source
        if isinstance(source, PictureSource):
            result.extend(picture for segment in source.pictures for picture in segment)
        else:
            result.append(source.values)
        if self.basis is not None:
            result.append(self.basis)
        if self.basis_t is not None:
            result.append(self.basis_t)
        if self.rope is not None:
            result.extend((self.rope.table.cos, self.rope.table.sin))
        return result


# ---------------------------------------------------------------------------------------------
# Completion handle
# ---------------------------------------------------------------------------------------------

_DEFERRED = []
_DEFERRED_LOCK = threading.RLock()


def _sweep_deferred():
    with _DEFERRED_LOCK:
        if _DEFERRED:
            _DEFERRED[:] = [(event, refs) for event, refs in _DEFERRED if not event.query()]


def pending_deferred():
    with _DEFERRED_LOCK:
        return len(_DEFERRED)


class RestoreHandle:
    """Completion of one :func:`reconstruct` call: a CUDA event recorded after the last write, and a
    keepalive of every input and temporary until :meth:`release` (or, when dropped unreleased, until
    the event completes)."""

    def __init__(self, *, event, stream, keepalive, stats):
        self._event = event
        self._stream = stream
        self._keepalive = keepalive
        self._released = False
        self.stats = stats

    @property
    def event(self):
        return self._event

    @property
    def stream(self):
        return self._stream

    @property
    def released(self):
        return self._released

    def query(self):
        return self._event is None or self._event.query()

    def synchronize(self):
        if self._event is not None:
            self._event.synchronize()

    def wait(self, stream=None):
        if self._event is None:
            return
        if stream is None:
            stream = torch.cuda.current_stream(self._stream.device)
        stream.wait_event(self._event)

    def release(self):
        if self._released:
            return
        self.synchronize()
        self._keepalive = None
        self._released = True
        _sweep_deferred()

    def __del__(self):
        try:
            if not self._released and self._event is not None and self._keepalive is not None:
                if not self._event.query():
                    with _DEFERRED_LOCK:
                        _DEFERRED.append((self._event, self._keepalive))
        except Exception:  # noqa: BLE001 - interpreter shutdown
            pass


# ---------------------------------------------------------------------------------------------
# Validation and the reference backend
# ---------------------------------------------------------------------------------------------


def _storage_key(tensor):
    try:
        return tensor.untyped_storage().data_ptr(), tensor.device
    except (RuntimeError, NotImplementedError):
        return tensor.data_ptr(), tensor.device


def _check_disjoint(jobs):
    """Reject jobs whose slots in the same destination view overlap (their writes would race)."""
    spans = {}
    for index, job in enumerate(jobs):
        view = job.destination
        tensor = view.tensor
        key = (*_storage_key(tensor), tensor.storage_offset(), tuple(tensor.shape), tensor.stride(),
               view.layout, view.batch_index)
        spans.setdefault(key, []).append((view.token_offset, view.token_offset + job.tokens, index))
    for intervals in spans.values():
        intervals.sort()
        for (_, stop, first), (start, _, second) in zip(intervals, intervals[1:]):
            if start < stop:
                raise ConfigurationError(f"jobs {first} and {second} write overlapping destination tokens")


def _validate(jobs):
    if isinstance(jobs, ReconstructionJob):
        jobs = (jobs,)
    if not isinstance(jobs, Sequence) or isinstance(jobs, (str, bytes)):
        raise ConfigurationError("jobs must be a sequence of ReconstructionJob")
    jobs = tuple(jobs)
    if any(not isinstance(job, ReconstructionJob) for job in jobs):
        raise ConfigurationError("jobs must be ReconstructionJob instances")
    devices = set()
    for job in jobs:
        devices.add(job.destination.tensor.device)
        source = job.source
        devices.add(source.device if isinstance(source, PictureSource) else source.values.device)
        if job.basis is not None:
            devices.add(job.basis.device)
    if len(devices) > 1:
        raise ConfigurationError("all job tensors (except RoPE tables) must share one device")
    _check_disjoint(jobs)
    return jobs, (devices.pop() if devices else None)


def unpack_pictures(source):
    """Quantized pixels ``[N, rank]`` of a :class:`PictureSource` (mosaic cell mapping)."""
    layout = source.layout
    frames, height, width, rank = layout["frames"], layout["height"], layout["width"], layout["rank"]
    columns, rows = layout["grid"]
    planes, slots = layout["planes"], layout["channels_per_segment"]
    values = torch.empty((frames, height, width, rank), dtype=torch.uint8, device=source.device)
    for segment, pictures in enumerate(source.pictures):
        first = segment * slots
        count = min(slots, rank - first)
        for frame, picture in enumerate(pictures):
            cropped = picture[:planes, :rows * height, :columns * width]
            tiled = cropped.reshape(planes, rows, height, columns, width)
            values[frame, :, :, first:first + count] = tiled.permute(2, 4, 1, 3, 0).reshape(height, width, -1)[:, :, :count]
    return values.reshape(-1, rank)


def dequantize(pixels, scale, offset):
    """``float(pixel) * scale + offset`` with the eager (multiply, then add) rounding."""
    scale = torch.from_numpy(np.ascontiguousarray(scale)).to(pixels.device)
    offset = torch.from_numpy(np.ascontiguousarray(offset)).to(pixels.device)
    return pixels.float().mul_(scale).add_(offset)


def reference_coefficients(job):
    source = job.source
    if isinstance(source, PictureSource):
        return dequantize(unpack_pictures(source), source.scale, source.offset)
    if isinstance(source, CoefficientSource):
        if source.quantized:
            return dequantize(source.values[:, :job.rank], source.scale[:job.rank], source.offset[:job.rank])
        return source.values[:, :job.rank].float()
    raise ConfigurationError("dense sources have no coefficients")


def rope_cos_sin(positions, grid, *, dtype=torch.float64, device=None):
    """Per-token ``(cos, sin)`` ``[N, head_dim // 2]`` of a job's positions."""
    table = positions.table
    device = table.cos.device if device is None else device
    cos = table.cos.to(device=device, dtype=dtype)
    sin = table.sin.to(device=device, dtype=dtype)
    frames, height, width = grid
    tokens = frames * height * width
    if table.sections is None:
        first = positions.rows
        return cos[first:first + tokens], sin[first:first + tokens]
    index = torch.arange(tokens, device=device)
    frame, rest = index // (height * width), index % (height * width)
    coordinates = (frame, rest // width, rest % width)
    out_cos = torch.empty((tokens, table.pairs), dtype=dtype, device=device)
    out_sin = torch.empty_like(out_cos)
    column = 0
    for axis, pairs in enumerate(table.sections):
        rows = positions.rows[axis] + coordinates[axis]
        out_cos[:, column:column + pairs] = cos[rows, column:column + pairs]
        out_sin[:, column:column + pairs] = sin[rows, column:column + pairs]
        column += pairs
    return out_cos, out_sin


def apply_rope_reference(values, positions, grid, *, dtype=torch.float64):
    """Rotate interleaved pairs of ``values[N, H, D]`` in ``dtype`` (complex product)."""
    cos, sin = rope_cos_sin(positions, grid, dtype=dtype, device=values.device)
    x = values.to(dtype)
    even, odd = x[..., 0::2], x[..., 1::2]
    cos, sin = cos[:, None, :], sin[:, None, :]
    out = torch.empty_like(x)
    out[..., 0::2] = even * cos - odd * sin
    out[..., 1::2] = even * sin + odd * cos
    return out


def _reference_job(job, compute, native_rope, native_rope_dtype):
    heads, head_dim = job.destination.heads, job.destination.head_dim
    tokens = job.tokens
    slot = job.destination.slot(tokens)
    if isinstance(job.source, DenseSource):
        values = job.source.values
    else:
        coefficients = reference_coefficients(job)
        basis = job.basis[:job.rank]
        values = coefficients.to(compute) @ basis.to(device=coefficients.device, dtype=compute)
    if native_rope is not None and job.rope is not None:
        dtype = slot.dtype if native_rope_dtype is None else native_rope_dtype
        result = native_rope(values.to(dtype).reshape(tokens, heads, head_dim), job)
        if not isinstance(result, torch.Tensor) or result.numel() != tokens * heads * head_dim:
            raise IntegrityError("native RoPE callable returned a tensor of the wrong size")
        slot.copy_(result.reshape(tokens, heads, head_dim))
        return
    values = values.reshape(tokens, heads, head_dim)
    if job.rope is not None:
        values = apply_rope_reference(values, job.rope, job.grid, dtype=compute)
    slot.copy_(values)


def reconstruct_reference(jobs, *, compute_dtype=torch.float64, native_rope=None, native_rope_dtype=None):
    """Plain-torch reference: FP64 (default) or FP32 math, then one cast."""
    jobs, _ = _validate(jobs)
    if compute_dtype not in (torch.float32, torch.float64):
        raise ConfigurationError("reference compute dtype must be float32 or float64")
    with torch.no_grad():
        for job in jobs:
            _reference_job(job, compute_dtype, native_rope, native_rope_dtype)


_UNIT_ROUNDOFF = {torch.bfloat16: 2.0 ** -8, torch.float16: 2.0 ** -11, torch.float32: 2.0 ** -24}
_OUTPUT_FLOOR = {torch.bfloat16: 2.0 ** -134, torch.float16: 2.0 ** -25, torch.float32: 2.0 ** -150}


def _gemm_gamma(precision, rank):
    """Relative GEMM error per unit of ``sum_k |a_k| |q_k|`` of each precision mode."""
    accumulate = (rank + 1) * 2.0 ** -24
    return {
        "fp32": accumulate,
        "tf32": 2.0 ** -10 + accumulate,
        "tf32x3": 2.0 ** -20 + 3 * accumulate,
        "fp16": 2.0 ** -11 + accumulate,
        "fp16x2": 2.0 ** -21 + 2 * accumulate,
        "bf16": 2.0 ** -7 + 2.0 ** -16 + accumulate,
        "reference32": accumulate,
    }[precision]


def reference_values(job):
    """FP64 values ``y*[N, C]`` a job writes before the final cast, and ``sum_k |p_k| |q_k|``."""
    tokens, heads, head_dim = job.tokens, job.destination.heads, job.destination.head_dim
    if isinstance(job.source, DenseSource):
        values = job.source.values.double()
        magnitude = torch.zeros_like(values)
    else:
        coefficients = reference_coefficients(job).double()
        basis = job.basis[:job.rank].to(device=coefficients.device, dtype=torch.float64)
        values = coefficients @ basis
        magnitude = coefficients.abs() @ basis.abs()
    if job.rope is not None:
        values = apply_rope_reference(values.reshape(tokens, heads, head_dim), job.rope, job.grid).reshape(tokens, -1)
        pairs = magnitude.reshape(tokens, -1, 2)
        magnitude = (pairs[..., 0] + pairs[..., 1]).repeat_interleave(2, dim=-1)
    return values, magnitude


def error_bound(job, precision, out_dtype=None):
    """Elementwise bound on ``|written - y*|`` (first-order): ``u_out |y*| + (1 + u_out) E + floor``
    with ``E = gamma(precision, rank) * S + 2**-21 (|y_e| + |y_o|)`` for RoPE jobs. Returns
    ``(y*, bound)`` in FP64."""
    values, magnitude = reference_values(job)
    out_dtype = job.destination.tensor.dtype if out_dtype is None else out_dtype
    unit = _UNIT_ROUNDOFF[out_dtype]
    rank = job.rank or 0
    error = _gemm_gamma(precision, rank) * magnitude
    if job.rope is not None:
        pairs = values.reshape(job.tokens, -1, 2).abs()
        error = error + 2.0 ** -21 * (pairs[..., 0] + pairs[..., 1]).repeat_interleave(2, dim=-1)
    return values, unit * values.abs() + (1 + unit) * error + _OUTPUT_FLOOR[out_dtype]


# ---------------------------------------------------------------------------------------------
# Fused sm_100a backend
# ---------------------------------------------------------------------------------------------

_BASIS_T_CACHE = OrderedDict()
_BASIS_T_LIMIT = 256
_BASIS_T_LOCK = threading.Lock()


def transposed_basis(basis, stream=None):
    """The fused kernel's B operand of an FP16 basis ``[R, C]``: ``Qt[C, ceil(R / 64) * 64]`` FP16,
    zero-padded, cached per basis tensor state."""
    key = (basis.data_ptr(), tuple(basis.shape), basis.stride(), basis.dtype, basis.device,
           None if basis.is_inference() else basis._version)
    with _BASIS_T_LOCK:
        hit = _BASIS_T_CACHE.get(key)
        if hit is not None:
            _BASIS_T_CACHE.move_to_end(key)
            return hit[0]
    rows, channels = basis.shape
    padded = ((rows + 63) // 64) * 64
    with torch.inference_mode(False), torch.no_grad():
        qt = torch.zeros((channels, padded), dtype=torch.float16, device=basis.device)
        qt[:, :rows].copy_(basis.t())
    with _BASIS_T_LOCK:
        _BASIS_T_CACHE[key] = (qt, basis)
        while len(_BASIS_T_CACHE) > _BASIS_T_LIMIT:
            _BASIS_T_CACHE.popitem(last=False)
    return qt


def _rope_fields(job, device, stream):
    """(rope, dense, row_stride, row_t, row_h, row_w, sec_t, sec_h, cos_ptr, sin_ptr, tensors)."""
    if job.rope is None:
        return (0, 0, 0, 0, 0, 0, 0, 0, 0, 0, ())
    table = job.rope.table
    cos, sin = table.kernel_tables_t(device, stream)
    if table.sections is None:
        return (1, 1, table.rows, job.rope.rows, 0, 0, 0, 0, cos.data_ptr(), sin.data_ptr(), (cos, sin))
    t_row, h_row, w_row = job.rope.rows
    sec_t, sec_h, _ = table.sections
    return (1, 0, table.rows, t_row, h_row, w_row, sec_t, sec_h, cos.data_ptr(), sin.data_ptr(), (cos, sin))


def _fused_factor_group(jobs, device, precision, stream, keepalive):
    """Describe the group's jobs to the launch plumbing (reelcache_b200/ops/restore.py)."""
    from .ops.restore import launch_factor_group

    items = []
    for job in jobs:
        source = job.source
        view = job.destination
        item = {"tokens": job.tokens, "rank": job.rank, "grid": job.grid, "basis": job.basis,
                "basis_t": job.basis_t,
                "dest": (view.address(), view.strides(), view.tensor.dtype, job.channels, view.head_dim)}
        if job.rope is None:
            item["rope"] = None
        else:
            item["rope"] = restore_rope_item(job.rope, job.grid, device, stream, keepalive)
        if job.basis.dtype != torch.float16:
            with torch.cuda.stream(stream):
                item["basis"] = job.basis[:job.rank].half().contiguous()
            keepalive.append(item["basis"])
        if isinstance(source, PictureSource):
            addresses = np.array([[picture.data_ptr() for picture in segment] for segment in source.pictures],
                                 dtype=np.int64).reshape(-1)
            item.update(kind="pictures", pictures=(addresses, source.plane_stride, source.row_stride, source.layout),
                        scale=source.scale, offset=source.offset)
        elif source.quantized:
            item.update(kind="u8", values=source.values, scale=source.scale, offset=source.offset)
        else:
            item.update(kind="f32", values=source.values, bound=source.bound)
        items.append(item)
    return launch_factor_group(items, device, precision, stream, keepalive)


def _fused_dense_group(jobs, device, stream, keepalive):
    from .ops._ext import ext

    rows = []
    for job in jobs:
        values = job.source.values
        if values.stride(1) != 1:
            with torch.cuda.stream(stream):
                values = values.contiguous()
            keepalive.append(values)
        view = job.destination
        ts, hs, ds = view.strides()
        rope = _rope_fields(job, device, stream)
        keepalive.extend(rope[10])
        rows.append([
            values.data_ptr(), view.address(), rope[8], rope[9], values.stride(0), ts, hs, ds,
            _OUT_CODE[values.dtype], _OUT_CODE[view.tensor.dtype], job.tokens, job.channels, view.head_dim,
            job.grid[1], job.grid[2], rope[0], rope[1], rope[2], rope[3], rope[4], rope[5], rope[6], rope[7],
            device.index if device.index is not None else torch.cuda.current_device(),
        ])
    with torch.cuda.stream(stream):
        ext().rope_store_launch(torch.tensor(rows, dtype=torch.int64))
    return 1


class _null:
    def __enter__(self):
        return self

    def __exit__(self, *_):
        return False


def _matrix_flops(jobs):
    return sum(2 * job.tokens * job.rank * job.channels for job in jobs if job.rank)


def _resolve_backend(backend, cuda):
    if backend == "reference" or (backend == "auto" and not cuda):
        return "reference"
    if not cuda:
        raise UnsupportedError(f"the {backend} backend needs CUDA tensors; use 'reference'")
    from .ops._ext import ext

    ext()  # raises UnsupportedError naming the missing library: never a silent fallback
    return "fused"


def reconstruct(jobs, *, backend="auto", precision="auto", stream=None, wait_events=(), native_rope=None,
                native_rope_dtype=None, compute_dtype=torch.float64, stage_events=None, config=None):
    """Reconstruct restored matrices into their native cache slots.

    One call should cover all restored chunks of a layer (K and V): the fused backend runs one
    persistent launch per 16 factorized jobs (and one per 48 dense jobs). ``stream`` (default:
    current) first waits on ``wait_events``. ``native_rope(pre_rope[N, H, D], job)`` replaces the
    built-in rotation for RoPE jobs (the exact engine path). Returns a :class:`RestoreHandle`.
    """
    _sweep_deferred()
    jobs, device = _validate(jobs)
    if backend not in BACKENDS:
        raise ConfigurationError(f"backend must be one of {BACKENDS}")
    if precision != "auto" and precision not in PRECISIONS:
        raise ConfigurationError(f"precision must be 'auto' or one of {PRECISIONS}")
    if native_rope is not None and not callable(native_rope):
        raise ConfigurationError("native_rope must be callable")
    stats = {"jobs": len(jobs), "matrices": len(jobs), "flops": _matrix_flops(jobs), "launches": 0}
    if not jobs:
        stats.update(backend="none", precision=None)
        return RestoreHandle(event=None, stream=None, keepalive=None, stats=stats)
    cuda = device.type == "cuda"
    backend = _resolve_backend(backend, cuda)
    if precision == "auto":
        # Every destination dtype takes the two-product split: its error bound does not depend on the
        # cancellation in sum_k a_k q_k, which a single FP16 product's bound does.
        precision = DEFAULT_PRECISION
    if backend == "fused" and precision not in KERNEL_PRECISIONS:
        raise UnsupportedError(f"the fused sm_100a kernel runs {KERNEL_PRECISIONS}; use backend='reference' "
                               f"for {precision}")
    if cuda:
        stream = torch.cuda.current_stream(device) if stream is None else stream
        if not isinstance(stream, torch.cuda.Stream) or stream.device != device:
            raise ConfigurationError("stream must be a torch.cuda.Stream on the jobs' device")
    elif stream is not None or wait_events:
        raise ConfigurationError("host execution takes no CUDA stream or events")
    keepalive = [tensor for job in jobs for tensor in job.tensors()]
    stats.update(backend=backend, precision=precision if backend != "reference" else str(compute_dtype))
    if cuda:
        for event in wait_events:
            stream.wait_event(event)
    if stage_events is not None and cuda:
        start = torch.cuda.Event(enable_timing=True)
        start.record(stream)
        stage_events.append(("start", start))
    if backend == "reference":
        with torch.cuda.stream(stream) if cuda else _null():
            reconstruct_reference(jobs, compute_dtype=compute_dtype, native_rope=native_rope,
                                  native_rope_dtype=native_rope_dtype)
    else:
        try:
            exact = [job for job in jobs if native_rope is not None and job.rope is not None]
            ordinary = [job for job in jobs if not (native_rope is not None and job.rope is not None)]
            factor = [job for job in ordinary if not isinstance(job.source, DenseSource)]
            dense = [job for job in ordinary if isinstance(job.source, DenseSource)]
            for i in range(0, len(factor), MAX_JOBS_PER_LAUNCH):
                stats["launches"] += _fused_factor_group(factor[i:i + MAX_JOBS_PER_LAUNCH], device, precision,
                                                         stream, keepalive)
            for i in range(0, len(dense), MAX_DENSE_JOBS_PER_LAUNCH):
                stats["launches"] += _fused_dense_group(dense[i:i + MAX_DENSE_JOBS_PER_LAUNCH], device, stream,
                                                        keepalive)
            if exact:
                stats["launches"] += _native_rope_jobs(exact, native_rope, native_rope_dtype, precision, device,
                                                       stream, keepalive)
        except BaseException:
            failed = torch.cuda.Event()
            failed.record(stream)
            with _DEFERRED_LOCK:
                _DEFERRED.append((failed, keepalive))
            raise
    if stage_events is not None and cuda:
        stop = torch.cuda.Event(enable_timing=True)
        stop.record(stream)
        stage_events.append(("fused", stop))
    event = None
    if cuda:
        event = torch.cuda.Event()
        event.record(stream)
    return RestoreHandle(event=event, stream=stream, keepalive=keepalive, stats=stats)


def _native_rope_jobs(jobs, native_rope, native_rope_dtype, precision, device, stream, keepalive):
    """Pre-RoPE reconstruction into scratch slots, then the engine's own RoPE callable into the slot."""
    launches = 0
    scratch_jobs = []
    pending = []
    for job in jobs:
        view = job.destination
        dtype = view.tensor.dtype if native_rope_dtype is None else native_rope_dtype
        with torch.cuda.stream(stream):
            scratch = torch.empty((job.tokens, view.heads, view.head_dim), dtype=dtype, device=device)
        keepalive.append(scratch)
        if isinstance(job.source, DenseSource) and job.source.values.dtype == dtype:
            pending.append((job, job.source.values.reshape(job.tokens, view.heads, view.head_dim)))
            continue
        scratch_jobs.append(ReconstructionJob(job.source, NativeView(scratch, "THD"), job.grid, job.basis, job.rank,
                                              None, job.label, job.basis_t))
        pending.append((job, scratch))
    factor = [j for j in scratch_jobs if not isinstance(j.source, DenseSource)]
    dense = [j for j in scratch_jobs if isinstance(j.source, DenseSource)]
    for i in range(0, len(factor), MAX_JOBS_PER_LAUNCH):
        launches += _fused_factor_group(factor[i:i + MAX_JOBS_PER_LAUNCH], device, precision, stream, keepalive)
    for i in range(0, len(dense), MAX_DENSE_JOBS_PER_LAUNCH):
        launches += _fused_dense_group(dense[i:i + MAX_DENSE_JOBS_PER_LAUNCH], device, stream, keepalive)
    with torch.cuda.stream(stream):
        for job, pre in pending:
            result = native_rope(pre, job)
            if not isinstance(result, torch.Tensor) or result.numel() != pre.numel():
                raise IntegrityError("native RoPE callable returned a tensor of the wrong size")
            job.destination.slot(job.tokens).copy_(result.reshape(pre.shape))
            keepalive.append(result)
    return launches


# ---------------------------------------------------------------------------------------------
# Warm-up
# ---------------------------------------------------------------------------------------------

WARMUP_SOURCES = ("pictures", "uint8", "float", "dense")
WARMUP_ROPE_MODES = ("none", "fused", "native")


@dataclass(frozen=True)
class WarmupShape:
    """One kind of launch group of the restore path (see :func:`warmup`)."""

    heads: int
    head_dim: int
    dtype: torch.dtype = torch.bfloat16
    layout: str = "BTHD"
    source: str = "pictures"
    rope: str = "fused"
    max_rank: int = 256

    def __post_init__(self):
        _int(self.heads, "heads", minimum=1)
        _int(self.head_dim, "head_dim", minimum=2)
        if self.dtype not in OUTPUT_DTYPES:
            raise ConfigurationError("warm-up dtype must be an output dtype")
        if self.layout not in LAYOUTS:
            raise ConfigurationError("warm-up layout must be a native layout")
        if self.source not in WARMUP_SOURCES:
            raise ConfigurationError(f"warm-up source must be one of {WARMUP_SOURCES}")
        if self.rope not in WARMUP_ROPE_MODES:
            raise ConfigurationError(f"warm-up rope must be one of {WARMUP_ROPE_MODES}")


def warmup(device, shapes, *, backend="auto", precision="auto", stream=None, **_ignored):
    """Load the module and set the kernels' shared-memory attributes ahead of the first restore by
    running one tiny job per shape (the sm_100a kernels are compiled ahead of time, so no JIT runs)."""
    device = torch.device(device)
    if device.type != "cuda":
        return {"warmed": 0}
    count = 0
    for shape in shapes:
        channels = shape.heads * shape.head_dim
        dest = torch.empty((1, 32, shape.heads, shape.head_dim), dtype=shape.dtype, device=device)
        if shape.layout == "THD":
            view = NativeView(dest[0], "THD")
        elif shape.layout == "BHTD":
            view = NativeView(dest.transpose(1, 2).contiguous(), "BHTD")
        else:
            view = NativeView(dest, "BTHD")
        grid = (1, 4, 8)
        rope = None
        if shape.rope == "fused":
            rope = RopePositions(RopeTable.wan(shape.head_dim, 64, device=device), (0, 0, 0))
        if shape.source == "dense":
            job = ReconstructionJob(DenseSource(torch.zeros(32, channels, dtype=shape.dtype, device=device)),
                                    view, grid, rope=rope)
        else:
            rank = 32
            basis = torch.zeros(rank, channels, dtype=torch.float16, device=device)
            if shape.source == "float":
                src = CoefficientSource(torch.zeros(32, rank, device=device), bound=1.0)
            else:
                src = CoefficientSource(torch.zeros(32, rank, dtype=torch.uint8, device=device),
                                        np.ones(rank, np.float32), np.zeros(rank, np.float32))
            job = ReconstructionJob(src, view, grid, basis, rope=rope)
        reconstruct([job], backend=backend, precision=precision, stream=stream).release()
        count += 1
    return {"warmed": count}


def kernel_error_bound(job, precision="fp16x2", out_dtype=None):
    """Elementwise bound of the fused sm_100a kernel (same first-order form as :func:`error_bound`).

    For 8-bit sources the kernel multiplies the exact centered pixel ``p - 128`` by the FP16 hi/lo split
    of ``s[k] Q[k, c]`` and adds the bias ``sum_k (o[k] + 128 s[k]) Q[k, c]``, so its rounding is
    charged to ``S' = sum_k (|a_k| + |o_k + 128 s_k|) |q_k|`` instead of ``sum_k |a_k| |q_k|`` (``a_k`` the
    dequantized coefficient); float sources keep the reference's ``S``. Returns ``(y*, bound)`` in FP64.
    """
    values, magnitude = reference_values(job)
    source = job.source
    quantized = isinstance(source, PictureSource) or (isinstance(source, CoefficientSource) and source.quantized)
    if quantized:
        scale = torch.from_numpy(np.asarray(source.scale[:job.rank], dtype=np.float64))
        offset = torch.from_numpy(np.asarray(source.offset[:job.rank], dtype=np.float64))
        shifted = (offset + 128.0 * scale).abs().to(magnitude.device)
        basis = job.basis[:job.rank].to(device=magnitude.device, dtype=torch.float64).abs()
        extra = (shifted @ basis).expand(job.tokens, -1)
        if job.rope is not None:
            pairs = extra.reshape(job.tokens, -1, 2)
            extra = (pairs[..., 0] + pairs[..., 1]).repeat_interleave(2, dim=-1)
        magnitude = magnitude + extra
    out_dtype = job.destination.tensor.dtype if out_dtype is None else out_dtype
    unit = _UNIT_ROUNDOFF[out_dtype]
    error = _gemm_gamma(precision, job.rank or 0) * magnitude
    if job.rope is not None:
        pairs = values.reshape(job.tokens, -1, 2).abs()
        error = error + 2.0 ** -21 * (pairs[..., 0] + pairs[..., 1]).repeat_interleave(2, dim=-1)
    return values, unit * values.abs() + (1 + unit) * error + _OUTPUT_FLOOR[out_dtype]
