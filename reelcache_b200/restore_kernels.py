"""The restore entry point: reconstruct many restored KV matrices straight into native cache slots.

Public names follow the reference's restore-kernel API (reelcache/restore_kernels.py: ``reconstruct``,
``RopeTable``, ``RestoreHandle``, ``warmup`` and the job classes re-exported from :mod:`.restore_jobs`), so
engine code written against it carries over. One :func:`reconstruct` call takes any number of jobs -- each one
chunk's K or V of one layer -- and, per job, writes ``cast(RoPE(dequantize(coefficients) @ basis[:rank]))``
(K) or ``cast(dequantize(coefficients) @ basis[:rank])`` (V) into its slot.

Backends: ``fused`` (CUDA; chosen by ``auto`` on CUDA) runs the sm_100a pipeline of csrc/restore -- an unpack
kernel turns 8-bit pixels (mosaic pictures or dense) into the exact FP16 operand ``p - 128``, a preparation
kernel folds each column's scale into a hi/lo FP16 split of the basis and its offset into a per-channel bias,
and a persistent TMA + tcgen05 GEMM adds the bias, rotates K from FP32 tables in its epilogue, casts and stores
with TMA. Dense sources go through csrc/restore/rope_store.cu. ``reference`` (chosen by ``auto`` on the CPU)
is the plain-torch FP64/FP32 computation of :mod:`.restore_reference`. Precisions of the fused kernel:
``fp16x2`` (two products, the default) and ``fp16`` (one); the bound each meets is
:func:`~reelcache_b200.restore_reference.kernel_error_bound`. A CUDA job never falls back silently: without
the native extension it raises :class:`~reelcache_b200.errors.UnsupportedError`.
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
from .restore_jobs import (COEFFICIENT_DTYPES, LAYOUTS, OUTPUT_DTYPES, CoefficientSource, DenseSource, NativeView,
                           PictureSource, ReconstructionJob, RopePositions, expand_affine, wan_sections)
from .restore_jobs import host_affine as _host_vector  # noqa: F401  (used by the fused backend's checks)
from .restore_reference import (OUTPUT_FLOOR as _OUTPUT_FLOOR, UNIT_ROUNDOFF as _UNIT_ROUNDOFF,
                                apply_rope_reference, dequantize, error_bound, gemm_gamma as _gemm_gamma,
                                kernel_error_bound, reconstruct_reference, reference_coefficients, reference_values,
                                rope_cos_sin, unpack_pictures)
from .restore_reference import check_disjoint as _check_disjoint  # noqa: F401
from .restore_reference import validate_jobs as _validate

PRECISIONS = ("fp32", "tf32", "tf32x3", "fp16", "fp16x2", "bf16")
KERNEL_PRECISIONS = ("fp16", "fp16x2")
BACKENDS = ("auto", "reference", "fused")
DEFAULT_PRECISION = "fp16x2"
MAX_JOBS_PER_LAUNCH = 16
MAX_DENSE_JOBS_PER_LAUNCH = 48
_OUT_CODE = {torch.bfloat16: 0, torch.float16: 1, torch.float32: 2}


def _nonnegative(value) -> bool:
    return type(value) is int and value >= 0


def _int(value, name, *, minimum=0):
    if type(value) is int and value >= minimum:
        return value
    raise ConfigurationError(f"{name}={value!r}: expected an int of at least {minimum}")


def _require_tensor(value, name):
    """``value`` if it is a strided tensor with storage (not a meta tensor)."""
    ok = isinstance(value, torch.Tensor) and value.layout == torch.strided and value.device.type != "meta"
    if not ok:
        raise ConfigurationError(f"{name}: expected a strided torch.Tensor with storage, got {type(value).__name__}")
    return value


def _axis_dims(head_dim: int) -> tuple[int, int, int]:
    """Rotary dims of the (frame, row, column) axes used by Wan and LongCat: the two spatial axes get
    ``2 * (head_dim // 6)`` each and the frame axis the rest (44 / 42 / 42 for head_dim 128)."""
    spatial = 2 * (head_dim // 6)
    return head_dim - 2 * spatial, spatial, spatial


def _separable(angle_tables, *, cos_sin=None):
    """``(cos, sin, sections, section_rows)`` of a separable table assembled from per-axis tables placed side by
    side; ``angle_tables`` hold angles ``[positions, pairs]`` (``cos_sin`` instead gives the per-axis
    ``(cos, sin)`` pairs). Cells past an axis's last position are NaN, so a lookup outside the axis shows."""
    parts = cos_sin if cos_sin is not None else [(a.cos(), a.sin()) for a in angle_tables]
    lengths = tuple(c.shape[0] for c, _ in parts)
    widths = tuple(c.shape[1] for c, _ in parts)
    first = parts[0][0]
    cos = torch.full((max(lengths), sum(widths)), float("nan"), dtype=first.dtype, device=first.device)
    sin = cos.clone()
    offset = 0
    for (c, s), width in zip(parts, widths):
        cos[:c.shape[0], offset:offset + width] = c
        sin[:s.shape[0], offset:offset + width] = s
        offset += width
    return cos, sin, widths, lengths


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


@dataclass(frozen=True, eq=False)
class RopeTable:
    """Rotation tables ``cos, sin [rows, head_dim // 2]`` for interleaved (even, odd) channel pairs.

    Dense (``sections=None``): row ``r`` holds the angles of position ``r``. Separable
    (``sections=(t, h, w)`` pair counts): the first ``t`` columns are indexed by frame, the next ``h`` by
    latent row and the last ``w`` by latent column, each from its own first row (``RopePositions.rows``);
    ``section_rows`` records how many rows each axis really has. Device copies in FP32 are cached per device
    (:meth:`kernel_tables`) and rebuilt when the tables are modified in place.
    """

    cos: torch.Tensor
    sin: torch.Tensor
    sections: tuple | None = None
    section_rows: tuple | None = None
    _device_cache: dict = field(default_factory=dict, init=False, repr=False, compare=False)

    def __post_init__(self):
        cos, sin = _require_tensor(self.cos, "RopeTable.cos"), _require_tensor(self.sin, "RopeTable.sin")
        same = (cos.shape == sin.shape and cos.dtype == sin.dtype and cos.device == sin.device)
        if not (same and cos.ndim == 2 and cos.numel() > 0 and cos.dtype in (torch.float32, torch.float64)):
            raise ConfigurationError(f"RopeTable: cos {tuple(cos.shape)} {cos.dtype} and sin {tuple(sin.shape)} "
                                     f"{sin.dtype} must be equal non-empty 2-D float32/float64 tensors on one device")
        rows, pairs = cos.shape
        if self.sections is None:
            if self.section_rows is not None:
                raise ConfigurationError("RopeTable: section_rows describes a separable table; give sections too")
            return
        sections = tuple(self.sections)
        if not (len(sections) == 3 and all(_nonnegative(v) for v in sections) and sum(sections) == pairs):
            raise ConfigurationError(f"RopeTable: sections {sections} must be three pair counts adding up to {pairs}")
        lengths = (rows,) * 3 if self.section_rows is None else tuple(self.section_rows)
        if not (len(lengths) == 3 and all(_nonnegative(v) and v <= rows for v in lengths)):
            raise ConfigurationError(f"RopeTable: section_rows {lengths} must be three counts of at most {rows}")
        object.__setattr__(self, "sections", sections)
        object.__setattr__(self, "section_rows", lengths)

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
        """From unit complex rotations ``[rows, head_dim // 2]`` (``sections="wan"``: the Wan 3-axis split)."""
        freqs = _require_tensor(freqs, "freqs")
        if not (freqs.is_complex() and freqs.ndim == 2):
            raise ConfigurationError(f"freqs: expected a 2-D complex tensor, got {tuple(freqs.shape)} {freqs.dtype}")
        parts = torch.view_as_real(freqs.resolve_conj())
        real_dtype = torch.float64 if freqs.dtype == torch.complex128 else torch.float32
        if sections == "wan":
            sections = wan_sections(freqs.shape[1])
        return cls(parts[..., 0].to(real_dtype).contiguous(), parts[..., 1].to(real_dtype).contiguous(), sections)

    @classmethod
    def from_axes(cls, temporal, height, width):
        """Separable table from per-axis complex rotations ``[positions, pairs]`` (frame, row, column)."""
        axes = [_require_tensor(v, "axis rotations") for v in (temporal, height, width)]
        if not all(v.is_complex() and v.ndim == 2 for v in axes):
            raise ConfigurationError("from_axes: each axis is a 2-D complex tensor [positions, pairs]")
        real_dtype = torch.float64 if all(v.dtype == torch.complex128 for v in axes) else torch.float32
        pairs = []
        for v in axes:
            parts = torch.view_as_real(v.resolve_conj()).to(real_dtype)
            pairs.append((parts[..., 0], parts[..., 1]))
        cos, sin, widths, lengths = _separable(None, cos_sin=pairs)
        return cls(cos, sin, widths, lengths)

    @classmethod
    def from_cos_sin(cls, cos, sin, sections=None):
        return cls(cos, sin, sections)

    @classmethod
    def wan(cls, head_dim, max_positions=1024, *, theta=10000.0, device="cpu"):
        """Wan / causal-Wan tables in FP64: axis ``a`` of rotary dim ``d_a`` turns pair ``j`` by
        ``position / theta ** (2 j / d_a)``; every axis has ``max_positions`` rows."""
        _int(head_dim, "head_dim", minimum=8)
        position = torch.arange(max_positions, dtype=torch.float64)
        angles = [torch.outer(position, 1.0 / theta ** (torch.arange(0, d, 2, dtype=torch.float64) / d))
                  for d in _axis_dims(head_dim)]
        joined = torch.cat(angles, dim=1)
        return cls(joined.cos().to(device), joined.sin().to(device), tuple(a.shape[1] for a in angles))

    @classmethod
    def longcat(cls, head_dim, num_frames, height, width, *, base=10000.0, device="cpu"):
        """LongCat-Video 3-D tables, computed in FP32 as its ``rope_3d`` does, one axis per grid extent."""
        _int(head_dim, "head_dim", minimum=8)
        if head_dim % 8:
            raise ConfigurationError(f"LongCat RoPE: head_dim {head_dim} is not a multiple of 8")
        angles = []
        for d, extent in zip(_axis_dims(head_dim), (num_frames, height, width)):
            _int(extent, "grid extent", minimum=1)
            frequency = 1.0 / (base ** (torch.arange(0, d, 2)[:d // 2].float() / d))
            angles.append(torch.outer(torch.arange(extent, dtype=torch.float32), frequency))
        cos, sin, widths, lengths = _separable(angles)
        return cls(cos.to(device), sin.to(device), widths, lengths)

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


# ---------------------------------------------------------------------------------------------
# Completion handle
# ---------------------------------------------------------------------------------------------

class _Graveyard:
    """Keepalives of handles dropped before their GPU work finished: each stays referenced until its event
    completes, so no tensor a queued kernel reads is freed under it. Swept on every restore call."""

    def __init__(self):
        self._lock = threading.RLock()
        self._entries: list = []

    def bury(self, event, refs) -> None:
        with self._lock:
            self._entries.append((event, refs))

    def sweep(self) -> None:
        with self._lock:
            self._entries = [(event, refs) for event, refs in self._entries if not event.query()]

    def __len__(self) -> int:
        with self._lock:
            return len(self._entries)


_GRAVEYARD = _Graveyard()


def _sweep_deferred():
    _GRAVEYARD.sweep()


def pending_deferred():
    """Number of dropped handles whose GPU work has not been seen to finish."""
    return len(_GRAVEYARD)


class RestoreHandle:
    """What one :func:`reconstruct` call returns: the event recorded after its last write on ``stream`` and
    the references that keep its inputs and temporaries alive. :meth:`release` waits for the event and drops
    them; a handle dropped without release hands them to the graveyard until the event completes.
    ``stats``: jobs, launches, FLOPs, backend and precision of the call."""

    def __init__(self, *, event, stream, keepalive, stats):
        self._event, self._stream, self._keepalive = event, stream, keepalive
        self._released = False
        self.stats = stats

    event = property(lambda self: self._event)
    stream = property(lambda self: self._stream)
    released = property(lambda self: self._released)

    def query(self):
        """True once every write of the call has finished (always True on the host path)."""
        return self._event.query() if self._event is not None else True

    def synchronize(self):
        if self._event is not None:
            self._event.synchronize()

    def wait(self, stream=None):
        """Order ``stream`` (default: the current stream of the call's device) after the call's writes."""
        if self._event is not None:
            (stream or torch.cuda.current_stream(self._stream.device)).wait_event(self._event)

    def release(self):
        if not self._released:
            self.synchronize()
            self._keepalive, self._released = None, True
            _GRAVEYARD.sweep()

    def __del__(self):
        try:
            unfinished = self._event is not None and self._keepalive is not None and not self._event.query()
            if not self._released and unfinished:
                _GRAVEYARD.bury(self._event, self._keepalive)
        except Exception:  # noqa: BLE001 -- torch may already be torn down at interpreter exit
            pass


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
    """``reference`` for host jobs (or on request); ``fused`` for CUDA jobs, which needs the native
    extension: a missing library raises (naming it) instead of quietly running the host math."""
    if backend == "reference" or (backend == "auto" and not cuda):
        return "reference"
    if not cuda:
        raise UnsupportedError(f"backend {backend!r} runs CUDA jobs only; these are on the host")
    from .ops._ext import ext

    ext()
    return "fused"


def _resolve_precision(precision, backend):
    if precision != "auto" and precision not in PRECISIONS:
        raise ConfigurationError(f"precision {precision!r}: expected 'auto' or one of {PRECISIONS}")
    # "auto" is the two-product split for every destination dtype: its bound does not grow with the
    # cancellation inside sum_k a_k q_k, while a single FP16 product's does.
    resolved = DEFAULT_PRECISION if precision == "auto" else precision
    if backend == "fused" and resolved not in KERNEL_PRECISIONS:
        raise UnsupportedError(f"the sm_100a restore kernel computes {KERNEL_PRECISIONS}; {resolved!r} is "
                               f"available with backend='reference'")
    return resolved


def _launch_fused(jobs, device, precision, stream, keepalive):
    """Launch factorized jobs in groups of ``MAX_JOBS_PER_LAUNCH`` and dense ones in groups of
    ``MAX_DENSE_JOBS_PER_LAUNCH``; returns the number of launches."""
    factor = [job for job in jobs if not isinstance(job.source, DenseSource)]
    dense = [job for job in jobs if isinstance(job.source, DenseSource)]
    launches = 0
    for first in range(0, len(factor), MAX_JOBS_PER_LAUNCH):
        launches += _fused_factor_group(factor[first:first + MAX_JOBS_PER_LAUNCH], device, precision, stream,
                                        keepalive)
    for first in range(0, len(dense), MAX_DENSE_JOBS_PER_LAUNCH):
        launches += _fused_dense_group(dense[first:first + MAX_DENSE_JOBS_PER_LAUNCH], device, stream, keepalive)
    return launches


def reconstruct(jobs, *, backend="auto", precision="auto", stream=None, wait_events=(), native_rope=None,
                native_rope_dtype=None, compute_dtype=torch.float64, stage_events=None, config=None):
    """Write every job's restored matrix into its native cache slot; returns a :class:`RestoreHandle`.

    Pass all restored chunks of a layer (its K and V) in one call: the fused backend issues one persistent
    launch per ``MAX_JOBS_PER_LAUNCH`` factorized jobs and per ``MAX_DENSE_JOBS_PER_LAUNCH`` dense ones.
    The work is queued on ``stream`` (default: the device's current stream) after ``wait_events``.
    ``native_rope(pre_rope [N, H, D], job)``, when given, rotates RoPE jobs with the engine's own function
    instead of the kernel's tables (those jobs reconstruct into scratch first). ``stage_events``, a list,
    receives ``("start", event)`` and ``("fused", event)`` timing events around the launches.
    """
    _GRAVEYARD.sweep()
    jobs, device = _validate(jobs)
    if backend not in BACKENDS:
        raise ConfigurationError(f"backend {backend!r}: expected one of {BACKENDS}")
    if native_rope is not None and not callable(native_rope):
        raise ConfigurationError("native_rope must be a callable (pre_rope, job) -> tensor")
    stats = {"jobs": len(jobs), "matrices": len(jobs), "flops": _matrix_flops(jobs), "launches": 0}
    if not jobs:
        return RestoreHandle(event=None, stream=None, keepalive=None,
                             stats={**stats, "backend": "none", "precision": None})
    cuda = device.type == "cuda"
    backend = _resolve_backend(backend, cuda)
    precision = _resolve_precision(precision, backend)
    if not cuda:
        if stream is not None or wait_events:
            raise ConfigurationError("host jobs run synchronously: pass no stream and no wait_events")
    else:
        stream = stream if stream is not None else torch.cuda.current_stream(device)
        if not (isinstance(stream, torch.cuda.Stream) and stream.device == device):
            raise ConfigurationError(f"stream must be a torch.cuda.Stream of {device}")
        for event in wait_events:
            stream.wait_event(event)
    keepalive = [tensor for job in jobs for tensor in job.tensors()]
    stats["backend"] = backend
    stats["precision"] = str(compute_dtype) if backend == "reference" else precision

    def mark(name):
        if stage_events is not None and cuda:
            event = torch.cuda.Event(enable_timing=True)
            event.record(stream)
            stage_events.append((name, event))

    mark("start")
    if backend == "reference":
        with torch.cuda.stream(stream) if cuda else _null():
            reconstruct_reference(jobs, compute_dtype=compute_dtype, native_rope=native_rope,
                                  native_rope_dtype=native_rope_dtype)
    else:
        by_engine = [native_rope is not None and job.rope is not None for job in jobs]
        engine_rope = [job for job, engine in zip(jobs, by_engine) if engine]
        try:
            stats["launches"] += _launch_fused([job for job, engine in zip(jobs, by_engine) if not engine], device,
                                               precision, stream, keepalive)
            if engine_rope:
                stats["launches"] += _native_rope_jobs(engine_rope, native_rope, native_rope_dtype, precision,
                                                       device, stream, keepalive)
        except BaseException:
            # kernels of earlier groups may still read the inputs: keep them until the stream passes here
            failed = torch.cuda.Event()
            failed.record(stream)
            _GRAVEYARD.bury(failed, keepalive)
            raise
    mark("fused")
    event = None
    if cuda:
        event = torch.cuda.Event()
        event.record(stream)
    return RestoreHandle(event=event, stream=stream, keepalive=keepalive, stats=stats)


def _native_rope_jobs(jobs, native_rope, native_rope_dtype, precision, device, stream, keepalive):
    """RoPE jobs rotated by the engine: reconstruct each without rotation into a ``[T, H, D]`` scratch (a
    dense source already in the scratch dtype is used as it is), then write ``native_rope(scratch, job)``
    into the slot."""
    staged, rotations = [], []
    for job in jobs:
        view = job.destination
        dtype = native_rope_dtype or view.tensor.dtype
        if isinstance(job.source, DenseSource) and job.source.values.dtype == dtype:
            rotations.append((job, job.source.values.reshape(job.tokens, view.heads, view.head_dim)))
            continue
        with torch.cuda.stream(stream):
            scratch = torch.empty((job.tokens, view.heads, view.head_dim), dtype=dtype, device=device)
        keepalive.append(scratch)
        staged.append(ReconstructionJob(job.source, NativeView(scratch, "THD"), job.grid, job.basis, job.rank,
                                        None, job.label, job.basis_t))
        rotations.append((job, scratch))
    launches = _launch_fused(staged, device, precision, stream, keepalive)
    with torch.cuda.stream(stream):
        for job, pre in rotations:
            rotated = native_rope(pre, job)
            if not isinstance(rotated, torch.Tensor) or rotated.numel() != pre.numel():
                raise IntegrityError(f"native_rope returned {getattr(rotated, 'shape', type(rotated))} for a "
                                     f"{tuple(pre.shape)} input")
            job.destination.slot(job.tokens).copy_(rotated.reshape(pre.shape))
            keepalive.append(rotated)
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
        for name, value, allowed in (("dtype", self.dtype, OUTPUT_DTYPES), ("layout", self.layout, LAYOUTS),
                                     ("source", self.source, WARMUP_SOURCES), ("rope", self.rope, WARMUP_ROPE_MODES)):
            if value not in allowed:
                raise ConfigurationError(f"WarmupShape.{name}={value!r}: expected one of {tuple(allowed)}")


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
