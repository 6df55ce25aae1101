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
