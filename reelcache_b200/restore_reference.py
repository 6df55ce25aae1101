"""Plain-torch reference of the restore and its documented error bounds.

The reference backend computes what a restore writes in FP64 (or FP32) with ordinary torch operations; the
bounds say how far a fused kernel's output may lie from it, elementwise. The bound's first-order form follows
the reference implementation's analysis (reelcache/restore_kernels.py:1176-1230): the output rounding
``u_out |y*|``, plus ``(1 + u_out)`` times the GEMM error ``gamma(precision, rank) * S`` with
``S = sum_k |a_k| |q_k|`` (per element, rotated like the values for K), plus ``2^-21 (|y_e| + |y_o|)`` for the
rotation of each interleaved pair, plus a floor below which the destination type cannot resolve anything.
"""

from __future__ import annotations

from collections.abc import Sequence

import numpy as np
import torch

from .errors import ConfigurationError, IntegrityError
from .restore_jobs import CoefficientSource, DenseSource, PictureSource, ReconstructionJob

UNIT_ROUNDOFF = {torch.bfloat16: 2.0 ** -8, torch.float16: 2.0 ** -11, torch.float32: 2.0 ** -24}
OUTPUT_FLOOR = {torch.bfloat16: 2.0 ** -134, torch.float16: 2.0 ** -25, torch.float32: 2.0 ** -150}
_ROTATION_ERROR = 2.0 ** -21
# (leading relative error of the products, number of accumulations charged at 2^-24 per term)
_PRODUCTS = {"fp32": (0.0, 1), "tf32": (2.0 ** -10, 1), "tf32x3": (2.0 ** -20, 3), "fp16": (2.0 ** -11, 1),
             "fp16x2": (2.0 ** -21, 2), "bf16": (2.0 ** -7 + 2.0 ** -16, 1), "reference32": (0.0, 1)}


def gemm_gamma(precision: str, rank: int) -> float:
    """Relative GEMM error per unit of ``sum_k |a_k| |q_k|`` in a precision mode."""
    lead, passes = _PRODUCTS[precision]
    return lead + passes * (rank + 1) * 2.0 ** -24


# -------------------------------------------------------------------------------------------------------------
# Validation shared by every backend
# -------------------------------------------------------------------------------------------------------------

def _storage(tensor):
    try:
        return tensor.untyped_storage().data_ptr(), tensor.device
    except (RuntimeError, NotImplementedError):
        return tensor.data_ptr(), tensor.device


def check_disjoint(jobs) -> None:
    """Jobs that write overlapping tokens of one destination view would race: reject them."""
    by_view: dict = {}
    for index, job in enumerate(jobs):
        view = job.destination
        t = view.tensor
        key = (*_storage(t), t.storage_offset(), tuple(t.shape), t.stride(), view.layout, view.batch_index)
        by_view.setdefault(key, []).append((view.token_offset, view.token_offset + job.tokens, index))
    for spans in by_view.values():
        spans.sort()
        for (_, end, first), (start, _, second) in zip(spans, spans[1:]):
            if start < end:
                raise ConfigurationError(f"jobs {first} and {second} write the same destination tokens")


def validate_jobs(jobs):
    """``(jobs tuple, device)`` after checking every job shares one device and no two writes overlap."""
    if isinstance(jobs, ReconstructionJob):
        jobs = (jobs,)
    if isinstance(jobs, (str, bytes)) or not isinstance(jobs, Sequence):
        raise ConfigurationError("jobs are a sequence of ReconstructionJob")
    jobs = tuple(jobs)
    if not all(isinstance(job, ReconstructionJob) for job in jobs):
        raise ConfigurationError("jobs are ReconstructionJob instances")
    devices = set()
    for job in jobs:
        source = job.source
        devices.add(job.destination.tensor.device)
        devices.add(source.device if isinstance(source, PictureSource) else source.values.device)
        if job.basis is not None:
            devices.add(job.basis.device)
    if len(devices) > 1:
        raise ConfigurationError(f"the jobs' tensors span devices {sorted(map(str, devices))}")
    check_disjoint(jobs)
    return jobs, next(iter(devices), None)


# -------------------------------------------------------------------------------------------------------------
# Coefficients and rotation
# -------------------------------------------------------------------------------------------------------------

def unpack_pictures(source: PictureSource) -> torch.Tensor:
    """The 8-bit coefficients ``[N, rank]`` of a picture source: column ``k`` of segment
    ``k // channels_per_segment`` lives in cell ``i = k % channels_per_segment`` -- plane ``i % planes``, grid
    cell ``divmod(i // planes, grid_columns)`` -- of each frame's picture."""
    lay = source.layout
    frames, height, width, rank = lay["frames"], lay["height"], lay["width"], lay["rank"]
    grid_columns = lay["grid"][0]
    planes, slots = lay["planes"], lay["channels_per_segment"]
    device = source.device
    cells = torch.arange(slots, device=device)
    plane_of = cells % planes
    grid_row, grid_col = torch.div(cells // planes, grid_columns, rounding_mode="floor"), (cells // planes) % grid_columns
    ys = torch.arange(height, device=device)
    xs = torch.arange(width, device=device)
    out = torch.empty((frames, height, width, rank), dtype=torch.uint8, device=device)
    for segment, pictures in enumerate(source.pictures):
        first = segment * slots
        used = min(slots, rank - first)
        p = plane_of[:used, None, None]
        r = (grid_row[:used] * height)[:, None, None] + ys[None, :, None]
        c = (grid_col[:used] * width)[:, None, None] + xs[None, None, :]
        for frame, picture in enumerate(pictures):
            out[frame, :, :, first:first + used] = picture[p, r, c].permute(1, 2, 0)
    return out.reshape(-1, rank)


def dequantize(pixels, scale, offset):
    """``float(pixel) * scale + offset``, rounded after the product and after the sum (no fused multiply-add)."""
    s = torch.from_numpy(np.ascontiguousarray(scale)).to(pixels.device)
    o = torch.from_numpy(np.ascontiguousarray(offset)).to(pixels.device)
    scaled = pixels.float() * s
    return scaled + o


def reference_coefficients(job) -> torch.Tensor:
    """The FP32 coefficient matrix ``[N, rank]`` a job reconstructs from."""
    source = job.source
    if isinstance(source, PictureSource):
        return dequantize(unpack_pictures(source), source.scale, source.offset)
    if isinstance(source, CoefficientSource):
        columns = source.values[:, :job.rank]
        if source.quantized:
            return dequantize(columns, source.scale[:job.rank], source.offset[:job.rank])
        return columns.float()
    raise ConfigurationError("a dense source has no coefficients")


def rope_cos_sin(positions, grid, *, dtype=torch.float64, device=None):
    """Per-token ``(cos, sin)`` ``[N, head_dim // 2]`` of a chunk at ``positions``: in a separable table pair
    ``j`` of the token at (frame, row, column) reads the row of its axis section, offset by the chunk's start."""
    table = positions.table
    device = table.cos.device if device is None else device
    cos = table.cos.to(device=device, dtype=dtype)
    sin = table.sin.to(device=device, dtype=dtype)
    frames, height, width = grid
    tokens = frames * height * width
    if table.sections is None:
        start = positions.rows
        return cos[start:start + tokens], sin[start:start + tokens]
    token = torch.arange(tokens, device=device)
    coords = torch.stack((token // (height * width), (token // width) % height, token % width))   # [3, N]
    axis_of_pair = torch.repeat_interleave(torch.arange(3, device=device),
                                           torch.tensor(table.sections, device=device))
    starts = torch.tensor(positions.rows, device=device)[axis_of_pair]                            # [pairs]
    rows = coords[axis_of_pair].t() + starts                                                      # [N, pairs]
    return torch.gather(cos, 0, rows), torch.gather(sin, 0, rows)


def apply_rope_reference(values, positions, grid, *, dtype=torch.float64):
    """``values[N, H, D]`` with every interleaved pair ``(2j, 2j + 1)`` rotated as the complex number
    ``x_2j + i x_2j+1`` times ``cos + i sin`` (computed in ``dtype``)."""
    cos, sin = rope_cos_sin(positions, grid, dtype=dtype, device=values.device)
    x = values.to(dtype)
    pairs = x.reshape(*x.shape[:-1], -1, 2)
    even, odd = pairs[..., 0], pairs[..., 1]
    c, s = cos[:, None, :], sin[:, None, :]
    return torch.stack((even * c - odd * s, even * s + odd * c), dim=-1).reshape(x.shape)


# -------------------------------------------------------------------------------------------------------------
# Reference restore
# -------------------------------------------------------------------------------------------------------------

def _pre_rope(job, compute):
    if isinstance(job.source, DenseSource):
        return job.source.values
    coefficients = reference_coefficients(job)
    basis = job.basis[:job.rank].to(device=coefficients.device, dtype=compute)
    return coefficients.to(compute) @ basis


def _restore_one(job, compute, native_rope, native_rope_dtype):
    heads, head_dim, tokens = job.destination.heads, job.destination.head_dim, job.tokens
    slot = job.destination.slot(tokens)
    values = _pre_rope(job, compute)
    if job.rope is not None and native_rope is not None:
        rotated = native_rope(values.to(native_rope_dtype or slot.dtype).reshape(tokens, heads, head_dim), job)
        if not isinstance(rotated, torch.Tensor) or rotated.numel() != tokens * heads * head_dim:
            raise IntegrityError("the native RoPE callable returned a tensor of another size")
        slot.copy_(rotated.reshape(tokens, heads, head_dim))
        return
    values = values.reshape(tokens, heads, head_dim)
    if job.rope is not None:
        values = apply_rope_reference(values, job.rope, job.grid, dtype=compute)
    slot.copy_(values)


def reconstruct_reference(jobs, *, compute_dtype=torch.float64, native_rope=None, native_rope_dtype=None):
    """The plain-torch restore: FP64 (default) or FP32 arithmetic, one cast into each slot."""
    jobs, _ = validate_jobs(jobs)
    if compute_dtype not in (torch.float32, torch.float64):
        raise ConfigurationError(f"the reference computes in float32 or float64, not {compute_dtype}")
    with torch.no_grad():
        for job in jobs:
            _restore_one(job, compute_dtype, native_rope, native_rope_dtype)


# -------------------------------------------------------------------------------------------------------------
# Error bounds
# -------------------------------------------------------------------------------------------------------------

def _rotate_magnitude(magnitude: torch.Tensor, tokens: int) -> torch.Tensor:
    """A rotation mixes each pair: both outputs are charged the sum of the pair's magnitudes."""
    pairs = magnitude.reshape(tokens, -1, 2)
    return pairs.sum(dim=-1).repeat_interleave(2, dim=-1)


def reference_values(job):
    """``(y*, S)`` in FP64: the values a job writes before the final cast, and ``sum_k |p_k| |q_k|``."""
    tokens, heads, head_dim = job.tokens, job.destination.heads, job.destination.head_dim
    if isinstance(job.source, DenseSource):
        values = job.source.values.double()
        magnitude = torch.zeros_like(values)
    else:
        p = reference_coefficients(job).double()
        q = job.basis[:job.rank].to(device=p.device, dtype=torch.float64)
        values, magnitude = p @ q, p.abs() @ q.abs()
    if job.rope is not None:
        values = apply_rope_reference(values.reshape(tokens, heads, head_dim), job.rope, job.grid).reshape(tokens, -1)
        magnitude = _rotate_magnitude(magnitude, tokens)
    return values, magnitude


def _assemble_bound(job, values, magnitude, precision, out_dtype):
    out_dtype = job.destination.tensor.dtype if out_dtype is None else out_dtype
    u = UNIT_ROUNDOFF[out_dtype]
    gemm = gemm_gamma(precision, job.rank or 0) * magnitude
    if job.rope is not None:
        gemm = gemm + _ROTATION_ERROR * _rotate_magnitude(values.abs(), job.tokens)
    return values, u * values.abs() + (1 + u) * gemm + OUTPUT_FLOOR[out_dtype]


def error_bound(job, precision, out_dtype=None):
    """``(y*, bound)`` in FP64: the elementwise bound on ``|written - y*|`` of a restore in ``precision``."""
    values, magnitude = reference_values(job)
    return _assemble_bound(job, values, magnitude, precision, out_dtype)


def kernel_error_bound(job, precision="fp16x2", out_dtype=None):
    """The fused sm_100a kernel's bound. For 8-bit sources the kernel multiplies the exact centered pixel
    ``p - 128`` by the FP16 split of ``s_k Q[k, c]`` and adds the bias ``sum_k (o_k + 128 s_k) Q[k, c]``, so its
    rounding is charged to ``S' = sum_k (|a_k| + |o_k + 128 s_k|) |q_k|`` (``a_k`` the dequantized
    coefficient); float sources keep ``S``."""
    values, magnitude = reference_values(job)
    source = job.source
    eight_bit = isinstance(source, PictureSource) or (isinstance(source, CoefficientSource) and source.quantized)
    if eight_bit:
        scale = np.asarray(source.scale[:job.rank], dtype=np.float64)
        offset = np.asarray(source.offset[:job.rank], dtype=np.float64)
        shift = torch.from_numpy(np.abs(offset + 128.0 * scale)).to(magnitude.device)
        q = job.basis[:job.rank].to(device=magnitude.device, dtype=torch.float64).abs()
        extra = (shift @ q).expand(job.tokens, -1)
        if job.rope is not None:
            extra = _rotate_magnitude(extra.contiguous(), job.tokens)
        magnitude = magnitude + extra
    return _assemble_bound(job, values, magnitude, precision, out_dtype)


__all__ = ["OUTPUT_FLOOR", "UNIT_ROUNDOFF", "apply_rope_reference", "check_disjoint", "dequantize", "error_bound",
           "gemm_gamma", "kernel_error_bound", "reconstruct_reference", "reference_coefficients", "reference_values",
           "rope_cos_sin", "unpack_pictures", "validate_jobs"]
