"""Launch plumbing of the fused sm_100a restore (csrc/restore/{unpack,prep,restore_sm100}.cu).

A launch group of factorized jobs runs as three kernels on the execution stream:

1. ``unpack``: 8-bit coefficients (mosaic pictures or a dense uint8 matrix) -> A = centered FP16
   pixels ``p - 128`` ``[N, K_pad]`` (exact), zero beyond the rank;
2. ``prep``: per job, Bt = FP16 hi/lo split of ``s[k] * Q[k, c] * 2^e`` ``[C, 2 K_pad]`` and the
   per-channel bias ``sum_k (o[k] + 128 s[k]) Q[k, c]`` (FP64 accumulation);
3. ``restore``: persistent TMA -> tcgen05 GEMM ``acc = A @ Bt^T`` (two FP16 products), epilogue
   ``acc * 2^-e + bias``, RoPE, cast, strided store into the native slots.

Float coefficient sources take A = FP16 hi/lo split of ``P * 2^e`` ``[N, 2 K_pad]`` against the plain
transposed basis ``[C, K_pad]`` (no bias). Scratch operands come from the caching allocator on the
execution stream and are kept alive by the caller's handle.
"""

from __future__ import annotations

import math
import struct

import numpy as np
import torch

from ..errors import ConfigurationError
from ._ext import ext, status_word

_OUT_CODE = {torch.bfloat16: 0, torch.float16: 1, torch.float32: 2}
_COLUMN_TABLES: dict = {}


def k_pad_of(rank: int) -> int:
    return (rank + 63) // 64 * 64


def column_tables(layout, plane_stride, row_stride, k_pad):
    """``(col_off, col_seg)`` int32 ``[k_pad]`` of a channel-tile layout: byte offset of each rank
    column's mosaic cell inside a picture (-1 beyond the rank) and its segment."""
    key = (layout["rank"], layout["planes"], tuple(layout["grid"]), layout["height"], layout["width"],
           layout["channels_per_segment"], plane_stride, row_stride, k_pad)
    hit = _COLUMN_TABLES.get(key)
    if hit is not None:
        return hit
    rank, planes = layout["rank"], layout["planes"]
    columns = layout["grid"][0]
    slots = layout["channels_per_segment"]
    k = np.arange(k_pad, dtype=np.int64)
    seg = k // slots
    cell = k - seg * slots
    plane = cell % planes
    cell //= planes
    off = plane * plane_stride + (cell // columns) * layout["height"] * row_stride + (cell % columns) * layout["width"]
    off = np.where(k < rank, off, -1)
    if off.max() >= 2 ** 31:
        raise ConfigurationError("picture planes exceed the unpack kernel's 32-bit cell offsets")
    hit = (off.astype(np.int32), np.where(k < rank, seg, 0).astype(np.int32))
    if len(_COLUMN_TABLES) > 1024:
        _COLUMN_TABLES.clear()
    _COLUMN_TABLES[key] = hit
    return hit


def prescale_exponent(bound: float) -> int:
    """Exponent e bringing ``bound * 2^e`` into (2^13, 2^14] (0 for a zero bound), clamped to +-100."""
    if not bound > 0 or not math.isfinite(bound):
        return 0
    return int(min(max(14 - math.ceil(math.log2(max(bound, 1e-30))), -100), 100))


class HostArena:
    """Pinned host staging of per-call device tables, uploaded with one copy on the stream."""

    def __init__(self):
        self.parts = []
        self.size = 0

    def add(self, array) -> int:
        array = np.ascontiguousarray(array)
        start = (self.size + 15) // 16 * 16
        self.parts.append((start, array))
        self.size = start + array.nbytes
        return start

    def upload(self, device, stream):
        host = torch.empty(max(self.size, 16), dtype=torch.uint8, pin_memory=True)
        view = host.numpy()
        for start, array in self.parts:
            view[start:start + array.nbytes] = np.frombuffer(array.tobytes(), dtype=np.uint8)
        with torch.cuda.stream(stream):
            dev = torch.empty(host.shape, dtype=torch.uint8, device=device)
            dev.copy_(host, non_blocking=True)
        return host, dev


_QMAX_CACHE: dict = {}


def basis_max_abs(basis: torch.Tensor) -> float:
    """max |Q| of a basis tensor (cached per tensor state; one device reduction per new basis)."""
    key = (basis.data_ptr(), tuple(basis.shape), basis.stride(), None if basis.is_inference() else basis._version)
    hit = _QMAX_CACHE.get(key)
    if hit is None:
        hit = float(basis.abs().amax().item())
        if len(_QMAX_CACHE) > 4096:
            _QMAX_CACHE.clear()
        _QMAX_CACHE[key] = hit
    return hit


def launch_factor_group(items, device, precision, stream, keepalive):
    """Run one fused restore over ``items``: dicts with keys ``kind`` ("pictures" | "u8" | "f32"),
    ``tokens``, ``rank``, ``grid`` (frames, height, width), ``basis`` (FP16 [R, C]), ``basis_t``
    (optional FP16 [C, k_pad]), ``qmax`` (optional), ``scale``/``offset`` (host float32 [rank]),
    ``dest`` (address, (ts, hs, ds), dtype, channels, head_dim), ``rope`` (8 ints + cos/sin pointers)
    and the source (``pictures`` (addresses, plane_stride, row_stride, layout) | ``values``).
    Returns the number of kernel launches."""
    passes = 2 if precision in ("fp16x2",) else 1
    arena = HostArena()
    unpack_rows, prep_rows = [], []
    a_ops, b_ops, inverse, rows = [], [], [], []
    sizes = []  # (a_elems, b_elems, bias_elems) of scratch per item
    plan = []
    for item in items:
        rank, tokens = item["rank"], item["tokens"]
        k_pad = k_pad_of(rank)
        channels = item["dest"][3]
        if item["kind"] == "f32":
            a_elems, b_elems, bias_elems = tokens * 2 * k_pad, 0, channels
        else:
            a_elems, b_elems, bias_elems = tokens * k_pad, channels * 2 * k_pad, channels
        plan.append((k_pad, a_elems, b_elems, bias_elems))
    # one scratch allocation: FP16 operands then FP32 biases (each slice 256-byte aligned)
    offsets = []
    cursor = 0
    for k_pad, a_elems, b_elems, bias_elems in plan:
        a_off = cursor
        cursor += (a_elems * 2 + 255) // 256 * 256
        b_off = cursor
        cursor += (b_elems * 2 + 255) // 256 * 256
        bias_off = cursor
        cursor += (bias_elems * 4 + 255) // 256 * 256
        offsets.append((a_off, b_off, bias_off))
    with torch.cuda.stream(stream):
        scratch = torch.empty(max(cursor, 256), dtype=torch.uint8, device=device)
    keepalive.append(scratch)
    base_scratch = scratch.data_ptr()
    pending_unpack = []
    pending_prep = []
    for item, (k_pad, a_elems, b_elems, bias_elems), (a_off, b_off, bias_off) in zip(items, plan, offsets):
        rank, tokens, channels = item["rank"], item["tokens"], item["dest"][3]
        bias_view = scratch[bias_off:bias_off + bias_elems * 4].view(torch.float32)
        if item["kind"] == "f32":
            values = item["values"]
            bound = item.get("bound")
            with torch.cuda.stream(stream):
                if bound is None:
                    bound = float(values[:, :rank].abs().amax().item())
                e = prescale_exponent(bound)
                a = scratch[a_off:a_off + a_elems * 2].view(torch.float16).view(tokens, 2 * k_pad)
                a.zero_()
                scaled = values[:, :rank].float() * (2.0 ** e)
                hi = scaled.half()
                a[:, :rank] = hi
                a[:, k_pad:k_pad + rank] = (scaled - hi.float()).half()
                bias_view.zero_()
                b = item.get("basis_t")
                if b is None:
                    from ..restore_kernels import transposed_basis
                    b = transposed_basis(item["basis"])
            keepalive.append(b)
            if b.shape[1] != k_pad:
                b = b[:, :k_pad]
        else:
            qmax = item.get("qmax")
            if qmax is None:
                qmax = basis_max_abs(item["basis"])
            smax = float(np.abs(item["scale"]).max(initial=0.0))
            e = prescale_exponent(smax * qmax)
            a = scratch[a_off:a_off + a_elems * 2].view(torch.float16).view(tokens, k_pad)
            b = scratch[b_off:b_off + b_elems * 2].view(torch.float16).view(channels, 2 * k_pad)
            if item["kind"] == "pictures":
                addresses, plane_stride, row_stride, layout = item["pictures"]
                col_off, col_seg = column_tables(layout, plane_stride, row_stride, k_pad)
                frames, height, width = item["grid"]
                pending_unpack.append([arena.add(addresses), arena.add(col_off), arena.add(col_seg), 0, a.data_ptr(),
                                       row_stride, tokens, k_pad, rank, frames, height, width])
            else:
                values = item["values"]
                frames, height, width = item["grid"]
                pending_unpack.append([-1, -1, -1, values.data_ptr(), a.data_ptr(), values.stride(0), tokens, k_pad,
                                       rank, frames, height, width])
            basis = item["basis"]
            scale_off = arena.add(np.ascontiguousarray(item["scale"][:rank], dtype=np.float32))
            offset_off = arena.add(np.ascontiguousarray(item["offset"][:rank], dtype=np.float32))
            bits = struct.unpack("<I", struct.pack("<f", float(2.0 ** e)))[0]
            pending_prep.append([basis.data_ptr(), scale_off, offset_off, b.data_ptr(), bias_view.data_ptr(),
                                 basis.stride(0), rank, k_pad, channels, bits])
            keepalive.append(basis)
        address, (ts, hs, ds), dtype, channels, head_dim = item["dest"]
        rope = item["rope"]
        row = [0] * 40
        row[0] = address
        row[1] = bias_view.data_ptr()
        row[2], row[3] = rope[8], rope[9]
        row[4], row[5], row[6] = ts, hs, ds
        row[7] = tokens
        row[8] = passes
        row[9], row[10], row[11] = item["grid"]
        row[12] = _OUT_CODE[dtype]
        row[13] = channels
        row[14] = head_dim
        row[15:23] = list(rope[:8])
        rows.append(row)
        a_ops.append(a)
        b_ops.append(b)
        inverse.append(2.0 ** -e)
    launches = 0
    if pending_unpack or pending_prep:
        host, dev = arena.upload(device, stream)
        keepalive.extend((host, dev))
        base = dev.data_ptr()
        for row in pending_unpack:
            for index in (0, 1, 2):
                row[index] = 0 if row[index] < 0 else row[index] + base
        for row in pending_prep:
            row[1] += base
            row[2] += base
        with torch.cuda.stream(stream):
            if pending_unpack:
                ext().unpack_launch(torch.tensor(pending_unpack, dtype=torch.int64), device.index)
                launches += 1
            if pending_prep:
                ext().prep_launch(torch.tensor(pending_prep, dtype=torch.int64), device.index)
                launches += 1
    with torch.cuda.stream(stream):
        ext().restore_launch(torch.tensor(rows, dtype=torch.int64), a_ops, b_ops,
                             torch.tensor(inverse, dtype=torch.float32), status_word(device))
    return launches + 1
