"""Launch plumbing of the fused sm_100a restore (csrc/restore/{unpack,prep,restore_sm100}.cu).

A set of factorized jobs runs as three kernels on the execution stream:

1. ``unpack``: 8-bit coefficients (mosaic pictures or a dense uint8 matrix) -> A = centered FP16
   pixels ``p - 128`` ``[N, K_pad]`` (exact), zero beyond the rank;
2. ``prep``: per job, Bt = FP16 hi/lo split of ``s[k] * Q[k, c] * 2^e`` ``[C, 2 K_pad]`` and the
   per-channel bias ``sum_k (o[k] + 128 s[k]) Q[k, c]`` (FP64 accumulation);
3. ``restore``: persistent TMA -> tcgen05 GEMM ``acc = A @ Bt^T`` (one or two FP16 products), epilogue
   ``acc * 2^-e + bias``, RoPE from per-token tables, cast, strided store into the native slots.

Float coefficient sources take A = FP16 hi/lo split of ``P * 2^e`` ``[N, 2 K_pad]`` against the plain
transposed basis ``[C, K_pad]`` (no bias).

:class:`RestoreProgram` plans many jobs once (scratch, operand preparation for every job in a few
batched launches) and then launches the GEMM group by group (e.g. one layer at a time, overlapped
with a forward), so the per-layer host cost is one native call.
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
MAX_RESTORE_JOBS = 48
MAX_AUX_JOBS = 48


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


class RestoreProgram:
    """Jobs planned once, prepared in batched launches, restored group by group.

    Each job (``add``) is a dict: ``kind`` ("pictures" | "u8" | "f32"), ``tokens``, ``rank``, ``grid``
    (frames, height, width), ``basis`` (FP16 [R, C]), optional ``basis_t`` (FP16 [C, k_pad]) and
    ``qmax``, ``scale``/``offset`` (host float32 [>= rank]), ``dest`` (address, (ts, hs, ds), dtype,
    channels, head_dim), ``rope`` (restore_kernels.restore_rope_item) or None, and the source
    (``pictures``: (addresses, plane_stride, row_stride, layout) | ``values``: device tensor, with optional
    ``runs`` = (run_len, run_stride, run_offset): token t reads coefficient row
    ``(t // run_len) * run_stride + run_offset + t % run_len`` -- one job restores a rank's block of a frame grid).
    """

    def __init__(self, device, stream, *, precision: str = "fp16x2"):
        self.device = torch.device(device)
        if self.device.type == "cuda" and self.device.index is None:
            self.device = torch.device("cuda", torch.cuda.current_device())
        self.stream = stream
        self.passes = 2 if precision == "fp16x2" else 1
        self.jobs: list[dict] = []
        self.groups: dict = {}
        self.keepalive: list = []
        self.prepared = False
        self.launches = 0
        self.scratch_bytes = 0
        self._batch_cache: dict = {}

    def add(self, job: dict, group=0) -> None:
        if self.prepared:
            raise ConfigurationError("jobs cannot be added after prepare()")
        self.groups.setdefault(group, []).append(len(self.jobs))
        self.jobs.append(job)

    def prepare(self, run_aux: bool = True) -> "RestoreProgram":
        """Allocate scratch, build every unpack / prep / restore table and (``run_aux``) run unpack + prep
        for every job in batched launches; otherwise each group's preparation runs with its launch
        (``launch(group, aux=True)``)."""
        stream, device = self.stream, self.device
        plan = []
        cursor = 0
        for job in self.jobs:
            rank, tokens, channels = job["rank"], job["tokens"], job["dest"][3]
            k_pad = k_pad_of(rank)
            if job["kind"] == "f32":
                sizes = (tokens * 2 * k_pad * 2, 0, channels * 4)
            elif job["kind"] == "a16":  # A already unpacked (e.g. in a peer's symmetric buffer)
                sizes = (0, channels * 2 * k_pad * 2, channels * 4)
            else:
                sizes = (tokens * k_pad * 2, channels * 2 * k_pad * 2, channels * 4)
            offsets = []
            for size in sizes:
                offsets.append(cursor)
                cursor += (size + 255) // 256 * 256
            plan.append((k_pad, offsets))
        with torch.cuda.stream(stream):
            scratch = torch.empty(max(cursor, 256), dtype=torch.uint8, device=device)
        self.keepalive.append(scratch)
        self.scratch_bytes = scratch.numel()
        arena = HostArena()
        unpack_rows, prep_rows = [], []
        unpack_owner, prep_owner = [], []  # job index of every row
        self.a_ops, self.b_ops, self.inverse, self.rows = [], [], [], []
        for job, (k_pad, (a_off, b_off, bias_off)) in zip(self.jobs, plan):
            rank, tokens, channels = job["rank"], job["tokens"], job["dest"][3]
            bias_view = scratch[bias_off:bias_off + channels * 4].view(torch.float32)
            if job["kind"] == "f32":
                values = job["values"]
                bound = job.get("bound")
                with torch.cuda.stream(stream):
                    if bound is None:
                        bound = float(values[:, :rank].abs().amax().item())
                    e = prescale_exponent(bound)
                    a = scratch[a_off:a_off + tokens * 2 * k_pad * 2].view(torch.float16).view(tokens, 2 * k_pad)
                    a.zero_()
                    scaled = values[:, :rank].float() * (2.0 ** e)
                    hi = scaled.half()
                    a[:, :rank] = hi
                    a[:, k_pad:k_pad + rank] = (scaled - hi.float()).half()
                    bias_view.zero_()
                    b = job.get("basis_t")
                    if b is None:
                        from ..restore_kernels import transposed_basis
                        b = transposed_basis(job["basis"])
                self.keepalive.append(b)
                b = b[:, :k_pad]
            else:
                qmax = job.get("qmax")
                if qmax is None:
                    qmax = basis_max_abs(job["basis"])
                smax = float(np.abs(job["scale"][:rank]).max(initial=0.0))
                e = prescale_exponent(smax * qmax)
                if job["kind"] != "a16":
                    a = scratch[a_off:a_off + tokens * k_pad * 2].view(torch.float16).view(tokens, k_pad)
                b = scratch[b_off:b_off + channels * 2 * k_pad * 2].view(torch.float16).view(channels, 2 * k_pad)
                frames, height, width = job["grid"]
                if job["kind"] == "a16":
                    a = job["a"]  # FP16 [tokens, k_pad] centered pixels, produced elsewhere
                    if a.dtype != torch.float16 or tuple(a.shape) != (tokens, k_pad):
                        raise ConfigurationError("a16 jobs take an FP16 [tokens, k_pad] A operand")
                    self.keepalive.append(a)
                elif job["kind"] == "pictures":
                    addresses, plane_stride, row_stride, layout = job["pictures"]
                    col_off, col_seg = column_tables(layout, plane_stride, row_stride, k_pad)
                    unpack_owner.append(len(self.rows))
                    unpack_rows.append([arena.add(addresses), arena.add(col_off), arena.add(col_seg), 0,
                                        a.data_ptr(), row_stride, tokens, k_pad, rank, frames, height, width, 0, 0, 0])
                else:
                    values = job["values"]
                    self.keepalive.append(values)
                    unpack_owner.append(len(self.rows))
                    runs = job.get("runs") or (0, 0, 0)   # (run_len, run_stride, run_offset): a row gather
                    if runs[0]:
                        last = (tokens - 1) // runs[0] * runs[1] + runs[2] + (tokens - 1) % runs[0]
                        if last >= values.shape[0] or min(runs) < 0:
                            raise ConfigurationError("row runs reach past the job's coefficient rows")
                    unpack_rows.append([-1, -1, -1, values.data_ptr(), a.data_ptr(), values.stride(0), tokens,
                                        k_pad, rank, frames, height, width, *runs])
                basis = job["basis"]
                scale_off = arena.add(np.ascontiguousarray(job["scale"][:rank], dtype=np.float32))
                offset_off = arena.add(np.ascontiguousarray(job["offset"][:rank], dtype=np.float32))
                bits = struct.unpack("<I", struct.pack("<f", float(2.0 ** e)))[0]
                prep_owner.append(len(self.rows))
                prep_rows.append([basis.data_ptr(), scale_off, offset_off, b.data_ptr(), bias_view.data_ptr(),
                                  basis.stride(0), rank, k_pad, channels, bits])
                self.keepalive.append(basis)
            address, (ts, hs, ds), dtype, channels, head_dim = job["dest"]
            row = [0] * 40
            row[0] = address
            row[1] = bias_view.data_ptr()
            rope = job.get("rope")
            if rope is not None and rope[0] == "packed":  # separable tables staged in shared memory
                row[2], row[17], row[18], row[19], row[20] = rope[1], rope[2], rope[3], rope[4], rope[5]
                row[15] = 2
            elif rope is not None:  # per-token FP32 rows [tokens, pairs]
                row[2], row[3], row[17] = rope[1], rope[2], rope[3]
                row[15] = 1
            row[4], row[5], row[6] = ts, hs, ds
            row[7] = tokens
            row[8] = self.passes
            row[9], row[10], row[11] = job["grid"]
            row[12] = _OUT_CODE[dtype]
            row[13] = channels
            row[14] = head_dim
            self.rows.append(row)
            self.a_ops.append(a)
            self.b_ops.append(b)
            self.inverse.append(2.0 ** -e)
        if unpack_rows or prep_rows:
            host, dev = arena.upload(device, stream)
            self.keepalive.extend((host, dev))
            base = dev.data_ptr()
            for row in unpack_rows:
                for index in (0, 1, 2):
                    row[index] = 0 if row[index] < 0 else row[index] + base
            for row in prep_rows:
                row[1] += base
                row[2] += base
        self.aux = _aux_tables(unpack_rows, prep_rows)
        self._aux_rows = (unpack_rows, unpack_owner, prep_rows, prep_owner)
        group_of = {}
        for group, indices in self.groups.items():
            for index in indices:
                group_of[index] = group
        self.group_aux = {}
        for group in self.groups:
            self.group_aux[group] = _aux_tables(
                [row for row, owner in zip(unpack_rows, unpack_owner) if group_of[owner] == group],
                [row for row, owner in zip(prep_rows, prep_owner) if group_of[owner] == group])
        if run_aux:
            self.run_aux(stream)
        # launch parameters (tensor maps included) encoded once per batch of <= 48 jobs
        self.blobs = {group: self._build_blobs(indices) for group, indices in self.groups.items()}
        self.keepalive.extend(self.a_ops)
        self.keepalive.extend(self.b_ops)
        self.prepared = True
        return self

    def _build_blobs(self, indices) -> list:
        blobs = []
        by_dtype: dict = {}
        for index in indices:  # one launch covers jobs of one output dtype
            by_dtype.setdefault(self.rows[index][12], []).append(index)
        batches = [same[i:i + MAX_RESTORE_JOBS] for same in by_dtype.values()
                   for i in range(0, len(same), MAX_RESTORE_JOBS)]
        for chunk in batches:
            blobs.append(ext().restore_build(torch.tensor([self.rows[j] for j in chunk], dtype=torch.int64),
                                             [self.a_ops[j] for j in chunk], [self.b_ops[j] for j in chunk],
                                             torch.tensor([self.inverse[j] for j in chunk], dtype=torch.float32)))
        return blobs

    def batches(self, groups=None) -> list[tuple]:
        """Consecutive groups (in insertion order) packed into batches of at most 48 jobs: the launch
        units of :meth:`launch_batch` when no per-group readiness is needed (a non-overlapped restore
        launches 6 CausVid layers per kernel instead of one)."""
        order = list(self.groups) if groups is None else list(groups)
        out, current, count = [], [], 0
        for group in order:
            n = len(self.groups[group])
            if current and count + n > MAX_RESTORE_JOBS:
                out.append(tuple(current))
                current, count = [], 0
            current.append(group)
            count += n
        if current:
            out.append(tuple(current))
        return out

    def _batch(self, groups: tuple):
        cached = self._batch_cache.get(groups)
        if cached is None:
            indices = [i for g in groups for i in self.groups[g]]
            members = set(indices)
            unpack_rows, unpack_owner, prep_rows, prep_owner = self._aux_rows
            aux = _aux_tables([row for row, owner in zip(unpack_rows, unpack_owner) if owner in members],
                              [row for row, owner in zip(prep_rows, prep_owner) if owner in members])
            cached = (self._build_blobs(indices), aux)
            self._batch_cache[groups] = cached
        return cached

    def launch_batch(self, groups, stream=None, *, aux: bool = False) -> int:
        """One restore launch (per output dtype and 48 jobs) covering every job of ``groups``; ``aux``
        first runs their unpack + basis preparation (batched too). Parameters are encoded once per
        distinct batch and reused."""
        if not self.prepared:
            self.prepare()
        blobs, (unpack_tables, prep_tables) = self._batch(tuple(groups))
        status = status_word(self.device)
        with torch.cuda.stream(stream or self.stream):
            if aux:
                for table in unpack_tables:
                    ext().unpack_launch(table, self.device.index)
                for table in prep_tables:
                    ext().prep_launch(table, self.device.index)
                self.launches += len(unpack_tables) + len(prep_tables)
            for blob in blobs:
                ext().restore_run(blob, self.device.index, status)
        self.launches += len(blobs)
        return len(blobs)

    def batch_launch_count(self, aux: bool = True) -> int:
        """Kernel launches of one pass of :meth:`launch_batch` over :meth:`batches`."""
        total = 0
        for groups in self.batches():
            blobs, (unpack_tables, prep_tables) = self._batch(groups)
            total += len(blobs) + (len(unpack_tables) + len(prep_tables) if aux else 0)
        return total

    def run_aux(self, stream=None, group=None) -> int:
        """(Re-)run the operand preparation of every job (or of one group's jobs): unpack of the 8-bit
        sources and basis prep."""
        unpack_tables, prep_tables = self.aux if group is None else self.group_aux[group]
        with torch.cuda.stream(stream or self.stream):
            for table in unpack_tables:
                ext().unpack_launch(table, self.device.index)
            for table in prep_tables:
                ext().prep_launch(table, self.device.index)
        self.launches += len(unpack_tables) + len(prep_tables)
        return len(unpack_tables) + len(prep_tables)

    def launch(self, group=0, stream=None, *, aux: bool = False) -> int:
        """Launch the restore GEMM of one group on ``stream`` (default: the program's stream); ``aux``
        first runs the group's unpack + basis preparation."""
        if not self.prepared:
            self.prepare()
        status = status_word(self.device)
        if aux:
            self.run_aux(stream, group)
        with torch.cuda.stream(stream or self.stream):
            for blob in self.blobs[group]:
                ext().restore_run(blob, self.device.index, status)
        self.launches += len(self.blobs[group])
        return len(self.blobs[group])

    def launch_all(self, stream=None) -> int:
        return sum(self.launch(group, stream) for group in self.groups)


def _aux_tables(unpack_rows, prep_rows):
    return ([torch.tensor(unpack_rows[i:i + MAX_AUX_JOBS], dtype=torch.int64)
             for i in range(0, len(unpack_rows), MAX_AUX_JOBS)],
            [torch.tensor(prep_rows[i:i + MAX_AUX_JOBS], dtype=torch.int64)
             for i in range(0, len(prep_rows), MAX_AUX_JOBS)])


def launch_factor_group(items, device, precision, stream, keepalive):
    """Plan, prepare and launch ``items`` (see :class:`RestoreProgram`); returns the launch count."""
    program = RestoreProgram(device, stream, precision=precision)
    for item in items:
        program.add(item)
    program.prepare()
    program.launch_all()
    keepalive.append(program)
    return program.launches
