"""The allocation-free C entry point ``rc_restore_u8_noalloc`` (csrc/restore/noalloc.h), for callers that
cannot allocate device memory (an engine that owns all of it, code running while the allocator is locked or
trimming), against the existing fused restore entry point (``restore_kernels.reconstruct``): same kernels,
same parameters, so the restored slots are bitwise identical, on two calls in a row that reuse the fixed
scratch; both are also checked against the kernel's documented elementwise error bound, for one and two
FP16 products and for bfloat16 and FP32 destinations, and the calls leave torch's allocator untouched.
Collected last so it also runs after every other GPU test in one process."""

import ctypes

import numpy as np
import pytest
import torch

from reelcache_b200 import restore_kernels as rk

pytestmark = pytest.mark.gpu


class RcRestoreU8Job(ctypes.Structure):
    _fields_ = [
        ("coefficients", ctypes.c_void_p), ("coeff_stride", ctypes.c_int64), ("tokens", ctypes.c_int64),
        ("rank", ctypes.c_int64), ("basis", ctypes.c_void_p), ("basis_stride", ctypes.c_int64),
        ("scale", ctypes.c_void_p), ("offset", ctypes.c_void_p), ("scale_basis_bound", ctypes.c_double),
        ("destination", ctypes.c_void_p), ("dst_token_stride", ctypes.c_int64), ("dst_head_stride", ctypes.c_int64),
        ("dst_dim_stride", ctypes.c_int64), ("out_dtype", ctypes.c_int64), ("channels", ctypes.c_int64),
        ("head_dim", ctypes.c_int64), ("rope_pack", ctypes.c_void_p), ("grid_t", ctypes.c_int64),
        ("grid_h", ctypes.c_int64), ("grid_w", ctypes.c_int64), ("sec_t", ctypes.c_int64), ("sec_h", ctypes.c_int64),
        ("rope_entries", ctypes.c_int64), ("passes", ctypes.c_int64), ("status", ctypes.c_void_p),
    ]


def _entry():
    from reelcache_b200.ops._ext import ext

    lib = ctypes.CDLL(ext().__file__)
    fn = lib.rc_restore_u8_noalloc
    fn.restype = ctypes.c_int
    fn.argtypes = [ctypes.POINTER(RcRestoreU8Job), ctypes.c_int, ctypes.c_void_p, ctypes.c_char_p, ctypes.c_size_t]
    return fn


def _job(device, seed, rank, rope):
    grid = (3, 30, 52)
    tokens, heads, head_dim = grid[0] * grid[1] * grid[2], 12, 128
    rng = np.random.default_rng(seed)
    pixels = torch.from_numpy(rng.integers(0, 256, (tokens, rank), dtype=np.uint8)).to(device)
    scale = rng.uniform(0.001, 0.05, rank).astype(np.float32)
    offset = rng.uniform(-3.0, 3.0, rank).astype(np.float32)
    basis = (torch.from_numpy(rng.standard_normal((rank, heads * head_dim)).astype(np.float32)) / 40).half().to(device)
    table = rk.RopeTable.wan(head_dim, 64, device=device)
    rows = (3, 0, 0)
    return grid, tokens, heads, head_dim, pixels, scale, offset, basis, table, rows


_DTYPE_CODES = {torch.bfloat16: 0, torch.float16: 1, torch.float32: 2}


def _restore_both(fn, device, seed, rank, rope, passes=1, out_dtype=torch.bfloat16):
    grid, tokens, heads, head_dim, pixels, scale, offset, basis, table, rows = _job(device, seed, rank, rope)
    expected = torch.zeros((1, tokens, heads, head_dim), dtype=out_dtype, device=device)
    precision = "fp16x2" if passes == 2 else "fp16"
    job = rk.ReconstructionJob(rk.CoefficientSource(pixels, scale, offset), rk.NativeView(expected), grid, basis,
                               rope=rk.RopePositions(table, rows) if rope else None)
    rk.reconstruct([job], backend="fused", precision=precision).synchronize()

    got = torch.full_like(expected, float("nan"))
    scale_d = torch.from_numpy(scale).to(device)
    offset_d = torch.from_numpy(offset).to(device)
    status = torch.zeros(1, dtype=torch.int32, device=device)
    c = RcRestoreU8Job()
    c.coefficients, c.coeff_stride, c.tokens, c.rank = pixels.data_ptr(), pixels.stride(0), tokens, rank
    c.basis, c.basis_stride = basis.data_ptr(), basis.stride(0)
    c.scale, c.offset = scale_d.data_ptr(), offset_d.data_ptr()
    c.scale_basis_bound = float(np.abs(scale).max()) * float(basis.abs().amax().item())
    view = rk.NativeView(got)
    c.destination = view.address()
    c.dst_token_stride, c.dst_head_stride, c.dst_dim_stride = view.strides()
    c.out_dtype, c.channels, c.head_dim = _DTYPE_CODES[out_dtype], heads * head_dim, head_dim
    keep = []
    if rope:
        pack, (sec_t, sec_h, entries) = table.packed_tables(rows, grid, device)
        keep.append(pack)
        c.rope_pack, c.sec_t, c.sec_h, c.rope_entries = pack.data_ptr(), sec_t, sec_h, entries
    c.grid_t, c.grid_h, c.grid_w = grid
    c.passes = passes
    c.status = status.data_ptr()
    error = ctypes.create_string_buffer(256)
    stream = torch.cuda.current_stream(device)
    torch.cuda.synchronize(device)
    allocated = torch.cuda.memory_allocated(device)
    code = fn(ctypes.byref(c), device.index, ctypes.c_void_p(stream.cuda_stream), error, len(error))
    assert code == 0, error.value.decode()
    assert torch.cuda.memory_allocated(device) == allocated  # nothing drawn from torch's allocator
    torch.cuda.synchronize(device)
    assert int(status.item()) == 0
    # the documented bound of the fused kernel, checked on what the allocation-free call wrote
    values, bound = rk.kernel_error_bound(job, precision)
    written = got.reshape(tokens, -1).double()
    assert float(((written - values).abs() - bound).max()) <= 0
    return expected, got


def test_noalloc_matches_fused_entry_point_twice(cuda_device):
    fn = _entry()
    # setup-only call (what a caller does before any stream capture)
    assert fn(None, cuda_device.index, None, None, 0) == 0
    for seed, rank, rope in ((1, 64, True), (2, 200, False)):
        expected, got = _restore_both(fn, cuda_device, seed, rank, rope)
        assert torch.equal(got, expected)


@pytest.mark.parametrize("passes,out_dtype", [(2, torch.bfloat16), (2, torch.float32), (1, torch.float32)])
def test_noalloc_precisions_and_destinations(cuda_device, passes, out_dtype):
    fn = _entry()
    for seed, rank, rope in ((3, 96, True), (4, 257, True)):
        expected, got = _restore_both(fn, cuda_device, seed, rank, rope, passes=passes, out_dtype=out_dtype)
        assert torch.equal(got, expected)


def test_noalloc_rejects_oversized_job(cuda_device):
    fn = _entry()
    c = RcRestoreU8Job()
    c.coefficients = c.basis = c.scale = c.offset = c.destination = 1  # never dereferenced: rejected first
    c.tokens, c.rank, c.coeff_stride = 200000, 256, 256
    c.basis_stride, c.channels, c.head_dim = 1536, 1536, 128
    c.passes, c.out_dtype = 1, 0
    error = ctypes.create_string_buffer(256)
    code = fn(ctypes.byref(c), cuda_device.index, None, error, len(error))
    assert code == 2 and b"scratch" in error.value
