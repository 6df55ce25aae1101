"""Restore-kernel API on CPU: reference backend, picture unpacking, error-bound bookkeeping."""

import numpy as np
import pytest
import torch

from reelcache_b200 import _hevc
from reelcache_b200 import restore_kernels as rk
from reelcache_b200.errors import ConfigurationError

from .restore_support import picture_job


def test_unpack_pictures_inverts_mosaic():
    job, pixels = picture_job("cpu", rank=70, heads=1, frames=2, height=6, width=10)
    unpacked = rk.unpack_pictures(job.source)
    assert torch.equal(unpacked, torch.from_numpy(pixels))


def test_reference_backend_matches_fp64_values():
    job, _ = picture_job("cpu", rank=40, heads=2, frames=2, height=5, width=7, out_dtype=torch.float32)
    rk.reconstruct([job], backend="reference").release()
    values, bound = rk.error_bound(job, "fp16x2")
    written = job.destination.slot(job.tokens).reshape(job.tokens, -1).double()
    assert torch.all((written - values).abs() <= bound + 1e-6 * values.abs().max())


def test_overlapping_destinations_rejected():
    job, _ = picture_job("cpu", rank=8, heads=1, frames=1, height=4, width=4, capacity=32)
    other = rk.ReconstructionJob(job.source, rk.NativeView(job.destination.tensor, "BTHD", 8), job.grid, job.basis)
    with pytest.raises(ConfigurationError):
        rk.reconstruct([job, other], backend="reference")


def test_quantize_dequantize_covering():
    rng = np.random.default_rng(3)
    values = rng.standard_normal((200, 12)).astype(np.float32)
    pixels, affine, layout = _hevc.quantize_coefficients(values, "per_channel")
    restored = _hevc.dequantize_coefficients(pixels, affine, layout)
    assert np.all(np.abs(restored - values) <= affine[0] * 0.5 + 1e-6)
    assert np.all(np.float32(255) * affine[0] + affine[1] >= values.max(0))


def test_rope_wan_sections():
    table = rk.RopeTable.wan(128, 16)
    assert table.sections == (22, 21, 21)
    assert table.pairs == 64


def test_packed_rope_tables_match_token_tables():
    table = rk.RopeTable.wan(128, 64)
    grid, rows = (3, 5, 7), (4, 2, 1)
    pack, (sec_t, sec_h, entries) = table.packed_tables(rows, grid, "cpu")
    cos, sin = table.token_tables(rows, grid, "cpu")
    frames, height, width = grid
    assert entries == frames * sec_t + height * sec_h + width * (table.pairs - sec_t - sec_h)
    assert pack.shape[0] == entries + entries % 2
    off_h, off_w = frames * sec_t, frames * sec_t + height * sec_h
    for n in range(frames * height * width):
        f, rem = divmod(n, height * width)
        y, x = divmod(rem, width)
        for q in range(table.pairs):
            if q < sec_t:
                e = f * sec_t + q
            elif q < sec_t + sec_h:
                e = off_h + y * sec_h + q - sec_t
            else:
                e = off_w + x * (table.pairs - sec_t - sec_h) + q - sec_t - sec_h
            assert pack[e, 0] == cos[n, q] and pack[e, 1] == sin[n, q]


def test_packed_rope_tables_fall_back():
    dense = rk.RopeTable.from_cos_sin(torch.rand(64, 64), torch.rand(64, 64))
    assert dense.packed_tables(0, (1, 2, 2), "cpu") is None
    wide = rk.RopeTable.wan(128, 4096)
    assert wide.packed_tables((0, 0, 0), (1, 2, rk.PACKED_ROPE_ENTRIES), "cpu") is None
