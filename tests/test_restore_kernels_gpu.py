"""Fused sm_100a restore kernel against the FP64 reference and its documented error bound."""

import numpy as np
import pytest
import torch

from reelcache_b200 import restore_kernels as rk

from .restore_support import picture_job

pytestmark = pytest.mark.gpu


def _check(job, precision="fp16x2"):
    values, bound = rk.kernel_error_bound(job, precision)
    written = job.destination.slot(job.tokens).reshape(job.tokens, -1).double()
    excess = ((written - values).abs() - bound).max().item()
    assert excess <= 0, excess


@pytest.mark.parametrize("rank,rope", [(96, True), (200, True), (33, False), (256, True)])
def test_fused_pictures_within_bound(cuda_device, rank, rope):
    from reelcache_b200.ops import _ext

    job, _ = picture_job(cuda_device, rank=rank, heads=4, rope=rope)
    handle = rk.reconstruct([job], backend="fused", precision="fp16x2")
    handle.synchronize()
    _ext.check_status(cuda_device)
    _check(job)
    handle.release()


def test_fused_group_of_jobs_k_and_v(cuda_device):
    from reelcache_b200.ops import _ext

    cache = torch.zeros((1, 3 * 4680, 12, 128), dtype=torch.bfloat16, device=cuda_device)
    table = rk.RopeTable.wan(128, 256, device=cuda_device)
    jobs = []
    for chunk in range(3):
        job, _ = picture_job(cuda_device, rank=64 + 32 * chunk, heads=12, destination=cache, token_offset=4680 * chunk,
                             table=table, rope_rows=(3 * chunk, 0, 0), seed=chunk)
        jobs.append(job)
    rk.reconstruct(jobs, backend="fused").synchronize()  # auto precision: the two-product fp16x2 split
    _ext.check_status(cuda_device)
    for job in jobs:
        _check(job, "fp16x2")


@pytest.mark.parametrize("layout", ["THD", "BHTD"])
def test_fused_layouts_and_fp16(cuda_device, layout):
    job, _ = picture_job(cuda_device, rank=128, heads=2, layout=layout, out_dtype=torch.float16)
    rk.reconstruct([job], backend="fused", precision="fp16").synchronize()
    _check(job, "fp16")


def test_fused_float_and_uint8_coefficients(cuda_device):
    job, pixels = picture_job(cuda_device, rank=80, heads=2, out_dtype=torch.float32)
    coeff = rk.reference_coefficients(job)
    fjob = rk.ReconstructionJob(rk.CoefficientSource(coeff.contiguous()), job.destination, job.grid, job.basis,
                                rope=job.rope)
    rk.reconstruct([fjob], backend="fused").synchronize()
    _check(fjob)
    u8 = torch.from_numpy(pixels).to(cuda_device)
    ujob = rk.ReconstructionJob(rk.CoefficientSource(u8, job.source.scale, job.source.offset), job.destination,
                                job.grid, job.basis, rope=job.rope)
    rk.reconstruct([ujob], backend="fused").synchronize()
    _check(ujob)


@pytest.mark.parametrize("kind", ["dense_table", "wide_grid"])
def test_fused_token_rope_fallback(cuda_device, kind):
    """Tables the epilogue cannot stage in shared memory take the per-token FP32 row path."""
    from reelcache_b200.ops import _ext

    if kind == "dense_table":
        angles = torch.rand(4 * 30 * 52 + 8, 64, dtype=torch.float64) * 6.0
        table = rk.RopeTable.from_cos_sin(torch.cos(angles).to(cuda_device), torch.sin(angles).to(cuda_device))
        job, _ = picture_job(cuda_device, rank=96, heads=2, table=table, rope_rows=5, frames=3)
    else:
        table = rk.RopeTable.wan(128, 6000, device=cuda_device)
        job, _ = picture_job(cuda_device, rank=64, heads=2, table=table, frames=1, height=2, width=5400)
        assert table.packed_tables((0, 0, 0), job.grid, cuda_device) is None
    rk.reconstruct([job], backend="fused", precision="fp16x2").synchronize()
    _ext.check_status(cuda_device)
    _check(job)


def test_dense_rope_store(cuda_device):
    from reelcache_b200.ops import _ext

    tokens, heads, d = 3 * 30 * 52, 4, 128
    values = torch.randn(tokens, heads * d, device=cuda_device, dtype=torch.bfloat16)
    dest = torch.zeros((1, tokens, heads, d), dtype=torch.bfloat16, device=cuda_device)
    table = rk.RopeTable.wan(d, 64, device=cuda_device)
    job = rk.ReconstructionJob(rk.DenseSource(values), rk.NativeView(dest), (3, 30, 52),
                               rope=rk.RopePositions(table, (2, 0, 0)))
    rk.reconstruct([job], backend="fused").synchronize()
    _ext.check_status(cuda_device)
    ref = rk.apply_rope_reference(values.reshape(tokens, heads, d), job.rope, job.grid).to(torch.bfloat16)
    assert torch.allclose(dest[0].float(), ref.float(), atol=2e-2, rtol=1e-2)
