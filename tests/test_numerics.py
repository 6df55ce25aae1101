"""Fitting numerics on CPU: FP32-accurate products, CholeskyQR2, factorization backends, projection and
basis reuse, FP64 spectra, lockstep reads, bounded eigensolves, exact source fingerprints and the opt-in
fitter levers."""

import math

import pytest
import torch

from reelcache_b200 import accel, deferred_reads, exact_blas, factorization, gpu_fitting, reuse, spectra
from reelcache_b200.errors import ConfigurationError
from reelcache_b200.lineage_commit import (FINGERPRINT_PRIME, fingerprint_terms, source_fingerprint,
                                           source_fingerprints)
from reelcache_b200.types import MatrixKey, ModelIdentity, TensorContext


def _low_rank(n=96, c=48, r=6, noise=1e-3, seed=0):
    g = torch.Generator().manual_seed(seed)
    return (torch.randn(n, r, generator=g) @ torch.randn(r, c, generator=g) * 0.5
            + noise * torch.randn(n, c, generator=g))


def _context(n, c, layer=0):
    model = ModelIdentity("numerics", "f0", 2, c, "THD", "float32")
    return TensorContext(model, MatrixKey(layer, "V"), 0, 1, 1, n, "none")


def test_mm_and_cholesky_qr2_host():
    a, b = torch.randn(37, 19, dtype=torch.float64), torch.randn(19, 23, dtype=torch.float64)
    got = exact_blas.mm(a.float(), b.float())
    assert got.dtype == torch.float32
    assert torch.allclose(got.double(), a @ b, atol=1e-5, rtol=1e-5)
    x = torch.randn(64, 12)
    q = exact_blas.cholesky_qr2(x)
    assert torch.allclose(q.t() @ q, torch.eye(12), atol=1e-5)
    # same span as x
    assert torch.allclose(q @ (q.t() @ x), x, atol=1e-4)
    with pytest.raises(ConfigurationError):
        exact_blas.mm(torch.ones(2, 3), torch.ones(2, 3))


def test_fit_basis_backends_and_projection():
    x = _low_rank()
    ctx = _context(*x.shape)
    exact = factorization.fit_basis(x, ctx, 6, method="exact")
    rand = factorization.fit_basis(x, ctx, 6, method="randomized", seed=3)
    gram = factorization.fit_basis(x, ctx, 6, method="gram")
    for factors in (exact, rand, gram):
        assert factors.basis.dtype == torch.float16 and factors.basis.shape == (6, 48)
        assert factors.metrics["projection_relative_residual"] < 5e-3
        # canonical signs: the largest-magnitude entry of every row is positive
        top = factors.basis.float().gather(1, factors.basis.float().abs().argmax(1, keepdim=True))
        assert bool((top > 0).all())
    again = factorization.fit_basis(x, ctx, 6, method="randomized", seed=3)
    assert torch.equal(again.basis, rand.basis)
    projection = factorization.project_onto_basis(x, exact.basis, rank=4)
    assert projection.coefficients.shape == (96, 4) and projection.relative_residual > 1e-3
    assert 1.0 <= factorization.fast_condition_bound(exact.basis) < 1.01
    assert factorization.basis_condition_bound(exact.basis) <= factorization.fast_condition_bound(exact.basis) + 1e-6
    with pytest.raises(ConfigurationError):
        factorization.fit_basis(x, ctx, 0)


def test_rank_directions_and_anchor_detector():
    x = _low_rank(n=128, c=64, r=10)
    ctx = _context(*x.shape)
    fit = factorization.fit_rank_directions(x, 16, seed=1)
    full = factorization.fit_rank_directions(x, 16, solver="gram_eigh")
    assert fit.required_rank(0.99) == full.required_rank(0.99) <= 10
    assert abs(fit.energy_fraction(10) - full.energy_fraction(10)) < 1e-5
    spec = factorization.DetectorSpec(initial_width=4, stop_energy=0.999)
    acquisition = factorization.acquire_anchor_directions(x, ctx, spec)
    assert acquisition.status == "reached" and acquisition.width >= 10 and acquisition.attempts >= 2
    assert acquisition.to_dict()["detector"] == spec.fingerprint()
    assert factorization.DetectorSpec.from_dict(spec.to_dict()) == spec


def test_reuse_gate():
    x = _low_rank(seed=4)
    ctx = _context(*x.shape)
    parent = factorization.fit_basis(x, ctx, 6, method="exact").basis
    accepted = reuse.try_reuse_basis(x, ctx, parent, 0.99)
    assert accepted.accepted and accepted.captured_energy > 0.99
    other = _low_rank(seed=9)
    rejected = reuse.try_reuse_basis(other, ctx, parent, 0.99)
    assert not rejected.accepted and rejected.reason == "below_threshold"
    factors = reuse.factorize_tensor(other, ctx, 6, reuse_basis=parent, reuse_threshold=0.99, method="exact")
    assert factors.metrics["reuse_accepted"] is False and factors.metrics["reuse_reason"] == "below_threshold"
    with pytest.raises(ConfigurationError):
        reuse.validate_threshold(1.5)


def test_spectra_streaming_matches_svd(tmp_path):
    x = _low_rank(n=200, c=32, r=5, noise=1e-2)
    result = spectra.exact_spectrum(x, tile_rows=64)
    assert result.rows == 200 and result.channels == 32
    assert abs(result.total_energy - float(x.double().square().sum())) < 1e-9 * result.total_energy
    check = spectra.direct_svd_crosscheck(x, result)
    assert check["max_eigenvalue_difference"] < 1e-10
    assert check["svd_r95"] == check["gram_r95"] == result.r95
    bracket = result.rank_at(0.95)
    assert bracket.low <= bracket.rank <= bracket.high
    digest = spectra.write_spectrum_json(result, tmp_path / "s.json")
    assert len(digest) == 64
    assert spectra.SpectrumResult.from_dict(result.to_dict()).eigenvalues == result.eigenvalues


def test_lockstep_rounds_and_exceptions():
    def routine(value, fail=False):
        a = torch.tensor(float(value))
        (got,) = yield (a,)
        if fail:
            raise ValueError(f"routine {value}")
        (got2, vec) = yield (a * 2, torch.arange(3.0))
        return got + got2 + float(vec.sum())

    before = dict(deferred_reads.STATS)
    assert deferred_reads.run_lockstep([routine(i) for i in range(5)]) == [3 * i + 3.0 for i in range(5)]
    assert deferred_reads.STATS["rounds"] - before["rounds"] == 2
    with pytest.raises(ValueError, match="routine 1"):
        deferred_reads.run_lockstep([routine(0), routine(1, fail=True), routine(2, fail=True)])

    def batched(value):
        result = yield deferred_reads.BatchedCall("sum", lambda payloads: [sum(payloads)] * len(payloads), value)
        return result

    assert deferred_reads.run_lockstep([batched(1), batched(2), batched(3)]) == [6, 6, 6]
    work = deferred_reads.TileWorkspace()
    a = work.get("t", (4, 4), torch.float32, "cpu")
    b = work.get("t", (2, 2), torch.float32, "cpu")
    assert a.untyped_storage().data_ptr() == b.untyped_storage().data_ptr()


def test_projection_routines_match_direct():
    x = _low_rank(seed=5)
    rows = factorization.fit_basis(x, None, 6, method="exact").basis
    total = float(x.double().square().sum())
    (energy, coefficients), = deferred_reads.run_lockstep([deferred_reads.stored_energy_routine(x, rows, total)])
    projection = factorization.project_onto_basis(x, rows)
    assert abs(energy - (1 - projection.relative_residual ** 2)) < 1e-9
    assert torch.allclose(coefficients, projection.coefficients)


def test_bounded_eigh_sub_batches():
    mats = torch.randn(6, 8, 8)
    mats = mats @ mats.transpose(1, 2)
    bounded = gpu_fitting.BoundedEigh("t", gpu_fitting.torch_rows_eigh,
                                      total_memory=gpu_fitting.eigh_workspace_bytes(2, 8, "t") * 4,
                                      memory_fraction=0.25)
    values, rows = bounded(mats)
    assert bounded.last["sub_batch"] == 2 and bounded.last["solver_calls"] == 3
    ref_values, ref_vectors = torch.linalg.eigh(mats)
    assert torch.allclose(values, ref_values, atol=1e-4)
    recon = rows.transpose(1, 2) @ torch.diag_embed(values) @ rows
    assert torch.allclose(recon, mats, atol=1e-3)
    fixed = gpu_fitting.BoundedEigh("t", gpu_fitting.torch_rows_eigh, sub_batch_size=lambda n: 4)
    fixed(mats)
    assert fixed.last["reason"] == "fixed" and fixed.last["solver_calls"] == 2
    label, solver = gpu_fitting.select_eigh_solver("torch_loop")
    assert label == "torch_eigh_loop_explicit"
    with pytest.raises(ConfigurationError):
        gpu_fitting.select_eigh_solver("magma")
    bases = gpu_fitting.gram_bases([_low_rank(seed=1), _low_rank(seed=2)], [3, 5])
    assert [tuple(b.shape) for b in bases] == [(3, 48), (5, 48)]


def test_gpu_fitter_validation():
    with pytest.raises(ConfigurationError):
        gpu_fitting.GPUFitter(gpu_id=0, gpu_uuid="nope")
    with pytest.raises(ConfigurationError):
        gpu_fitting.GPUFitter(gpu_id=0, gpu_uuid="GPU-x", method="magic")
    fitter = gpu_fitting.GPUFitter(gpu_id=0, gpu_uuid="GPU-x", method="gram_batched")
    assert fitter.prefit_stats["batches"] == 0


def _fingerprint_loops(m: torch.Tensor) -> list[int]:
    """The checksum definition written out element by element (independent of the vectorized paths)."""
    wide = m.element_size() == 4
    bits = m.contiguous().view(torch.int32 if wide else torch.int16).tolist()
    combos = ((37, 101, False), (613, 211, False), (1, 17, True))
    totals = [0] * (6 if wide else 3)
    for r, row in enumerate(bits):
        parts = [[v & 0xFFFF for v in row], [v >> 16 for v in row]] if wide else [row]
        for pi, part in enumerate(parts):
            for ci, (a, b, square) in enumerate(combos):
                s = sum((t * t if square else t) * ((c * a + 7) % 1021 + 1) for c, t in enumerate(part))
                totals[pi * 3 + ci] += (s % FINGERPRINT_PRIME) * ((r * b + 3) % 1019 + 1)
    return [t % FINGERPRINT_PRIME for t in totals]


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
def test_source_fingerprint_definition(dtype):
    m = (torch.randn(9, 13) * 100).to(dtype)
    assert fingerprint_terms(m).tolist() == _fingerprint_loops(m)
    text = source_fingerprint(m)
    assert text.startswith(f"fp1:9x13:{m.dtype}:")
    assert len(text.split(":")[-1]) == 8 * (6 if dtype == torch.float32 else 3)
    other = m.clone()
    other.view(-1)[5] = other.view(-1)[5] * 2 + 1
    assert source_fingerprint(other) != text
    assert source_fingerprints({"a": m, "b": other}) == {"a": text, "b": source_fingerprint(other)}


def test_accel_options():
    assert accel.parse_fitter_fp64("on") == frozenset()
    assert accel.parse_fitter_fp64("off") == frozenset(accel.OFF_PASSES)
    assert accel.parse_fitter_fp64("fp32:energy+span") == {"energy", "span"}
    with pytest.raises(ConfigurationError):
        accel.parse_fitter_fp64("fp32:warp")
    with pytest.raises(ConfigurationError):
        accel.FitterAccel(cuda_graphs=True)
    options = accel.FitterAccel(fp32_passes=frozenset({"energy"}))
    with accel.scope(options):
        assert accel.current() is options and accel.fp32("energy") and not accel.fp32("span")
    assert accel.current() is None
    assert float(accel.sumsq64(torch.tensor([[3.0, 4.0]]))) == 25.0
    # Neumann span energy equals the direct <G^-1, M> for nearly orthonormal rows
    x = _low_rank(seed=7)
    rows = factorization.fit_basis(x, None, 6, method="exact").basis
    p = x @ rows.float().t()
    q = rows.double()
    direct = float(torch.trace(torch.linalg.inv(q @ q.t()) @ (p.double().t() @ p.double())))
    total = float(x.double().square().sum())
    value = accel.span_energy_fp32(p, rows, total)
    assert value is not None and math.isclose(value, direct / total, rel_tol=1e-6)


def test_row_shard_spectrum_matches_whole_matrix():
    from reelcache_b200.spectra import exact_spectrum, row_shard, spectrum_from_row_shards
    g = torch.Generator().manual_seed(0)
    x = torch.randn(300, 8, generator=g) @ torch.randn(8, 48, generator=g) + 1e-3 * torch.randn(300, 48, generator=g)
    whole = exact_spectrum(x)
    shards = [row_shard(x[a:b], rank=r, row_start=a) for r, (a, b) in enumerate(((0, 100), (100, 170), (170, 300)))]
    merged = spectrum_from_row_shards(list(reversed(shards)))
    assert merged.rows == 300 and merged.r95 == whole.r95 and merged.r99 == whole.r99
    assert max(abs(a - b) for a, b in zip(merged.eigenvalues, whole.eigenvalues)) <= 1e-9 * whole.total_energy
    diagnostics = merged.metrics["diagnostics"]
    assert diagnostics["asymmetry"] < 1e-12 and diagnostics["trace_residual"] < 1e-10
    with pytest.raises(Exception):
        spectrum_from_row_shards([shards[0], shards[2]])   # a gap
