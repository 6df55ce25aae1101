"""sm_100a fitter kernels against FP64 PyTorch references: the split-bf16 FP32-accurate GEMM, the batched
Jacobi eigensolver, the fused square sums, the exact fingerprint kernel and the Dot2 GEMM; and the planner
and GPU fitter paths that use them."""

import pytest
import torch

pytestmark = pytest.mark.gpu


@pytest.fixture(autouse=True)
def _cuda():
    if not torch.cuda.is_available():
        pytest.skip("needs a GPU")
    from reelcache_b200.ops import _ext
    _ext.ext()  # fail loudly when the extension is missing on a GPU box


def _err(got, ref):
    return float((got.double() - ref).norm() / ref.norm())


@pytest.mark.parametrize("m,k,n", [(256, 4680, 192), (37, 19, 23), (1536, 1536, 96), (5, 8, 1)])
def test_split_gemm_is_fp32_accurate(m, k, n):
    from reelcache_b200 import exact_blas
    g = torch.Generator(device="cuda").manual_seed(m + k + n)
    a = torch.randn(m, k, device="cuda", generator=g)
    b = torch.randn(k, n, device="cuda", generator=g)
    ref = a.double() @ b.double()
    got = exact_blas.mm(a, b)
    torch.backends.cuda.matmul.allow_tf32 = False
    sgemm = a @ b
    assert exact_blas.STATS["mm_split_bf16"] > 0
    # as accurate as an IEEE FP32 GEMM (within a small factor), far better than one bf16 product
    assert _err(got, ref) <= 4 * _err(sgemm, ref) + 1e-7
    assert _err(got, ref) < 2e-6
    # transposed operand layouts
    got_t = exact_blas.mm(a.t().contiguous().t(), b.t().contiguous().t())
    assert torch.equal(got_t, got)


def test_split_gemm_with_bf16_left_operand_matches_the_six_product_path():
    """A bf16 left operand takes the three-segment split; the result equals the six-segment split of the same
    values converted to FP32 (the three dropped products are exactly zero) and stays FP32-accurate."""
    from reelcache_b200 import exact_blas
    g = torch.Generator(device="cuda").manual_seed(7)
    a = torch.randn(4680, 1536, device="cuda", generator=g).bfloat16()
    b = torch.randn(1536, 64, device="cuda", generator=g)
    got = exact_blas.mm(a, b)
    assert torch.allclose(got, exact_blas.mm(a.float(), b), rtol=2e-6, atol=1e-5)
    assert _err(got, a.double() @ b.double()) < 2e-6


@pytest.mark.parametrize("k", [64, 4680, 28080])
def test_promoted_accumulation_matches_sgemm(k):
    from reelcache_b200.ops.fitter import matmul_promoted
    from reelcache_b200.ops.gemm import matmul_tn
    a = torch.randn(256, k, device="cuda").bfloat16().abs()
    b = torch.randn(200, k, device="cuda").bfloat16().abs()
    ref = a.double() @ b.double().t()
    torch.backends.cuda.matmul.allow_tf32 = False
    sgemm = _err(a.float() @ b.float().t(), ref)
    promoted = _err(matmul_promoted(a, b), ref)
    assert promoted <= 4 * sgemm + 1e-7, (promoted, sgemm, _err(matmul_tn(a, b), ref))


@pytest.mark.parametrize("n", [2, 7, 64, 129, 160])
def test_jacobi_eigh_matches_fp64(n):
    from reelcache_b200.ops.fitter import jacobi_eigh
    g = torch.Generator(device="cuda").manual_seed(n)
    x = torch.randn(6, 3 * n, n, device="cuda", generator=g)
    x[:, :, : n // 2] *= 10.0  # spread spectrum
    mats = x.transpose(1, 2) @ x
    values, vectors, info, sweeps = jacobi_eigh(mats)
    assert bool((info == 0).all()), (info, sweeps)
    ref = torch.linalg.eigvalsh(mats.double())
    scale = ref.abs().amax(1, keepdim=True)
    # an FP32 solver: eigenvalues to a few FP32 ulps of ||A||, like cuSOLVER's FP32 eigh on the same input
    cusolver = float(((torch.linalg.eigvalsh(mats).double() - ref).abs() / scale).max())
    assert float(((values.double() - ref).abs() / scale).max()) < max(1e-5, 4 * cusolver)
    eye = torch.eye(n, device="cuda", dtype=torch.float64)
    v = vectors.double()
    assert float((v.transpose(1, 2) @ v - eye).abs().max()) < 1e-5
    recon = v @ torch.diag_embed(values.double()) @ v.transpose(1, 2)
    assert float(((recon - mats.double()).norm(dim=(1, 2)) / mats.double().norm(dim=(1, 2))).max()) < 1e-5
    assert bool(torch.all(values[:, 1:] >= values[:, :-1]))


def test_jacobi_solver_selection_and_fallback_counts():
    from reelcache_b200 import gpu_fitting
    mats = torch.randn(4, 40, 40, device="cuda")
    mats = mats @ mats.transpose(1, 2)
    label, solver = gpu_fitting.select_eigh_solver("jacobi")
    before = gpu_fitting.STATS["jacobi_matrices"]
    values, rows = solver(mats)
    assert label == "jacobi_sm100" and gpu_fitting.STATS["jacobi_matrices"] == before + 4
    ref = torch.linalg.eigvalsh(mats.double())
    assert torch.allclose(values.double(), ref, rtol=1e-5, atol=1e-3)
    big = torch.eye(200, device="cuda").unsqueeze(0)
    with pytest.raises(Exception):
        gpu_fitting.jacobi_rows_eigh(big)
    v2, _ = gpu_fitting.rows_eigh(big)  # auto: cuSOLVER beyond the kernel's size
    assert torch.allclose(v2, torch.ones_like(v2))


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16, torch.float32])
def test_sq_partials(dtype):
    from reelcache_b200.ops.fitter import sq_partials
    x = (torch.randn(1001, 333, device="cuda") * 3).to(dtype)
    r = torch.randn(1001, 333, device="cuda")
    out = sq_partials(x, r, 2.5).sum(0)
    xd = x.double()
    assert abs(float(out[0]) - float((xd / 2.5).square().sum())) < 1e-5 * float((xd / 2.5).square().sum())
    ref_d = float(((xd - r.double()) / 2.5).square().sum())
    assert abs(float(out[1]) - ref_d) < 1e-5 * ref_d
    assert float(out[2]) == 0.0
    x2 = x.clone()
    x2[500, 7] = float("inf")
    assert float(sq_partials(x2).sum(0)[2]) > 0
    # strided (transposed) views
    xt = x.t()
    assert abs(float(sq_partials(xt).sum(0)[0]) - float(xd.square().sum())) < 1e-5 * float(xd.square().sum())


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32, torch.float16])
def test_fingerprint_kernel_equals_host(dtype):
    from reelcache_b200.lineage_commit import _fingerprint_terms_host, fingerprint_terms, source_fingerprint
    x = (torch.randn(4680, 1536, device="cuda") * 50).to(dtype)
    assert torch.equal(fingerprint_terms(x).cpu(), _fingerprint_terms_host(x.cpu()))
    assert source_fingerprint(x) == source_fingerprint(x.cpu())


def test_dot2_gemm_is_compensated():
    from reelcache_b200.ops.fitter import dot2_gemm
    x = torch.randn(300, 2000, device="cuda")
    rows = torch.randn(70, 2000, device="cuda")
    ref = x.double() @ rows.double().t()
    got = dot2_gemm(x, rows)
    # correctly rounded to FP32 up to a couple of ulps
    assert float(((got.double() - ref).abs() / ref.abs().clamp_min(1e-3)).median()) < 1e-7
    torch.backends.cuda.matmul.allow_tf32 = False
    assert _err(got, ref) < _err(x @ rows.t(), ref)


def test_planner_uses_jacobi_and_fitter_gram_batched():
    from reelcache_b200 import gpu_fitting
    from reelcache_b200.rank_method import RankMethodConfig, plan_chunk
    from reelcache_b200.types import CodecSpec, MatrixKey, ModelIdentity, TensorContext, energy_targets
    model = ModelIdentity("fit", "f", 2, 256, "THD", "bfloat16")
    g = torch.Generator(device="cuda").manual_seed(0)
    matrices, contexts = {}, {}
    for layer in range(2):
        for target in ("K", "V"):
            key = MatrixKey(layer, target)
            base = torch.randn(1024, 24, device="cuda", generator=g) @ torch.randn(24, 256, device="cuda", generator=g)
            matrices[key] = (base + 0.01 * torch.randn(1024, 256, device="cuda", generator=g)).to(torch.bfloat16)
            contexts[key] = TensorContext(model, key, 0, 4, 16, 16, "pre_rope" if target == "K" else "none")
    cfg = RankMethodConfig(energy_targets("causvid"), CodecSpec("svd_hevc", 32))
    before = gpu_fitting.STATS["jacobi_calls"]
    plans = plan_chunk(matrices, contexts, cfg, None, {}, {})
    assert gpu_fitting.STATS["jacobi_calls"] > before
    for key, plan in plans.items():
        assert plan.energy.stored_factor_energy >= cfg.targets.for_target(key.target) - 1e-6
    uuid = "GPU-" + str(torch.cuda.get_device_properties(0).uuid).removeprefix("GPU-")
    fitter = gpu_fitting.GPUFitter(gpu_id=0, gpu_uuid=uuid, method="gram_batched")
    items = {key: (matrices[key].float(), contexts[key], 24) for key in matrices}
    fitter.prefit(items)
    factors = fitter.fit(items[MatrixKey(0, "K")][0], contexts[MatrixKey(0, "K")], 24)
    assert fitter.prefit_stats["hits"] == 1 and factors.metrics["projection_relative_residual"] < 0.05


@pytest.mark.parametrize("rank", [37, 64, 300])
def test_device_finalization_matches_host(rank):
    import numpy as np
    from reelcache_b200.node_packets import finalize_tile
    g = torch.Generator().manual_seed(rank)
    coefficients = torch.randn(3 * 30 * 52, rank, generator=g) * 3
    host = finalize_tile(coefficients, (3, 30, 52))
    device = finalize_tile(coefficients.cuda(), (3, 30, 52)).to_host()
    assert np.array_equal(device.canvas, host.canvas)
    assert np.array_equal(device.affine, host.affine)
