"""tcgen05 GEMM numerics against an fp32 PyTorch reference of the same op."""

import pytest
import torch

pytestmark = pytest.mark.gpu


def _ref(a, b, bias=None):
    out = a.float() @ b.float().t()
    if bias is not None:
        out = out + bias.float()
    return out


@pytest.mark.parametrize("m,n,k", [(128, 256, 64), (300, 520, 200), (4680, 1536, 1536), (77, 4608, 1536),
                                   (1000, 8960, 1536), (4680, 1536, 8960)])
def test_gemm_store_matches_fp32(cuda_device, m, n, k):
    from reelcache_b200.ops import gemm, _ext

    torch.manual_seed(0)
    a = torch.randn(m, k, device=cuda_device, dtype=torch.bfloat16)
    b = torch.randn(n, k, device=cuda_device, dtype=torch.bfloat16)
    out = gemm.matmul_tn(a, b, out_dtype=torch.float32)
    torch.cuda.synchronize()
    _ext.check_status(cuda_device)
    ref = _ref(a, b)
    err = (out - ref).abs().max().item()
    scale = (a.float().abs() @ b.float().abs().t()).max().item()
    assert err <= 1e-5 * scale + 1e-3, (err, scale)


@pytest.mark.parametrize("bn", [128, 192, 256])
def test_gemm_bias_tiles(cuda_device, bn):
    from reelcache_b200.ops import gemm, _ext

    torch.manual_seed(1)
    a = torch.randn(520, 384, device=cuda_device, dtype=torch.bfloat16)
    b = torch.randn(700, 384, device=cuda_device, dtype=torch.bfloat16)
    bias = torch.randn(700, device=cuda_device, dtype=torch.bfloat16)
    out = gemm.linear(a, b, bias, bn=bn)
    torch.cuda.synchronize()
    _ext.check_status(cuda_device)
    ref = _ref(a, b, bias)
    assert torch.allclose(out.float(), ref, atol=0.25, rtol=2e-2)


@pytest.mark.parametrize("m", [333, 1100])
def test_gemm_gelu_and_gated_residual(cuda_device, m):
    """Fused GELU and gated-residual epilogues; ``m`` = 1100 leaves a partial last row tile."""
    from reelcache_b200.ops import gemm, _ext

    torch.manual_seed(2)
    x = torch.randn(m, 256, device=cuda_device, dtype=torch.bfloat16)
    w = torch.randn(512, 256, device=cuda_device, dtype=torch.bfloat16) * 0.05
    bias = torch.randn(512, device=cuda_device, dtype=torch.bfloat16)
    out = gemm.linear_gelu(x, w, bias)
    ref = torch.nn.functional.gelu(_ref(x, w, bias), approximate="tanh")
    torch.cuda.synchronize()
    assert torch.allclose(out.float(), ref, atol=3e-2, rtol=2e-2)
    w2 = torch.randn(256, 512, device=cuda_device, dtype=torch.bfloat16) * 0.05
    bias2 = torch.randn(256, device=cuda_device, dtype=torch.bfloat16)
    gate = torch.randn(256, device=cuda_device, dtype=torch.float32)
    resid = torch.randn(m, 256, device=cuda_device, dtype=torch.bfloat16)
    expect = resid.float() + _ref(out, w2, bias2) * gate
    gemm.linear_gated_residual(out, w2, bias2, gate, resid)
    torch.cuda.synchronize()
    _ext.check_status(cuda_device)
    assert torch.allclose(resid.float(), expect, atol=6e-2, rtol=2e-2)


_PAIR_SCRIPT = """
import sys, torch
sys.path.insert(0, {root!r})
from reelcache_b200.ops import gemm, _ext
torch.manual_seed(3)
dev = torch.device("cuda", 0)
worst = 0.0
for bn in (128, 192, 256):
    for m, n, k, epi in ((1300, 1000, 320, "bias"), (1100, 520, 256, "gelu"), (700, 264, 512, "gated")):
        a = torch.randn(m, k, device=dev, dtype=torch.bfloat16)
        b = torch.randn(n, k, device=dev, dtype=torch.bfloat16) * 0.05
        bias = torch.randn(n, device=dev, dtype=torch.bfloat16)
        ref = a.float() @ b.float().t() + bias.float()
        if epi == "bias":
            out = gemm.linear(a, b, bias, bn=bn, out_dtype=torch.float32).float()
        elif epi == "gelu":
            out = gemm.linear_gelu(a, b, bias).float()
            ref = torch.nn.functional.gelu(ref, approximate="tanh")
        else:
            gate = torch.randn(n, device=dev)
            resid = torch.randn(m, n, device=dev, dtype=torch.bfloat16)
            ref = resid.float() + ref * gate
            out = gemm.linear_gated_residual(a, b, bias, gate, resid).float()
        torch.cuda.synchronize()
        _ext.check_status(dev)
        worst = max(worst, ((out - ref).abs() / (0.05 + 0.02 * ref.abs())).max().item())
print("worst", worst)
assert worst <= 1.0, worst
"""


def test_gemm_pair_kernel(cuda_device):
    """The opt-in paired-CTA kernel (tcgen05 cta_group::2, 256-row tiles; REELCACHE_GEMM_PAIRS=1, read once per
    process, hence a child process) on partial row / column tiles with each N tile and epilogue."""
    import os
    import subprocess
    import sys
    from pathlib import Path

    root = str(Path(__file__).resolve().parents[1])
    env = dict(os.environ, REELCACHE_GEMM_PAIRS="1")
    run = subprocess.run([sys.executable, "-c", _PAIR_SCRIPT.format(root=root)], env=env, capture_output=True,
                         text=True, timeout=300)
    assert run.returncode == 0, run.stdout + run.stderr

