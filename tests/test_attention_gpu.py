"""The sm_100a tcgen05 flash-attention forward against an FP32 PyTorch softmax(Q K^T) V reference (and cuDNN's
fused SDPA for scale): ragged query and key counts, strided K/V cache views, the CausVid self- and cross-attention
shapes."""

import math

import pytest
import torch

pytestmark = pytest.mark.gpu


@pytest.fixture(autouse=True)
def _cuda():
    if not torch.cuda.is_available():
        pytest.skip("needs a GPU")
    from reelcache_b200.ops import _ext
    assert hasattr(_ext.ext(), "attention_fwd")


def _reference(q, k, v, scale):
    qf, kf, vf = (t.float().permute(1, 0, 2) for t in (q, k, v))
    p = torch.softmax(qf @ kf.transpose(1, 2) * scale, dim=-1)
    return (p @ vf).permute(1, 0, 2)


@pytest.mark.parametrize("tq,tk,heads", [(200, 77, 2), (128, 512, 3), (4680, 4680, 2), (333, 1000, 1),
                                         (4680, 18720, 12)])
def test_attention_matches_fp32(tq, tk, heads):
    from reelcache_b200.ops import _ext
    from reelcache_b200.ops.attention import attention
    g = torch.Generator(device="cuda").manual_seed(tq + tk)
    q = torch.randn(tq, heads, 128, device="cuda", generator=g).bfloat16()
    cache_k = torch.randn(tk + 64, heads, 128, device="cuda", generator=g).bfloat16() * 2
    cache_v = torch.randn(tk + 64, heads, 128, device="cuda", generator=g).bfloat16()
    k, v = cache_k[:tk], cache_v[:tk]            # cache views (row stride of the full buffer)
    scale = 1.0 / math.sqrt(128)
    got = attention(q, k, v, backend="fused", scale=scale)
    _ext.check_status(q.device)
    ref = _reference(q, k, v, scale)
    err = float((got.float() - ref).norm() / ref.norm())
    sdpa = attention(q, k, v, backend="sdpa", scale=scale)
    err_sdpa = float((sdpa.float() - ref).norm() / ref.norm())
    assert err < max(2e-2, 3 * err_sdpa), (err, err_sdpa)
    assert torch.isfinite(got.float()).all()


def test_attention_peaked_scores_rescale():
    """Rows whose maximum grows block after block exercise the lazy O rescaling."""
    from reelcache_b200.ops.attention import attention
    tq, tk, heads = 256, 1024, 2
    q = torch.ones(tq, heads, 128, device="cuda").bfloat16() * 0.25
    ramp = torch.linspace(0, 6, tk, device="cuda").view(tk, 1, 1)
    k = (torch.ones(tk, heads, 128, device="cuda") * ramp).bfloat16()
    v = torch.randn(tk, heads, 128, device="cuda").bfloat16()
    got = attention(q, k, v, backend="fused", scale=1.0)
    ref = _reference(q, k, v, 1.0)
    assert float((got.float() - ref).norm() / ref.norm()) < 2e-2


@pytest.mark.parametrize("tq,tk,ranges", [(300, 1000, 2), (4680, 4680, 3), (256, 2000, 4), (700, 390, 3)])
def test_attention_key_ranges_match_fp32(tq, tk, ranges):
    """Key ranges forced through the option word: each range's normalized partial output and log2-sum-exp,
    combined by the merge kernel, equal the single-pass result."""
    from reelcache_b200.ops import _ext
    from reelcache_b200.ops.attention import attention
    g = torch.Generator(device="cuda").manual_seed(7 * tq + tk)
    heads = 3
    q = torch.randn(tq, heads, 128, device="cuda", generator=g).bfloat16()
    k = torch.randn(tk, heads, 128, device="cuda", generator=g).bfloat16() * 2
    v = torch.randn(tk, heads, 128, device="cuda", generator=g).bfloat16()
    scale = 1.0 / math.sqrt(128)
    got = attention(q, k, v, backend="fused", scale=scale, options=ranges)
    single = attention(q, k, v, backend="fused", scale=scale, options=1)
    _ext.check_status(q.device)
    ref = _reference(q, k, v, scale)
    assert float((got.float() - ref).norm() / ref.norm()) < 2e-2
    assert float((got.float() - single.float()).abs().max()) < 3e-2


def test_attention_fma_exponentials_match_fp32():
    """A quarter of the exponentials on the FMA pipe (cubic fit of 2^f) stays within bf16 rounding of P."""
    from reelcache_b200.ops import _ext
    from reelcache_b200.ops.attention import OPT_POLY_EXP, attention
    g = torch.Generator(device="cuda").manual_seed(11)
    q = torch.randn(1000, 2, 128, device="cuda", generator=g).bfloat16()
    k = torch.randn(3000, 2, 128, device="cuda", generator=g).bfloat16() * 2
    v = torch.randn(3000, 2, 128, device="cuda", generator=g).bfloat16()
    got = attention(q, k, v, backend="fused", scale=0.1, options=OPT_POLY_EXP)
    _ext.check_status(q.device)
    ref = _reference(q, k, v, 0.1)
    assert float((got.float() - ref).norm() / ref.norm()) < 2e-2
