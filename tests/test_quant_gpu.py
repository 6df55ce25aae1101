"""Device quantization is bitwise equal to the host covering-affine quantization."""

import numpy as np
import pytest
import torch

from reelcache_b200 import _hevc

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("normalization", ["per_channel", "global", "leading_columns"])
def test_device_quantize_matches_host(cuda_device, normalization):
    from reelcache_b200.ops.quant import quantize_device

    rng = np.random.default_rng(0)
    values = (rng.standard_normal((4680, 96)) * rng.uniform(0.01, 10, 96)).astype(np.float32)
    pixels, affine, layout = _hevc.quantize_coefficients(values, normalization, 0.25)
    dpix, daff, dlay = quantize_device(torch.from_numpy(values).to(cuda_device), normalization, 0.25)
    assert np.array_equal(affine, daff) and layout == dlay
    assert np.array_equal(pixels, dpix)
