"""Device finalization of coefficient tiles (csrc/fit/quantize.cu): per-column extrema on the GPU, the
covering FP32 affine on the host from the copied extrema (the reference's ``_covering_affine``), then
an FP64 ``rint`` quantization on the GPU that is bitwise equal to ``_hevc.quantize_coefficients``."""

from __future__ import annotations

import numpy as np
import torch

from .. import _hevc
from ..errors import ConfigurationError
from ._ext import ext


def column_extrema(p: torch.Tensor) -> tuple[np.ndarray, np.ndarray]:
    p = p.float().contiguous()
    lo = torch.empty(p.shape[1], dtype=torch.float32, device=p.device)
    hi = torch.empty_like(lo)
    bad = torch.zeros(1, dtype=torch.int32, device=p.device)
    ext().colminmax(p, lo, hi, bad)
    packed = torch.cat([lo, hi, bad.float()]).cpu().numpy()
    if packed[-1] != 0:
        raise ConfigurationError("coefficients must be finite")
    r = p.shape[1]
    return packed[:r].copy(), packed[r:2 * r].copy()


def quantize_device(p: torch.Tensor, normalization: str = "per_channel", protected_fraction: float = 1.0,
                    *, out: torch.Tensor | None = None, as_numpy: bool = True):
    """``(pixels, affine [2, records], layout)``; pixels are a host numpy array unless ``as_numpy=False``."""
    p = p.float().contiguous()
    lo, hi = column_extrema(p)
    layout = _hevc.normalization_layout(p.shape[1], normalization, protected_fraction)
    affine = _hevc.affine_for(lo, hi, layout)
    scale, offset = _hevc.expanded_affine(affine, layout, p.shape[1])
    scale_t = torch.from_numpy(np.ascontiguousarray(scale, dtype=np.float32)).to(p.device)
    offset_t = torch.from_numpy(np.ascontiguousarray(offset, dtype=np.float32)).to(p.device)
    if out is None:
        out = torch.empty(p.shape, dtype=torch.uint8, device=p.device)
    ext().quantize_columns(p, scale_t, offset_t, out)
    pixels = out[:, :p.shape[1]]
    return (pixels.cpu().numpy() if as_numpy else pixels), affine, layout
