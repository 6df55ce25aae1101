"""One tiny end-to-end pass of the flagship path on a CUDA device (used by the driver's smoke check):
restore a compressed chunk history into a KV cache with the fused sm_100a kernel and run one tcgen05
GEMM, checking both against fp64 / fp32 references."""

from __future__ import annotations

import numpy as np
import torch

from . import _hevc
from . import restore_kernels as rk
from .ops import _ext, gemm


def run(device):
    torch.manual_seed(0)
    rng = np.random.default_rng(0)
    frames, height, width, rank, heads, head_dim = 1, 8, 16, 64, 2, 128
    tokens = frames * height * width
    values = rng.standard_normal((tokens, rank)).astype(np.float32)
    pixels, affine, norm = _hevc.quantize_coefficients(values, "per_channel")
    layout = _hevc.video_layout(frames, height, width, rank)
    canvases = torch.from_numpy(_hevc.mosaic_all(pixels, layout)).to(device)
    scale, offset = rk.expand_affine(affine, norm, rank)
    source = rk.PictureSource.from_canvases(canvases, layout, [[s] for s in range(layout["segments"])], (0, 0),
                                            scale, offset)
    basis = (torch.randn(rank, heads * head_dim) / 16).half().to(device)
    cache = torch.zeros((1, tokens, heads, head_dim), dtype=torch.bfloat16, device=device)
    table = rk.RopeTable.wan(head_dim, 32, device=device)
    job = rk.ReconstructionJob(source, rk.NativeView(cache), (frames, height, width), basis,
                               rope=rk.RopePositions(table, (0, 0, 0)))
    rk.reconstruct([job], backend="fused", precision="fp16x2").release()  # the precision its bound describes
    _ext.check_status(device)
    expect, bound = rk.kernel_error_bound(job, "fp16x2")
    got = cache[0].reshape(tokens, -1).double()
    assert bool(((got - expect).abs() <= bound).all()), "fused restore exceeded its error bound"
    a = torch.randn(256, 128, device=device, dtype=torch.bfloat16)
    b = torch.randn(192, 128, device=device, dtype=torch.bfloat16)
    out = gemm.matmul_tn(a, b)
    torch.cuda.synchronize(device)
    _ext.check_status(device)
    ref = a.float() @ b.float().t()
    assert torch.allclose(out, ref, atol=1e-2, rtol=1e-3), "tcgen05 GEMM mismatch"
    return {"restore_max_err": float((got - expect).abs().max()), "gemm_max_err": float((out - ref).abs().max())}
