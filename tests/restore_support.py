"""Synthetic restore jobs shared by the CPU and GPU restore tests."""

import numpy as np
import torch

from reelcache_b200 import _hevc
from reelcache_b200 import restore_kernels as rk


def picture_job(device, *, frames=3, height=30, width=52, rank=96, heads=4, head_dim=128, rows=None, seed=0,
                rope=True, out_dtype=torch.bfloat16, layout="BTHD", token_offset=0, capacity=None,
                destination=None, table=None, rope_rows=(0, 0, 0)):
    rng = np.random.default_rng(seed)
    channels = heads * head_dim
    tokens = frames * height * width
    values = rng.standard_normal((tokens, rank)).astype(np.float32) * rng.uniform(0.1, 4.0, rank).astype(np.float32)
    pixels, affine, norm = _hevc.quantize_coefficients(values, "per_channel")
    lay = _hevc.video_layout(frames, height, width, rank, "yuv444p")
    canvases = torch.from_numpy(_hevc.mosaic_all(pixels, lay)).to(device)
    indices = [[s * frames + f for f in range(frames)] for s in range(lay["segments"])]
    scale, offset = rk.expand_affine(affine, norm, rank)
    source = rk.PictureSource.from_canvases(canvases, lay, indices, (0, 0), scale, offset)
    basis_rows = rows or rank
    q = torch.from_numpy(rng.standard_normal((basis_rows, channels)).astype(np.float32) / np.sqrt(channels))
    basis = q.to(torch.float16).to(device)
    if destination is None:
        cap = capacity or tokens + token_offset
        if layout == "BHTD":
            destination = torch.zeros((1, heads, cap, head_dim), dtype=out_dtype, device=device)
        elif layout == "THD":
            destination = torch.zeros((cap, heads, head_dim), dtype=out_dtype, device=device)
        else:
            destination = torch.zeros((1, cap, heads, head_dim), dtype=out_dtype, device=device)
    view = rk.NativeView(destination, layout, token_offset)
    positions = None
    if rope:
        table = table or rk.RopeTable.wan(head_dim, 128, device=device)
        positions = rk.RopePositions(table, rope_rows)
    job = rk.ReconstructionJob(source, view, (frames, height, width), basis, rope=positions)
    return job, pixels
