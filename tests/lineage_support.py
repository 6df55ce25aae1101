"""Tiny models and drifting low-rank chunks (the shape of the reference's step6 fixtures)."""

import math

import torch

from reelcache_b200.rank_method import RankMethodConfig
from reelcache_b200.types import CodecSpec, MatrixKey, ModelIdentity, TensorContext, energy_targets

MODEL = ModelIdentity("tiny-dit", "tiny-fp-1", 2, 128, "BTHD", "bfloat16")
FRAMES, HEIGHT, WIDTH = 2, 8, 16
TOKENS = FRAMES * HEIGHT * WIDTH


def method(**overrides):
    base = dict(targets=energy_targets("causvid"), codec=CodecSpec("svd_hevc", 32), solver="gram_eigh")
    base.update(overrides)
    return RankMethodConfig(**base)


def chunk(index, *, seed=0, drift=0.15, rank=12, model=MODEL, dtype=torch.float32):
    """Matrices whose dominant subspace drifts slowly from chunk to chunk."""
    gen = torch.Generator().manual_seed(seed)
    channels = model.channels_for("K")
    base = torch.linalg.qr(torch.randn(channels, channels, generator=gen))[0]
    matrices, contexts = {}, {}
    for layer in range(model.layers):
        for target in ("K", "V"):
            g = torch.Generator().manual_seed(seed * 1000 + layer * 10 + (target == "V") + 7 * index)
            angle = drift * index
            mix = torch.linalg.qr(torch.eye(channels) + angle * torch.randn(channels, channels, generator=g) * 0.1)[0]
            q = (base @ mix)[:, :rank].t()
            sigma = torch.tensor([1.0 / (i + 1) for i in range(rank)])
            u = torch.randn(TOKENS, rank, generator=g)
            x = (u * sigma) @ q + 1e-3 * torch.randn(TOKENS, channels, generator=g)
            key = MatrixKey(layer, target)
            matrices[key] = x.to(dtype)
            contexts[key] = TensorContext(model, key, index * TOKENS, FRAMES, HEIGHT, WIDTH,
                                          "pre_rope" if target == "K" else "none")
    return matrices, contexts


def relative_error(a, b):
    return float((a.float() - b.float()).norm() / b.float().norm())
