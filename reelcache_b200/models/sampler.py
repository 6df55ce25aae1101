"""Chunk-wise causal generation with a few-step DMD flow sampler and the archival / restore seams
(reference: causal_wan/sampling.py:20-100 and sglang_stages.py:229-939; SGLang patch 0016 for the
layer-overlapped restore).

Per chunk: ``len(timesteps)`` denoising forwards (CausVid: 1000, 757, 522) predict the flow
``v = eps - x0`` with ``x_t = (1 - s) x0 + s eps`` (``s = t / 1000``), re-noising the predicted ``x0``
between steps; then one clean forward at ``t = 0`` writes the chunk's K/V into its cache slot and
hands the normalized pre-RoPE K and the V of every layer to the capture hook (the archive seam).
"""

from __future__ import annotations

from dataclasses import dataclass, field
from typing import Callable

import torch

from .causal_wan import CausalWanDiT, KVCache

CAUSVID_TIMESTEPS = (1000.0, 757.0, 522.0)


@dataclass
class ChunkResult:
    index: int
    latents: torch.Tensor          # denoised x0 [in_dim, F, H, W] (FP32)
    events: dict = field(default_factory=dict)


class ChunkGenerator:
    """Drives :class:`CausalWanDiT` chunk by chunk over one :class:`KVCache`."""

    def __init__(self, model: CausalWanDiT, cache: KVCache, text_kv, *, timesteps=CAUSVID_TIMESTEPS, seed: int = 0,
                 attention_backend: str = "auto", group=None):
        """``group``: a Ulysses sequence-parallel process group (the cache is then this rank's
        :class:`~reelcache_b200.models.causal_wan.SPKVCache`; every rank draws the same noise)."""
        self.group = group
        self.model = model
        self.cache = cache
        self.text_kv = text_kv
        self.timesteps = tuple(timesteps)
        self.generator = torch.Generator(device=model.device).manual_seed(seed)
        self.attention_backend = attention_backend

    def _forward(self, *args, **kwargs):
        if self.group is None:
            return self.model.forward_chunk(*args, **kwargs)
        return self.model.forward_chunk_sp(*args, group=self.group, **kwargs)

    def noise(self) -> torch.Tensor:
        cfg = self.model.cfg
        return torch.randn((cfg.in_dim, cfg.frames_per_chunk, cfg.latent_height, cfg.latent_width),
                           generator=self.generator, device=self.model.device)

    def denoise(self, index: int, *, layer_wait: Callable | None = None) -> torch.Tensor:
        """The chunk's denoised latents (the "first new chunk"); the first forward may wait per layer on
        an overlapped restore (``layer_wait``)."""
        x = self.noise()
        x0 = x
        for step, t in enumerate(self.timesteps):
            sigma = t / 1000.0
            flow = self._forward(x, t, index, self.cache, self.text_kv,
                                            layer_wait=layer_wait if step == 0 else None,
                                            attention_backend=self.attention_backend)
            x0 = x - sigma * flow
            if step + 1 < len(self.timesteps):
                nxt = self.timesteps[step + 1] / 1000.0
                x = (1.0 - nxt) * x0 + nxt * self.noise()
        return x0

    def commit_clean(self, index: int, latents: torch.Tensor, *, capture: Callable | None = None) -> None:
        """The clean (t = 0) forward: writes the chunk's clean K/V into its slot; ``capture(layer, k_pre, v)``
        receives the archive inputs."""
        self._forward(latents, 0.0, index, self.cache, self.text_kv, capture=capture,
                                 attention_backend=self.attention_backend)
        self.cache.length = max(self.cache.length, (index + 1) * self.model.cfg.chunk_tokens)

    def generate(self, index: int, *, capture: Callable | None = None, layer_wait: Callable | None = None) -> ChunkResult:
        latents = self.denoise(index, layer_wait=layer_wait)
        self.commit_clean(index, latents, capture=capture)
        return ChunkResult(index, latents)
