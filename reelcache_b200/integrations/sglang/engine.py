"""Chunk engines behind the serving bridge.

An engine owns the model side of the seam: it allocates a native KV cache, generates one chunk
(denoising forwards, then the clean forward whose per-layer pre-RoPE K / V go to the capture
builder), and installs restored history into a cache. The bridge is engine-agnostic.

* :class:`CausalWanEngine` -- the CausVid-shaped DiT of :mod:`reelcache_b200.models` on one GPU; it
  installs archived history with the fused sm_100a restore (:class:`LineageRestorer`), layer by layer,
  overlapped with the first forward of the next chunk.
* :class:`SyntheticEngine` -- deterministic synthetic low-rank K / V on any device (CPU tests and
  host-side workload runs); its "forward" folds a digest of the attended history into the output,
  so divergent histories produce divergent chunks.
"""

from __future__ import annotations

import hashlib
from dataclasses import dataclass
from typing import Any, Callable

import torch

from ...errors import UnsupportedError
from ...types import MatrixKey, ModelIdentity
from .capture import CleanChunkBuilder
from .profiles import ModelProfile


@dataclass
class InstallResult:
    """Handle of an installed (possibly still running) history restore."""

    wait: Callable[..., None]  # wait(layer[, stream])
    join: Callable[[], Any]
    stats: dict


class SyntheticEngine:
    def __init__(self, profile: ModelProfile, identity: ModelIdentity, device="cpu", *, rank: int = 6, seed: int = 0,
                 dtype=torch.float32):
        self.profile = profile
        self.identity = identity
        self.device = torch.device(device)
        self.rank = rank
        self.seed = seed
        self.dtype = dtype

    def new_cache(self, capacity_chunks: int) -> dict:
        tokens = capacity_chunks * self.profile.chunk_tokens
        c = self.profile.channels
        return {"k": [torch.zeros(tokens, c, dtype=self.dtype, device=self.device) for _ in range(self.profile.num_layers)],
                "v": [torch.zeros(tokens, c, dtype=self.dtype, device=self.device) for _ in range(self.profile.num_layers)],
                "end": 0}

    def _bases(self, layer: int, target: str) -> torch.Tensor:
        g = torch.Generator().manual_seed(self.seed * 7919 + layer * 2 + (target == "V"))
        q = torch.linalg.qr(torch.randn(self.profile.channels, self.rank, generator=g))[0]
        return q.t().contiguous()

    def history_digest(self, cache: dict, tokens: int) -> int:
        if tokens == 0:
            return 0
        k = cache["k"][0][:tokens].double()
        return int(torch.round(k.abs().sum() * 1e3).item()) & 0x7FFFFFFF

    def generate_chunk(self, cache: dict, index: int, builder: CleanChunkBuilder, *, request_seed: int = 0,
                       layer_wait: Callable[[int], None] | None = None) -> torch.Tensor:
        per_chunk = self.profile.chunk_tokens
        if layer_wait is not None:
            for layer in range(self.profile.num_layers):
                layer_wait(layer)
        digest = self.history_digest(cache, index * per_chunk)
        g = torch.Generator().manual_seed((request_seed * 1_000_003 + index * 9176 + digest) & 0x7FFFFFFF)
        start = index * per_chunk
        for layer in range(self.profile.num_layers):
            for target in ("K", "V"):
                coeff = torch.randn(per_chunk, self.rank, generator=g) * torch.tensor(
                    [1.0 / (i + 1) for i in range(self.rank)])
                matrix = (coeff @ self._bases(layer, target)).to(self.dtype).to(self.device)
                (cache["k"] if target == "K" else cache["v"])[layer][start:start + per_chunk] = matrix
            builder.capture_layer(layer, cache["k"][layer][start:start + per_chunk].clone(),
                                  cache["v"][layer][start:start + per_chunk].clone())
        cache["end"] = start + per_chunk
        return torch.tensor([float(digest), float(index)])

    def install(self, cache: dict, archive, head_ref: str, plan, *, overlapped: bool = True) -> InstallResult:
        """Dense history from the archive (raw tier first, then the CPU reference decode)."""
        stats = archive.install_dense(cache, head_ref, plan, self.profile.num_layers)
        return InstallResult(lambda layer: None, lambda: stats, stats)


class CausalWanEngine:
    """The CausVid-shaped DiT on one GPU (full-history visibility)."""

    def __init__(self, model, text_kv, profile: ModelProfile, identity: ModelIdentity, *, attention_backend="auto"):
        if profile.visibility != "full_history":
            raise UnsupportedError("the CausVid-shaped DiT attends to its full history; sink-window profiles need "
                                   "a windowed cache")
        self.model = model
        self.text_kv = text_kv
        self.profile = profile
        self.identity = identity
        self.device = model.device
        self.attention_backend = attention_backend

    def new_cache(self, capacity_chunks: int):
        from ...models.causal_wan import KVCache
        return KVCache(self.model.cfg, capacity_chunks, self.device)

    def generate_chunk(self, cache, index: int, builder: CleanChunkBuilder, *, request_seed: int = 0,
                       layer_wait=None) -> torch.Tensor:
        from ...models.sampler import ChunkGenerator
        gen = ChunkGenerator(self.model, cache, self.text_kv, timesteps=self.profile.timesteps,
                             seed=request_seed * 1_000_003 + index, attention_backend=self.attention_backend)
        latents = gen.denoise(index, layer_wait=layer_wait)

        def capture(layer, k_pre, v):
            builder.capture_layer(layer, k_pre.clone(), v.clone())

        gen.commit_clean(index, latents, capture=capture)
        return latents

    def install(self, cache, archive, head_ref: str, plan, *, overlapped: bool = True) -> InstallResult:
        from .restore import LineageInstall
        cfg = self.model.cfg

        def destination(layer, which):
            return cache.k[layer] if which == "K" else cache.v[layer]

        install = LineageInstall(plan=plan, destination=destination,
                                 rope_rows=lambda chunk: (cfg.frames_per_chunk * chunk, 0, 0), table=self.model.rope,
                                 tokens_per_frame=cfg.grid_h * cfg.grid_w)
        result = archive.restore_into(head_ref, install, plan, overlapped=overlapped)

        def join():
            stats = result.join()
            result.lease.close()
            return stats

        # the DiT calls wait(layer, stream): the stream is ordered after the layer's restore events
        return InstallResult(lambda layer, stream=None: result.wait(layer, stream), join, result.stats)


def model_identity_for(profile: ModelProfile, fingerprint: str) -> ModelIdentity:
    return ModelIdentity(profile.backbone, fingerprint, profile.num_layers, profile.channels, "BTHD",
                         profile.native_dtype)


def digest_tensor(t: torch.Tensor) -> str:
    return hashlib.sha256(t.detach().float().cpu().numpy().tobytes()).hexdigest()
