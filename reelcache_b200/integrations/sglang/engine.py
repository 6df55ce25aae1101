"""Chunk engines behind the serving bridge.

An engine owns the model side of the seam (:mod:`.seam`): it allocates a native KV cache, generates one
chunk (denoising forwards, then the clean forward whose per-layer pre-RoPE K / V go to the capture
scope), replays a recorded chunk's clean forward from its stored latents (``restore_mode="recompute"``),
re-runs a recache window under a new prompt, and installs restored history into a cache. The bridge is
engine-agnostic.

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
from .profiles import ModelProfile


@dataclass
class InstallResult:
    """Handle of an installed (possibly still running) history restore."""

    wait: Callable[..., None]  # wait(layer[, stream])
    join: Callable[[], Any]
    stats: dict


def prompt_scale(prompt: str | None) -> float:
    """A deterministic per-prompt gain of the synthetic engine's K / V (1.0 for the default conditioning)."""
    if prompt is None:
        return 1.0
    return 1.0 + (int(hashlib.sha256(prompt.encode()).hexdigest()[:8], 16) % 97) / 128.0


class SyntheticEngine:
    """Synthetic low-rank K / V; a chunk's K / V are a function of its latents and its prompt only, so a replay
    from stored latents or a recache under another prompt reproduces them bit for bit."""

    def __init__(self, profile: ModelProfile, identity: ModelIdentity, device="cpu", *, rank: int = 6, seed: int = 0,
                 dtype=torch.float32):
        self.profile = profile
        self.identity = identity
        self.device = torch.device(device)
        self.rank = rank
        self.seed = seed
        self.dtype = dtype
        self.forwards = {"generate": 0, "replay": 0, "recache": 0}

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

    def _write(self, cache: dict, index: int, latents: torch.Tensor, prompt: str | None, capture=None, *,
               write: bool = True) -> None:
        per_chunk = self.profile.chunk_tokens
        start = index * per_chunk
        gain = prompt_scale(prompt)
        for layer in range(self.profile.num_layers):
            rows = {}
            for target in ("K", "V"):
                scale = gain if target == "K" else 1.0 / gain
                rows[target] = ((latents * scale) @ self._bases(layer, target)).to(self.dtype).to(self.device)
                if write:
                    (cache["k"] if target == "K" else cache["v"])[layer][start:start + per_chunk] = rows[target]
            if capture is not None:
                capture(layer, rows["K"].clone(), rows["V"].clone())
        if write:
            cache["end"] = max(cache.get("end", 0), start + per_chunk)

    def generate_chunk(self, cache: dict, index: int, capture, *, request_seed: int = 0,
                       layer_wait: Callable[..., None] | None = None, prompt: str | None = None) -> torch.Tensor:
        """Latents from a generator folded with a digest of the attended history, then the clean write."""
        per_chunk = self.profile.chunk_tokens
        if layer_wait is not None:
            for layer in range(self.profile.num_layers):
                layer_wait(layer)
        digest = self.history_digest(cache, index * per_chunk)
        g = torch.Generator().manual_seed((request_seed * 1_000_003 + index * 9176 + digest) & 0x7FFFFFFF)
        latents = torch.randn(per_chunk, self.rank, generator=g) * torch.tensor(
            [1.0 / (i + 1) for i in range(self.rank)])
        self._write(cache, index, latents, prompt, None if capture is None else capture.capture_layer)
        self.forwards["generate"] += 1
        return latents

    def replay_chunk(self, cache: dict, index: int, latents: torch.Tensor, *, prompt: str | None = None) -> None:
        """The clean forward of a recorded chunk from its stored latents (recompute restore)."""
        self._write(cache, index, latents.cpu(), prompt)
        self.forwards["replay"] += 1

    def recache(self, cache: dict, plan, capture, *, prompt: str | None, latents) -> None:
        """Re-run the window's chunks under ``prompt``; only the written chunks' K / V are stored (and captured as
        one range per layer)."""
        chunk_frames = self.profile.chunk_frames
        first, write, end = (plan.window_start_frame // chunk_frames, plan.write_start_frame // chunk_frames,
                             plan.end_frame // chunk_frames)
        pieces: dict[int, list] = {}
        for index in range(first, end):
            written = index >= write

            def keep(layer, k, v, written=written):
                if written:
                    pieces.setdefault(layer, []).append((k, v))
            self._write(cache, index, latents[index].cpu(), prompt, keep, write=written)
        if capture is not None:
            for layer in range(self.profile.num_layers):
                parts = pieces.get(layer, [])
                if parts:
                    capture.capture_layer(layer, torch.cat([k for k, _ in parts]), torch.cat([v for _, v in parts]))
        self.forwards["recache"] += 1

    def install(self, cache: dict, archive, head_ref: str, plan, *, overlapped: bool = True) -> InstallResult:
        """Dense history from the archive (raw tier first, then the CPU reference decode)."""
        stats = archive.install_dense(cache, head_ref, plan, self.profile.num_layers)
        return InstallResult(lambda layer, stream=None: None, lambda: stats, stats)


class CausalWanEngine:
    """The CausVid-shaped DiT on one GPU (full-history visibility). ``prompts`` maps a prompt to its text K / V
    (default: ``text_kv`` for every prompt)."""

    def __init__(self, model, text_kv, profile: ModelProfile, identity: ModelIdentity, *, attention_backend="auto",
                 prompts: Callable[[str], Any] | None = None):
        if profile.visibility != "full_history":
            raise UnsupportedError("the CausVid-shaped DiT attends to its full history; sink-window profiles need "
                                   "a windowed cache")
        self.model = model
        self.text_kv = text_kv
        self.prompts = prompts
        self.profile = profile
        self.identity = identity
        self.device = model.device
        self.attention_backend = attention_backend

    def _text(self, prompt: str | None):
        return self.text_kv if prompt is None or self.prompts is None else self.prompts(prompt)

    def new_cache(self, capacity_chunks: int):
        from ...models.causal_wan import KVCache
        return KVCache(self.model.cfg, capacity_chunks, self.device)

    def _generator(self, cache, prompt, seed: int = 0):
        from ...models.sampler import ChunkGenerator
        return ChunkGenerator(self.model, cache, self._text(prompt), timesteps=self.profile.timesteps, seed=seed,
                              attention_backend=self.attention_backend)

    def generate_chunk(self, cache, index: int, capture, *, request_seed: int = 0, layer_wait=None,
                       prompt: str | None = None) -> torch.Tensor:
        gen = self._generator(cache, prompt, request_seed * 1_000_003 + index)
        latents = gen.denoise(index, layer_wait=layer_wait)

        def take(layer, k_pre, v):
            capture.capture_layer(layer, k_pre.clone(), v.clone())

        gen.commit_clean(index, latents, capture=None if capture is None else take)
        return latents

    def replay_chunk(self, cache, index: int, latents: torch.Tensor, *, prompt: str | None = None) -> None:
        """The chunk's clean (t = 0) forward from its stored latents: rebuilds its K / V in the cache."""
        self._generator(cache, prompt).commit_clean(index, latents.to(self.device))

    def recache(self, cache, plan, capture, *, prompt: str | None, latents) -> None:
        """The written chunks' clean forwards, in order, under the new prompt (the DiT is causal, so the kept sink
        and the earlier written chunks are what each re-run chunk attends to); captured as one range per layer."""
        chunk_frames = self.profile.chunk_frames
        gen = self._generator(cache, prompt)
        pieces: dict[int, list] = {}

        def take(layer, k_pre, v):
            pieces.setdefault(layer, []).append((k_pre.clone(), v.clone()))

        for index in range(plan.write_start_frame // chunk_frames, plan.end_frame // chunk_frames):
            gen.commit_clean(index, latents[index].to(self.device), capture=take)
        if capture is not None:
            for layer, parts in sorted(pieces.items()):
                capture.capture_layer(layer, torch.cat([k for k, _ in parts]), torch.cat([v for _, v in parts]))

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
