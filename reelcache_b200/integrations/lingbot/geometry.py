"""LingBot-World-Fast geometry (reference: integrations/lingbot/README.md:4-8, reelcache_lingbot/lb_model.py:121-160).

40 transformer blocks, 40 heads of 128 channels (5,120 KV channels per layer), chunks of 3 latent frames, a
480 x 832 video at a 16-pixel latent patch (30 x 52 = 1,560 tokens per latent frame, 4,680 per chunk), attention
over a window of ``window_latents`` latent frames (21 by default: 7 chunks) plus optional sink frames.
"""

from __future__ import annotations

from dataclasses import dataclass, replace

from ...types import ModelIdentity


@dataclass(frozen=True)
class LingBotGeometry:
    layers: int = 40
    heads: int = 40
    head_dim: int = 128
    frames_per_chunk: int = 3
    latent_height: int = 30
    latent_width: int = 52
    window_latents: int = 21
    sink_latents: int = 0
    dtype: str = "bfloat16"
    name: str = "lingbot-world-fast"
    fingerprint: str = "wan2.2-i2v-a14b-fast"

    def __post_init__(self):
        for field in ("layers", "heads", "head_dim", "frames_per_chunk", "latent_height", "latent_width",
                      "window_latents"):
            value = getattr(self, field)
            if type(value) is not int or value < 1:
                raise ValueError(f"LingBot geometry: {field} must be a positive integer, got {value!r}")
        if self.window_latents % self.frames_per_chunk or self.sink_latents % self.frames_per_chunk:
            raise ValueError("LingBot geometry: the window and the sink hold whole chunks")
        if self.head_dim % 2:
            raise ValueError("LingBot geometry: RoPE rotates channel pairs, head_dim must be even")

    @property
    def channels(self) -> int:
        return self.heads * self.head_dim

    @property
    def frame_tokens(self) -> int:
        return self.latent_height * self.latent_width

    @property
    def chunk_tokens(self) -> int:
        return self.frames_per_chunk * self.frame_tokens

    @property
    def window_chunks(self) -> int:
        return self.window_latents // self.frames_per_chunk

    @property
    def sink_chunks(self) -> int:
        return self.sink_latents // self.frames_per_chunk

    def chunk_bytes(self, element_bytes: int = 2) -> int:
        """Bytes of one chunk's K and V over every layer in the native cache."""
        return 2 * self.layers * self.chunk_tokens * self.channels * element_bytes

    def identity(self) -> ModelIdentity:
        return ModelIdentity(self.name, self.fingerprint, self.layers, self.channels, "BTHD", self.dtype)

    def scaled(self, **overrides) -> "LingBotGeometry":
        """The same geometry with some fields replaced (tests and stand-ins run smaller versions)."""
        return replace(self, **overrides)


LINGBOT_WORLD_FAST = LingBotGeometry()
