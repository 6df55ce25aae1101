"""LingBot's shared self-attention cache, the chunk KV capture / install hooks, and a stand-in world model
(reference: integrations/lingbot/runtime/lingbot_rt.py ChunkKV, reelcache_lingbot/lb_model.py:96-160, 414-456).

* :class:`SharedWindowCache` -- the one persistent self-attention cache of the model: per layer a K and a V
  tensor ``[1, slots * chunk_tokens, heads, head_dim]`` (BTHD). Chunk ``c`` lives in slot ``c`` while ``c`` is a
  sink chunk, else in slot ``sink + (c - sink) % window``; generating chunk ``n`` attends the sink chunks and the
  ``window - 1`` chunks before ``n``. Keys are stored after RoPE at the chunk's absolute frame position.
* :class:`ChunkKV` -- hooks on ``blocks[l].self_attn`` that capture a chunk's pre-RoPE K (the output of the key
  normalization when the attention has one, else of the key projection) and V (the value projection) during its
  clean pass, and install rows into the cache. Works on any module tree with that layout (the Wan blocks of the
  official pipeline included); ``remove()`` takes every hook off.
* :class:`StandInWorldModel` -- a small causal video transformer of the same interface (q / k / v / o projections,
  q / k RMSNorm, Wan 3-axis RoPE, windowed attention over the shared cache) used where the official pipeline and
  its weights are absent: CPU tests and GPU-sized smoke runs of the archive and the overlapped restore.
"""

from __future__ import annotations

from typing import Sequence

import torch

from ... import restore_kernels as rk
from ...restore_reference import apply_rope_reference
from .geometry import LingBotGeometry


class SharedWindowCache:
    """Sink + rolling-window slots of whole chunks, K and V per layer."""

    def __init__(self, geometry: LingBotGeometry, device, dtype=torch.bfloat16):
        self.geometry = geometry
        self.slots = geometry.sink_chunks + geometry.window_chunks
        rows = self.slots * geometry.chunk_tokens
        shape = (1, rows, geometry.heads, geometry.head_dim)
        self.k = [torch.zeros(shape, device=device, dtype=dtype) for _ in range(geometry.layers)]
        self.v = [torch.zeros(shape, device=device, dtype=dtype) for _ in range(geometry.layers)]
        self.resident: dict[int, int] = {}  # slot -> chunk index held

    def slot(self, chunk: int) -> int:
        g = self.geometry
        if chunk < 0:
            raise ValueError(f"chunk index {chunk} is negative")
        if chunk < g.sink_chunks:
            return chunk
        return g.sink_chunks + (chunk - g.sink_chunks) % g.window_chunks

    def place(self, chunk: int) -> tuple[int, int]:
        """First and end row of chunk ``chunk``'s slot."""
        start = self.slot(chunk) * self.geometry.chunk_tokens
        return start, start + self.geometry.chunk_tokens

    def attended(self, chunk: int) -> list[int]:
        """Chunks visible while generating ``chunk``: the sink, then the window ending with ``chunk``."""
        g = self.geometry
        sink = list(range(min(g.sink_chunks, chunk)))
        first = max(g.sink_chunks, chunk - g.window_chunks + 1)
        return sink + list(range(first, chunk + 1))

    def rows(self, chunks: Sequence[int]) -> torch.Tensor:
        """Row indices of ``chunks`` in the cache, in the given order."""
        parts = [torch.arange(*self.place(c)) for c in chunks]
        return torch.cat(parts) if parts else torch.empty(0, dtype=torch.long)

    def destination(self, layer: int, target: str) -> torch.Tensor:
        return self.k[layer] if target == "K" else self.v[layer]

    def nbytes(self) -> int:
        return sum(t.numel() * t.element_size() for t in self.k + self.v)


class ChunkKV:
    """Capture / install adapter around a model whose ``blocks[l].self_attn`` has ``k`` and ``v`` projections.

    ``arm()`` before a chunk's clean pass; ``take()`` after it returns per-layer pre-RoPE K and V ``[tokens,
    channels]`` (detached; cloned so a later forward cannot overwrite them)."""

    def __init__(self, blocks: Sequence[torch.nn.Module]):
        self.blocks = list(blocks)
        self._armed = False
        self._k: dict[int, torch.Tensor] = {}
        self._v: dict[int, torch.Tensor] = {}
        self._handles = []
        for layer, block in enumerate(self.blocks):
            attn = block.self_attn
            key_module = attn.norm_k if hasattr(attn, "norm_k") else attn.k
            self._handles.append(key_module.register_forward_hook(self._capture(self._k, layer)))
            self._handles.append(attn.v.register_forward_hook(self._capture(self._v, layer)))

    def _capture(self, bucket: dict, layer: int):
        def hook(_module, _inputs, output):
            if self._armed:
                bucket[layer] = output.detach().reshape(-1, output.shape[-1]).clone()
        return hook

    def arm(self) -> None:
        self._k.clear()
        self._v.clear()
        self._armed = True

    def take(self) -> tuple[list[torch.Tensor], list[torch.Tensor]]:
        self._armed = False
        layers = len(self.blocks)
        if len(self._k) != layers or len(self._v) != layers:
            raise RuntimeError(f"captured K for {len(self._k)} and V for {len(self._v)} of {layers} layers: the clean "
                               "pass did not run every block")
        k = [self._k.pop(layer) for layer in range(layers)]
        v = [self._v.pop(layer) for layer in range(layers)]
        return k, v

    def remove(self) -> None:
        handles, self._handles = self._handles, []
        for handle in handles:
            handle.remove()


class _RMSNorm(torch.nn.Module):
    def __init__(self, dim: int):
        super().__init__()
        self.weight = torch.nn.Parameter(torch.ones(dim))

    def forward(self, x):
        xf = x.float()
        return (xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + 1e-6) * self.weight).to(x.dtype)


class _SelfAttention(torch.nn.Module):
    def __init__(self, channels: int):
        super().__init__()
        self.q = torch.nn.Linear(channels, channels)
        self.k = torch.nn.Linear(channels, channels)
        self.v = torch.nn.Linear(channels, channels)
        self.o = torch.nn.Linear(channels, channels)
        self.norm_q = _RMSNorm(channels)
        self.norm_k = _RMSNorm(channels)

    def forward(self, y):
        """The projections of one chunk: normalized q, pre-RoPE (normalized) k and v. Forward pre-hooks on this
        module (an overlapped restore's layer wait) run before them."""
        return self.norm_q(self.q(y)), self.norm_k(self.k(y)), self.v(y)


class _Block(torch.nn.Module):
    def __init__(self, channels: int):
        super().__init__()
        self.norm = _RMSNorm(channels)
        self.self_attn = _SelfAttention(channels)


class StandInWorldModel(torch.nn.Module):
    """A small LingBot-shaped model: ``generate(chunk, x)`` runs one chunk's clean pass over the shared cache."""

    def __init__(self, geometry: LingBotGeometry, device="cpu", dtype=torch.bfloat16, seed: int = 0):
        super().__init__()
        self.geometry = geometry
        with torch.random.fork_rng(devices=[]):  # seeded weights without touching the caller's generator
            torch.manual_seed(seed)
            self.blocks = torch.nn.ModuleList(_Block(geometry.channels) for _ in range(geometry.layers))
        self.to(device=device, dtype=dtype)
        self.device = torch.device(device)
        self.dtype = dtype
        self.cache = SharedWindowCache(geometry, device, dtype)
        frames = 4096
        self.rope_table = rk.RopeTable.wan(geometry.head_dim, max(frames, geometry.latent_height,
                                                                  geometry.latent_width))
        self.kv = ChunkKV(self.blocks)
        self.overlap = None

    # -- positions and the cache -----------------------------------------------------------------------------------

    def grid(self) -> tuple[int, int, int]:
        g = self.geometry
        return g.frames_per_chunk, g.latent_height, g.latent_width

    def rope_positions(self, chunk: int) -> rk.RopePositions:
        return rk.RopePositions(self.rope_table, (chunk * self.geometry.frames_per_chunk, 0, 0))

    def rope(self, values: torch.Tensor, chunk: int) -> torch.Tensor:
        """``values [tokens, heads, head_dim]`` rotated at chunk ``chunk``'s absolute frame positions."""
        return apply_rope_reference(values, self.rope_positions(chunk), self.grid()).to(values.dtype)

    def destination_tensors(self, layer: int) -> tuple[torch.Tensor, torch.Tensor]:
        return self.cache.k[layer], self.cache.v[layer]

    def install_rows(self, layer: int, chunk: int, k_pre: torch.Tensor, v: torch.Tensor) -> None:
        """Write one chunk's K (rotated here) and V into its slot of layer ``layer``."""
        g = self.geometry
        start, end = self.cache.place(chunk)
        k = self.rope(k_pre.reshape(-1, g.heads, g.head_dim), chunk)
        self.cache.k[layer][0, start:end] = k.to(self.dtype)
        self.cache.v[layer][0, start:end] = v.reshape(-1, g.heads, g.head_dim).to(self.dtype)
        self.cache.resident[self.cache.slot(chunk)] = chunk

    def attention_modules(self) -> list[torch.nn.Module]:
        return [block.self_attn for block in self.blocks]

    # -- the overlapped restore seam ---------------------------------------------------------------------------

    def attach_overlapped_restore(self, session) -> None:
        session.attach(self.attention_modules())
        self.overlap = session

    def join_overlapped_restore(self):
        session, self.overlap = self.overlap, None
        return None if session is None else session.join()

    def abort_overlapped_restore(self) -> None:
        session, self.overlap = self.overlap, None
        if session is not None:
            session.abort()

    # -- one chunk ---------------------------------------------------------------------------------------------------

    @torch.no_grad()
    def generate(self, chunk: int, x: torch.Tensor, *, capture: bool = True):
        """Clean pass of chunk ``chunk`` on input tokens ``x [chunk_tokens, channels]``: each block writes the
        chunk's K / V into its slot and attends the visible chunks. Returns the output tokens and, with
        ``capture``, the per-layer pre-RoPE K and V. A pending overlapped restore is joined before returning."""
        g = self.geometry
        if x.shape != (g.chunk_tokens, g.channels):
            raise ValueError(f"chunk input must be [{g.chunk_tokens}, {g.channels}], got {list(x.shape)}")
        if capture:
            self.kv.arm()
        visible = self.cache.rows(self.cache.attended(chunk)).to(self.device)
        h = x.to(self.device, self.dtype)
        try:
            for layer, block in enumerate(self.blocks):
                attn = block.self_attn
                q, k_pre, v = attn(block.norm(h))  # an overlapped restore's wait for this layer runs first
                start, end = self.cache.place(chunk)
                self.cache.k[layer][0, start:end] = self.rope(k_pre.reshape(-1, g.heads, g.head_dim), chunk)
                self.cache.v[layer][0, start:end] = v.reshape(-1, g.heads, g.head_dim)
                qh = self.rope(q.reshape(-1, g.heads, g.head_dim), chunk).permute(1, 0, 2)
                kh = self.cache.k[layer][0, visible].permute(1, 0, 2)
                vh = self.cache.v[layer][0, visible].permute(1, 0, 2)
                out = torch.nn.functional.scaled_dot_product_attention(qh.unsqueeze(0), kh.unsqueeze(0),
                                                                       vh.unsqueeze(0))[0]
                h = h + attn.o(out.permute(1, 0, 2).reshape(-1, g.channels))
            self.cache.resident[self.cache.slot(chunk)] = chunk
        except BaseException:
            self.abort_overlapped_restore()
            raise
        self.join_overlapped_restore()
        if capture:
            return h, self.kv.take()
        return h, None
