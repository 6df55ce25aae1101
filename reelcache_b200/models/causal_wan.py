"""From-scratch CausVid-shaped causal video DiT (Wan2.1-T2V-1.3B geometry) on the sm_100a kernels.

Geometry (reference: reelcache_sglang_models/causal_wan/profiles.py:26-36, 475): 30 blocks, width
1536, 12 heads x 128, FFN 8960, text width 4096 (512 tokens), patch (1, 2, 2), 480x832 video ->
latent 60x104 -> 30x52 = 1560 tokens per latent frame, 3 latent frames (4680 tokens) per chunk.

Block math (reference: causal_wan/sglang_dit.py:203-296; SGLang patch 0001:570-690 for RoPE): AdaLN
6-way modulation ``modulation + e0``; LayerNorm -> modulate -> fused QKV GEMM -> RMSNorm across all
heads on q and k (weights) -> 3-axis interleaved RoPE (44/42/42 dims, theta 10000) -> attention over
the causal KV cache (bidirectional inside the chunk) -> out-projection with gated residual;
LayerNorm(affine) -> cross-attention to the cached text K/V -> residual; LayerNorm -> modulate ->
GELU(tanh) FFN -> gated residual. Head: LayerNorm -> modulate -> Linear(1536 -> 64) -> unpatchify.

Every GEMM is the tcgen05 kernel with a fused epilogue (bias, GELU, gated residual); norms,
modulation, q/k-norm + RoPE + KV-cache writes are the kernels in csrc/model. Weights are random
(deterministic seed): performance and the archival path depend only on the shapes.
"""

from __future__ import annotations

import math
from dataclasses import dataclass

import torch

from ..ops import attention as attn_ops
from ..ops import gemm, norms
from ..restore_kernels import RopeTable


@dataclass(frozen=True)
class WanConfig:
    layers: int = 30
    dim: int = 1536
    heads: int = 12
    head_dim: int = 128
    ffn: int = 8960
    in_dim: int = 16
    out_dim: int = 16
    text_dim: int = 4096
    text_len: int = 512
    freq_dim: int = 256
    patch: tuple = (1, 2, 2)
    eps: float = 1e-6
    latent_height: int = 60
    latent_width: int = 104
    frames_per_chunk: int = 3
    rope_theta: float = 10000.0

    @property
    def grid_h(self) -> int:
        return self.latent_height // self.patch[1]

    @property
    def grid_w(self) -> int:
        return self.latent_width // self.patch[2]

    @property
    def tokens_per_frame(self) -> int:
        return self.grid_h * self.grid_w

    @property
    def chunk_tokens(self) -> int:
        return self.frames_per_chunk * self.tokens_per_frame

    @property
    def patch_dim(self) -> int:
        return self.in_dim * self.patch[0] * self.patch[1] * self.patch[2]

    def scaled(self, **overrides) -> "WanConfig":
        values = {k: getattr(self, k) for k in self.__dataclass_fields__}
        values.update(overrides)
        return WanConfig(**values)


WAN21_T2V_1_3B = WanConfig()
CAUSVID = WAN21_T2V_1_3B


def sinusoidal(t: torch.Tensor, dim: int) -> torch.Tensor:
    """Wan's timestep embedding ``[cos(t w), sin(t w)]`` with ``w = 10000^(-i / (dim/2))`` (FP64 -> FP32)."""
    half = dim // 2
    freqs = torch.pow(10000.0, -torch.arange(half, dtype=torch.float64, device=t.device) / half)
    angles = t.double()[..., None] * freqs
    return torch.cat([torch.cos(angles), torch.sin(angles)], dim=-1).float()


class KVCache:
    """Per-layer native caches ``[1, capacity, heads, head_dim]`` (BTHD, contiguous) for K (post-RoPE)
    and V, with chunk-granular slots: chunk ``i`` occupies tokens ``[i * chunk_tokens, (i+1) * chunk_tokens)``."""

    def __init__(self, cfg: WanConfig, capacity_chunks: int, device, dtype=torch.bfloat16):
        self.cfg = cfg
        self.capacity = capacity_chunks * cfg.chunk_tokens
        self.k = [torch.zeros((1, self.capacity, cfg.heads, cfg.head_dim), dtype=dtype, device=device)
                  for _ in range(cfg.layers)]
        self.v = [torch.zeros_like(self.k[0]) for _ in range(cfg.layers)]
        self.length = 0  # tokens of valid history

    def rows(self, layer: int, which: str) -> torch.Tensor:
        """``[capacity, C]`` row view of one cache tensor."""
        t = self.k[layer] if which == "K" else self.v[layer]
        return t.view(self.capacity, self.cfg.dim)

    @property
    def nbytes(self) -> int:
        return 2 * self.cfg.layers * self.k[0].numel() * self.k[0].element_size()


class SPKVCache(KVCache):
    """A Ulysses rank's native caches: every token of the history for this rank's ``heads / world`` heads
    (``[1, capacity, heads / world, head_dim]``), the "heads" layout a sequence-parallel restore writes."""

    def __init__(self, cfg: WanConfig, capacity_chunks: int, device, *, world: int, rank: int,
                 dtype=torch.bfloat16):
        if cfg.heads % world:
            raise ValueError("heads must divide evenly across the Ulysses ranks")
        self.cfg = cfg
        self.world, self.rank = world, rank
        self.heads = cfg.heads // world
        self.capacity = capacity_chunks * cfg.chunk_tokens
        self.k = [torch.zeros((1, self.capacity, self.heads, cfg.head_dim), dtype=dtype, device=device)
                  for _ in range(cfg.layers)]
        self.v = [torch.zeros_like(self.k[0]) for _ in range(cfg.layers)]
        self.length = 0

    def rows(self, layer: int, which: str) -> torch.Tensor:
        t = self.k[layer] if which == "K" else self.v[layer]
        return t.view(self.capacity, self.heads * self.cfg.head_dim)


class CausalWanDiT:
    """The causal DiT (weights as plain tensors; forward uses the sm_100a ops)."""

    def __init__(self, cfg: WanConfig = CAUSVID, device="cuda", *, seed: int = 0, dtype=torch.bfloat16):
        self.cfg = cfg
        self.device = torch.device(device)
        gen = torch.Generator(device=self.device).manual_seed(seed)
        d, f = cfg.dim, cfg.ffn

        def w(out_f, in_f, std=None):
            std = std if std is not None else 1.0 / math.sqrt(in_f)
            return (torch.randn((out_f, in_f), generator=gen, device=self.device) * std).to(dtype).to(self.device)

        def b(n, std=0.02):
            return (torch.randn(n, generator=gen, device=self.device) * std).to(dtype).to(self.device)

        def vec(n, mean=1.0, std=0.05):
            return (mean + torch.randn(n, generator=gen, device=self.device) * std).float().to(self.device)

        self.patch_w, self.patch_b = w(d, cfg.patch_dim), b(d)
        self.time_w1, self.time_b1 = w(d, cfg.freq_dim), b(d)
        self.time_w2, self.time_b2 = w(d, d), b(d)
        self.tproj_w, self.tproj_b = w(6 * d, d, std=0.02 / math.sqrt(d)), b(6 * d, std=0.01)
        self.text_w1, self.text_b1 = w(d, cfg.text_dim), b(d)
        self.text_w2, self.text_b2 = w(d, d), b(d)
        self.blocks = []
        for _ in range(cfg.layers):
            blk = {
                "modulation": (torch.randn((6, d), generator=gen, device=self.device) * (0.1 / math.sqrt(d))).float().to(self.device),
                "qkv_w": w(3 * d, d), "qkv_b": b(3 * d), "norm_q": vec(d), "norm_k": vec(d),
                "o_w": w(d, d), "o_b": b(d), "norm3_w": vec(d), "norm3_b": vec(d, 0.0, 0.02),
                "cq_w": w(d, d), "cq_b": b(d), "ck_w": w(d, d), "ck_b": b(d), "cv_w": w(d, d), "cv_b": b(d),
                "cnorm_q": vec(d), "cnorm_k": vec(d), "co_w": w(d, d), "co_b": b(d),
                "ffn1_w": w(f, d), "ffn1_b": b(f), "ffn2_w": w(d, f), "ffn2_b": b(d),
            }
            self.blocks.append(blk)
        self.head_mod = (torch.randn((2, d), generator=gen, device=self.device) * (0.1 / math.sqrt(d))).float().to(self.device)
        self.head_w, self.head_b = w(cfg.patch_dim, d), b(cfg.patch_dim)
        pairs = cfg.head_dim // 2
        self.rope = RopeTable.wan(cfg.head_dim, 1024, theta=cfg.rope_theta, device=self.device)
        assert self.rope.pairs == pairs

    # -- conditioning ------------------------------------------------------------------------------------------

    def encode_text(self, context: torch.Tensor) -> list[tuple[torch.Tensor, torch.Tensor]]:
        """Per-layer cross-attention K/V ``[text_len, dim]`` of a text embedding ``[text_len, text_dim]``
        (computed once per request, as the reference's cached cross-attention)."""
        c = gemm.linear_gelu(context.to(torch.bfloat16), self.text_w1, self.text_b1)
        c = gemm.linear(c, self.text_w2, self.text_b2)
        kv = []
        for blk in self.blocks:
            k = norms.rms_norm(gemm.linear(c, blk["ck_w"], blk["ck_b"]), blk["cnorm_k"], eps=self.cfg.eps)
            v = gemm.linear(c, blk["cv_w"], blk["cv_b"])
            kv.append((k, v))
        return kv

    def time_modulation(self, t: float) -> tuple[torch.Tensor, torch.Tensor]:
        """``(e [dim], e0 [6, dim])`` FP32 of a timestep."""
        emb = sinusoidal(torch.tensor([float(t)], device=self.device), self.cfg.freq_dim).to(torch.bfloat16)
        e = gemm.linear(emb, self.time_w1, self.time_b1)
        e = torch.nn.functional.silu(e.float()).to(torch.bfloat16)
        e = gemm.linear(e, self.time_w2, self.time_b2)
        e0 = gemm.linear(torch.nn.functional.silu(e.float()).to(torch.bfloat16), self.tproj_w, self.tproj_b,
                         out_dtype=torch.float32)
        return e.float().reshape(-1), e0.reshape(6, self.cfg.dim)

    def token_rope(self, chunk_index: int):
        """Per-token cos/sin ``[chunk_tokens, pairs]`` of a chunk's positions (frame offset = 3 * index)."""
        cfg = self.cfg
        grid = (cfg.frames_per_chunk, cfg.grid_h, cfg.grid_w)
        return self.rope.token_tables((cfg.frames_per_chunk * chunk_index, 0, 0), grid, self.device)

    # -- forward -----------------------------------------------------------------------------------------------

    def patchify(self, latents: torch.Tensor) -> torch.Tensor:
        """``[in_dim, F, H, W]`` -> ``[F * H/2 * W/2, in_dim * 4]``."""
        cfg = self.cfg
        c, frames, h, w = latents.shape
        x = latents.reshape(c, frames, h // 2, 2, w // 2, 2).permute(1, 2, 4, 0, 3, 5)
        return x.reshape(frames * (h // 2) * (w // 2), cfg.patch_dim)

    def unpatchify(self, x: torch.Tensor) -> torch.Tensor:
        cfg = self.cfg
        frames = x.shape[0] // cfg.tokens_per_frame
        out = x.reshape(frames, cfg.grid_h, cfg.grid_w, cfg.out_dim, 2, 2).permute(3, 0, 1, 4, 2, 5)
        return out.reshape(cfg.out_dim, frames, cfg.latent_height, cfg.latent_width)

    def forward_chunk(self, latents: torch.Tensor, t: float, chunk_index: int, cache: KVCache, text_kv, *,
                      capture=None, layer_wait=None, attention_backend: str = "auto") -> torch.Tensor:
        """One forward of the chunk at ``chunk_index`` with timestep ``t``: writes the chunk's K (post-RoPE)
        and V into its cache slot and attends over ``[0, slot_end)``. ``capture(layer, k_pre, v)`` receives
        the normalized pre-RoPE K and V rows of every layer (clean pass). ``layer_wait(layer, stream)``
        blocks the stream until layer ``layer``'s restored history is written (overlapped restore).
        Returns the flow prediction ``[in_dim, F, H, W]`` (FP32)."""
        cfg = self.cfg
        tokens = cfg.chunk_tokens
        start = chunk_index * tokens
        end = start + tokens
        if end > cache.capacity:
            raise ValueError("chunk exceeds the KV cache capacity")
        x = gemm.linear(self.patchify(latents).to(torch.bfloat16).contiguous(), self.patch_w, self.patch_b)
        e, e0 = self.time_modulation(t)
        cos_tok, sin_tok = self.token_rope(chunk_index)
        q = torch.empty((tokens, cfg.dim), dtype=torch.bfloat16, device=self.device)
        k_pre = torch.empty_like(q) if capture is not None else None
        stream = torch.cuda.current_stream(self.device)
        for layer, blk in enumerate(self.blocks):
            mod = blk["modulation"] + e0
            y = norms.ln_modulate(x, shift=mod[0], scale=mod[1], eps=cfg.eps)
            qkv = gemm.linear(y, blk["qkv_w"], blk["qkv_b"])
            k_rows = cache.rows(layer, "K")[start:end]
            v_rows = cache.rows(layer, "V")[start:end]
            norms.qkv_norm_rope(qkv, blk["norm_q"], blk["norm_k"], cos_tok, sin_tok, q, k_rows, v_rows,
                                head_dim=cfg.head_dim, k_pre=k_pre, eps=cfg.eps)
            if capture is not None:
                capture(layer, k_pre, v_rows)
            if layer_wait is not None:
                layer_wait(layer, stream)
            o = attn_ops.attention(q.view(tokens, cfg.heads, cfg.head_dim), cache.k[layer][0, :end],
                                   cache.v[layer][0, :end], backend=attention_backend)
            gemm.linear_gated_residual(o.view(tokens, cfg.dim), blk["o_w"], blk["o_b"], mod[2].contiguous(), x)
            y = norms.ln_modulate(x, weight=blk["norm3_w"], bias=blk["norm3_b"], eps=cfg.eps)
            cq = norms.rms_norm(gemm.linear(y, blk["cq_w"], blk["cq_b"]), blk["cnorm_q"], eps=cfg.eps)
            ck, cv = text_kv[layer]
            co = attn_ops.attention(cq.view(tokens, cfg.heads, cfg.head_dim), ck.view(-1, cfg.heads, cfg.head_dim),
                                    cv.view(-1, cfg.heads, cfg.head_dim), backend=attention_backend)
            gemm.linear_gated_residual(co.view(tokens, cfg.dim), blk["co_w"], blk["co_b"], None, x)
            y = norms.ln_modulate(x, shift=mod[3], scale=mod[4], eps=cfg.eps)
            h = gemm.linear_gelu(y, blk["ffn1_w"], blk["ffn1_b"])
            gemm.linear_gated_residual(h, blk["ffn2_w"], blk["ffn2_b"], mod[5].contiguous(), x)
        shift = (self.head_mod[0] + e).contiguous()
        scale = (self.head_mod[1] + e).contiguous()
        y = norms.ln_modulate(x, shift=shift, scale=scale, eps=cfg.eps)
        out = gemm.linear(y, self.head_w, self.head_b, out_dtype=torch.float32)
        return self.unpatchify(out)

    def forward_chunk_sp(self, latents: torch.Tensor, t: float, chunk_index: int, cache: SPKVCache, text_kv, *,
                         group, capture=None, layer_wait=None, attention_backend: str = "auto") -> torch.Tensor:
        """:meth:`forward_chunk` under Ulysses sequence parallelism over ``group``: this rank projects, normalizes
        and ropes its contiguous ``tokens / world`` rows (the full-width q / k RMSNorm needs every head of a
        token, so it runs before the head split), one all-to-all per layer hands every rank all tokens of its
        ``heads / world`` heads (K and V land in its cache slot), attention runs over the full history of those
        heads, one all-to-all returns the outputs to their token rows, and cross-attention and the FFN stay on
        the rank's rows. ``capture(layer, k_pre, v)`` receives this rank's token rows (all heads). Returns the
        full flow prediction on every rank (one all-gather)."""
        import torch.distributed as dist
        cfg = self.cfg
        world, rank = cache.world, cache.rank
        tokens = cfg.chunk_tokens
        if tokens % world:
            raise ValueError("the chunk's tokens must divide evenly across the Ulysses ranks")
        n_loc, hp, d = tokens // world, cache.heads, cfg.head_dim
        rows = slice(rank * n_loc, (rank + 1) * n_loc)
        start = chunk_index * tokens
        end = start + tokens
        if end > cache.capacity:
            raise ValueError("chunk exceeds the KV cache capacity")
        x = gemm.linear(self.patchify(latents)[rows].to(torch.bfloat16).contiguous(), self.patch_w, self.patch_b)
        e, e0 = self.time_modulation(t)
        cos_tok, sin_tok = self.token_rope(chunk_index)
        cos_loc, sin_loc = cos_tok[rows].contiguous(), sin_tok[rows].contiguous()
        q = torch.empty((n_loc, cfg.dim), dtype=torch.bfloat16, device=self.device)
        k_loc, v_loc = torch.empty_like(q), torch.empty_like(q)
        k_pre = torch.empty_like(q) if capture is not None else None
        send = torch.empty((world, 3, n_loc, hp, d), dtype=torch.bfloat16, device=self.device)
        recv = torch.empty_like(send)
        back = torch.empty((world, n_loc, hp, d), dtype=torch.bfloat16, device=self.device)
        stream = torch.cuda.current_stream(self.device)
        for layer, blk in enumerate(self.blocks):
            mod = blk["modulation"] + e0
            y = norms.ln_modulate(x, shift=mod[0], scale=mod[1], eps=cfg.eps)
            qkv = gemm.linear(y, blk["qkv_w"], blk["qkv_b"])
            norms.qkv_norm_rope(qkv, blk["norm_q"], blk["norm_k"], cos_loc, sin_loc, q, k_loc, v_loc,
                                head_dim=d, k_pre=k_pre, eps=cfg.eps)
            if capture is not None:
                capture(layer, k_pre, v_loc)
            for index, part in enumerate((q, k_loc, v_loc)):   # [n_loc, world, hp, d] -> [world, n_loc, hp, d]
                send[:, index].copy_(part.view(n_loc, world, hp, d).transpose(0, 1))
            dist.all_to_all_single(recv, send, group=group)
            cache.k[layer][0, start:end].view(world, n_loc, hp, d).copy_(recv[:, 1])
            cache.v[layer][0, start:end].view(world, n_loc, hp, d).copy_(recv[:, 2])
            if layer_wait is not None:
                layer_wait(layer, stream)
            o = attn_ops.attention(recv[:, 0].reshape(tokens, hp, d), cache.k[layer][0, :end],
                                   cache.v[layer][0, :end], backend=attention_backend)
            dist.all_to_all_single(back, o.view(world, n_loc, hp, d), group=group)
            o_loc = back.transpose(0, 1).reshape(n_loc, cfg.dim)
            gemm.linear_gated_residual(o_loc, blk["o_w"], blk["o_b"], mod[2].contiguous(), x)
            y = norms.ln_modulate(x, weight=blk["norm3_w"], bias=blk["norm3_b"], eps=cfg.eps)
            cq = norms.rms_norm(gemm.linear(y, blk["cq_w"], blk["cq_b"]), blk["cnorm_q"], eps=cfg.eps)
            ck, cv = text_kv[layer]
            co = attn_ops.attention(cq.view(n_loc, cfg.heads, d), ck.view(-1, cfg.heads, d),
                                    cv.view(-1, cfg.heads, d), backend=attention_backend)
            gemm.linear_gated_residual(co.view(n_loc, cfg.dim), blk["co_w"], blk["co_b"], None, x)
            y = norms.ln_modulate(x, shift=mod[3], scale=mod[4], eps=cfg.eps)
            h = gemm.linear_gelu(y, blk["ffn1_w"], blk["ffn1_b"])
            gemm.linear_gated_residual(h, blk["ffn2_w"], blk["ffn2_b"], mod[5].contiguous(), x)
        shift = (self.head_mod[0] + e).contiguous()
        scale = (self.head_mod[1] + e).contiguous()
        y = norms.ln_modulate(x, shift=shift, scale=scale, eps=cfg.eps)
        out = gemm.linear(y, self.head_w, self.head_b, out_dtype=torch.float32)
        full = torch.empty((world, n_loc, out.shape[1]), dtype=out.dtype, device=self.device)
        dist.all_gather_into_tensor(full, out.contiguous(), group=group)
        return self.unpatchify(full.view(tokens, out.shape[1]))

    def flops_per_forward(self, history_tokens: int) -> float:
        cfg = self.cfg
        t, d, f = cfg.chunk_tokens, cfg.dim, cfg.ffn
        linear = 2 * t * (3 * d * d + d * d + d * d + d * d + 2 * d * f)
        attention = 4 * t * (history_tokens + t) * d + 4 * t * cfg.text_len * d
        return cfg.layers * (linear + attention)
