"""LongCat-Video-shaped DiT (48 x 4096, 32 heads x 128, 720p -> 45 x 80 = 3600 tokens per latent frame)
with context parallelism and the conditioning-cache seam (the counterpart of reference
reelcache_sglang_models/longcat_video/dit_core.py:41-476 and conditioning_cache.py:56-460).

Block (``LongCatVideoBlock``): AdaLN in FP32 (LayerNorm -> ``x * (1 + scale) + shift`` from the
timestep embedding) -> self-attention: fused qkv GEMM, per-head RMSNorm (FP32) on q and k, then the
**conditioning-cache branch**: the cached pre-RoPE K/V of the conditioning frames are concatenated in
front of the current K/V and RoPE is applied at read time (3-axis LongCat tables) -> attention ->
output projection -> gated residual -> cross-attention over the text -> residual -> SwiGLU FFN -> gated
residual. Final layer in FP32.

Context parallelism (``cp_group``): each rank keeps the spatial block of every frame that
``RowShard`` assigns it; self-attention runs Ulysses all-to-alls (heads scattered, sequence gathered)
on q, k, v and the inverse on the output; cross-attention and the FFN stay local; the final output is
gathered. Every rank holds (and restores) only its rows of the conditioning cache.

Weights are random (no checkpoint binding). On CUDA the GEMMs, RMSNorms and attention run on the
package's sm_100a ops; ``use_kernels=False`` runs the same math in plain torch (CPU tests, reference).
"""

from __future__ import annotations

import math
from dataclasses import dataclass, replace
from typing import Any, Callable, Protocol, Sequence

import torch
import torch.nn.functional as F

from ..parallel.context_parallel import RowShard, gather_tokens, ulysses_in, ulysses_out


def dist_rank(group) -> int:
    import torch.distributed as dist
    return dist.get_rank(group)
from ..restore_kernels import RopeTable


@dataclass(frozen=True)
class LongCatConfig:
    layers: int = 48
    dim: int = 4096
    heads: int = 32
    head_dim: int = 128
    ffn: int = 11008
    text_dim: int = 4096
    text_len: int = 512
    in_channels: int = 16
    latent_height: int = 90
    latent_width: int = 160
    frames_per_chunk: int = 4
    freq_dim: int = 256
    eps: float = 1e-6

    @property
    def grid(self) -> tuple[int, int]:
        return (self.latent_height // 2, self.latent_width // 2)

    @property
    def tokens_per_frame(self) -> int:
        return self.grid[0] * self.grid[1]

    @property
    def patch_dim(self) -> int:
        return self.in_channels * 4

    def scaled(self, **overrides) -> "LongCatConfig":
        return replace(self, **overrides)


LONGCAT_720P = LongCatConfig()


@dataclass(frozen=True)
class ConditioningCacheEpoch:
    """One segment's conditioning cache identity: ``frames`` conditioning latent frames starting at
    ``first_frame`` of the video."""

    epoch_id: str
    segment_index: int
    first_frame: int
    frames: int


class LongCatConditioningCache:
    """Per-layer pre-RoPE K and V ``[tokens, heads, head_dim]`` of the conditioning frames (this rank's
    rows under context parallelism)."""

    def __init__(self, epoch: ConditioningCacheEpoch, k: Sequence[torch.Tensor], v: Sequence[torch.Tensor]):
        if len(k) != len(v):
            raise ValueError("one K and one V per layer")
        self.epoch = epoch
        self.k = list(k)
        self.v = list(v)

    @property
    def tokens(self) -> int:
        return self.k[0].shape[0]

    @property
    def nbytes(self) -> int:
        return sum(t.numel() * t.element_size() for t in self.k + self.v)


class ConditioningCacheBackend(Protocol):
    """The seam a pipeline calls: ``restore(epoch)`` returns a cache (or None: build it), and
    ``on_cache_built(cache)`` hands a freshly built cache to the archive."""

    def restore(self, epoch: ConditioningCacheEpoch) -> LongCatConditioningCache | None: ...

    def on_cache_built(self, cache: LongCatConditioningCache) -> None: ...


class _Ops:
    """GEMM / RMSNorm / attention on the sm_100a kernels (CUDA) or plain torch."""

    def __init__(self, kernels: bool):
        self.kernels = kernels

    def linear(self, x, w, b=None, out_dtype=torch.bfloat16):
        if self.kernels:
            from ..ops import gemm
            return gemm.linear(x.contiguous(), w, b, out_dtype=out_dtype)
        y = x.float() @ w.float().t()
        if b is not None:
            y = y + b.float()
        return y.to(out_dtype)

    def rms_norm_heads(self, x, weight, eps):
        """Per-head RMSNorm in FP32 of ``[tokens, heads, head_dim]``."""
        if self.kernels:
            from ..ops.norms import head_norm_rope
            return head_norm_rope(x, weight, eps=eps)
        xf = x.float()
        return (xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + eps) * weight.float()).to(x.dtype)

    def norm_rope(self, x, weight, cos, sin, eps, *, out=None):
        """Per-head RMSNorm (``weight`` None: none) then RoPE of ``[tokens, heads, head_dim]``: one fused kernel on
        CUDA (FP32 throughout), two eager steps otherwise."""
        if self.kernels:
            from ..ops.norms import head_norm_rope
            return head_norm_rope(x, weight, cos, sin, eps=eps, out=out)
        y = _rope(self.rms_norm_heads(x, weight, eps) if weight is not None else x, cos, sin)
        if out is not None:
            out.copy_(y)
            return out
        return y

    def rope(self, x, cos, sin):
        return self.norm_rope(x, None, cos, sin, 0.0)

    def attention(self, q, k, v):
        """``[Tq, H, D]`` x ``[Tk, H, D]`` -> ``[Tq, H, D]`` (non-causal)."""
        if self.kernels:
            from ..ops import attention as attn_ops
            return attn_ops.attention(q, k, v)
        scale = 1.0 / math.sqrt(q.shape[-1])
        s = torch.einsum("qhd,khd->hqk", q.float(), k.float()) * scale
        return torch.einsum("hqk,khd->qhd", s.softmax(-1), v.float()).to(q.dtype)


def _rope(x: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor) -> torch.Tensor:
    """Interleaved-pair rotation of ``[tokens, heads, head_dim]`` by per-token ``[tokens, pairs]`` tables."""
    xf = x.float().reshape(*x.shape[:-1], -1, 2)
    c, s = cos[:, None, :], sin[:, None, :]
    e, o = xf[..., 0], xf[..., 1]
    return torch.stack((e * c - o * s, e * s + o * c), dim=-1).reshape(x.shape).to(x.dtype)


class LongCatDiT:
    def __init__(self, cfg: LongCatConfig = LONGCAT_720P, device="cuda", *, seed: int = 0, dtype=torch.bfloat16,
                 use_kernels: bool | None = None, max_frames: int = 64):
        self.cfg = cfg
        self.device = torch.device(device)
        self.dtype = dtype
        self.ops = _Ops(self.device.type == "cuda" if use_kernels is None else use_kernels)
        gen = torch.Generator(device="cpu").manual_seed(seed)
        d, f, hd = cfg.dim, cfg.ffn, cfg.head_dim

        def w(out_f, in_f, std=None):
            std = std if std is not None else 1.0 / math.sqrt(in_f)
            return (torch.randn((out_f, in_f), generator=gen) * std).to(dtype).to(self.device)

        def b(n, std=0.02):
            return (torch.randn(n, generator=gen) * std).to(dtype).to(self.device)

        def vec(n, mean=1.0, std=0.05):
            return (mean + torch.randn(n, generator=gen) * std).float().to(self.device)

        self.patch_w, self.patch_b = w(d, cfg.patch_dim), b(d)
        self.t_w1, self.t_b1 = w(d, cfg.freq_dim), b(d)
        self.t_w2, self.t_b2 = w(d, d), b(d)
        self.text_w, self.text_b = w(d, cfg.text_dim), b(d)
        self.blocks = []
        for _ in range(cfg.layers):
            self.blocks.append({
                "ada_w": w(6 * d, d, std=0.02 / math.sqrt(d)), "ada_b": b(6 * d, std=0.01),
                "qkv_w": w(3 * d, d), "qkv_b": b(3 * d), "q_norm": vec(hd), "k_norm": vec(hd),
                "proj_w": w(d, d), "proj_b": b(d),
                "cq_w": w(d, d), "cq_b": b(d), "ckv_w": w(2 * d, d), "ckv_b": b(2 * d),
                "cq_norm": vec(hd), "ck_norm": vec(hd), "cproj_w": w(d, d), "cproj_b": b(d),
                "w1": w(f, d), "w3": w(f, d), "w2": w(d, f),
            })
        self.final_ada_w, self.final_ada_b = w(2 * d, d, std=0.02 / math.sqrt(d)), b(2 * d, std=0.01)
        self.final_w, self.final_b = w(cfg.patch_dim, d), b(cfg.patch_dim)
        self.rope = RopeTable.longcat(hd, max_frames, cfg.grid[0], cfg.grid[1], device=self.device)

    # -- embeddings ---------------------------------------------------------------------------------------------

    def timestep(self, t: float) -> torch.Tensor:
        half = self.cfg.freq_dim // 2
        freqs = torch.exp(-math.log(10000.0) * torch.arange(half, device=self.device, dtype=torch.float32) / half)
        args = float(t) * freqs
        emb = torch.cat([torch.cos(args), torch.sin(args)]).to(self.dtype)[None]
        h = F.silu(self.ops.linear(emb, self.t_w1, self.t_b1).float()).to(self.dtype)
        return self.ops.linear(h, self.t_w2, self.t_b2)  # [1, d]

    def encode_text(self, context: torch.Tensor) -> torch.Tensor:
        return self.ops.linear(context.to(self.dtype), self.text_w, self.text_b)

    def patchify(self, latents: torch.Tensor) -> torch.Tensor:
        c, frames, h, w = latents.shape
        x = latents.reshape(c, frames, h // 2, 2, w // 2, 2).permute(1, 2, 4, 0, 3, 5)
        return x.reshape(frames * (h // 2) * (w // 2), self.cfg.patch_dim)

    def unpatchify(self, x: torch.Tensor, frames: int) -> torch.Tensor:
        gh, gw = self.cfg.grid
        out = x.reshape(frames, gh, gw, self.cfg.in_channels, 2, 2).permute(3, 0, 1, 4, 2, 5)
        return out.reshape(self.cfg.in_channels, frames, gh * 2, gw * 2)

    def rope_tables(self, first_frame: int, frames: int, shard: RowShard | None):
        """Per-token cos/sin ``[tokens, pairs]`` of frames ``first_frame..+frames`` (this rank's rows)."""
        gh, gw = self.cfg.grid
        cos, sin = self.rope.token_tables((first_frame, 0, 0), (frames, gh, gw), self.device)
        if shard is not None:
            index = shard.token_index().to(self.device)
            cos, sin = cos.index_select(0, index), sin.index_select(0, index)
        return cos, sin

    # -- forward --------------------------------------------------------------------------------------------------

    def _ulysses_cache(self, cache: LongCatConditioningCache, shards, cp_group):
        """Per layer, the conditioning cache in Ulysses layout ``[all cache rows, heads / cp, d]`` (rank-major,
        RoPE applied to K): one NCCL all-to-all per layer and epoch, reused by every forward of the epoch."""
        key = (id(cache), cache.epoch.epoch_id)
        memo = getattr(self, "_ulysses_memo", None)
        if memo is not None and memo[0] == key:
            return memo[1]
        cshards = [RowShard(sh.rank, sh.cp, cache.epoch.frames, *self.cfg.grid) for sh in shards]
        rank = dist_rank(cp_group)
        cos_c, sin_c = self.rope_tables(cache.epoch.first_frame, cache.epoch.frames, cshards[rank])
        layers = [(ulysses_in(self.ops.rope(cache.k[layer].to(self.dtype), cos_c, sin_c).contiguous(), cp_group),
                   ulysses_in(cache.v[layer].to(self.dtype).contiguous(), cp_group)) for layer in range(len(self.blocks))]
        self._ulysses_memo = (key, layers)
        return layers

    def forward(self, latents: torch.Tensor, t: float, text: torch.Tensor | None, *, first_frame: int = 0,
                cache: LongCatConditioningCache | None = None, cp_group=None, return_kv: bool = False,
                ulysses=None):
        """Flow prediction ``[C, F, H, W]`` (FP32) of ``latents`` (frames ``first_frame..``) attending to the
        conditioning cache; ``return_kv`` also returns this forward's per-layer pre-RoPE (K, V).

        ``ulysses``: a :class:`~reelcache_b200.parallel.ulysses_fused.FusedUlysses` of ``cp_group`` -- the
        self-attention's all-to-alls then run fused into the QKV and output-projection GEMMs over NVLink
        peer memory (q/k norm and RoPE after the scatter, on this rank's heads of every token) instead of
        NCCL around the GEMMs."""
        import torch.distributed as dist
        cfg = self.cfg
        if ulysses is not None and (cp_group is None or return_kv):
            raise ValueError("the fused Ulysses path needs a context-parallel group and no K/V capture")
        frames = latents.shape[1]
        shard = shards = None
        if cp_group is not None:
            cp, rank = dist.get_world_size(cp_group), dist.get_rank(cp_group)
            shards = [RowShard(r, cp, frames, *cfg.grid) for r in range(cp)]
            shard = shards[rank]
        tokens = self.patchify(latents.float()).to(self.dtype)
        if shard is not None:
            tokens = shard.local(tokens)
        x = self.ops.linear(tokens, self.patch_w, self.patch_b).float()     # residual stream in FP32
        temb = self.timestep(t)
        cos_cur, sin_cur = self.rope_tables(first_frame, frames, shard)
        if cache is not None:
            cshard = None if shard is None else RowShard(shard.rank, shard.cp, cache.epoch.frames, *cfg.grid)
            cos_c, sin_c = self.rope_tables(cache.epoch.first_frame, cache.epoch.frames, cshard)
        n, h, hd = x.shape[0], cfg.heads, cfg.head_dim
        if ulysses is not None:  # RoPE rows of every rank's tokens in rank-major (gathered) order
            tables = [self.rope_tables(first_frame, frames, sh) for sh in shards]
            cos_g, sin_g = torch.cat([c for c, _ in tables]), torch.cat([s_ for _, s_ in tables])
            cache_u = self._ulysses_cache(cache, shards, cp_group) if cache is not None else None
        kvs = []
        for layer, blk in enumerate(self.blocks):
            mod = self.ops.linear(F.silu(temb.float()).to(self.dtype), blk["ada_w"], blk["ada_b"],
                                  out_dtype=torch.float32).reshape(6, cfg.dim)
            y = F.layer_norm(x, (cfg.dim,), eps=cfg.eps) * (1 + mod[1]) + mod[0]
            if ulysses is not None:
                if blk.get("lora", {}).keys() & {"qkv", "proj"}:
                    raise ValueError("LoRA branches on qkv / proj need the unfused Ulysses path (ulysses=None)")
                rows = ulysses.world * n
                q_u, k_u, _ = ulysses.qkv(y.to(self.dtype), blk["qkv_w"], blk["qkv_b"])
                q = self.ops.norm_rope(q_u, blk["q_norm"], cos_g, sin_g, cfg.eps)
                self.ops.norm_rope(k_u, blk["k_norm"], cos_g, sin_g, cfg.eps, out=k_u)  # in place: row by row
                if cache_u is not None:
                    ulysses.set_cache(*cache_u[layer])
                k_all, v_all = ulysses.kv_all(rows)
                ulysses.local["o"][:rows].copy_(self.ops.attention(q, k_all, v_all).reshape(rows, -1))
                ulysses.out(x, blk["proj_w"], blk["proj_b"], mod[2])
                self._cross_and_ffn(x, blk, mod, text, n)
                continue
            qkv = self._proj(blk, "qkv", y.to(self.dtype), blk["qkv_w"], blk["qkv_b"]).reshape(n, 3, h, hd)
            q = self.ops.rms_norm_heads(qkv[:, 0], blk["q_norm"], cfg.eps)
            k = self.ops.rms_norm_heads(qkv[:, 1], blk["k_norm"], cfg.eps)
            v = qkv[:, 2]
            if return_kv:
                kvs.append((k.clone(), v.clone()))
            if cache is not None:  # conditioning-cache branch: RoPE applied at read time
                k_all = torch.cat([self.ops.rope(cache.k[layer].to(k.dtype), cos_c, sin_c),
                                   self.ops.rope(k, cos_cur, sin_cur)])
                v_all = torch.cat([cache.v[layer].to(v.dtype), v])
            else:
                k_all, v_all = self.ops.rope(k, cos_cur, sin_cur), v
            q = self.ops.rope(q, cos_cur, sin_cur)
            if shard is not None:
                o = ulysses_out(self.ops.attention(ulysses_in(q, cp_group), ulysses_in(k_all.contiguous(), cp_group),
                                                   ulysses_in(v_all.contiguous(), cp_group)), cp_group)
            else:
                o = self.ops.attention(q, k_all, v_all)
            x = x + mod[2] * self._proj(blk, "proj", o.reshape(n, cfg.dim), blk["proj_w"], blk["proj_b"]).float()
            self._cross_and_ffn(x, blk, mod, text, n)
        fmod = self.ops.linear(F.silu(temb.float()).to(self.dtype), self.final_ada_w, self.final_ada_b,
                               out_dtype=torch.float32).reshape(2, cfg.dim)
        y = (F.layer_norm(x, (cfg.dim,), eps=cfg.eps) * (1 + fmod[1]) + fmod[0]).to(self.dtype)
        out = self.ops.linear(y, self.final_w, self.final_b, out_dtype=torch.float32)
        if shard is not None:
            out = gather_tokens(out, shards, cp_group)
        pred = self.unpatchify(out, frames)
        return (pred, kvs) if return_kv else pred

    # -- LoRA ------------------------------------------------------------------------------------------------------

    def _proj(self, blk: dict, name: str, x: torch.Tensor, w: torch.Tensor, b: torch.Tensor | None = None):
        """A projection of the block plus its LoRA branches (none attached: the plain GEMM)."""
        out = self.ops.linear(x, w, b)
        if "lora" not in blk:
            return out
        from .longcat_lora import apply_branches
        return apply_branches(blk, name, x, out, self.ops.linear)

    def attach_lora(self, state_dict, *, multiplier: float = 1.0) -> list[str]:
        """Attach the branches of a native LongCat LoRA state dict (e.g. ``cfg_step_lora``); returns the targeted
        module paths. Branches stay separate from the weights (models/longcat_lora.py)."""
        from .longcat_lora import attach
        return attach(self.blocks, state_dict, multiplier=multiplier, dtype=self.dtype, device=self.device)

    def detach_loras(self) -> int:
        from .longcat_lora import detach
        return detach(self.blocks)

    def set_loras_enabled(self, enabled: bool) -> None:
        from .longcat_lora import set_enabled
        set_enabled(self.blocks, enabled)

    def _cross_and_ffn(self, x: torch.Tensor, blk: dict, mod: torch.Tensor, text: torch.Tensor, n: int) -> None:
        """Cross-attention over the text (skipped when ``text`` is None) and the SwiGLU FFN on this rank's
        rows, in place on ``x``."""
        cfg = self.cfg
        h, hd = cfg.heads, cfg.head_dim
        if text is not None:
            y = F.layer_norm(x, (cfg.dim,), eps=cfg.eps).to(self.dtype)
            cq = self.ops.rms_norm_heads(self._proj(blk, "cq", y, blk["cq_w"], blk["cq_b"]).reshape(n, h, hd),
                                         blk["cq_norm"], cfg.eps)
            ckv = self._proj(blk, "ckv", text, blk["ckv_w"], blk["ckv_b"]).reshape(-1, 2, h, hd)
            ck = self.ops.rms_norm_heads(ckv[:, 0], blk["ck_norm"], cfg.eps)
            co = self.ops.attention(cq, ck, ckv[:, 1])
            x.add_(self._proj(blk, "cproj", co.reshape(n, cfg.dim), blk["cproj_w"], blk["cproj_b"]).float())
        y = (F.layer_norm(x, (cfg.dim,), eps=cfg.eps) * (1 + mod[4]) + mod[3]).to(self.dtype)
        hidden = (F.silu(self._proj(blk, "w1", y, blk["w1"]).float())
                  * self._proj(blk, "w3", y, blk["w3"]).float()).to(self.dtype)
        x.add_(mod[5] * self._proj(blk, "w2", hidden, blk["w2"]).float())

    def build_conditioning_cache(self, cond_latents: torch.Tensor, epoch: ConditioningCacheEpoch,
                                 *, cp_group=None) -> LongCatConditioningCache:
        """One forward over the conditioning latents at ``t = 0`` returning their per-layer pre-RoPE K/V.

        The forward skips cross-attention (no text) and places the frames at segment-local positions
        (first frame 0), as reference reelcache_sglang_models/longcat_video/dit_core.py:452 does: the cache
        then depends only on the weights and the latents, which is what makes the content key of a segment
        (model fingerprint, latents digest, grid) identify it across sessions, prompts and video offsets.
        The epoch's ``first_frame`` is applied at read time, when RoPE rotates the cached K."""
        _, kvs = self.forward(cond_latents, 0.0, None, first_frame=0, cp_group=cp_group, return_kv=True)
        return LongCatConditioningCache(epoch, [k for k, _ in kvs], [v for _, v in kvs])

    def flops_per_forward(self, tokens: int, cache_tokens: int) -> float:
        cfg = self.cfg
        d, f = cfg.dim, cfg.ffn
        linear = 2 * tokens * (3 * d * d + d * d + d * d + d * d + 3 * d * f)
        attention = 4 * tokens * (tokens + cache_tokens) * d + 4 * tokens * cfg.text_len * d
        return cfg.layers * (linear + attention)


class ReelCacheConditioningCacheBackend:
    """The conditioning-cache seam over the archive: a built cache is committed as a **segment** node of
    the session's lineage (rank method, node pack); ``restore(epoch)`` rebuilds the cache from the
    newest segment node of that epoch (this rank's rows only under CP), or returns None."""

    def __init__(self, runtime, lineage: str, method, *, head_dim: int, grid: tuple[int, int], device="cpu",
                 cp_shard: RowShard | None = None, restorer="auto"):
        """``restorer``: a :class:`~reelcache_b200.archive_restore.LineageRestorer` on ``device``; with it a
        segment restores on the fused sm_100a kernels, each CP rank gathering only its rows of the coefficient
        tiles (:func:`shard_runs`), instead of decoding every row on the host. ``"auto"`` (default) creates one
        on the first restore when ``device`` is a CUDA device; ``None`` keeps the host decode (FP32 reference)."""
        self.restorer = restorer
        self.runtime = runtime
        self.lineage = lineage
        self.method = method
        self.device = torch.device(device)
        self.cp_shard = cp_shard
        self.head_dim = head_dim
        self.grid = grid
        self.segments: dict[str, str] = {}   # epoch id -> node ref
        self.stats = {"built": 0, "restored": 0, "missed": 0}

    def on_cache_built(self, cache: LongCatConditioningCache) -> str:
        from ..types import MatrixKey, TensorContext
        epoch = cache.epoch
        matrices, contexts = {}, {}
        for layer in range(len(cache.k)):
            for target, t in (("K", cache.k[layer]), ("V", cache.v[layer])):
                key = MatrixKey(layer, target)
                matrices[key] = t.reshape(t.shape[0], -1)
                contexts[key] = TensorContext(self.runtime.model, key, 0, epoch.frames, *self.grid,
                                              "pre_rope" if target == "K" else "none")
        commit = self.runtime.commit_segment(self.lineage, f"segment-{epoch.segment_index}", matrices, contexts,
                                             method=self.method, epoch_id=epoch.epoch_id, device=self.device,
                                             details={"first_frame": epoch.first_frame})
        self.segments[epoch.epoch_id] = commit.node_ref
        self.stats["built"] += 1
        return commit.node_ref

    def restore(self, epoch: ConditioningCacheEpoch, node_ref: str | None = None) -> LongCatConditioningCache | None:
        """``node_ref`` names the segment node directly (a fork or a resumed session restores another session's
        epoch, whose id differs); otherwise the node this backend committed for ``epoch``."""
        from ..types import MatrixKey
        node = node_ref or self.segments.get(epoch.epoch_id)
        if node is None:
            self.stats["missed"] += 1
            return None
        if self.restorer == "auto":
            self.restorer = None
            if self.device.type == "cuda":
                from ..archive_restore import LineageRestorer
                self.restorer = LineageRestorer(self.runtime, self.device)
        if self.restorer is not None and self.device.type == "cuda":
            return self._restore_fused(epoch, node)
        ks, vs = [], []
        packs: dict = {}
        for layer in range(self.runtime.model.layers):
            k, v = (self.runtime.acquire_node_history(node, MatrixKey(layer, t), device=self.device,
                                                      dtype=torch.bfloat16, packs=packs) for t in ("K", "V"))
            if self.cp_shard is not None:
                index = RowShard(self.cp_shard.rank, self.cp_shard.cp, epoch.frames, *self.grid).token_index()
                k, v = k.index_select(0, index.to(k.device)), v.index_select(0, index.to(v.device))
            ks.append(k.reshape(k.shape[0], -1, self.head_dim))
            vs.append(v.reshape(v.shape[0], -1, self.head_dim))
        self.stats["restored"] += 1
        return LongCatConditioningCache(epoch, ks, vs) if ks else None

    def _restore_fused(self, epoch: ConditioningCacheEpoch, node: str) -> LongCatConditioningCache:
        """The segment's K / V straight from its node pack on the fused kernels (no RoPE: the cache is pre-RoPE),
        this rank's rows only."""
        model = self.runtime.model
        h, w = self.grid
        shard = self.cp_shard if self.cp_shard is None else RowShard(self.cp_shard.rank, self.cp_shard.cp,
                                                                      epoch.frames, h, w)
        runs = shard_runs(shard, epoch.frames, h, w)
        tokens = sum(job[1] for job in runs)
        heads = model.channels_for("K") // self.head_dim
        ks = [torch.empty((1, tokens, heads, self.head_dim), dtype=torch.bfloat16, device=self.device)
              for _ in range(model.layers)]
        vs = [torch.empty_like(k) for k in ks]
        stream = torch.cuda.current_stream(self.device)
        program = self.restorer.gather_program(node, lambda layer, t: ks[layer] if t == "K" else vs[layer], runs,
                                               stream=stream)
        program.prepare()
        program.launch_all()
        self.stats["restored"] += 1
        self.stats["fused"] = self.stats.get("fused", 0) + 1
        self.last_program = program  # keeps the staging alive until the caller's stream moves on
        return LongCatConditioningCache(epoch, [k[0] for k in ks], [v[0] for v in vs])


def shard_runs(shard: RowShard | None, frames: int, height: int, width: int) -> list[tuple[int, int, int, int, int]]:
    """Row-run gathers ``(dest_row, tokens, run_len, run_stride, run_offset)`` that read a CP rank's block of a
    ``frames x height x width`` token grid in its local order (frame-major, then rows, then columns): one job when
    the block spans whole rows or whole columns of every frame, else one job per frame."""
    if shard is None:
        total = frames * height * width
        return [(0, total, total, total, 0)]
    rows, cols = shard.block
    bh, bw = rows.stop - rows.start, cols.stop - cols.start
    per_frame = height * width
    if bh == height:        # column block: runs of bw columns, one per (frame, row)
        return [(0, frames * bh * bw, bw, width, cols.start)]
    if bw == width:         # row block: one run of bh whole rows per frame
        return [(0, frames * bh * bw, bh * width, per_frame, rows.start * width)]
    return [(f * bh * bw, bh * bw, bw, width, f * per_frame + rows.start * width + cols.start) for f in range(frames)]
