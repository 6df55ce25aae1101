"""Plain-PyTorch FP32 reference of the causal DiT forward (the numerics oracle of the fused-kernel
model in :mod:`reelcache_b200.models.causal_wan`; same weights, same block math)."""

from __future__ import annotations

import math

import torch

from .causal_wan import CausalWanDiT, sinusoidal


def _ln(x, eps, weight=None, bias=None):
    y = torch.nn.functional.layer_norm(x, (x.shape[-1],), eps=eps)
    if weight is not None:
        y = y * weight + bias
    return y


def _rms(x, w, eps):
    return x * torch.rsqrt(x.square().mean(-1, keepdim=True) + eps) * w


def _rope(x, cos, sin):
    """``x[T, H, D]`` interleaved pairs, ``cos/sin[T, D/2]``."""
    even, odd = x[..., 0::2], x[..., 1::2]
    c, s = cos[:, None, :], sin[:, None, :]
    out = torch.empty_like(x)
    out[..., 0::2] = even * c - odd * s
    out[..., 1::2] = even * s + odd * c
    return out


def _attn(q, k, v):
    scale = 1.0 / math.sqrt(q.shape[-1])
    scores = torch.einsum("qhd,khd->hqk", q, k) * scale
    return torch.einsum("hqk,khd->qhd", scores.softmax(-1), v)


def reference_forward(model: CausalWanDiT, latents, t, chunk_index, history_k, history_v, context):
    """FP32 forward of one chunk. ``history_k/v``: per-layer post-RoPE K and V ``[T_hist, H, D]`` FP32.
    Returns ``(flow [in_dim, F, H, W], k_pre per layer, v per layer, k_post per layer)``."""
    cfg = model.cfg
    f32 = lambda w: w.float()  # noqa: E731
    x = model.patchify(latents).float() @ f32(model.patch_w).t() + f32(model.patch_b)
    emb = sinusoidal(torch.tensor([float(t)], device=latents.device), cfg.freq_dim)
    e = torch.nn.functional.silu(emb @ f32(model.time_w1).t() + f32(model.time_b1))
    e = e @ f32(model.time_w2).t() + f32(model.time_b2)
    e0 = (torch.nn.functional.silu(e) @ f32(model.tproj_w).t() + f32(model.tproj_b)).reshape(6, cfg.dim)
    e = e.reshape(-1)
    c = torch.nn.functional.gelu(context.float() @ f32(model.text_w1).t() + f32(model.text_b1), approximate="tanh")
    c = c @ f32(model.text_w2).t() + f32(model.text_b2)
    cos, sin = model.token_rope(chunk_index)
    tokens = cfg.chunk_tokens
    k_pres, vs, k_posts = [], [], []
    for layer, blk in enumerate(model.blocks):
        mod = blk["modulation"] + e0
        y = _ln(x, cfg.eps) * (1 + mod[1]) + mod[0]
        qkv = y @ f32(blk["qkv_w"]).t() + f32(blk["qkv_b"])
        q, k, v = qkv.split(cfg.dim, dim=-1)
        q = _rms(q, blk["norm_q"], cfg.eps).reshape(tokens, cfg.heads, cfg.head_dim)
        k_pre = _rms(k, blk["norm_k"], cfg.eps)
        k = k_pre.reshape(tokens, cfg.heads, cfg.head_dim)
        q, k = _rope(q, cos, sin), _rope(k, cos, sin)
        v = v.reshape(tokens, cfg.heads, cfg.head_dim)
        keys = torch.cat([history_k[layer], k]) if history_k is not None else k
        values = torch.cat([history_v[layer], v]) if history_v is not None else v
        o = _attn(q, keys, values).reshape(tokens, cfg.dim)
        x = x + (o @ f32(blk["o_w"]).t() + f32(blk["o_b"])) * mod[2]
        y = _ln(x, cfg.eps, blk["norm3_w"], blk["norm3_b"])
        cq = _rms(y @ f32(blk["cq_w"]).t() + f32(blk["cq_b"]), blk["cnorm_q"], cfg.eps)
        ck = _rms(c @ f32(blk["ck_w"]).t() + f32(blk["ck_b"]), blk["cnorm_k"], cfg.eps)
        cv = c @ f32(blk["cv_w"]).t() + f32(blk["cv_b"])
        co = _attn(cq.reshape(tokens, cfg.heads, cfg.head_dim), ck.reshape(-1, cfg.heads, cfg.head_dim),
                   cv.reshape(-1, cfg.heads, cfg.head_dim)).reshape(tokens, cfg.dim)
        x = x + co @ f32(blk["co_w"]).t() + f32(blk["co_b"])
        y = _ln(x, cfg.eps) * (1 + mod[4]) + mod[3]
        h = torch.nn.functional.gelu(y @ f32(blk["ffn1_w"]).t() + f32(blk["ffn1_b"]), approximate="tanh")
        x = x + (h @ f32(blk["ffn2_w"]).t() + f32(blk["ffn2_b"])) * mod[5]
        k_pres.append(k_pre)
        vs.append(v.reshape(tokens, cfg.dim))
        k_posts.append(k)
    y = _ln(x, cfg.eps) * (1 + model.head_mod[1] + e) + model.head_mod[0] + e
    out = y @ f32(model.head_w).t() + f32(model.head_b)
    return model.unpatchify(out), k_pres, vs, k_posts
