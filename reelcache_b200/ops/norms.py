"""DiT block elementwise ops on sm_100a (csrc/model/norms.cu): AdaLN LayerNorm + modulation, fused
q/k RMSNorm + RoPE writing straight into the KV-cache slots, and RMSNorm."""

from __future__ import annotations

import torch

from ._ext import ext


def ln_modulate(x, *, shift=None, scale=None, weight=None, bias=None, eps=1e-6, out=None):
    """``LayerNorm(x) * (1 + scale) + shift`` for bf16 ``x[T, C]`` (fp32 vectors)."""
    x2 = x.reshape(-1, x.shape[-1])
    out = torch.empty_like(x2) if out is None else out.reshape(-1, x.shape[-1])
    ext().ln_modulate(x2, out, shift, scale, weight, bias, float(eps))
    return out.reshape(x.shape)


def qkv_norm_rope(qkv, wq, wk, cos_tok, sin_tok, q_out, k_cache, v_cache, *, head_dim, k_pre=None, eps=1e-6):
    """From fused ``qkv[T, 3C]``: ``q_out = RoPE(RMSNorm(q) wq)``; ``k_pre = RMSNorm(k) wk`` (optional
    capture); ``k_cache = RoPE(k_pre)``; ``v_cache = v`` (all ``[T, C]`` row views)."""
    ext().qkv_norm_rope(qkv, wq, wk, cos_tok, sin_tok, q_out, k_pre, k_cache, v_cache, int(head_dim), float(eps))


def rms_norm(x, w, *, eps=1e-6, out=None):
    x2 = x.reshape(-1, x.shape[-1])
    out = torch.empty_like(x2) if out is None else out.reshape(-1, x.shape[-1])
    ext().rms_norm(x2, out, w, float(eps))
    return out.reshape(x.shape)


def head_norm_rope(x, weight=None, cos=None, sin=None, *, eps=1e-6, out=None):
    """Per-head RMSNorm (``weight`` [head_dim], optional) then interleaved-pair RoPE (``cos`` / ``sin``
    [tokens, head_dim / 2], optional) of ``x[tokens, heads, head_dim]`` in one pass; FP32 math, bf16 out."""
    out = torch.empty(x.shape, dtype=torch.bfloat16, device=x.device) if out is None else out
    ext().head_norm_rope(x, out, None if weight is None else weight.float().contiguous(),
                         None if cos is None else cos.float().contiguous(),
                         None if sin is None else sin.float().contiguous(), float(eps))
    return out
