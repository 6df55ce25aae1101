"""Attention entry point of the DiT: queries of the current chunk against keys/values of the causal
KV cache (bidirectional within the chunk) or of the cached text tokens.

``backend="fused"`` is the sm_100a tcgen05 flash-attention kernel (csrc/model/attention_sm100.cu: 256
queries per CTA as two 128-row tiles sharing every K / V block, TMA producer, single-thread MMA issuer,
one softmax warpgroup per tile in ping-pong with the tensor core, S, P and O in TMEM -- P is the A operand
of the P V MMA -- lazy rescaling, and key ranges merged in FP32 when one CTA per query pair would leave
the last wave of SMs idle); ``"sdpa"`` is PyTorch's scaled_dot_product_attention (cuDNN's fused kernel
on B200). ``"auto"`` selects ``AUTO_BACKEND``.

``options`` (fused only): bits 0-3 force the number of key ranges (0: chosen from the SM count),
``OPT_POLY_EXP`` computes an eighth of the exponentials with a polynomial on the FMA pipe, ``OPT_NO_TURNS``
lets the two softmax warpgroups run their exponentials at the same time.
"""

from __future__ import annotations

import math

import torch

from . import _ext


def _fused_available() -> bool:
    return _ext.available() and hasattr(_ext.ext(), "attention_fwd")


OPT_POLY_EXP = 16
OPT_NO_TURNS = 128
AUTO_BACKEND = "sdpa"


def attention(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, *, backend: str = "auto",
              scale: float | None = None, options: int = 0) -> torch.Tensor:
    """``softmax(q k^T * scale) v`` for ``q[Tq, H, D]``, ``k, v[Tk, H, D]`` (any row strides); returns
    ``[Tq, H, D]`` bf16."""
    scale = 1.0 / math.sqrt(q.shape[-1]) if scale is None else scale
    if backend == "auto":
        backend = AUTO_BACKEND
    if backend == "fused":
        out = torch.empty((q.shape[0], q.shape[1], q.shape[2]), dtype=torch.bfloat16, device=q.device)
        _ext.ext().attention_fwd(q, k, v, out, float(scale), _ext.status_word(q.device), int(options))
        return out
    qh = q.permute(1, 0, 2).unsqueeze(0)
    kh = k.permute(1, 0, 2).unsqueeze(0)
    vh = v.permute(1, 0, 2).unsqueeze(0)
    out = torch.nn.functional.scaled_dot_product_attention(qh, kh, vh, scale=scale)
    return out[0].permute(1, 0, 2).contiguous()
