"""Attention entry point of the DiT: queries of the current chunk against keys/values of the causal
KV cache (bidirectional within the chunk) or of the cached text tokens.

``backend="fused"`` is the sm_100a tcgen05 flash-attention kernel (csrc/model/attention_sm100.cu: TMA
producer, single-thread MMA issuer, two softmax warpgroups splitting the KV blocks, S and O in TMEM, lazy
rescaling); ``"sdpa"`` is PyTorch's scaled_dot_product_attention (cuDNN's fused kernel on B200). ``"auto"``
selects ``sdpa`` on CUDA: measured on B200 the fused kernel reaches about half of cuDNN's throughput (its
per-block shared-memory traffic -- P written to and re-read from shared memory, K/V tiles read once per
128 queries -- and the exp pipe bound it), so it is selected only explicitly.
"""

from __future__ import annotations

import math

import torch

from . import _ext


def _fused_available() -> bool:
    return _ext.available() and hasattr(_ext.ext(), "attention_fwd")


def attention(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, *, backend: str = "auto",
              scale: float | None = None) -> torch.Tensor:
    """``softmax(q k^T * scale) v`` for ``q[Tq, H, D]``, ``k, v[Tk, H, D]`` (any row strides); returns
    ``[Tq, H, D]`` bf16."""
    scale = 1.0 / math.sqrt(q.shape[-1]) if scale is None else scale
    if backend == "auto":
        backend = "sdpa"
    if backend == "fused":
        out = torch.empty((q.shape[0], q.shape[1], q.shape[2]), dtype=torch.bfloat16, device=q.device)
        _ext.ext().attention_fwd(q, k, v, out, float(scale), _ext.status_word(q.device))
        return out
    qh = q.permute(1, 0, 2).unsqueeze(0)
    kh = k.permute(1, 0, 2).unsqueeze(0)
    vh = v.permute(1, 0, 2).unsqueeze(0)
    out = torch.nn.functional.scaled_dot_product_attention(qh, kh, vh, scale=scale)
    return out[0].permute(1, 0, 2).contiguous()
