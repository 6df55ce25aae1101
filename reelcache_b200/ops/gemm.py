"""tcgen05 GEMM entry points (csrc/gemm/gemm_sm100.cu).

``linear(x, w)`` computes ``x @ w.T`` for bf16 ``x[M, K]`` and a Linear weight ``w[N, K]`` with
fp32 accumulation in TMEM and one of the fused epilogues below.
"""

from __future__ import annotations

import torch

from ._ext import ext, status_word

STORE, BIAS, BIAS_GELU, BIAS_GATE_RESID = 0, 1, 2, 3


def linear(x, weight, bias=None, *, out=None, out_dtype=torch.bfloat16, alpha=1.0, bn=0):
    """``alpha * x @ weight.T (+ bias)``; x, weight bf16 with unit inner stride."""
    shape = x.shape
    x2 = x.reshape(-1, shape[-1])
    if out is None:
        out = torch.empty((x2.shape[0], weight.shape[0]), dtype=out_dtype, device=x.device)
    ext().gemm_bf16_tn(x2, weight, out, BIAS if bias is not None else STORE, bias, None, None, float(alpha), bn,
                       status_word(x.device))
    return out.reshape(*shape[:-1], weight.shape[0])


def linear_gelu(x, weight, bias, *, out=None):
    """``gelu_tanh(x @ weight.T + bias)`` in one kernel."""
    shape = x.shape
    x2 = x.reshape(-1, shape[-1])
    if out is None:
        out = torch.empty((x2.shape[0], weight.shape[0]), dtype=torch.bfloat16, device=x.device)
    ext().gemm_bf16_tn(x2, weight, out, BIAS_GELU, bias, None, None, 1.0, 0, status_word(x.device))
    return out.reshape(*shape[:-1], weight.shape[0])


def linear_gated_residual(x, weight, bias, gate, residual):
    """``residual += (x @ weight.T + bias) * gate`` (in place on ``residual``; gate fp32 [N] or None)."""
    x2 = x.reshape(-1, x.shape[-1])
    r2 = residual.view(-1, residual.shape[-1])
    ext().gemm_bf16_tn(x2, weight, r2, BIAS_GATE_RESID, bias, gate, r2, 1.0, 0, status_word(x.device))
    return residual


def matmul_tn(a, b, *, out_dtype=torch.float32, alpha=1.0):
    """``alpha * a @ b.T`` for bf16 K-major operands, fp32 (or bf16) output."""
    out = torch.empty((a.shape[0], b.shape[0]), dtype=out_dtype, device=a.device)
    ext().gemm_bf16_tn(a, b, out, STORE, None, None, None, float(alpha), 0, status_word(a.device))
    return out
