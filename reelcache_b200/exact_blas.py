"""FP32-accurate products and triangular solves, independent of the TF32 flags (the counterpart of
reference reelcache/exact_blas.py:1-20 for the rationale, :171 ``mm``, :224 ``trsm_right_upper``).

The reference reaches IEEE FP32 by calling cuBLAS SGEMM with the default math mode. On sm_100a the
tensor cores do the same work faster: each FP32 operand is split into three bfloat16 parts
(``x = hi + mid + lo`` exactly to 24 bits), the parts are laid out as K-concatenated segments and one
tcgen05 GEMM with FP32 accumulation in TMEM evaluates ``hh + hm + mh + mm + hl + lh`` -- every cross
product down to 2^-16 relative, so the result carries the error of an FP32 GEMM (the dropped terms are
below 2^-24 relative). CPU tensors use torch's FP32 matmul (IEEE on the host).

``trsm_right_upper(x, r)`` = ``x @ inv(r)`` for upper-triangular ``r``: the small ``k x k`` inverse is
formed in FP64 by triangular substitution and applied with :func:`mm`. ``cholesky_qr2`` orthonormalizes
columns with two CholeskyQR passes -- FP32-accurate Gram, FP64 Cholesky and FP64 triangular solve -- and falls
back to Householder QR when a Gram is not positive definite.
"""

from __future__ import annotations

import contextlib

import torch

from .errors import ConfigurationError

#: Counters of the calls by path (tests and telemetry read them).
STATS = {"mm_split_bf16": 0, "mm_host": 0, "mm_tf32_guarded": 0, "trsm": 0, "cholesky_qr2": 0, "qr_fallbacks": 0}


@contextlib.contextmanager
def _no_tf32():
    old = torch.backends.cuda.matmul.allow_tf32, torch.backends.cudnn.allow_tf32
    torch.backends.cuda.matmul.allow_tf32 = False
    torch.backends.cudnn.allow_tf32 = False
    try:
        yield
    finally:
        torch.backends.cuda.matmul.allow_tf32, torch.backends.cudnn.allow_tf32 = old


def _native_ok(a: torch.Tensor) -> bool:
    if not a.is_cuda:
        return False
    from .ops import _ext
    return _ext.available()


def mm(a: torch.Tensor, b: torch.Tensor) -> torch.Tensor:
    """FP32-accurate ``a @ b`` of 2-D floating matrices (FP32 result)."""
    if a.ndim != 2 or b.ndim != 2 or a.shape[1] != b.shape[0]:
        raise ConfigurationError(f"mm needs [M, K] @ [K, N], got {tuple(a.shape)} @ {tuple(b.shape)}")
    if a.device != b.device:
        raise ConfigurationError("mm operands must share a device")
    if a.shape[0] == 0 or b.shape[1] == 0 or a.shape[1] == 0:
        return torch.zeros((a.shape[0], b.shape[1]), dtype=torch.float32, device=a.device)
    if _native_ok(a):
        from .ops.fitter import mm_fp32
        STATS["mm_split_bf16"] += 1
        return mm_fp32(a, b)
    if a.is_cuda:
        STATS["mm_tf32_guarded"] += 1
        with _no_tf32():
            return a.float() @ b.float()
    STATS["mm_host"] += 1
    return a.float() @ b.float()


def gram(x: torch.Tensor) -> torch.Tensor:
    """Symmetric FP32-accurate ``x^T x``."""
    g = mm(x.t(), x)
    return 0.5 * (g + g.t())


def trsm_right_upper(x: torch.Tensor, r: torch.Tensor) -> torch.Tensor:
    """``x @ inv(r)`` for an upper-triangular ``r[k, k]`` (FP32 result)."""
    if r.ndim != 2 or r.shape[0] != r.shape[1] or x.shape[1] != r.shape[0]:
        raise ConfigurationError("trsm_right_upper needs x[C, k] and an upper-triangular r[k, k]")
    STATS["trsm"] += 1
    eye = torch.eye(r.shape[0], dtype=torch.float64, device=r.device)
    inverse = torch.linalg.solve_triangular(r.double(), eye, upper=True)
    return mm(x, inverse.float())


def _canonical(q: torch.Tensor, r: torch.Tensor) -> torch.Tensor:
    signs = torch.sign(torch.diagonal(r))
    signs[signs == 0] = 1
    return q * signs.to(q.dtype)


def householder_qr(b: torch.Tensor) -> torch.Tensor:
    """Column-orthonormal ``Q`` of ``b[C, k]`` by Householder QR in FP32 (signs canonical)."""
    q, r = torch.linalg.qr(b.float())
    return _canonical(q, r)


def cholesky_qr2_routine(b: torch.Tensor):
    """Lockstep routine form of :func:`cholesky_qr2`: both passes are queued, then the factorizations' status and
    the result's finiteness are read in one host round (yielded); a Gram that is not positive definite in either
    pass (or a non-finite result) gives the Householder basis, as when each pass is checked on the spot."""
    STATS["cholesky_qr2"] += 1
    q = b.float()
    status = None
    for _ in range(2):
        # the factorization reads the upper triangle only, so the Gram needs no symmetrization; the triangular
        # solve runs in FP64 (q R^-1 directly, no explicit inverse)
        factor, info = torch.linalg.cholesky_ex(mm(q.t(), q).double(), upper=True)
        status = info if status is None else status + info
        q = torch.linalg.solve_triangular(factor, q.double(), upper=True, left=False).float()
    (bad,) = yield ((status != 0) | ~torch.isfinite(q).all(),)
    if bad:
        STATS["qr_fallbacks"] += 1
        return householder_qr(b)
    return q


def cholesky_qr2(b: torch.Tensor) -> torch.Tensor:
    """Column-orthonormal basis of ``b[C, k]`` by two CholeskyQR passes (FP64 Cholesky of the FP32-accurate
    Gram, FP32-accurate triangular solve); Householder QR when a Gram is not positive definite."""
    from .deferred_reads import run_one
    return run_one(cholesky_qr2_routine(b))


__all__ = ["STATS", "cholesky_qr2", "cholesky_qr2_routine", "gram", "householder_qr", "mm", "trsm_right_upper"]
