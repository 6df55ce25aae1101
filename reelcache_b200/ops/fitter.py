"""Fitter kernels (csrc/fit/fitter.cu): split-bf16 operands of the FP32-accurate tensor-core GEMM, the
batched Jacobi eigensolver, fused square sums, exact source fingerprints and the compensated Dot2 GEMM.

Every entry point takes CUDA tensors and raises when the extension is missing (no silent fallback); the
callers in :mod:`reelcache_b200.exact_blas`, :mod:`reelcache_b200.gpu_fitting` and
:mod:`reelcache_b200.accel` choose between these kernels and the CPU paths explicitly.
"""

from __future__ import annotations

import torch

from ._ext import ext

#: K-concatenated parts of the A and B operands (0 hi, 1 mid, 2 lo): lh + hl + mm + mh + hm + hh, the
#: small cross products first.
SPLIT_A = (2, 0, 1, 1, 0, 0)
SPLIT_B = (0, 2, 1, 0, 1, 0)
JACOBI_MAX_N = 160
SQ_ROWS = 8
FP_ROWS = 8


def _round8(k: int) -> int:
    return (int(k) + 7) // 8 * 8


def split_operand(x: torch.Tensor, parts) -> tuple[torch.Tensor, int]:
    """bf16 ``[R, len(parts) * kp]`` of FP32 ``x[R, K]`` (any unit-stride layout); returns (out, kp)."""
    x = x if x.dtype == torch.float32 else x.float()
    if x.stride(1) != 1 and x.stride(0) != 1:
        x = x.contiguous()
    kp = _round8(x.shape[1])
    out = torch.empty((x.shape[0], len(parts) * kp), dtype=torch.bfloat16, device=x.device)
    ext().split_bf16x3(x, out, kp, list(parts))
    return out, kp


def matmul_promoted(a: torch.Tensor, b: torch.Tensor, *, alpha: float = 1.0) -> torch.Tensor:
    """``alpha * a @ b.T`` for bf16 K-major operands with the tensor-core partials promoted to IEEE FP32
    adds every 128 K-elements (csrc/gemm/gemm_exact.cu)."""
    from ._ext import status_word
    out = torch.empty((a.shape[0], b.shape[0]), dtype=torch.float32, device=a.device)
    ext().gemm_bf16_promoted(a, b, out, float(alpha), status_word(a.device))
    return out


#: A bf16 left operand is its own hi part (mid = lo = 0): three segments a x (lo, mid, hi of b) carry every
#: nonzero cross product of the six, so the GEMM's K halves with the same result.
SPLIT_A_BF16 = (0, 0, 0)
SPLIT_B_BF16 = (2, 1, 0)


class _SplitCache:
    """Split operands of tensors that are multiplied again and again (a Gram matrix through a subspace iteration,
    a source matrix through its projections), kept while the tensor lives and is unchanged.

    An entry is keyed by the operand's root tensor (held weakly: a freed tensor's entry never matches the tensor
    that reuses its memory), its view geometry, the split parts and the root's version counter (an in-place write
    invalidates it); entries are bounded in bytes, least recently used first out."""

    def __init__(self, max_bytes: int = 4 << 30):
        import threading
        from collections import OrderedDict
        self.max_bytes = max_bytes
        self._entries: "OrderedDict[tuple, tuple]" = OrderedDict()
        self._bytes = 0
        self._lock = threading.Lock()
        self.hits = self.misses = 0

    @staticmethod
    def _key(x: torch.Tensor, parts) -> tuple:
        root = x._base if x._base is not None else x
        return (id(root), x.data_ptr(), tuple(x.shape), tuple(x.stride()), x.dtype, tuple(parts)), root

    def get(self, x: torch.Tensor, parts) -> torch.Tensor:
        import weakref
        key, root = self._key(x, parts)
        with self._lock:
            entry = self._entries.get(key)
            if entry is not None:
                ref, version, value = entry
                if ref() is root and version == root._version:
                    self._entries.move_to_end(key)
                    self.hits += 1
                    return value
                self._bytes -= value.numel() * value.element_size()
                del self._entries[key]
        value, _ = split_operand(x, parts)
        size = value.numel() * value.element_size()
        with self._lock:
            self.misses += 1
            if size <= self.max_bytes // 4:
                self._entries[key] = (weakref.ref(root), root._version, value)
                self._bytes += size
                while self._bytes > self.max_bytes and self._entries:
                    _, (_, _, old) = self._entries.popitem(last=False)
                    self._bytes -= old.numel() * old.element_size()
            self._sweep()
        return value

    def _sweep(self) -> None:
        """Drop entries whose tensors died (called under the lock)."""
        for key in [k for k, (ref, _, _) in self._entries.items() if ref() is None]:
            value = self._entries.pop(key)[2]
            self._bytes -= value.numel() * value.element_size()

    def clear(self) -> None:
        with self._lock:
            self._entries.clear()
            self._bytes = 0


SPLITS = _SplitCache()


def mm_fp32(a: torch.Tensor, b: torch.Tensor) -> torch.Tensor:
    """FP32-accurate ``a @ b`` (``a[M, K]``, ``b[K, N]``): split-bf16 operands (reused while an operand's tensor is
    unchanged), one tcgen05 GEMM with promoted accumulation."""
    parts_a, parts_b = (SPLIT_A_BF16, SPLIT_B_BF16) if a.dtype == torch.bfloat16 else (SPLIT_A, SPLIT_B)
    a_split = SPLITS.get(a, parts_a)
    b_split = SPLITS.get(b.t(), parts_b)
    return matmul_promoted(a_split, b_split)


def jacobi_eigh(mats: torch.Tensor, *, max_sweeps: int = 30, tol: float = 2.0 ** -23):
    """Batched symmetric eigendecomposition of FP32 ``[B, n, n]`` (n <= 160): ascending values ``[B, n]``,
    column eigenvectors ``[B, n, n]``, per-matrix status (0 converged, 1 sweep limit, 2 non-finite) and
    sweep counts."""
    if mats.dim() == 2:
        mats = mats.unsqueeze(0)
    mats = mats.float().contiguous()
    batch, n = int(mats.shape[0]), int(mats.shape[1])
    values = torch.empty((batch, n), dtype=torch.float32, device=mats.device)
    vectors = torch.empty((batch, n, n), dtype=torch.float32, device=mats.device)
    info = torch.empty((batch,), dtype=torch.int32, device=mats.device)
    sweeps = torch.empty((batch,), dtype=torch.int32, device=mats.device)
    ext().jacobi_eigh(mats, values, vectors, info, sweeps, int(max_sweeps), float(tol))
    return values, vectors, info, sweeps


def sq_partials(x: torch.Tensor, reconstructed: torch.Tensor | None = None, scale: float = 0.0) -> torch.Tensor:
    """``[ceil(rows / 8), 3]`` FP64 partials: ``sum (x/s)^2``, ``sum ((x - r)/s)^2``, non-finite flag
    (``scale`` 0: no division)."""
    blocks = -(-int(x.shape[0]) // SQ_ROWS)
    out = torch.empty((blocks, 3), dtype=torch.float64, device=x.device)
    r = reconstructed
    if r is not None and r.dtype != torch.float32:
        r = r.float()
    ext().sq_partials(x, r, float(scale), out)
    return out


def fingerprint_partials(x: torch.Tensor, row_start: int, prime: int) -> torch.Tensor:
    """``[ceil(rows / 8), 6]`` int64 fingerprint partials of a 16- or 32-bit matrix's bit patterns."""
    bits = x.detach().view(torch.int32 if x.element_size() == 4 else torch.int16)
    blocks = -(-int(x.shape[0]) // FP_ROWS)
    out = torch.empty((blocks, 6), dtype=torch.int64, device=x.device)
    ext().fingerprint_partials(bits, out, int(row_start), int(prime))
    return out


def dot2_gemm(x: torch.Tensor, rows: torch.Tensor) -> torch.Tensor:
    """``x @ rows.T`` (FP32) with compensated (Dot2) accumulation, deterministic."""
    x32 = x.float()
    r32 = rows.float()
    x32 = x32 if x32.stride(1) == 1 else x32.contiguous()
    r32 = r32 if r32.stride(1) == 1 else r32.contiguous()
    out = torch.empty((x32.shape[0], r32.shape[0]), dtype=torch.float32, device=x.device)
    ext().dot2_gemm(x32, r32, out)
    return out
