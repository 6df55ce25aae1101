"""First-parent basis reuse with a projection gate (the counterpart of reference reelcache/reuse.py:48
``try_reuse_basis`` and :106 ``factorize_tensor``).

A child matrix may reuse its parent's stored basis when projecting on those FP16 rows keeps at least the
reuse threshold of the energy: ``1 - rel_residual^2 >= threshold``. The gate is conservative: the measured
captured energy must clear the threshold by an FP32 band (``REUSE_BAND``) so rounding can never flip an
acceptance. Rejections record their reason; :func:`factorize_tensor` falls back to a fresh fit.
"""

from __future__ import annotations

import math
import time
from dataclasses import dataclass

import torch

from .errors import ConfigurationError
from .factorization import (Factors, Projection, RankProjectionError, fit_basis, project_onto_basis,
                            validate_matrix, validate_rank)
from .types import TensorContext

REUSE_BAND = 1e-6


@dataclass(frozen=True)
class ReuseDecision:
    accepted: bool
    reason: str
    projection: Projection | None
    captured_energy: float | None
    seconds: float


def validate_threshold(threshold: float) -> float:
    if isinstance(threshold, bool) or not isinstance(threshold, (int, float)):
        raise ConfigurationError("reuse threshold must be a number")
    threshold = float(threshold)
    if not math.isfinite(threshold) or not 0.0 < threshold < 1.0:
        raise ConfigurationError("reuse threshold must lie in (0, 1)")
    return threshold


def try_reuse_basis(tensor: torch.Tensor, context: TensorContext | None, basis: torch.Tensor, threshold: float, *,
                    rank: int | None = None, max_condition: float = 1e6) -> ReuseDecision:
    """Project on the parent's stored rows and accept iff the captured energy clears the threshold."""
    started = time.perf_counter()
    threshold = validate_threshold(threshold)
    validate_matrix(tensor, context)

    def reject(reason: str, projection: Projection | None = None, captured: float | None = None) -> ReuseDecision:
        return ReuseDecision(False, reason, projection, captured, time.perf_counter() - started)

    if basis is None:
        return reject("no_parent_basis")
    if basis.ndim != 2 or basis.shape[1] != tensor.shape[1]:
        return reject("channel_mismatch")
    try:
        projection = project_onto_basis(tensor, basis.to(tensor.device), rank=rank, max_condition=max_condition)
    except RankProjectionError:
        return reject("ill_conditioned")
    if projection.zero_input:
        return ReuseDecision(True, "zero_input", projection, 1.0, time.perf_counter() - started)
    captured = 1.0 - projection.relative_residual ** 2
    if captured < threshold + REUSE_BAND:
        return reject("below_threshold", projection, captured)
    return ReuseDecision(True, "accepted", projection, captured, time.perf_counter() - started)


def factorize_tensor(tensor: torch.Tensor, context: TensorContext | None, rank: int, *,
                     reuse_basis: torch.Tensor | None = None, reuse_threshold: float | None = None,
                     method: str = "auto", seed: int = 0, power_iterations: int = 2) -> Factors:
    """Reuse the parent's basis when the gate accepts it, else fit a fresh one; metrics record the path."""
    started = time.perf_counter()
    validate_rank(rank, tuple(tensor.shape))
    attempts = 0
    reason = "no_reuse_requested"
    if reuse_basis is not None and reuse_threshold is not None:
        attempts = 1
        decision = try_reuse_basis(tensor, context, reuse_basis, reuse_threshold)
        reason = decision.reason
        if decision.accepted:
            projection = decision.projection
            return Factors(reuse_basis, projection.coefficients, int(reuse_basis.shape[0]), {
                "reuse_attempts": 1, "reuse_accepted": True, "reuse_reason": reason,
                "reuse_seconds": decision.seconds, "reuse_captured_energy": decision.captured_energy,
                "projection_relative_residual": projection.relative_residual,
                "total_factorization_seconds": time.perf_counter() - started})
    factors = fit_basis(tensor, context, rank, method=method, seed=seed, power_iterations=power_iterations)
    metrics = {**factors.metrics, "reuse_attempts": attempts, "reuse_accepted": False, "reuse_reason": reason,
               "reuse_rejections": attempts, "total_factorization_seconds": time.perf_counter() - started}
    return Factors(factors.basis, factors.coefficients, factors.rank, metrics)


__all__ = ["REUSE_BAND", "ReuseDecision", "factorize_tensor", "try_reuse_basis", "validate_threshold"]
