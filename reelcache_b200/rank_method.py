"""Energy-targeted rank selection, verification and basis reuse (the paper's Algorithm 1; reference:
reelcache/rank_method.py:1-56 for the method, :130-320 for its configuration).

Conventions: canonical matrices ``A[N, C]``; stored row bases ``Q[r, C]`` in FP16; coefficients
``P = A.float() @ Q.float().T`` in FP32; reconstruction ``P @ Q``. Per matrix and energy target ``E_t``:

* **Anchor and prediction.** An ``m``-direction sketch ``S`` (QR-stabilized subspace iteration of the
  Gram matrix, ``q`` power iterations, private generator) gives ``E_m = ||A S||^2 / ||A||^2``. If
  ``E_m >= E_t`` the first bucket is predicted; otherwise ``x = ln((1 - E_m) / (1 - E_t))`` and
  ``r_hat = exp(a + b x)`` from the pinned learner of the regime (fresh or residual).
* **Fit, verify, grow, trim.** Candidate directions come from the Gram matrix (``gram_eigh``: full
  eigendecomposition; ``topk_rr``: predicted bucket + margin directions refined by a few Gram
  products and one small Rayleigh-Ritz solve). The predicted bucket is verified on the actual stored
  representation (FP16 rows, FP32 coefficients, direct residual); a short bucket grows one bucket at a
  time, an over-wide one is trimmed to the smallest bucket whose stored representation verifies.
* **Inherit, certify, augment, refit.** With an active basis the chunk is projected on the stored
  rows; ``e = 1 - ||R||^2 / ||A||^2``. If ``e >= E_t`` the shortest bucket-aligned prefix that verifies
  is shared. Otherwise the residual is fitted at ``(E_t - e) / (1 - e)``, re-orthogonalized against the
  inherited span and verified on ``A``. The refit rule (``paper``: refit iff the augmented chunk is
  estimated to store more bytes than a fresh fit; ``cumulative``: ski-rental debt) may start a new group.

Energies are accumulated in FP64 (fused square-sum kernel on CUDA). The Gram products of bf16 sources run on
the sm_100a tcgen05 GEMM (bf16 products are exact, FP32 accumulation); every other product is FP32-accurate
(:func:`reelcache_b200.exact_blas.mm`: split-bf16 tcgen05 GEMM on CUDA), and the Rayleigh-Ritz eigenproblems
run on the batched Jacobi kernel (FP64 LAPACK on the host).
"""

from __future__ import annotations

import contextlib
import threading

import math
import time
from dataclasses import dataclass, field, replace
from typing import Any, Mapping

import numpy as np
import torch

from . import exact_blas
from .errors import ConfigurationError
from .predictor_registry import RegistryView
from .types import (RANK_BUCKET, ActiveBasisBinding, CodecSpec, EnergyReport, EnergyTargets, FitObservation,
                    MatrixKey, PredictorKey, TensorContext, canonical_digest)

METHOD_SCHEMA = "reelcache.rank_method.v1"
SOLVERS = ("gram_eigh", "topk_rr")
REFIT_RULES = ("cumulative", "paper")
DECISIONS = ("fresh", "share", "augment", "refit", "zero_input", "diagnostic_full_width")
MATMUL_PRECISIONS = ("fp32", "fp32_verified_fp64")
ORTHOGONALIZERS = ("batched", "householder")
FIXED_BASES = ("fitted", "identity")


@dataclass(frozen=True)
class RankMethodConfig:
    """Versioned configuration of the rank method (paper defaults m = 32, q = 2)."""

    targets: EnergyTargets
    codec: CodecSpec
    anchor_rank: int = RANK_BUCKET
    bucket: int = RANK_BUCKET
    power_iterations: int = 2
    tile_rows: int = 1024
    seed: int = 0
    reuse: bool = True
    refit: bool = True
    solver: str = "topk_rr"
    decision_band: float = 1e-6
    trim_slack: float = 1e-5
    coefficient_bytes_proxy: float | None = None
    metadata_bytes_estimate: int = 4096
    batch_size: int = 60
    rate_lag: int = 0
    matmul_precision: str = "fp32"
    topk_margin: int = 64
    topk_steps: int = 3
    refit_rule: str = "paper"
    refit_debt_on_share: bool = False
    refit_hysteresis: float = 1.0
    fixed_rank_k: int | None = None
    fixed_rank_v: int | None = None
    fixed_basis: str = "fitted"
    orthogonalizer: str = "batched"

    def __post_init__(self) -> None:
        if not isinstance(self.targets, EnergyTargets):
            raise ConfigurationError("rank method requires explicit EnergyTargets")
        if not isinstance(self.codec, CodecSpec) or self.codec.kind not in ("svd", "svd_hevc"):
            raise ConfigurationError("the rank method encodes svd or svd_hevc coefficient packets")
        if self.solver not in SOLVERS:
            raise ConfigurationError(f"solver must be one of {SOLVERS}")
        if self.refit_rule not in REFIT_RULES:
            raise ConfigurationError(f"refit_rule must be one of {REFIT_RULES}")
        if self.matmul_precision not in MATMUL_PRECISIONS:
            raise ConfigurationError(f"matmul_precision must be one of {MATMUL_PRECISIONS}")
        if self.fixed_basis not in FIXED_BASES:
            raise ConfigurationError(f"fixed_basis must be one of {FIXED_BASES}")
        if self.orthogonalizer not in ORTHOGONALIZERS:
            raise ConfigurationError(f"orthogonalizer must be one of {ORTHOGONALIZERS}")
        for name, low, high in (("anchor_rank", 1, 4096), ("bucket", 1, 4096), ("power_iterations", 0, 8),
                                ("tile_rows", 1, 1 << 20), ("batch_size", 1, 256), ("rate_lag", 0, 8),
                                ("topk_margin", 0, 4096), ("topk_steps", 0, 16)):
            value = getattr(self, name)
            if type(value) is not int or not low <= value <= high:
                raise ConfigurationError(f"{name} must be an integer in [{low}, {high}]")
        if (self.fixed_rank_k is not None or self.fixed_rank_v is not None or self.fixed_basis != "fitted") \
                and self.reuse:
            raise ConfigurationError("fixed-rank and identity arms need reuse=False")

    def fixed_rank(self, target: str) -> int | None:
        return self.fixed_rank_k if target == "K" else self.fixed_rank_v

    def to_dict(self) -> dict[str, Any]:
        data = {"schema": METHOD_SCHEMA, "targets": self.targets.to_dict(), "codec": self.codec.to_dict(),
                "anchor_rank": self.anchor_rank, "bucket": self.bucket, "power_iterations": self.power_iterations,
                "tile_rows": self.tile_rows, "seed": self.seed, "reuse": self.reuse, "refit": self.refit,
                "solver": self.solver, "decision_band": self.decision_band, "trim_slack": self.trim_slack,
                "coefficient_bytes_proxy": self.coefficient_bytes_proxy,
                "metadata_bytes_estimate": self.metadata_bytes_estimate, "matmul_precision": self.matmul_precision,
                "topk_margin": self.topk_margin, "topk_steps": self.topk_steps}
        if self.refit_rule != "paper":
            data.update(refit_rule=self.refit_rule, refit_debt_on_share=self.refit_debt_on_share,
                        refit_hysteresis=self.refit_hysteresis)
        for name in ("fixed_rank_k", "fixed_rank_v"):
            if getattr(self, name) is not None:
                data[name] = getattr(self, name)
        if self.fixed_basis != "fitted":
            data["fixed_basis"] = self.fixed_basis
        if self.orthogonalizer != "batched":
            data["orthogonalizer"] = self.orthogonalizer
        return data

    @property
    def fingerprint(self) -> str:
        return canonical_digest(self.to_dict())


# ---------------------------------------------------------------------------------------------
# Numerics
# ---------------------------------------------------------------------------------------------


def gram(x: torch.Tensor) -> torch.Tensor:
    """FP32 ``X^T X`` of ``x[N, C]``: one tcgen05 bf16 GEMM for bf16 CUDA sources (exact products,
    partials promoted to IEEE FP32 adds every 128 rows), the FP32-accurate split GEMM of :mod:`exact_blas`
    otherwise."""
    if x.is_cuda and x.dtype == torch.bfloat16 and x.shape[0] % 8 == 0:
        from .ops import _ext
        if _ext.available():
            from .ops.fitter import matmul_promoted
            xt = x.t().contiguous()
            g = matmul_promoted(xt, xt)
            return 0.5 * (g + g.t())
    return exact_blas.gram(x)


def _sum_squares(x: torch.Tensor, r: torch.Tensor | None = None) -> torch.Tensor:
    """Device FP64 ``[sum x^2, sum (x - r)^2]`` (the fused square-sum kernel on CUDA)."""
    if x.is_cuda:
        from .ops import _ext
        if _ext.available():
            from .ops.fitter import sq_partials
            return sq_partials(x, r).sum(0)[:2]
    xf = x.double()
    resid = (xf - r.double()).square().sum() if r is not None else torch.zeros((), dtype=torch.float64)
    return torch.stack([xf.square().sum(), resid])


def _jacobi_batch(mats: list[torch.Tensor]) -> list[tuple[torch.Tensor, torch.Tensor]]:
    """One Jacobi launch for a round's Rayleigh-Ritz problems of one size (each matrix is solved by its own
    CTA, so a matrix's eigenpairs do not depend on the batch it rides in). Returns per matrix the FP32
    ascending values, row eigenvectors and the convergence status (0 converged)."""
    from .gpu_fitting import _count
    from .ops.fitter import jacobi_eigh
    values, vectors, info, _ = jacobi_eigh(torch.stack([m.float() for m in mats]))
    _count("jacobi_calls")
    _count("jacobi_matrices", len(mats))
    return [(values[i], vectors[i], info[i]) for i in range(len(mats))]


def _rr_eigh_routine(t: torch.Tensor):
    """Descending eigenvalues (FP64) and column eigenvectors (FP32) of a symmetric ``k x k`` matrix: the
    sm_100a Jacobi kernel on CUDA for k <= 160 (batched with the round's other problems of the same size; an
    unconverged matrix is re-solved by LAPACK / cuSOLVER), FP64 LAPACK/cuSOLVER otherwise."""
    from .deferred_reads import BatchedCall
    from .gpu_fitting import JACOBI_MAX_N
    if t.is_cuda and t.shape[0] <= JACOBI_MAX_N:
        from .ops import _ext
        if _ext.available():
            values, columns, info = yield BatchedCall(("rr_eigh", t.shape[0], t.device), _jacobi_batch, t)
            (status,) = yield (info,)
            if status != 0:
                values, columns = torch.linalg.eigh(t.float())
            return values.flip(0).double(), columns.flip(1).contiguous()
    values, vectors = torch.linalg.eigh(t.double())
    order = torch.argsort(values, descending=True)
    return values[order], vectors[:, order].float()


_ORTHO = threading.local()


@contextlib.contextmanager
def orthogonalizer_scope(name: str):
    """Select the orthogonalizer of the planning calls made on this thread inside the scope."""
    previous = getattr(_ORTHO, "name", "batched")
    _ORTHO.name = name
    try:
        yield
    finally:
        _ORTHO.name = previous


def _orthonormalize_routine(b: torch.Tensor):
    """Column-orthonormal basis of ``b[C, k]``: CholeskyQR2 (``batched``: FP32-accurate tensor-core Grams and
    triangular solves, one host round for both passes' status, Householder only when a Gram is not positive
    definite) or Householder QR in FP32; signs canonical (positive diagonal of R) either way."""
    if getattr(_ORTHO, "name", "batched") == "householder":
        return exact_blas.householder_qr(b)
    return (yield from exact_blas.cholesky_qr2_routine(b))


def _generator(seed: int, key: MatrixKey, salt: str) -> torch.Generator:
    digest = canonical_digest({"seed": seed, "key": key.to_dict(), "salt": salt})
    gen = torch.Generator(device="cpu")
    gen.manual_seed(int(digest[:15], 16))
    return gen


def anchor_sketch_routine(g: torch.Tensor, m: int, q: int, gen: torch.Generator):
    """``orth(G^(q+1) Omega)`` with a private Gaussian ``Omega[C, m]``."""
    channels = g.shape[0]
    omega = torch.randn((channels, min(m, channels)), generator=gen, dtype=torch.float32).to(g.device)
    s = yield from _orthonormalize_routine(exact_blas.mm(g, omega))
    for _ in range(q):
        s = yield from _orthonormalize_routine(exact_blas.mm(g, s))
    return s


def span_energy_routine(g: torch.Tensor, s: torch.Tensor, total: float):
    """``||A S||^2 / ||A||^2 = trace(S^T G S) / trace(G)`` for column-orthonormal ``S``."""
    if total <= 0:
        return 1.0
    (value,) = yield ((exact_blas.mm(g, s) * s).sum(dtype=torch.float64),)
    return value / total


def fp16_rows(directions: torch.Tensor) -> torch.Tensor:
    """FP16 stored rows ``[k, C]`` of FP32 column directions ``[C, k]``."""
    return directions.t().contiguous().to(torch.float16)


def stored_energy_routine(x: torch.Tensor, rows: torch.Tensor, total: float, tile_rows: int = 16384):
    """Energy of the actual stored representation: FP16 ``rows``, FP32 ``P = A Q^T``, direct residual
    ``||A - P Q||^2`` accumulated in FP64 over row tiles. Returns (energy, P)."""
    q = rows.float()
    qt = q.t()
    if x.shape[0] <= tile_rows:  # one tile: the projection is the coefficient matrix itself
        coefficients = exact_blas.mm(x, qt)
        residual = _sum_squares(x, exact_blas.mm(coefficients, q))[1]
    else:
        coefficients = torch.empty((x.shape[0], rows.shape[0]), dtype=torch.float32, device=x.device)
        residual = None
        for start in range(0, x.shape[0], tile_rows):
            a = x[start:start + tile_rows]
            p = exact_blas.mm(a, qt)
            coefficients[start:start + tile_rows] = p
            part = _sum_squares(a, exact_blas.mm(p, q))[1]
            residual = part if residual is None else residual + part
    if total <= 0:
        return 1.0, coefficients
    (value,) = yield (residual,)
    return 1.0 - value / total, coefficients


def prefix_energies_routine(x: torch.Tensor, rows: torch.Tensor, coefficients: torch.Tensor, prefixes, total: float,
                            tile_rows: int = 16384):
    """Stored energies of the row prefixes ``rows[:c]`` (``c`` ascending) in one pass: the coefficients of a prefix
    are the leading columns of ``coefficients = A Q^T``, and its reconstruction grows by one block of rows at a
    time, each prefix's direct residual summed in FP64 -- one host round for every prefix."""
    q = rows.float()
    sums = []
    for start in range(0, x.shape[0], tile_rows):
        a = x[start:start + tile_rows]
        p = coefficients[start:start + tile_rows]
        recon = torch.zeros(a.shape, dtype=torch.float32, device=a.device)
        previous = 0
        for index, c in enumerate(prefixes):
            recon += exact_blas.mm(p[:, previous:c], q[previous:c])
            previous = c
            part = _sum_squares(a, recon)[1]
            sums[index:index + 1] = [part if len(sums) <= index else sums[index] + part]
        del recon
    (values,) = yield (torch.stack(sums),)
    return [1.0 - float(v) / total for v in values]


def _bucketed(rank: float, bucket: int, limit: int) -> int:
    if not math.isfinite(rank):
        return limit
    return int(min(limit, max(bucket, math.ceil(max(rank, 1.0) / bucket) * bucket)))


@dataclass
class Fit:
    directions: torch.Tensor      # [C, k] FP32 column-orthonormal, energy ordered
    energies: torch.Tensor        # [k] FP64 eigen/Ritz values (descending)
    exact: bool                   # True when the directions span the full width


def fit_directions_routine(g: torch.Tensor, wanted: int, cfg: RankMethodConfig, gen: torch.Generator,
                           warm: torch.Tensor | None = None):
    """Energy-ordered candidate directions of a Gram matrix."""
    channels = g.shape[0]
    k = min(channels, wanted + cfg.topk_margin)
    if cfg.solver == "gram_eigh" or k >= channels or 2 * k > channels:
        values, vectors = torch.linalg.eigh(g.double())
        order = torch.argsort(values, descending=True)
        return Fit(vectors[:, order].float(), values[order].clamp_min(0), True)
    start = torch.randn((channels, k), generator=gen, dtype=torch.float32).to(g.device)
    if warm is not None:
        cols = min(k, warm.shape[1])
        start[:, :cols] = warm[:, :cols]
    b = yield from _orthonormalize_routine(exact_blas.mm(g, start))
    for _ in range(cfg.topk_steps):
        b = yield from _orthonormalize_routine(exact_blas.mm(g, b))
    t = exact_blas.mm(b.t(), exact_blas.mm(g, b))
    t = 0.5 * (t + t.t())
    values, vectors = yield from _rr_eigh_routine(t)
    directions = exact_blas.mm(b, vectors)
    directions = yield from _orthonormalize_routine(directions)
    return Fit(directions, values.clamp_min(0), False)


def _sync(routine_factory):
    """The blocking form of a routine (one host read per yield)."""
    from .deferred_reads import run_one

    def call(*args, **kwargs):
        return run_one(routine_factory(*args, **kwargs))
    call.__name__ = routine_factory.__name__.replace("_routine", "")
    call.__doc__ = routine_factory.__doc__
    return call


anchor_sketch = _sync(anchor_sketch_routine)
span_energy = _sync(span_energy_routine)
stored_energy = _sync(stored_energy_routine)
fit_directions = _sync(fit_directions_routine)
_rr_eigh = _sync(_rr_eigh_routine)
_orthonormalize = _sync(_orthonormalize_routine)


# ---------------------------------------------------------------------------------------------
# Plans
# ---------------------------------------------------------------------------------------------


@dataclass
class MatrixPlan:
    """The planner's decision for one matrix (device tensors stay on the planning device)."""

    entry: Any
    context: TensorContext
    decision: str
    rows: torch.Tensor              # full stored view [rank_view, C] FP16 (inherited rows first)
    new_rows: torch.Tensor | None   # rows to store as a new version block (None: shared)
    parent_version: str | None      # version the new block extends (augment) / the shared version
    rank_view: int
    coefficients: torch.Tensor      # FP32 P [N, rank_view]
    energy: EnergyReport
    observation: FitObservation | None
    binding: ActiveBasisBinding     # binding after this chunk (version_ref filled in at store time)
    details: dict = field(default_factory=dict)

    def decision_record(self) -> dict[str, Any]:
        """The content part of the decision (run timings excluded: they never enter content ids)."""
        return {"decision": self.decision, **{k: v for k, v in self.details.items() if k != "planner_seconds"}}


def _predict(view: RegistryView | None, pkey: PredictorKey, anchor: float, target: float, cfg: RankMethodConfig,
             limit: int) -> tuple[int, float | None, float | None, Any]:
    """(predicted bucket, x, predicted rank, use)."""
    if anchor >= target:
        return min(cfg.anchor_rank, limit), None, None, None
    x = math.log((1.0 - anchor) / (1.0 - target))
    if view is None:
        return _bucketed(cfg.anchor_rank, cfg.bucket, limit), x, None, None
    use = view.predict(pkey, x)
    return _bucketed(use.predicted_rank, cfg.bucket, limit), x, use.predicted_rank, use


def _fresh_routine(x: torch.Tensor, g: torch.Tensor, total: float, target: float, cfg: RankMethodConfig,
           view: RegistryView | None, pkey: PredictorKey, key: MatrixKey, *, inherited: torch.Tensor | None = None,
           full_x: torch.Tensor | None = None, full_total: float | None = None, full_target: float | None = None):
    """Fit ``x`` (the matrix, or the residual after inherited rows) to ``target``; when ``inherited``
    is given the combined rows are verified on ``full_x`` at ``full_target``.

    Returns (rows_new [k, C] FP16, energy_report, coefficients, observation_fields, details)."""
    channels = x.shape[1]
    gen = _generator(cfg.seed, key, pkey.regime)
    sketch = yield from anchor_sketch_routine(g, cfg.anchor_rank, cfg.power_iterations, gen)
    anchor = min(max((yield from span_energy_routine(g, sketch, total)), 0.0), 1.0 - 1e-12)
    limit = channels - (0 if inherited is None else inherited.shape[0])
    predicted, xval, predicted_rank, use = _predict(view, pkey, anchor, target, cfg, limit)
    fit = yield from fit_directions_routine(g, predicted, cfg, gen, warm=sketch)
    (cumulative,) = yield (torch.cumsum(fit.energies, 0) / max(total, 1e-300),)   # host FP64 vector
    available = fit.directions.shape[1]
    ideal_rank = int(np.searchsorted(cumulative, target - cfg.decision_band, side="left")) + 1
    ideal_rank = min(ideal_rank, available)
    verify_x = x if inherited is None else full_x
    verify_total = total if inherited is None else full_total
    verify_target = target if inherited is None else full_target

    def rows_at(rank):
        new = fp16_rows(fit.directions[:, :rank])
        if inherited is None:
            return new, new
        return new, torch.cat([inherited, new], 0)

    # smallest bucket reaching the ideal target (Eckart-Young), then grow until the stored rows verify
    rank = min(max(_bucketed(ideal_rank, cfg.bucket, limit), 1), available)
    rank = min(rank, predicted) if cumulative[min(predicted, available) - 1] >= target - cfg.trim_slack else rank
    grown = 0
    while True:
        new, rows = rows_at(rank)
        energy, coefficients = yield from stored_energy_routine(verify_x, rows, verify_total, cfg.tile_rows)
        if energy >= verify_target - cfg.decision_band or rank >= available:
            break
        rank = min(rank + cfg.bucket, available)
        grown += 1
    report = EnergyReport(verify_target, min(float(cumulative[rank - 1]) if inherited is None else energy, 1.0),
                          min(energy, 1.0 + 1e-7), None, ideal_rank, _bucketed(ideal_rank, cfg.bucket, limit),
                          rows.shape[0])
    details = {"anchor_energy": anchor, "predicted_bucket": predicted, "observed_rank": ideal_rank,
               "grown_buckets": grown, "solver": cfg.solver}
    observation = None
    if xval is not None and xval > 0 and target < 1.0 and anchor < target:
        observation = {"anchor_energy": anchor, "target_energy": target, "x": xval, "observed_rank": ideal_rank,
                       "predicted_rank": predicted_rank,
                       "prediction_revision": None if use is None else use.revision}
    return new, report, coefficients, observation, details


def _bytes_estimate(tokens: int, rank: int, new_rows: int, channels: int, cfg: RankMethodConfig,
                    rate: float | None) -> float:
    per_value = rate if rate is not None else (cfg.coefficient_bytes_proxy or 1.0)
    return tokens * rank * per_value + new_rows * channels * 2 + 8 * rank + cfg.metadata_bytes_estimate


def plan_matrix_routine(matrix: torch.Tensor, context: TensorContext, cfg: RankMethodConfig,
                        view: RegistryView | None, binding: ActiveBasisBinding, inherited_rows: torch.Tensor | None, *,
                        entry: Any = None, source_id: str | None = None, chunk_id: str = "chunk",
                        model_fingerprint: str | None = None):
    """Plan one matrix against its lineage's active binding (``inherited_rows``: its stored view). A lockstep
    routine: it yields each group of device values whose host copies its next decision needs."""
    started = time.perf_counter()
    entry = context.key if entry is None else entry
    key = context.key
    x = matrix.reshape(context.token_count, context.channels)
    tokens, channels = x.shape
    target = cfg.targets.for_target(key.target)
    (total,) = yield (_sum_squares(x)[0],)
    fingerprint = model_fingerprint or context.model.fingerprint
    pkey_fresh = PredictorKey(fingerprint, key.layer, key.target, tokens, channels, cfg.solver, "sketch", "fresh")
    pkey_resid = replace(pkey_fresh, regime="residual")
    source_id = source_id or canonical_digest({"chunk": chunk_id, "key": key.to_dict()})

    def observation_of(fields, pkey):
        if fields is None:
            return None
        return FitObservation(pkey, source_id, fields["anchor_energy"], fields["target_energy"], fields["x"],
                              max(1, int(fields["observed_rank"])), fields["predicted_rank"],
                              fields["prediction_revision"])

    if total == 0.0:
        rows = torch.zeros((1, channels), dtype=torch.float16, device=x.device)
        rows[0, 0] = 1.0
        report = EnergyReport(target, 1.0, 1.0, None, 0, 0, 1, zero_input=True)
        return MatrixPlan(entry, context, "zero_input", rows, rows, None, 1,
                          torch.zeros((tokens, 1), dtype=torch.float32, device=x.device), report, None,
                          ActiveBasisBinding(), {"reason": "zero_input"})

    fixed = cfg.fixed_rank(key.target)
    if cfg.fixed_basis == "identity" or fixed is not None:
        if cfg.fixed_basis == "identity":
            rows = torch.eye(channels, dtype=torch.float16, device=x.device)
            reason = "identity_basis"
        else:
            g = gram(x)
            values, vectors = torch.linalg.eigh(g.double())
            order = torch.argsort(values, descending=True)
            rows = fp16_rows(vectors[:, order[:min(fixed, channels)]].float())
            reason = "fixed_rank_policy"
        energy, coefficients = yield from stored_energy_routine(x, rows, total, cfg.tile_rows)
        report = EnergyReport(target, min(energy, 1.0), min(energy, 1.0), None, None, 0, rows.shape[0],
                              diagnostic_full_width=True)
        return MatrixPlan(entry, context, "fresh", rows, rows, None, rows.shape[0], coefficients, report, None,
                          ActiveBasisBinding(), {"reason": reason, "diagnostic": True})

    g = None
    # -------- inherit / certify / augment --------
    if cfg.reuse and inherited_rows is not None and binding.version_ref is not None:
        inherited_rows = inherited_rows.to(x.device)
        energy_all, coefficients_all = yield from stored_energy_routine(x, inherited_rows, total, cfg.tile_rows)
        if energy_all >= target - cfg.decision_band:
            # shortest bucket-aligned prefix that verifies
            rank = inherited_rows.shape[0]
            candidates = list(range(cfg.bucket, rank, cfg.bucket))
            chosen, chosen_energy, chosen_p = rank, energy_all, coefficients_all
            if candidates:
                energies = yield from prefix_energies_routine(x, inherited_rows, coefficients_all, candidates, total,
                                                              cfg.tile_rows)
                for candidate, energy_c in zip(candidates, energies):
                    if energy_c >= target - cfg.decision_band:
                        chosen, chosen_energy = candidate, energy_c
                        chosen_p = coefficients_all[:, :candidate].contiguous()
                        break
            report = EnergyReport(target, min(chosen_energy, 1.0), min(chosen_energy, 1.0), None, None,
                                  _bucketed(chosen, cfg.bucket, channels), chosen)
            return MatrixPlan(entry, context, "share", inherited_rows[:chosen], None, binding.version_ref, chosen,
                              chosen_p, report, None, binding,
                              {"inherited_energy": energy_all, "planner_seconds": time.perf_counter() - started})
        # augment: fit the residual at (E_t - e) / (1 - e)
        q = inherited_rows.float()
        residual = x.float() - exact_blas.mm(coefficients_all, q)
        (r_total,) = yield (_sum_squares(residual)[0],)
        residual_target = min(max((target - energy_all) / max(1.0 - energy_all, 1e-300), 1e-6), 1.0)
        rg = gram(residual)
        new, report, coefficients, fields, details = yield from _fresh_routine(
            residual, rg, r_total, residual_target, cfg, view, pkey_resid, key, inherited=inherited_rows,
            full_x=x, full_total=total, full_target=target)
        # re-orthogonalize the new rows against the inherited span (two Gram-Schmidt passes in FP32)
        w = new.float()
        for _ in range(2):
            w = w - exact_blas.mm(exact_blas.mm(w, q.t()), q)
        w = (yield from _orthonormalize_routine(w.t())).t()
        new = w.to(torch.float16)
        rows = torch.cat([inherited_rows, new], 0)
        energy, coefficients = yield from stored_energy_routine(x, rows, total, cfg.tile_rows)
        report = replace(report, stored_factor_energy=min(energy, 1.0), ideal_subspace_energy=min(energy, 1.0),
                         rank_view=rows.shape[0])
        augment_plan = MatrixPlan(entry, context, "augment", rows, new, binding.version_ref, rows.shape[0],
                                  coefficients, report, observation_of(fields, pkey_resid),
                                  replace(binding, refit_debt=binding.refit_debt if cfg.refit_rule == "cumulative"
                                          else 0.0),
                                  {**details, "inherited_energy": energy_all, "residual_target": residual_target})
        if not cfg.refit or binding.fresh_rank is None:
            augment_plan.details["planner_seconds"] = time.perf_counter() - started
            return augment_plan
        # refit rule
        rate = binding.coefficient_rate
        b_aug = _bytes_estimate(tokens, rows.shape[0], new.shape[0], channels, cfg, rate)
        b_fresh = _bytes_estimate(tokens, binding.fresh_rank, binding.fresh_rank, channels, cfg, rate)
        excess = _bytes_estimate(tokens, rows.shape[0], 0, channels, cfg, rate) - \
            _bytes_estimate(tokens, binding.fresh_rank, 0, channels, cfg, rate)
        cost = binding.fresh_rank * channels * 2
        if cfg.refit_rule == "paper":
            refit = b_aug > b_fresh
        else:
            refit = b_aug > b_fresh or binding.refit_debt + excess >= cfg.refit_hysteresis * cost
        estimate = {"schema": "reelcache.refit_estimate.v1" if cfg.refit_rule == "paper"
                    else "reelcache.refit_estimate.v2", "augmented_bytes": b_aug, "fresh_bytes": b_fresh,
                    "debt_before": binding.refit_debt, "excess": excess, "cost": cost}
        if not refit:
            debt = binding.refit_debt + max(0.0, excess) if cfg.refit_rule == "cumulative" else 0.0
            augment_plan.binding = replace(binding, refit_debt=debt)
            augment_plan.details.update(refit_estimate=estimate, planner_seconds=time.perf_counter() - started)
            return augment_plan
        g = gram(x)
        new, report, coefficients, fields, details = yield from _fresh_routine(x, g, total, target, cfg, view,
                                                                               pkey_fresh, key)
        return MatrixPlan(entry, context, "refit", new, new, None, new.shape[0], coefficients, report,
                          observation_of(fields, pkey_fresh),
                          ActiveBasisBinding(None, 0, None, new.shape[0], chunk_id),
                          {**details, "refit_estimate": estimate, "planner_seconds": time.perf_counter() - started})

    # -------- fresh fit --------
    g = gram(x) if g is None else g
    new, report, coefficients, fields, details = yield from _fresh_routine(x, g, total, target, cfg, view, pkey_fresh,
                                                                           key)
    details["planner_seconds"] = time.perf_counter() - started
    return MatrixPlan(entry, context, "fresh", new, new, None, new.shape[0], coefficients, report,
                      observation_of(fields, pkey_fresh), ActiveBasisBinding(None, 0, None, new.shape[0], chunk_id),
                      details)


plan_matrix = _sync(plan_matrix_routine)


def plan_chunk(matrices: Mapping[Any, torch.Tensor], contexts: Mapping[Any, TensorContext], cfg: RankMethodConfig,
               view: RegistryView | None, bindings: Mapping[Any, ActiveBasisBinding],
               inherited: Mapping[Any, torch.Tensor | None], *, chunk_id: str = "chunk",
               device: Any = None) -> dict[Any, MatrixPlan]:
    """Plan every matrix of a chunk (entries in canonical order), ``cfg.batch_size`` matrices in lockstep: the
    matrices of a group run their decision routines together, so each round of host reads (an energy, a
    factorization status, a cumulative spectrum) is one device-to-host transfer for the whole group, and the
    round's Rayleigh-Ritz problems of one size share one Jacobi launch. Each matrix's kernels, host values and
    decisions are those of planning it alone (``batch_size=1``)."""
    from .deferred_reads import run_lockstep
    entries = sorted(contexts, key=_entry_order)
    plans: dict[Any, MatrixPlan] = {}
    with orthogonalizer_scope(cfg.orthogonalizer):
        for start in range(0, len(entries), cfg.batch_size):
            group = entries[start:start + cfg.batch_size]
            routines, lanes = [], None
            for index, entry in enumerate(group):
                matrix = matrices[entry]
                if device is not None:
                    matrix = matrix.to(device)
                routine = plan_matrix_routine(matrix, contexts[entry], cfg, view,
                                              bindings.get(entry, ActiveBasisBinding()), inherited.get(entry),
                                              entry=entry, chunk_id=chunk_id)
                if matrix.is_cuda and len(group) > 1:
                    lanes = lanes or _stream_lanes(matrix.device, min(PLANNER_STREAMS, len(group)))
                    routine = _on_stream(routine, lanes[index % len(lanes)])
                routines.append(routine)
            for entry, plan in zip(group, run_lockstep(routines)):
                plans[entry] = plan
            if lanes:
                current = torch.cuda.current_stream(lanes[0].device)
                for lane in lanes:
                    current.wait_stream(lane)
    return plans


#: CUDA streams a lockstep group spreads its matrices over: a matrix's planning kernels are small (thin
#: ``C x k`` products, k x k factorizations) and fill a fraction of the SMs, so several matrices run side by side.
PLANNER_STREAMS = 8
_LANES: dict = {}


def _stream_lanes(device: torch.device, count: int) -> list:
    """Side streams of ``device`` (created once per device), each ordered after the current stream's work."""
    lanes = _LANES.setdefault(device, [])
    while len(lanes) < count:
        lanes.append(torch.cuda.Stream(device))
    current = torch.cuda.current_stream(device)
    for lane in lanes[:count]:
        lane.wait_stream(current)
    return lanes[:count]


def _on_stream(routine, stream):
    """Run a routine's device work on ``stream``. Each step first orders the stream after the current one (a
    batched call of the round ran there), and the current stream waits for the step's work before the round's
    host reads and batched calls are issued on it; errors of a batched call are thrown into the routine."""
    current = torch.cuda.current_stream(stream.device)
    send, throw = None, None
    while True:
        stream.wait_stream(current)
        with torch.cuda.stream(stream):
            try:
                request = routine.throw(throw) if throw is not None else routine.send(send)
            except StopIteration as stop:
                return stop.value
        current.wait_stream(stream)
        try:
            send, throw = (yield request), None
        except Exception as error:  # noqa: BLE001 - delivered to the wrapped routine
            send, throw = None, error


def _entry_order(e) -> tuple:
    if isinstance(e, MatrixKey):
        return e.layer, e.target, ""
    return e[0].layer, e[0].target, e[1]
