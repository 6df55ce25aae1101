"""Deterministic factorization in the canonical channel domain (the counterpart of reference
reelcache/factorization.py: ``DetectorSpec`` :74, ``project_onto_basis`` :318, ``fit_basis`` :445-562,
``fit_rank_directions`` :728, ``acquire_anchor_directions`` :925).

* :func:`fit_basis` fits an ordered basis of a matrix ``X[N, C]``, rounds it to FP16 once and projects on
  those stored bytes. Backends: ``exact`` (FP64 SVD), ``randomized`` (seeded range finder with a private
  generator + reduced SVD), ``gram`` (FP32-accurate Gram + batched eigensolver: the sm_100a Jacobi kernel
  for C <= 160, cuSOLVER beyond), ``torch_lowrank`` and the cuSOLVER SVD drivers ``gesvd``/``gesvdj``/
  ``gesvda`` (CUDA only, measured baselines). ``auto`` picks ``exact`` for small problems, else
  ``randomized``.
* :func:`project_onto_basis` computes ``P = X Q^T`` with the stored FP16 rows promoted to FP32 and a tiled
  *direct* residual ``||X - P Q||`` accumulated in FP64 (fused square-sum kernel on CUDA), with a
  condition bound of the stored rows.
* :func:`fit_rank_directions` / :func:`acquire_anchor_directions` give energy-ordered candidate directions
  and the fixed anchor detector (width doubling until the captured energy reaches ``stop_energy``).
"""

from __future__ import annotations

import hashlib
import math
import platform
import time
from dataclasses import asdict, dataclass, field
from typing import Any, Mapping

import torch

from . import exact_blas
from .errors import ConfigurationError, UnsupportedError
from .types import TensorContext, canonical_digest

GPU_METHODS = ("gesvd", "gesvdj", "gesvda", "torch_lowrank", "gram")
METHODS = ("auto", "exact", "randomized") + GPU_METHODS
EXACT_LIMIT = 256


# ---------------------------------------------------------------------------------------------------------
# detector recipe
# ---------------------------------------------------------------------------------------------------------

def _backend_fingerprint() -> str:
    return canonical_digest({"torch": str(torch.__version__), "cuda": str(torch.version.cuda),
                             "machine": platform.machine()})


@dataclass(frozen=True)
class DetectorSpec:
    """The fixed anchor-acquisition recipe (solver, widths, seeds, energies) with its identity."""

    solver: str = "qr_q2"
    device: str = "cpu"
    compute_dtype: str = "float32"
    norm_recipe: str = "scaled_original_fp64"
    power_iterations: int = 2
    initial_width: int = 128
    width_growth: int = 2
    width_cap: str = "min_rows_channels"
    energy_denominator: str = "full_original_frobenius_norm"
    stop_energy: float = 0.99
    feature_energies: tuple[float, ...] = (0.95, 0.99)
    base_seed: int = 0
    seed_recipe: str = "sha256_geometry_key_position_plus_attempt_v1"
    tile_rows: int = 1024
    cpu_threads: int = 1
    backend_fingerprint: str = field(default_factory=_backend_fingerprint)
    schema_version: str = "reelcache.fixed_anchor_detector.v1"

    def __post_init__(self) -> None:
        if self.solver != "qr_q2" or self.compute_dtype != "float32":
            raise ConfigurationError("the anchor detector is the FP32 QR subspace iteration (qr_q2)")
        if self.device not in ("cpu", "cuda"):
            raise ConfigurationError("detector device must be cpu or cuda")
        if not 0 <= self.power_iterations <= 8 or self.initial_width < 1 or self.width_growth < 2:
            raise ConfigurationError("invalid detector iteration count or widths")
        if not 0.0 < self.stop_energy < 1.0 or any(not 0.0 < e < 1.0 for e in self.feature_energies):
            raise ConfigurationError("detector energies must lie in (0, 1)")
        object.__setattr__(self, "feature_energies", tuple(float(e) for e in self.feature_energies))
        if self.tile_rows < 1 or self.cpu_threads < 1:
            raise ConfigurationError("tile_rows and cpu_threads must be positive")

    def fingerprint(self) -> str:
        return canonical_digest(self.to_dict())

    def to_dict(self) -> dict[str, Any]:
        data = asdict(self)
        data["feature_energies"] = list(self.feature_energies)
        return data

    @classmethod
    def from_dict(cls, value: Mapping[str, Any]) -> "DetectorSpec":
        data = dict(value)
        data["feature_energies"] = tuple(data.get("feature_energies", (0.95, 0.99)))
        return cls(**data)

    def validate_runtime(self) -> None:
        if self.backend_fingerprint != _backend_fingerprint():
            raise ConfigurationError("the anchor detector was recorded on another torch/CUDA build")

    def seed_for(self, context: TensorContext, attempt: int = 0) -> int:
        digest = hashlib.sha256(canonical_digest({
            "base": self.base_seed, "key": context.key.to_dict(), "token_start": context.token_start,
            "geometry": [context.frames, context.height, context.width], "attempt": attempt}).encode()).hexdigest()
        return int(digest[:15], 16)


# ---------------------------------------------------------------------------------------------------------
# results
# ---------------------------------------------------------------------------------------------------------

@dataclass
class Projection:
    coefficients: torch.Tensor
    relative_residual: float
    source_norm: float
    residual_norm: float
    zero_input: bool
    condition_bound: float
    seconds: float
    coefficient_seconds: float = 0.0
    guard_seconds: float = 0.0
    condition_seconds: float = 0.0


@dataclass(frozen=True)
class Factors:
    basis: torch.Tensor            # [rank, C] FP16 stored rows
    coefficients: torch.Tensor     # [N, rank] FP32
    rank: int
    metrics: dict[str, Any] = field(default_factory=dict)


class RankFitError(ConfigurationError):
    def __init__(self, message: str, metrics: Mapping[str, Any]):
        super().__init__(message)
        self.metrics = dict(metrics)


class RankProjectionError(ConfigurationError):
    def __init__(self, message: str, metrics: Mapping[str, Any]):
        super().__init__(message)
        self.metrics = dict(metrics)

    def __reduce__(self):
        return (type(self), (str(self), self.metrics))


class DetectorAcquisitionError(ConfigurationError):
    def __init__(self, message: str, metrics: Mapping[str, Any]):
        super().__init__(message)
        self.metrics = dict(metrics)

    def __reduce__(self):
        return (type(self), (str(self), self.metrics))


# ---------------------------------------------------------------------------------------------------------
# validation
# ---------------------------------------------------------------------------------------------------------

def tensor_sha256(tensor: torch.Tensor, *, tile_rows: int = 1024) -> str:
    """SHA-256 of a matrix's dtype, shape and row-major bytes (read in row tiles)."""
    value = tensor.detach()
    digest = hashlib.sha256(f"{str(value.dtype).removeprefix('torch.')}:{list(value.shape)}".encode())
    for start in range(0, value.shape[0], tile_rows):
        tile = value[start:start + tile_rows].contiguous().cpu()
        digest.update(tile.view(torch.uint8).reshape(-1).numpy().tobytes())
    return digest.hexdigest()


def validate_matrix(tensor: torch.Tensor, context: TensorContext | None = None, *, lossy: bool = False,
                    check_values: bool = True) -> torch.Tensor:
    """A nonempty floating 2-D matrix of the context's geometry (finite unless ``check_values`` is off)."""
    if not isinstance(tensor, torch.Tensor) or tensor.ndim != 2 or min(tensor.shape) < 1:
        raise ConfigurationError("factorization needs a nonempty 2-D matrix")
    if not tensor.is_floating_point():
        raise ConfigurationError("factorization needs a floating-point matrix")
    if context is not None and tuple(tensor.shape) != (context.token_count, context.channels):
        raise ConfigurationError(f"matrix shape {tuple(tensor.shape)} differs from its context "
                                 f"({context.token_count}, {context.channels})")
    if check_values and not bool(torch.isfinite(tensor).all()):
        raise ConfigurationError("factorization needs finite values")
    return tensor


def validate_rank(rank: int, shape: tuple[int, int]) -> int:
    if type(rank) is not int or not 1 <= rank <= min(shape):
        raise ConfigurationError(f"rank must be an integer in [1, {min(shape)}]")
    return rank


def validate_stored_basis(basis: torch.Tensor, channels: int) -> torch.Tensor:
    if not isinstance(basis, torch.Tensor) or basis.ndim != 2 or basis.shape[1] != channels or basis.shape[0] < 1:
        raise ConfigurationError("a stored basis is a nonempty [rank, channels] matrix")
    if basis.dtype != torch.float16:
        raise ConfigurationError("a stored basis is FP16")
    if not bool(torch.isfinite(basis).all()):
        raise ConfigurationError("stored basis is not finite")
    return basis


# ---------------------------------------------------------------------------------------------------------
# condition bounds and projection
# ---------------------------------------------------------------------------------------------------------

def basis_condition_bound(basis: torch.Tensor) -> float:
    """2-norm condition number of the stored rows (FP64 Gram eigenvalues)."""
    q = basis.double()
    values = torch.linalg.eigvalsh(q @ q.t())
    low, high = float(values[0]), float(values[-1])
    return math.inf if low <= 0 else math.sqrt(high / low)


def fast_condition_bound(basis: torch.Tensor) -> float:
    """Upper bound of the condition number from the Gershgorin radius of ``Q Q^T - I`` (FP32-accurate
    products): ``sqrt((1 + eta) / (1 - eta))``, infinite when ``eta >= 1``."""
    q = basis.float()
    delta = exact_blas.mm(q, q.t())
    delta.diagonal().sub_(1.0)
    eta = float(delta.abs().sum(1).max())
    return math.inf if not math.isfinite(eta) or eta >= 1.0 else math.sqrt((1.0 + eta) / (1.0 - eta))


def _sumsq(x: torch.Tensor, r: torch.Tensor | None = None) -> tuple[float, float]:
    """(sum x^2, sum (x - r)^2) accumulated in FP64 (fused kernel on CUDA)."""
    if x.is_cuda:
        from .ops import _ext
        if _ext.available():
            from .ops.fitter import sq_partials
            totals = sq_partials(x, r).sum(0)
            return float(totals[0]), float(totals[1])
    xf = x.double()
    source = float(xf.square().sum())
    residual = float((xf - r.double()).square().sum()) if r is not None else 0.0
    return source, residual


def project_onto_basis(tensor: torch.Tensor, basis: torch.Tensor, *, rank: int | None = None, tile_rows: int = 1024,
                       max_condition: float = 1e6, _condition_bound: float | None = None) -> Projection:
    """Project once on the stored FP16 rows and measure a tiled direct residual (FP64 sums)."""
    started = time.perf_counter()
    validate_matrix(tensor)
    stored = validate_stored_basis(basis, tensor.shape[1])
    if rank is not None:
        stored = stored[:validate_rank(rank, (stored.shape[0], stored.shape[1]))]
    guard = time.perf_counter()
    bound = fast_condition_bound(stored) if _condition_bound is None else float(_condition_bound)
    condition_seconds = time.perf_counter() - guard
    if bound > max_condition:
        raise RankProjectionError("stored basis is too ill-conditioned to project on",
                                  {"condition_bound": bound, "max_condition": max_condition})
    q = stored.to(tensor.device).float()
    coefficients = torch.empty((tensor.shape[0], q.shape[0]), dtype=torch.float32, device=tensor.device)
    source = residual = 0.0
    coefficient_seconds = 0.0
    for start in range(0, tensor.shape[0], tile_rows):
        a = tensor[start:start + tile_rows]
        t0 = time.perf_counter()
        p = exact_blas.mm(a, q.t())
        coefficients[start:start + a.shape[0]] = p
        coefficient_seconds += time.perf_counter() - t0
        s, r = _sumsq(a, exact_blas.mm(p, q))
        source += s
        residual += r
    zero = source == 0.0
    return Projection(coefficients, 0.0 if zero else math.sqrt(residual / source), math.sqrt(source),
                      math.sqrt(residual), zero, bound, time.perf_counter() - started, coefficient_seconds,
                      0.0, condition_seconds)


def _canonical_signs(basis: torch.Tensor) -> torch.Tensor:
    """Rows flipped so each row's largest-magnitude entry is positive."""
    index = basis.abs().argmax(dim=1, keepdim=True)
    signs = torch.sign(torch.gather(basis, 1, index))
    signs[signs == 0] = 1
    return basis * signs


# ---------------------------------------------------------------------------------------------------------
# fitting
# ---------------------------------------------------------------------------------------------------------

def _private_generator(seed: int, device) -> torch.Generator:
    gen = torch.Generator(device=device)
    gen.manual_seed(int(seed))
    return gen


def _randomized_rows(x: torch.Tensor, rank: int, seed: int, power_iterations: int) -> torch.Tensor:
    """Top ``rank`` right singular rows by a seeded range finder (FP32-accurate products) + reduced SVD."""
    n, c = x.shape
    width = min(c, n, rank + max(8, rank // 4))
    gen = _private_generator(seed, x.device if x.is_cuda else "cpu")
    omega = torch.randn((c, width), generator=gen, device=x.device, dtype=torch.float32)
    y = exact_blas.cholesky_qr2(exact_blas.mm(x, omega))
    for _ in range(power_iterations):
        z = exact_blas.cholesky_qr2(exact_blas.mm(x.t(), y))
        y = exact_blas.cholesky_qr2(exact_blas.mm(x, z))
    b = exact_blas.mm(y.t(), x)                       # [width, C]
    _, _, vh = torch.linalg.svd(b.double(), full_matrices=False)
    return vh[:rank].float()


def _gram_rows(x: torch.Tensor, rank: int) -> torch.Tensor:
    from .gpu_fitting import gram_bases
    (rows,) = gram_bases([x.float()], [rank])
    return rows


def fit_basis(tensor: torch.Tensor, context: TensorContext | None, rank: int, *, method: str = "auto",
              seed: int = 0, power_iterations: int = 2) -> Factors:
    """Fit an ordered basis, round it once to FP16, then project on those bytes."""
    started = time.perf_counter()
    value = validate_matrix(tensor, context)
    validate_rank(rank, tuple(value.shape))
    if method not in METHODS:
        raise ConfigurationError(f"unsupported factorization method {method!r}")
    if method in GPU_METHODS and method != "gram" and value.device.type != "cuda":
        raise UnsupportedError(f"the {method} backend requires CUDA input")
    if type(seed) is not int or not 0 <= seed < 2 ** 63:
        raise ConfigurationError("seed must be a nonnegative 63-bit integer")
    chosen = method
    if method == "auto":
        chosen = "exact" if min(value.shape) <= EXACT_LIMIT or 2 * rank >= min(value.shape) else "randomized"
    x = value.float()
    decomposition = time.perf_counter()
    if chosen == "exact":
        _, _, vh = torch.linalg.svd(x.double(), full_matrices=False)
        rows = vh[:rank].float()
    elif chosen == "randomized":
        rows = _randomized_rows(x, rank, seed, power_iterations)
    elif chosen == "gram":
        rows = _gram_rows(x, rank)
    elif chosen == "torch_lowrank":
        gen_state = torch.random.get_rng_state()
        try:
            torch.manual_seed(seed)
            _, _, v = torch.svd_lowrank(x, q=min(min(x.shape), rank + 8), niter=power_iterations)
        finally:
            torch.random.set_rng_state(gen_state)
        rows = v[:, :rank].t()
    else:
        _, _, vh = torch.linalg.svd(x, full_matrices=False, driver=chosen)
        rows = vh[:rank]
    decomposition_seconds = time.perf_counter() - decomposition
    basis = _canonical_signs(rows).to(torch.float16).contiguous()
    if not bool(torch.isfinite(basis).all()):
        raise ConfigurationError("fitted basis is not finite in stored FP16")
    projection = project_onto_basis(value, basis)
    return Factors(basis, projection.coefficients, rank, {
        "factorization_method": chosen, "factorization_seed": seed,
        "power_iterations": power_iterations if chosen == "randomized" else 0,
        "decomposition_seconds": decomposition_seconds, "projection_seconds": projection.seconds,
        "projection_relative_residual": projection.relative_residual,
        "basis_condition_bound": projection.condition_bound, "zero_input": projection.zero_input,
        "fit_seconds": time.perf_counter() - started})


# ---------------------------------------------------------------------------------------------------------
# energies and candidate directions
# ---------------------------------------------------------------------------------------------------------

@dataclass(frozen=True)
class SourceEnergy:
    total: float                 # sum of squares (FP64)
    finite: bool
    seconds: float


def measure_source_energy(tensor: torch.Tensor, *, tile_rows: int = 4096) -> SourceEnergy:
    started = time.perf_counter()
    total = 0.0
    finite = True
    for start in range(0, tensor.shape[0], tile_rows):
        tile = tensor[start:start + tile_rows]
        if tile.is_cuda:
            from .ops import _ext
            if _ext.available():
                from .ops.fitter import sq_partials
                sums = sq_partials(tile).sum(0)
                total += float(sums[0])
                finite = finite and float(sums[2]) == 0.0
                continue
        finite = finite and bool(torch.isfinite(tile).all())
        total += float(tile.double().square().sum())
    return SourceEnergy(total, finite, time.perf_counter() - started)


@dataclass
class DirectionFit:
    directions: torch.Tensor      # [C, k] FP32 column-orthonormal, energy ordered
    energies: torch.Tensor        # [k] FP64 captured energies per direction (descending)
    source_energy: float
    exact: bool = False

    def __post_init__(self) -> None:
        if self.directions.shape[1] != self.energies.shape[0]:
            raise ConfigurationError("one energy per direction")

    @property
    def width(self) -> int:
        return int(self.directions.shape[1])

    def required_rank(self, energy_target: float) -> int | None:
        """Smallest prefix capturing ``energy_target`` of the source energy (None: the width does not)."""
        if self.source_energy <= 0:
            return 1
        cumulative = torch.cumsum(self.energies.double(), 0) / self.source_energy
        hits = torch.nonzero(cumulative >= energy_target)
        return int(hits[0]) + 1 if hits.numel() else None

    def energy_fraction(self, rank: int) -> float:
        if self.source_energy <= 0:
            return 1.0
        return float(self.energies[:rank].double().sum()) / self.source_energy


def rank_fit_workspace_bytes(rows: int, channels: int, width: int) -> int:
    """Device bytes of :func:`fit_rank_directions` (Gram, sketch, split operands)."""
    return 4 * channels * channels + 16 * channels * width + 24 * rows * channels


def rank_projection_workspace_bytes(rows: int, channels: int, rank: int, tile_rows: int = 1024) -> int:
    return 4 * rows * rank + 8 * min(rows, tile_rows) * channels + 4 * rank * channels


def fit_rank_directions(tensor: torch.Tensor, width: int, *, seed: int = 0, power_iterations: int = 2,
                        solver: str = "topk_rr", steps: int = 3) -> DirectionFit:
    """Energy-ordered candidate directions of ``X``: full Gram eigendecomposition (``gram_eigh``) or a seeded
    block subspace iteration of the Gram refined by one Rayleigh-Ritz solve (``topk_rr``)."""
    from .gpu_fitting import rows_eigh
    x = validate_matrix(tensor).float()
    channels = x.shape[1]
    width = max(1, min(int(width), channels))
    g = exact_blas.gram(x)
    total = float(torch.diagonal(g).double().sum())
    if solver == "gram_eigh" or 2 * width > channels:
        values, rows = rows_eigh(g.unsqueeze(0))
        values, rows = values[0].flip(0), rows[0].flip(0)
        directions = rows[:width].t().contiguous()
        return DirectionFit(directions, values[:width].double().clamp_min(0), total, exact=True)
    if solver != "topk_rr":
        raise ConfigurationError("solver must be gram_eigh or topk_rr")
    gen = _private_generator(seed, "cpu")
    b = torch.randn((channels, width), generator=gen, dtype=torch.float32).to(x.device)
    b = exact_blas.cholesky_qr2(exact_blas.mm(g, b))
    for _ in range(max(steps, power_iterations)):
        b = exact_blas.cholesky_qr2(exact_blas.mm(g, b))
    t = exact_blas.mm(b.t(), exact_blas.mm(g, b))
    t = 0.5 * (t + t.t())
    values, rows = rows_eigh(t.unsqueeze(0))
    values, rows = values[0].flip(0), rows[0].flip(0)
    directions = exact_blas.mm(b, rows.t().contiguous())
    return DirectionFit(exact_blas.cholesky_qr2(directions), values.double().clamp_min(0), total)


def project_rank_directions(tensor: torch.Tensor, directions: torch.Tensor, rank: int) -> Projection:
    """Projection of ``X`` on the FP16 rounding of the first ``rank`` directions."""
    rows = directions[:, :rank].t().contiguous().to(torch.float16)
    return project_onto_basis(tensor, rows)


@dataclass
class AnchorAcquisition:
    spec: DetectorSpec
    fit: DirectionFit
    width: int
    attempts: int
    status: str                      # "reached" | "capped"
    feature_ranks: dict = field(default_factory=dict)

    def __post_init__(self) -> None:
        if self.status not in ("reached", "capped"):
            raise ConfigurationError("anchor status is reached or capped")

    @property
    def directions(self) -> torch.Tensor:
        return self.fit.directions

    def rank_at(self, tau: float) -> int | None:
        return self.fit.required_rank(tau)

    def to_dict(self) -> dict[str, Any]:
        return {"detector": self.spec.fingerprint(), "width": self.width, "attempts": self.attempts,
                "status": self.status, "feature_ranks": {f"{k:.4f}": v for k, v in self.feature_ranks.items()},
                "captured_energy": self.fit.energy_fraction(self.width)}


def acquire_anchor_directions(tensor: torch.Tensor, context: TensorContext, spec: DetectorSpec | None = None, *,
                              max_bytes: int | None = None) -> AnchorAcquisition:
    """The fixed anchor detector: subspace iteration at ``initial_width``, growing by ``width_growth`` until
    the captured energy reaches ``stop_energy`` or the width hits ``min(rows, channels)``."""
    spec = spec or DetectorSpec()
    x = validate_matrix(tensor, context)
    cap = min(x.shape)
    width = min(spec.initial_width, cap)
    attempt = 0
    while True:
        if max_bytes is not None and rank_fit_workspace_bytes(x.shape[0], x.shape[1], width) > max_bytes:
            raise DetectorAcquisitionError("anchor acquisition exceeds its workspace budget",
                                           {"width": width, "max_bytes": max_bytes})
        fit = fit_rank_directions(x, width, seed=spec.seed_for(context, attempt),
                                  power_iterations=spec.power_iterations, steps=spec.power_iterations)
        attempt += 1
        if fit.energy_fraction(width) >= spec.stop_energy or width >= cap:
            status = "reached" if fit.energy_fraction(width) >= spec.stop_energy else "capped"
            ranks = {tau: fit.required_rank(tau) for tau in spec.feature_energies}
            return AnchorAcquisition(spec, fit, width, attempt, status, ranks)
        width = min(cap, width * spec.width_growth)


__all__ = ["AnchorAcquisition", "DetectorAcquisitionError", "DetectorSpec", "DirectionFit", "Factors",
           "Projection", "RankFitError", "RankProjectionError", "SourceEnergy", "acquire_anchor_directions",
           "basis_condition_bound", "fast_condition_bound", "fit_basis", "fit_rank_directions",
           "measure_source_energy", "project_onto_basis", "project_rank_directions", "rank_fit_workspace_bytes",
           "rank_projection_workspace_bytes", "tensor_sha256", "validate_matrix", "validate_rank",
           "validate_stored_basis"]
