"""Reference FP64 energy spectra (the counterpart of reference reelcache/spectra.py:
``StreamingGramAccumulator`` :873, ``exact_spectrum`` :1142, ``direct_svd_crosscheck`` :1210).

Measurement only: the uncentered energy spectrum of ``X[N, C]`` from an FP64 Gram accumulated over row tiles
(each tile widened to FP64 before its product, so the Gram is exact up to FP64 rounding), its eigenvalues
by LAPACK ``eigvalsh``, the ranks that reach energy thresholds (with a bracket that accounts for the FP64
rounding budget of the cumulative sums), and an SVD cross-check. The planner never calls this module; it is
the CPU oracle the tests and the rank study compare against.
"""

from __future__ import annotations

import hashlib
import json
import math
import os
from dataclasses import dataclass, field
from typing import Any, Mapping

import torch

from .errors import ConfigurationError, IntegrityError

SCHEMA = "reelcache.spectrum.v1"


class SpectrumNumericalError(IntegrityError):
    def __init__(self, *args: Any, metrics: Mapping[str, Any] | None = None) -> None:
        super().__init__(*args)
        self._metrics = dict(metrics) if metrics is not None else None

    @property
    def metrics(self) -> Mapping[str, Any] | None:
        return self._metrics


@dataclass(frozen=True)
class RankBracket:
    """Rank reaching ``tau`` and its bracket under the FP64 rounding budget of the cumulative energies."""

    tau: float
    rank: int | None
    low: int | None
    high: int | None

    def to_dict(self) -> dict[str, Any]:
        return {"tau": self.tau, "rank": self.rank, "low": self.low, "high": self.high}


def _gamma(count: int) -> float:
    unit = 2.0 ** -53
    return count * unit / (1.0 - count * unit)


def _rank_bracket(values: tuple[float, ...], total: float, tau: float, budget: float) -> RankBracket:
    if not 0.0 < tau <= 1.0:
        raise ConfigurationError("energy thresholds lie in (0, 1]")
    if total <= 0.0:
        return RankBracket(tau, 0, 0, 0)
    target = tau * total
    running = 0.0
    rank = low = high = None
    for index, value in enumerate(values, start=1):
        running += value
        if low is None and running >= target - budget:
            low = index
        if rank is None and running >= target:
            rank = index
        if high is None and running >= target + budget:
            high = index
            break
    return RankBracket(tau, rank, low, high)


@dataclass
class SpectrumResult:
    rows: int
    channels: int
    eigenvalues: tuple[float, ...]        # descending, clamped at 0
    total_energy: float                   # trace of the Gram (= ||X||_F^2 in FP64)
    dc_energy: float                      # energy of the column means (N * ||mean||^2)
    source_sha256: str
    rounding_budget: float = 0.0
    metrics: dict = field(default_factory=dict)

    def __post_init__(self) -> None:
        if len(self.eigenvalues) != self.channels:
            raise ConfigurationError("one eigenvalue per channel")
        if not math.isfinite(self.total_energy) or self.total_energy < 0:
            raise SpectrumNumericalError("spectrum energy is not a finite nonnegative number")

    @property
    def zero_energy(self) -> bool:
        return self.total_energy == 0.0

    @property
    def dc_energy_fraction(self) -> float:
        return 0.0 if self.zero_energy else self.dc_energy / self.total_energy

    def rank_at(self, tau: float) -> RankBracket:
        return _rank_bracket(self.eigenvalues, sum(self.eigenvalues), tau, self.rounding_budget)

    @property
    def r95(self) -> int | None:
        return self.rank_at(0.95).rank

    @property
    def r99(self) -> int | None:
        return self.rank_at(0.99).rank

    def energy(self, rank: int) -> float:
        total = sum(self.eigenvalues)
        return 1.0 if total == 0 else sum(self.eigenvalues[:rank]) / total

    def to_dict(self) -> dict[str, Any]:
        return {"schema": SCHEMA, "rows": self.rows, "channels": self.channels,
                "eigenvalues": list(self.eigenvalues), "total_energy": self.total_energy,
                "dc_energy": self.dc_energy, "source_sha256": self.source_sha256,
                "rounding_budget": self.rounding_budget, "metrics": self.metrics,
                "r95": self.r95, "r99": self.r99}

    @classmethod
    def from_dict(cls, payload: Mapping[str, Any]) -> "SpectrumResult":
        if payload.get("schema") != SCHEMA:
            raise ConfigurationError("not a spectrum record")
        return cls(int(payload["rows"]), int(payload["channels"]), tuple(float(v) for v in payload["eigenvalues"]),
                   float(payload["total_energy"]), float(payload["dc_energy"]), str(payload["source_sha256"]),
                   float(payload.get("rounding_budget", 0.0)), dict(payload.get("metrics", {})))


def write_spectrum_json(result: SpectrumResult, path: str | os.PathLike[str]) -> str:
    """Write the record atomically; returns the SHA-256 of the written bytes."""
    data = json.dumps(result.to_dict(), sort_keys=True, separators=(",", ":"), allow_nan=False).encode()
    tmp = f"{os.fspath(path)}.tmp"
    with open(tmp, "wb") as handle:
        handle.write(data)
        handle.flush()
        os.fsync(handle.fileno())
    os.replace(tmp, path)
    return hashlib.sha256(data).hexdigest()


class StreamingGramAccumulator:
    """FP64 ``X^T X``, column sums and a SHA-256 of the rows, accumulated tile by tile in row order."""

    def __init__(self, channels: int):
        if type(channels) is not int or channels < 1:
            raise ConfigurationError("channels must be a positive integer")
        self.channels = channels
        self.gram = torch.zeros((channels, channels), dtype=torch.float64)
        self.column_sums = torch.zeros(channels, dtype=torch.float64)
        self.rows = 0
        self._hasher = hashlib.sha256()
        self._sealed = False

    def add(self, tile: torch.Tensor) -> None:
        if self._sealed:
            raise ConfigurationError("the accumulator is finalized")
        if tile.ndim != 2 or tile.shape[1] != self.channels or not tile.is_floating_point():
            raise ConfigurationError("tiles are floating [rows, channels] matrices")
        host = tile.detach().cpu().contiguous()
        if not bool(torch.isfinite(host).all()):
            raise SpectrumNumericalError("spectrum source is not finite")
        self._hasher.update(host.view(torch.uint8).reshape(-1).numpy().tobytes())
        x = host.double()
        self.gram += x.t() @ x
        self.column_sums += x.sum(0)
        self.rows += int(x.shape[0])

    def finalize(self) -> SpectrumResult:
        self._sealed = True
        g = 0.5 * (self.gram + self.gram.t())
        values = torch.linalg.eigvalsh(g).flip(0).clamp_min(0.0)
        total = float(torch.diagonal(g).sum())
        mean = self.column_sums / max(1, self.rows)
        dc = float(self.rows * mean.square().sum())
        budget = _gamma(self.rows + self.channels) * total
        return SpectrumResult(self.rows, self.channels, tuple(float(v) for v in values), total, dc,
                              self._hasher.hexdigest(), budget, {"algorithm": "fp64_streaming_gram_eigvalsh"})


@dataclass(frozen=True)
class SpectrumDiagnostics:
    """The numerical health of one spectrum: the Gram's asymmetry before symmetrization, the most negative
    eigenvalue before clamping, the trace against the eigenvalue sum, all relative to the total energy, and the
    FP64 rounding budget the rank brackets use."""

    asymmetry: float
    negative_eigenvalue: float
    trace_residual: float
    rounding_budget: float

    @classmethod
    def of(cls, gram: torch.Tensor, values: torch.Tensor, total: float, budget: float) -> "SpectrumDiagnostics":
        scale = max(total, 1e-300)
        return cls(float((gram - gram.t()).abs().max()) / scale, float(min(0.0, float(values.min()))) / scale,
                   abs(total - float(values.sum())) / scale, budget)

    def to_dict(self) -> dict[str, float]:
        return {"asymmetry": self.asymmetry, "negative_eigenvalue": self.negative_eigenvalue,
                "trace_residual": self.trace_residual, "rounding_budget": self.rounding_budget}


@dataclass
class SpectrumRowShard:
    """One rank's rows of a sequence-parallel matrix, reduced to what its spectrum needs: the rows' FP64 Gram and
    column sums, the first row's index, the row count and the SHA-256 of the rows."""

    rank: int
    row_start: int
    rows: int
    gram: torch.Tensor
    column_sums: torch.Tensor
    sha256: str


def row_shard(tensor: torch.Tensor, *, rank: int, row_start: int, tile_rows: int = 1024) -> SpectrumRowShard:
    """This rank's :class:`SpectrumRowShard` of ``tensor`` (its rows ``[row_start, row_start + rows)``)."""
    accumulator = StreamingGramAccumulator(int(tensor.shape[1]))
    for start in range(0, tensor.shape[0], tile_rows):
        accumulator.add(tensor[start:start + tile_rows])
    return SpectrumRowShard(rank, row_start, accumulator.rows, accumulator.gram, accumulator.column_sums,
                            accumulator._hasher.hexdigest())


def spectrum_from_row_shards(shards) -> SpectrumResult:
    """The spectrum of a matrix whose rows are split over ranks, from every rank's shard: the shards must tile the
    rows without gaps or overlaps; Grams and column sums are summed in row order (deterministic), the source digest
    is the SHA-256 of the shards' digests in row order, and the result carries its diagnostics."""
    shards = sorted(shards, key=lambda shard: shard.row_start)
    if not shards:
        raise ConfigurationError("a spectrum needs at least one row shard")
    channels = int(shards[0].gram.shape[0])
    cursor = 0
    gram = torch.zeros((channels, channels), dtype=torch.float64)
    sums = torch.zeros(channels, dtype=torch.float64)
    digest = hashlib.sha256()
    for shard in shards:
        if shard.row_start != cursor or shard.gram.shape != (channels, channels):
            raise ConfigurationError("row shards must tile the matrix rows in order, with one channel count")
        cursor += shard.rows
        gram += shard.gram.double()
        sums += shard.column_sums.double()
        digest.update(bytes.fromhex(shard.sha256))
    symmetric = 0.5 * (gram + gram.t())
    raw_values = torch.linalg.eigvalsh(symmetric).flip(0)
    total = float(torch.diagonal(symmetric).sum())
    if not math.isfinite(total):
        raise SpectrumNumericalError("row-shard spectrum energy is not finite")
    budget = _gamma(cursor + channels) * total
    diagnostics = SpectrumDiagnostics.of(gram, raw_values, total, budget)
    mean = sums / max(1, cursor)
    return SpectrumResult(cursor, channels, tuple(float(v) for v in raw_values.clamp_min(0.0)), total,
                          float(cursor * mean.square().sum()), digest.hexdigest(), budget,
                          {"algorithm": "fp64_row_shard_gram_eigvalsh", "shards": len(shards),
                           "diagnostics": diagnostics.to_dict()})


def exact_spectrum(tensor: torch.Tensor, *, tile_rows: int = 1024) -> SpectrumResult:
    if tensor.ndim != 2 or min(tensor.shape) < 1:
        raise ConfigurationError("spectra take a nonempty matrix")
    accumulator = StreamingGramAccumulator(int(tensor.shape[1]))
    for start in range(0, tensor.shape[0], tile_rows):
        accumulator.add(tensor[start:start + tile_rows])
    return accumulator.finalize()


def direct_svd_crosscheck(tensor: torch.Tensor, result: SpectrumResult | None = None) -> dict[str, float]:
    """FP64 SVD of the matrix against the Gram spectrum: max relative difference of the squared singular
    values on the energy scale, and of the captured energies at 95 % / 99 %."""
    x = tensor.detach().cpu().double()
    result = result or exact_spectrum(tensor)
    singular = torch.linalg.svdvals(x).square()
    values = torch.tensor(result.eigenvalues[:singular.numel()], dtype=torch.float64)
    scale = max(result.total_energy, 1e-300)
    return {"max_eigenvalue_difference": float((singular - values).abs().max() / scale),
            "svd_r95": _rank_bracket(tuple(singular.tolist()), float(singular.sum()), 0.95, 0.0).rank or 0,
            "gram_r95": result.r95 or 0,
            "svd_r99": _rank_bracket(tuple(singular.tolist()), float(singular.sum()), 0.99, 0.0).rank or 0,
            "gram_r99": result.r99 or 0}


__all__ = ["RankBracket", "SpectrumNumericalError", "SpectrumResult", "StreamingGramAccumulator",
           "direct_svd_crosscheck", "exact_spectrum", "write_spectrum_json"]
