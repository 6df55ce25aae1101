"""Opt-in fitter levers (the counterpart of reference reelcache/accel_b.py: options :1-52, ``OFF_PASSES`` :70,
``dot2_gemm`` :233, ``green_stream`` :271, kernels :318-455, ``energy_fp32`` :521, ``residual_fp32`` :530,
``span_energy_fp32`` :570, ``fingerprint_terms_fused`` :606).

Every option defaults to off; :func:`scope` applies a :class:`FitterAccel` to the archival routines of the
calling thread. The reference's Triton kernels are the sm_100a kernels of ``csrc/fit/fitter.cu`` here:

* ``sq_partials`` (fused scaled sums of squares, residual sums and a non-finite flag, FP64 partials) backs
  :func:`energy_fp32`, :func:`residual_fp32` and :func:`sumsq64`;
* ``fingerprint_partials`` (exact int64) backs :func:`fingerprint_terms_fused`;
* ``dot2_gemm`` (Ogita-Rump-Oishi compensated FP32 products) backs :func:`dot2_gemm`.

``fitter_fp64="off"`` selects the FP32 replacements of the FP64 measurement passes (:data:`OFF_PASSES`);
``span`` evaluates ``<G^-1, M>`` by a Neumann series of ``D = Q Q^T - I`` when ``eta = max_i sum_j |D_ij|``
is small. Green contexts (``green_sms``) give the fitter a stream limited to that many SMs. CUDA-graph replay
of the FP64 passes is not provided (the reference documents it as harmful and off).
"""

from __future__ import annotations

import contextlib
import dataclasses
import math
import threading
from typing import Any

import torch

from .errors import ConfigurationError

FP32_PASSES = ("products", "products_verify", "products_recon", "products_df", "residual", "energy", "span",
               "planner")
OFF_PASSES = ("products_verify", "products_recon", "residual", "energy", "span", "planner")
GREEN_WORKQUEUES = ("balanced", "device_ctx")
SPAN_ETA_MAX = 0.05
SPAN_TOLERANCE = 1e-10
SPAN_MAX_TERMS = 12


def parse_fitter_fp64(value: Any) -> frozenset:
    """``"on"`` (FP64 passes), ``"off"`` (:data:`OFF_PASSES` in FP32) or ``"fp32:<pass>[+<pass>...]"``."""
    if value == "on":
        return frozenset()
    if value == "off":
        return frozenset(OFF_PASSES)
    if isinstance(value, str) and value.startswith("fp32:"):
        names = [name for name in value[5:].split("+") if name]
        if names and all(name in FP32_PASSES for name in names):
            return frozenset(names)
    raise ConfigurationError(f"fitter_fp64 must be 'on', 'off' or 'fp32:<pass>[+<pass>...]' from {FP32_PASSES}")


@dataclasses.dataclass(frozen=True)
class FitterAccel:
    green_sms: int | None = None
    green_workqueue: str | None = None
    cuda_graphs: bool = False
    graph_memory_bytes: int | None = None
    fused_fingerprints: bool = False
    finalize_on_fit_device: bool = False
    fp32_passes: frozenset = frozenset()

    def __post_init__(self) -> None:
        if self.green_sms is not None and (type(self.green_sms) is not int or self.green_sms < 1):
            raise ConfigurationError("fitter_green_context_sms must be None or a positive SM count")
        if self.green_workqueue is not None and self.green_workqueue not in GREEN_WORKQUEUES:
            raise ConfigurationError(f"fitter_green_workqueue must be None or one of {GREEN_WORKQUEUES}")
        if self.green_workqueue is not None and self.green_sms is None:
            raise ConfigurationError("fitter_green_workqueue needs fitter_green_context_sms")
        for name in ("cuda_graphs", "fused_fingerprints", "finalize_on_fit_device"):
            if type(getattr(self, name)) is not bool:
                raise ConfigurationError(f"{name} must be a bool")
        if self.cuda_graphs:
            raise ConfigurationError("CUDA-graph replay of the fitter's FP64 passes is not provided")
        passes = frozenset(self.fp32_passes)
        if not passes <= set(FP32_PASSES):
            raise ConfigurationError(f"unknown FP32 passes {sorted(passes - set(FP32_PASSES))}")
        object.__setattr__(self, "fp32_passes", passes)

    @property
    def default(self) -> bool:
        return self == FitterAccel()

    def to_dict(self) -> dict[str, Any]:
        data = dataclasses.asdict(self)
        data["fp32_passes"] = sorted(self.fp32_passes)
        return data

    @classmethod
    def from_config(cls, config: Any) -> "FitterAccel | None":
        accel = cls(green_sms=getattr(config, "fitter_green_context_sms", None),
                    green_workqueue=getattr(config, "fitter_green_workqueue", None),
                    fused_fingerprints=getattr(config, "fused_fingerprints", False),
                    finalize_on_fit_device=getattr(config, "finalize_on_fit_device", False),
                    fp32_passes=parse_fitter_fp64(getattr(config, "fitter_fp64", "on")))
        return None if accel.default else accel


_LOCAL = threading.local()
_STATS_LOCK = threading.Lock()
STATS: dict[str, int] = {"energy_fused": 0, "residual_fused_tiles": 0, "span_neumann": 0, "span_fallbacks": 0,
                         "span_terms": 0, "fingerprints_fused": 0, "dot2_gemms": 0}


def _count(name: str, value: int = 1) -> None:
    with _STATS_LOCK:
        STATS[name] = STATS.get(name, 0) + value


def stats() -> dict[str, int]:
    with _STATS_LOCK:
        return dict(STATS)


@contextlib.contextmanager
def scope(accel: FitterAccel | None, *, fit_device: Any = None):
    previous = (getattr(_LOCAL, "accel", None), getattr(_LOCAL, "fit_device", None))
    _LOCAL.accel = accel
    _LOCAL.fit_device = None if fit_device is None else torch.device(fit_device)
    try:
        yield
    finally:
        _LOCAL.accel, _LOCAL.fit_device = previous


def current() -> FitterAccel | None:
    return getattr(_LOCAL, "accel", None)


def fp32(name: str, tensor: torch.Tensor | None = None) -> bool:
    accel = current()
    if accel is None or name not in accel.fp32_passes:
        return False
    return tensor is None or (isinstance(tensor, torch.Tensor) and tensor.is_cuda)


def _native(x: torch.Tensor) -> bool:
    if not x.is_cuda:
        return False
    from .ops import _ext
    return _ext.available()


def sumsq64(x: torch.Tensor) -> torch.Tensor:
    """0-d FP64 ``sum(x * x)``: FP32 squares accumulated in FP64 (fused kernel on CUDA)."""
    if not _native(x) or x.ndim != 2:
        return torch.sum(x.float() * x.float(), dtype=torch.float64)
    from .ops.fitter import sq_partials
    return sq_partials(x).sum(0)[0]


def energy_fp32(tensor: torch.Tensor, scale: float) -> tuple[torch.Tensor, torch.Tensor]:
    """(0-d FP64 ``sum (x/scale)^2``, 0-d bool finite) in one fused kernel."""
    from .ops.fitter import sq_partials
    _count("energy_fused")
    totals = sq_partials(tensor, None, scale).sum(0)
    return totals[0], totals[2] == 0


def residual_fp32(tensor: torch.Tensor, coefficients: torch.Tensor, rows32: torch.Tensor, tile_rows: int,
                  scale: float) -> tuple[torch.Tensor, torch.Tensor]:
    """(source, error) 0-d FP64 sums over residual tiles with FP32-accurate reconstructions."""
    from .exact_blas import mm
    from .ops.fitter import sq_partials
    totals = None
    tiles = 0
    for start in range(0, int(tensor.shape[0]), tile_rows):
        stop = min(start + tile_rows, int(tensor.shape[0]))
        part = sq_partials(tensor[start:stop], mm(coefficients[start:stop], rows32), scale).sum(0)
        totals = part if totals is None else totals + part
        tiles += 1
    _count("residual_fused_tiles", tiles)
    return totals[0], totals[1]


def dot2_gemm(tensor: torch.Tensor, rows: torch.Tensor) -> torch.Tensor:
    from .ops.fitter import dot2_gemm as kernel
    _count("dot2_gemms")
    return kernel(tensor, rows)


def span_energy_fp32(coefficients: torch.Tensor, rows16: torch.Tensor, source_energy: float) -> float | None:
    """``<G^-1, M> / source_energy`` with ``G = Q Q^T`` (FP16 rows) and ``M = P^T P`` by the Neumann series
    ``||P||^2 + sum_k (-1)^k tr(D^k M)``, ``D = G - I``; None when ``eta > SPAN_ETA_MAX`` (the caller then
    uses the FP64 Cholesky path)."""
    from .exact_blas import mm
    q = rows16.to(device=coefficients.device, dtype=torch.float32)
    delta = mm(q, q.t())
    diagonal = torch.sum(q.double() * q.double(), dim=1)
    delta.diagonal().copy_((diagonal - 1.0).float())
    eta = float(delta.abs().sum(1).max())
    if not math.isfinite(eta) or eta > SPAN_ETA_MAX:
        _count("span_fallbacks")
        return None
    terms = 0
    while terms < SPAN_MAX_TERMS and eta ** (terms + 1) / (1.0 - eta) > SPAN_TOLERANCE:
        terms += 1
    p = coefficients.float()
    work = mm(p.t(), p)
    traces = []
    for _ in range(terms):
        work = mm(delta, work)
        traces.append(torch.sum(work.diagonal(), dtype=torch.float64))
    values = torch.stack([sumsq64(p)] + traces).tolist()
    total = values[0] + sum((-1.0) ** (k + 1) * v for k, v in enumerate(values[1:]))
    if not math.isfinite(total):
        _count("span_fallbacks")
        return None
    _count("span_neumann")
    _count("span_terms", terms)
    return total / source_energy


def fused_fingerprints(tensor: torch.Tensor) -> bool:
    accel = current()
    return accel is not None and accel.fused_fingerprints and _native(tensor)


def fingerprint_terms_fused(tensor: torch.Tensor, prime: int, tile_elements: int) -> torch.Tensor:
    """Exact fingerprint terms (int64 ``[3]`` or ``[6]`` mod ``prime``) with one kernel per row tile."""
    from .ops.fitter import fingerprint_partials
    rows, columns = (int(size) for size in tensor.shape)
    wide = tensor.element_size() == 4
    tile_rows = max(1, tile_elements // columns)
    totals = None
    for start in range(0, rows, tile_rows):
        part = fingerprint_partials(tensor[start:start + tile_rows], start, prime).sum(0)
        totals = part if totals is None else totals + part
    _count("fingerprints_fused")
    return totals[:6 if wide else 3].remainder(prime)


_GREEN: dict = {}
_GREEN_LOCK = threading.Lock()


def green_stream(device: Any, sms: int, workqueue: str | None = None):
    """The stream of this process's green context of ``sms`` SMs on ``device`` (created once, kept)."""
    device = torch.device(device)
    if device.type != "cuda":
        raise ConfigurationError("a green context needs a CUDA device")
    index = device.index if device.index is not None else torch.cuda.current_device()
    key = (index, int(sms), workqueue)
    with _GREEN_LOCK:
        entry = _GREEN.get(key)
        if entry is None:
            try:
                from torch.cuda import green_contexts
            except ImportError as exc:
                raise ConfigurationError(f"torch {torch.__version__} has no green contexts") from exc
            kwargs: dict[str, Any] = {"num_sms": int(sms), "device_id": index}
            if workqueue is not None:
                kwargs["workqueue_scope"] = workqueue
            try:
                with torch.cuda.device(index):
                    context = green_contexts.GreenContext.create(**kwargs)
                    stream = context.Stream()
            except Exception as exc:  # noqa: BLE001 - surfaced as a configuration error
                raise ConfigurationError(f"a green context of {sms} SMs is unsupported here: {exc}") from exc
            entry = _GREEN[key] = (context, stream)
    return entry[1]


__all__ = ["FP32_PASSES", "FitterAccel", "OFF_PASSES", "current", "dot2_gemm", "energy_fp32",
           "fingerprint_terms_fused", "fp32", "fused_fingerprints", "green_stream", "parse_fitter_fp64",
           "residual_fp32", "scope", "span_energy_fp32", "stats", "sumsq64"]
