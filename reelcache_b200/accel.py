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
    """The FP32-replaced passes named by the ``fitter_fp64`` setting: ``"on"`` keeps every measurement pass in
    FP64, ``"off"`` moves :data:`OFF_PASSES` to FP32, ``"fp32:a+b"`` moves exactly the listed passes."""
    presets = {"on": frozenset(), "off": frozenset(OFF_PASSES)}
    if value in presets:
        return presets[value]
    listed = value.removeprefix("fp32:").split("+") if isinstance(value, str) and value.startswith("fp32:") else []
    listed = [name for name in listed if name]
    if listed and set(listed) <= set(FP32_PASSES):
        return frozenset(listed)
    raise ConfigurationError(f"fitter_fp64={value!r}: use 'on', 'off' or 'fp32:' followed by '+'-joined names "
                             f"from {FP32_PASSES}")


@dataclasses.dataclass(frozen=True)
class FitterAccel:
    """Opt-in fitter levers; the all-default instance means "none" (:meth:`from_config` returns None)."""

    green_sms: int | None = None
    green_workqueue: str | None = None
    cuda_graphs: bool = False
    graph_memory_bytes: int | None = None
    fused_fingerprints: bool = False
    finalize_on_fit_device: bool = False
    fp32_passes: frozenset = frozenset()

    def __post_init__(self) -> None:
        problems = []
        if not (self.green_sms is None or (type(self.green_sms) is int and self.green_sms > 0)):
            problems.append(f"green_sms={self.green_sms!r} is not None or an SM count >= 1")
        if self.green_workqueue is not None:
            if self.green_workqueue not in GREEN_WORKQUEUES:
                problems.append(f"green_workqueue={self.green_workqueue!r} is not one of {GREEN_WORKQUEUES}")
            if self.green_sms is None:
                problems.append("green_workqueue applies to a green context: set green_sms too")
        flags = ("cuda_graphs", "fused_fingerprints", "finalize_on_fit_device")
        problems += [f"{flag}={getattr(self, flag)!r} is not a bool" for flag in flags
                     if type(getattr(self, flag)) is not bool]
        if self.cuda_graphs is True:
            problems.append("cuda_graphs: graph replay of the FP64 passes is not offered (it slows them down)")
        passes = frozenset(self.fp32_passes)
        if passes - set(FP32_PASSES):
            problems.append(f"fp32_passes names unknown passes {sorted(passes - set(FP32_PASSES))}")
        if problems:
            raise ConfigurationError("FitterAccel: " + "; ".join(problems))
        object.__setattr__(self, "fp32_passes", passes)

    @property
    def default(self) -> bool:
        return self == FitterAccel()

    def to_dict(self) -> dict[str, Any]:
        return {**dataclasses.asdict(self), "fp32_passes": sorted(self.fp32_passes)}

    @classmethod
    def from_config(cls, config: Any) -> "FitterAccel | None":
        """The levers a runtime config selects (its ``fitter_*`` / fingerprint / finalize fields), or None."""
        read = lambda name, default: getattr(config, name, default)  # noqa: E731
        accel = cls(green_sms=read("fitter_green_context_sms", None),
                    green_workqueue=read("fitter_green_workqueue", None),
                    fused_fingerprints=read("fused_fingerprints", False),
                    finalize_on_fit_device=read("finalize_on_fit_device", False),
                    fp32_passes=parse_fitter_fp64(read("fitter_fp64", "on")))
        return None if accel.default else accel


class _Counters:
    """Thread-safe event counts of the accelerated paths (exposed as :func:`stats`)."""

    NAMES = ("energy_fused", "residual_fused_tiles", "span_neumann", "span_fallbacks", "span_terms",
             "fingerprints_fused", "dot2_gemms")

    def __init__(self):
        self._lock = threading.Lock()
        self.values = dict.fromkeys(self.NAMES, 0)

    def add(self, name: str, amount: int = 1) -> None:
        with self._lock:
            self.values[name] = self.values.get(name, 0) + amount

    def snapshot(self) -> dict[str, int]:
        with self._lock:
            return dict(self.values)


_LOCAL = threading.local()
_COUNTERS = _Counters()
STATS = _COUNTERS.values


def _count(name: str, value: int = 1) -> None:
    _COUNTERS.add(name, value)


def stats() -> dict[str, int]:
    return _COUNTERS.snapshot()


@contextlib.contextmanager
def scope(accel: FitterAccel | None, *, fit_device: Any = None):
    """Apply ``accel`` (and the fit device) to the archival routines this thread runs inside the block."""
    saved = getattr(_LOCAL, "accel", None), getattr(_LOCAL, "fit_device", None)
    _LOCAL.accel, _LOCAL.fit_device = accel, (torch.device(fit_device) if fit_device is not None else None)
    try:
        yield
    finally:
        _LOCAL.accel, _LOCAL.fit_device = saved


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


def _make_green_stream(index: int, sms: int, workqueue: str | None):
    try:
        from torch.cuda import green_contexts
    except ImportError as exc:
        raise ConfigurationError(f"green contexts need a newer torch than {torch.__version__}") from exc
    options: dict[str, Any] = {"num_sms": sms, "device_id": index}
    if workqueue is not None:
        options["workqueue_scope"] = workqueue
    try:
        with torch.cuda.device(index):
            context = green_contexts.GreenContext.create(**options)
            return context, context.Stream()
    except Exception as exc:  # noqa: BLE001 -- the driver's refusal becomes a configuration error
        raise ConfigurationError(f"cuda:{index} refused a green context of {sms} SMs: {exc}") from exc


def green_stream(device: Any, sms: int, workqueue: str | None = None):
    """A stream of a green context limited to ``sms`` SMs on ``device``; one context per (device, SMs,
    work queue), created on first use and kept for the life of the process."""
    device = torch.device(device)
    if device.type != "cuda":
        raise ConfigurationError(f"green contexts exist on CUDA devices, not {device}")
    index = torch.cuda.current_device() if device.index is None else device.index
    key = (index, int(sms), workqueue)
    with _GREEN_LOCK:
        if key not in _GREEN:
            _GREEN[key] = _make_green_stream(index, int(sms), workqueue)
        return _GREEN[key][1]


__all__ = ["FP32_PASSES", "FitterAccel", "OFF_PASSES", "current", "dot2_gemm", "energy_fp32",
           "fingerprint_terms_fused", "fp32", "fused_fingerprints", "green_stream", "parse_fitter_fp64",
           "residual_fp32", "scope", "span_energy_fp32", "stats", "sumsq64"]
