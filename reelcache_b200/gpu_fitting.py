"""GPU fitting: batched eigensolvers and the owner-thread fitter (the counterpart of reference
reelcache/gpu_fitting.py: ``BoundedEigh`` :100, ``select_eigh_solver`` :238, ``gram_bases`` :276,
``GPUFitter`` :298-520; and of reelcache/cusolver_eigh.py, whose cuSOLVER batched eigh is the baseline here).

Solvers map stacked symmetric FP32 ``[b, n, n]`` to ``(values, row_vectors)`` with ascending values and the
eigenvector of ``values[:, j]`` in ``row_vectors[:, j, :]``:

* ``jacobi`` -- the sm_100a batched Jacobi kernel (one CTA per matrix, matrix and vectors in shared memory,
  n <= 160, per-matrix convergence status); the default for the Rayleigh-Ritz problems of the planner.
* ``torch_batched`` -- ``torch.linalg.eigh`` on the whole batch (cuSOLVER): the measured baseline and the
  solver for n > 160 (full Grams).
* ``torch_loop`` -- one ``torch.linalg.eigh`` per matrix, an explicit diagnostic.

``auto`` runs ``jacobi`` where it applies (CUDA, extension present, n <= 160) and ``torch_batched``
otherwise; matrices whose Jacobi status is not "converged" are re-solved by ``torch_batched`` and counted.
:class:`BoundedEigh` cuts a batch into sub-batches that fit a device-memory bound; a fixed sub-batch size
makes each matrix's result independent of its batch companions.
"""

from __future__ import annotations

import contextlib
import os
import threading
import time
from typing import Any, Callable

import torch

from .errors import CapacityError, ConfigurationError, StateError, UnsupportedError

EIGH_SOLVERS = ("auto", "jacobi", "torch_batched", "torch_loop")
GPU_FIT_METHODS = ("randomized", "gram_batched", "gram", "exact", "torch_lowrank", "gesvd", "gesvdj", "gesvda")
EIGH_MEMORY_FRACTION = 0.25
JACOBI_MAX_N = 160
STATS = {"jacobi_calls": 0, "jacobi_matrices": 0, "jacobi_fallbacks": 0, "torch_calls": 0}
_STATS_LOCK = threading.Lock()


def _count(name: str, value: int = 1) -> None:
    with _STATS_LOCK:
        STATS[name] = STATS.get(name, 0) + value


def _jacobi_ok(mats: torch.Tensor) -> bool:
    if not mats.is_cuda or mats.shape[-1] > JACOBI_MAX_N:
        return False
    from .ops import _ext
    return _ext.available()


def torch_rows_eigh(mats: torch.Tensor):
    _count("torch_calls")
    values, columns = torch.linalg.eigh(mats)
    return values, columns.transpose(-1, -2)


def torch_loop_eigh(mats: torch.Tensor):
    pairs = [torch.linalg.eigh(m) for m in mats]
    _count("torch_calls", len(pairs))
    return torch.stack([v for v, _ in pairs]), torch.stack([c.transpose(0, 1) for _, c in pairs])


def jacobi_rows_eigh(mats: torch.Tensor, *, max_sweeps: int = 30, refine_unconverged: bool = True):
    """The sm_100a Jacobi kernel; unconverged matrices re-solved by ``torch.linalg.eigh`` when asked."""
    if not _jacobi_ok(mats):
        raise UnsupportedError("the Jacobi kernel needs a CUDA batch with n <= 160 and the native extension")
    from .ops.fitter import jacobi_eigh
    values, vectors, info, _ = jacobi_eigh(mats, max_sweeps=max_sweeps)
    _count("jacobi_calls")
    _count("jacobi_matrices", int(mats.shape[0]))
    if refine_unconverged:
        bad = torch.nonzero(info != 0).flatten()
        if bad.numel():
            _count("jacobi_fallbacks", int(bad.numel()))
            v2, c2 = torch.linalg.eigh(mats[bad].float())
            values[bad] = v2
            vectors[bad] = c2
    return values, vectors.transpose(-1, -2)


def rows_eigh(mats: torch.Tensor):
    """``auto``: Jacobi where it applies, cuSOLVER (or the host LAPACK) otherwise."""
    mats = mats.float()
    if _jacobi_ok(mats):
        return jacobi_rows_eigh(mats)
    return torch_rows_eigh(mats)


def default_eigh_sub_batch(n: int) -> int | None:
    """One matrix per call from n = 4096 on (cost-neutral there); None below (whole batch)."""
    return 1 if n >= 4096 else None


def eigh_workspace_bytes(batch: int, n: int, label: str) -> int:
    """Device bytes of one batched solve: copies of the inputs, values, vectors and the solver workspace
    (Jacobi keeps everything in shared memory; cuSOLVER's workspace is modeled as two more copies)."""
    copies = 3 if label.startswith("jacobi") else 5
    return batch * (copies * 4 * n * n + 8 * n)


class BoundedEigh:
    """A batched eigensolver called on sub-batches that a device-memory bound admits (the solver never
    changes). ``calls`` records each call's batch, n, sub-batch and reason; ``last`` the latest."""

    def __init__(self, label: str, solver: Callable, *, memory_fraction: float = EIGH_MEMORY_FRACTION,
                 workspace: Callable | None = None, total_memory: int | None = None,
                 sub_batch_size: Callable | None = None):
        problems = []
        if not 0 < memory_fraction <= 1:
            problems.append(f"memory_fraction={memory_fraction!r} is outside (0, 1]")
        if not (total_memory is None or (type(total_memory) is int and total_memory > 0)):
            problems.append(f"total_memory={total_memory!r} is not None or a byte count >= 1")
        if not (sub_batch_size is None or callable(sub_batch_size)):
            problems.append("sub_batch_size must be None or a callable n -> sub-batch size")
        if problems:
            raise ConfigurationError(f"BoundedEigh {label!r}: " + "; ".join(problems))
        self.label, self.solver, self.memory_fraction = label, solver, memory_fraction
        self._workspace = workspace or (lambda batch, n, device: eigh_workspace_bytes(batch, n, label))
        self.total_memory = total_memory
        self.sub_batch_size = sub_batch_size or default_eigh_sub_batch
        self.calls: list[dict] = []
        self.last: dict | None = None

    def derive(self, *, memory_fraction: float | None = None, total_memory: int | None = None) -> "BoundedEigh":
        return BoundedEigh(self.label, self.solver,
                           memory_fraction=self.memory_fraction if memory_fraction is None else memory_fraction,
                           workspace=self._workspace,
                           total_memory=self.total_memory if total_memory is None else total_memory,
                           sub_batch_size=self.sub_batch_size)

    def _budget(self, device) -> float | None:
        if self.total_memory is not None:
            return self.memory_fraction * self.total_memory
        if torch.device(device).type != "cuda":
            return None
        return self.memory_fraction * torch.cuda.get_device_properties(device).total_memory

    def sub_batch(self, batch: int, n: int, device) -> tuple[int, str]:
        fixed = self.sub_batch_size(n)
        budget = self._budget(device)
        if fixed is not None:
            if budget is not None and self._workspace(fixed, n, device) > budget:
                return fixed, "over_budget"
            return min(fixed, batch), "fixed"
        size = batch
        while size > 1 and budget is not None and self._workspace(size, n, device) > budget:
            size = (size + 1) // 2
        return size, "whole" if size == batch else "memory_bound"

    def __call__(self, mats: torch.Tensor):
        batch, n = int(mats.shape[0]), int(mats.shape[-1])
        size, reason = self.sub_batch(batch, n, mats.device)
        values, rows = [], []
        calls = 0
        for start in range(0, batch, size):
            v, r = self.solver(mats[start:start + size])
            values.append(v)
            rows.append(r)
            calls += 1
        self.last = {"batch": batch, "n": n, "sub_batch": size, "solver_calls": calls, "reason": reason,
                     "solver": self.label}
        self.calls.append(self.last)
        return torch.cat(values), torch.cat(rows)


def select_eigh_solver(solver: str = "auto", *, sub_batch_size=None):
    """``(label, eigh)`` for stacked FP32 symmetric matrices; never silently degrades: an explicit
    ``jacobi`` raises where the kernel cannot run."""
    if solver not in EIGH_SOLVERS:
        raise ConfigurationError(f"eigh solver must be one of {EIGH_SOLVERS}")
    if solver == "auto":
        return "auto_jacobi_sm100_or_cusolver", BoundedEigh("auto", rows_eigh, sub_batch_size=sub_batch_size)
    if solver == "jacobi":
        return "jacobi_sm100", BoundedEigh("jacobi_sm100", jacobi_rows_eigh, sub_batch_size=sub_batch_size)
    if solver == "torch_batched":
        return "torch_linalg_eigh_batched", BoundedEigh("torch_linalg_eigh_batched", torch_rows_eigh,
                                                        sub_batch_size=sub_batch_size)
    return "torch_eigh_loop_explicit", torch_loop_eigh


def gram_bases(sources, ranks, *, eigh=None):
    """Top-``rank`` right singular rows (FP32 ``[rank, C]``, descending energy) of each ``[rows, C]`` source by
    one batched eigensolve of their FP32-accurate Grams."""
    from .exact_blas import gram
    if not sources or len(sources) != len(ranks):
        raise ConfigurationError(f"{len(sources)} sources and {len(ranks)} ranks: give one rank per source")
    widths = sorted({int(x.shape[1]) for x in sources})
    if len(widths) != 1:
        raise ConfigurationError(f"one batched Gram solve needs one channel count, got {widths}")
    grams = torch.stack([gram(x) for x in sources])
    _, rows = (eigh or rows_eigh)(grams)
    return [rows[index, -rank:].flip(0) for index, rank in enumerate(ranks)]


class GPUFitter:
    """Owner-thread GPU fitting on one granted device (by index and UUID). ``gram_batched`` batch-solves the
    Grams of a whole chunk in :meth:`prefit`; each basis is consumed by the next :meth:`fit` of the same,
    unmodified tensor. :meth:`plan_chunk` runs the rank method's chunk planner on the fitter's device and
    stream."""

    def __init__(self, *, gpu_id: int, gpu_uuid: str, method: str = "randomized",
                 max_workspace_bytes: int = 2 * 1024 ** 3, seed: int = 0, power_iterations: int = 2,
                 batch_size: int = 60, side_stream: bool = False, shared: bool = False, eigh_solver: str = "auto"):
        def whole(value, low, high=None):
            return type(value) is int and value >= low and (high is None or value <= high)

        checks = (
            (whole(gpu_id, 0) and isinstance(gpu_uuid, str) and gpu_uuid.startswith("GPU-"),
             f"device index {gpu_id!r} and UUID {gpu_uuid!r} (a 'GPU-...' string) are both required"),
            (method in GPU_FIT_METHODS, f"method {method!r} is not one of {GPU_FIT_METHODS}"),
            (whole(max_workspace_bytes, 1), f"max_workspace_bytes={max_workspace_bytes!r} is not a byte count >= 1"),
            (whole(seed, 0), f"seed={seed!r} is not an int >= 0"),
            (whole(power_iterations, 0, 8), f"power_iterations={power_iterations!r} is not an int in [0, 8]"),
            (whole(batch_size, 1, 256), f"batch_size={batch_size!r} is not an int in [1, 256]"),
            (type(side_stream) is bool and type(shared) is bool, "side_stream and shared take True or False"),
            (eigh_solver in EIGH_SOLVERS, f"eigh_solver {eigh_solver!r} is not one of {EIGH_SOLVERS}"),
        )
        problems = [message for ok, message in checks if not ok]
        if problems:
            raise ConfigurationError("GPUFitter: " + "; ".join(problems))
        self.gpu_id, self.gpu_uuid, self.method = gpu_id, gpu_uuid, method
        self.max_workspace_bytes, self.seed, self.power_iterations = max_workspace_bytes, seed, power_iterations
        self.batch_size, self.eigh_solver = batch_size, eigh_solver
        self.shared = shared
        self.side_stream = side_stream or shared
        self._stream = None
        self._lock = threading.Lock()
        self.owner = (os.getpid(), threading.get_ident())
        self._prefit: dict = {}
        self.prefit_stats = {"batches": 0, "matrices": 0, "hits": 0, "misses": 0, "solver": None}

    def adopt_current_thread(self) -> None:
        self.clear_prefit()
        self.owner = (os.getpid(), threading.get_ident())

    def _check_owner(self) -> None:
        if self.shared:
            if self.owner[0] != os.getpid():
                raise StateError("a shared GPU fitter cannot cross processes")
            return
        if self.owner != (os.getpid(), threading.get_ident()):
            raise StateError("GPU fitting runs on its owner thread")

    def _device(self) -> torch.device:
        if not torch.cuda.is_available() or self.gpu_id >= torch.cuda.device_count():
            raise UnsupportedError("the GPU fitting device is unavailable")
        device = torch.device("cuda", self.gpu_id)
        actual = str(torch.cuda.get_device_properties(device).uuid).removeprefix("GPU-")
        if actual != self.gpu_uuid.removeprefix("GPU-"):
            raise ConfigurationError("the GPU fitting device differs from the granted UUID")
        return device

    def _scope(self, device):
        if self.side_stream and self._stream is None:
            self._stream = torch.cuda.Stream(device)
        stream = torch.cuda.stream(self._stream) if self.side_stream else contextlib.nullcontext()
        lock = self._lock if self.shared else contextlib.nullcontext()
        return lock, stream

    @staticmethod
    def _identity(tensor, context, rank):
        return (tensor.untyped_storage().data_ptr(), tensor.storage_offset(), tuple(tensor.shape),
                tuple(tensor.stride()), tensor.dtype, str(tensor.device), tensor._version, context, rank)

    @torch.no_grad()
    def prefit(self, items: dict) -> None:
        """Batch-solve bases for ``{key: (tensor, context, rank)}`` (``gram_batched`` only)."""
        from .factorization import _canonical_signs, validate_matrix, validate_rank
        self._check_owner()
        self.clear_prefit()
        if self.method != "gram_batched" or not items:
            return
        prepared = []
        for tensor, context, rank in items.values():
            validate_matrix(tensor, context, lossy=True, check_values=False)
            validate_rank(rank, tuple(tensor.shape))
            prepared.append((tensor, context, rank))
        channels = max(int(t.shape[1]) for t, _, _ in prepared)
        rows = max(int(t.shape[0]) for t, _, _ in prepared)
        per_item = 3 * 4 * channels * channels
        if 8 * rows * channels + per_item > self.max_workspace_bytes:
            raise CapacityError("batched GPU fitting exceeds its declared workspace budget")
        batch = min(self.batch_size, max(1, (self.max_workspace_bytes - 8 * rows * channels) // per_item))
        device = self._device()
        label, solver = select_eigh_solver(self.eigh_solver)
        self.prefit_stats["solver"] = label
        lock, stream = self._scope(device)
        with lock, torch.cuda.device(device), stream:
            for start in range(0, len(prepared), batch):
                group = prepared[start:start + batch]
                began = time.perf_counter()
                sources = [validate_matrix(t.to(device), c).float() for t, c, _ in group]
                bases = gram_bases(sources, [r for _, _, r in group], eigh=solver)
                bases = [_canonical_signs(b).to(torch.float16).contiguous() for b in bases]
                torch.cuda.current_stream(device).synchronize()
                share = (time.perf_counter() - began) / len(group)
                for (tensor, context, rank), basis in zip(group, bases):
                    if not bool(torch.isfinite(basis).all()):
                        raise ConfigurationError("fitted basis is not finite in stored FP16")
                    self._prefit[self._identity(tensor, context, rank)] = (tensor, basis, share)
                self.prefit_stats["batches"] += 1
                self.prefit_stats["matrices"] += len(group)

    def clear_prefit(self) -> None:
        self._prefit.clear()

    @torch.no_grad()
    def fit(self, tensor, context, rank, *, reuse_basis=None, reuse_threshold=None):
        """Fresh :class:`~reelcache_b200.factorization.Factors` (host tensors) of one matrix."""
        from .factorization import Factors, _canonical_signs, fit_basis, project_onto_basis, validate_matrix, \
            validate_rank
        self._check_owner()
        validate_matrix(tensor, context, lossy=True, check_values=False)
        validate_rank(rank, tuple(tensor.shape))
        if reuse_basis is not None or reuse_threshold is not None:
            raise UnsupportedError("GPU solver comparisons fit fresh bases")
        rows, channels = tensor.shape
        estimated = 32 * (rows * channels + channels * channels + rows * rank)
        if estimated > self.max_workspace_bytes:
            raise CapacityError("GPU fitting exceeds its declared workspace budget")
        device = self._device()
        started = time.perf_counter()
        lock, stream = self._scope(device)
        with lock, torch.cuda.device(device), stream:
            events = [torch.cuda.Event(enable_timing=True) for _ in range(4)]
            events[0].record()
            source = tensor.to(device)
            events[1].record()
            if self.method in ("gram_batched", "gram"):
                cached = self._prefit.pop(self._identity(tensor, context, rank), None)
                if cached is not None:
                    self.prefit_stats["hits"] += 1
                    basis = cached[1]
                else:
                    self.prefit_stats["misses"] += 1
                    (basis,) = gram_bases([validate_matrix(source, context).float()], [rank])
                    basis = _canonical_signs(basis).to(torch.float16).contiguous()
                projection = project_onto_basis(source, basis)
                factors = Factors(basis, projection.coefficients, rank, {
                    "factorization_method": "fp32_gram_eigh", "prefit_batched": cached is not None,
                    "projection_relative_residual": projection.relative_residual,
                    "basis_condition_bound": projection.condition_bound})
            else:
                factors = fit_basis(source, context, rank, method=self.method, seed=self.seed,
                                    power_iterations=self.power_iterations)
            events[2].record()
            basis, coefficients = factors.basis.cpu(), factors.coefficients.cpu()
            events[3].record()
            events[3].synchronize()
        metrics = {**factors.metrics, "gpu_fitting_backend": self.method, "gpu_fitting_uuid": self.gpu_uuid,
                   "gpu_fitting_workspace_estimate": estimated,
                   "gpu_fitting_h2d_ms": events[0].elapsed_time(events[1]),
                   "gpu_fitting_compute_ms": events[1].elapsed_time(events[2]),
                   "gpu_fitting_d2h_ms": events[2].elapsed_time(events[3]),
                   "gpu_fitting_wall_seconds": time.perf_counter() - started}
        return Factors(basis, coefficients, rank, metrics)

    @torch.no_grad()
    def plan_chunk(self, config, view, matrices, contexts, bindings, inherited, *, chunk_id: str = "chunk") -> Any:
        """The rank method's chunk plan (sketch, predict, fit, verify/grow/trim, share/augment/refit) on this
        fitter's device, stream and owner thread."""
        from .rank_method import plan_chunk
        self._check_owner()
        device = self._device()
        lock, stream = self._scope(device)
        with lock, torch.cuda.device(device), stream:
            plan = plan_chunk(matrices, contexts, config, view, bindings, inherited, chunk_id=chunk_id,
                              device=device)
        self.prefit_stats["solver"] = select_eigh_solver(self.eigh_solver)[0]
        return plan


__all__ = ["BoundedEigh", "EIGH_SOLVERS", "GPUFitter", "STATS", "default_eigh_sub_batch", "eigh_workspace_bytes",
           "gram_bases", "jacobi_rows_eigh", "rows_eigh", "select_eigh_solver", "torch_loop_eigh",
           "torch_rows_eigh"]
