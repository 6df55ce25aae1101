"""Lockstep routines with batched host reads (the counterpart of reference reelcache/deferred_reads.py:
``BatchedCall`` :50, ``read_host`` :77, ``run_lockstep`` :180, ``TileWorkspace`` :246, the projection /
energy / span routines :510-690).

A *routine* is a generator that queues device work and yields the tensors whose host values it needs next
(or a :class:`BatchedCall`); it is resumed with a tuple of host values (Python scalars for 0-d tensors,
float64 NumPy arrays otherwise) and finally returns its result. :func:`run_lockstep` advances many routines
together, so a round of reads costs one device-to-host transfer per device instead of one synchronization
per matrix and value -- under contention with a forward on the same GPU every host synchronization waits
for the queued work, so the number of rounds, not the number of matrices, sets the planner's latency.
"""

from __future__ import annotations

import math
import threading
from contextlib import contextmanager
from collections.abc import Generator, Iterable, Sequence
from typing import Any

import numpy as np
import torch

from .errors import ConfigurationError, IntegrityError

Routine = Generator[Sequence[torch.Tensor], tuple, Any]


class BatchedCall:
    """A request for device work batched with the round's other calls of the same ``key``: ``run(payloads)``
    runs once per key (payloads in routine order) and returns one result per payload."""

    __slots__ = ("key", "run", "payload")

    def __init__(self, key: Any, run, payload: Any):
        self.key, self.run, self.payload = key, run, payload


def _host_value(values: np.ndarray, tensor: torch.Tensor):
    if tensor.ndim == 0:
        value = values[0]
        if tensor.dtype == torch.bool:
            return bool(value)
        return float(value) if tensor.dtype.is_floating_point else int(value)
    values = values.reshape(tuple(tensor.shape))
    return values.astype(bool) if tensor.dtype == torch.bool else values


STATS = {"rounds": 0, "transfers": 0, "values": 0}
_STATS_LOCK = threading.Lock()
_STEP = threading.local()


def set_step_hook(hook) -> None:
    """Install ``hook()`` (None: remove) for this thread: :func:`run_lockstep` calls it between rounds, where no
    device read is pending and no lock is held -- the step boundary at which a pause of the caller's GPU work
    lands."""
    _STEP.hook = hook


def yield_point() -> None:
    """A step boundary outside the lockstep runner (long host loops call it): runs this thread's step hook."""
    hook = getattr(_STEP, "hook", None)
    if hook is not None:
        hook()


def step_phase(label: str) -> None:
    """Name the phase this thread's GPU work is in (reported by a pause that times out)."""
    _STEP.phase = label


def current_phase() -> str | None:
    return getattr(_STEP, "phase", None)


@contextmanager
def blocked_wait(label: str):
    """Mark a wait that allocates nothing (a host read's synchronization, a staging-slot wait): its end is a step
    boundary, so the step hook runs there."""
    previous = getattr(_STEP, "phase", None)
    _STEP.phase = f"wait:{label}"
    try:
        yield
    finally:
        _STEP.phase = previous
        yield_point()


def read_host(requests: Sequence[Sequence[torch.Tensor]]) -> list[tuple]:
    """Host values of every tensor of every request, one transfer per device (values travel as float64,
    exact for every 16/32-bit float, boolean and small integer)."""
    output: list[list] = [[None] * len(request) for request in requests]
    by_device: dict[torch.device, list] = {}
    for row, request in enumerate(requests):
        for column, tensor in enumerate(request):
            if not isinstance(tensor, torch.Tensor):
                raise ConfigurationError("lockstep reads take tensors")
            by_device.setdefault(tensor.device, []).append((row, column, tensor))
    for items in by_device.values():
        parts = [tensor.detach().reshape(-1).to(torch.float64) for _, _, tensor in items]
        flat = (torch.cat(parts) if len(parts) > 1 else parts[0]).cpu().numpy()
        with _STATS_LOCK:
            STATS["transfers"] += 1
            STATS["values"] += int(flat.size)
        offset = 0
        for (row, column, tensor), part in zip(items, parts):
            count = part.numel()
            output[row][column] = _host_value(flat[offset:offset + count], tensor)
            offset += count
    return [tuple(row) for row in output]


def _serve(requests: list) -> tuple[list, dict[int, BaseException]]:
    results: list = [None] * len(requests)
    raised: dict[int, BaseException] = {}
    reads = [i for i, request in enumerate(requests) if not isinstance(request, BatchedCall)]
    if reads:
        for i, values in zip(reads, read_host([requests[i] for i in reads])):
            results[i] = values
    groups: dict[Any, list[int]] = {}
    for i, request in enumerate(requests):
        if isinstance(request, BatchedCall):
            groups.setdefault(request.key, []).append(i)
    for positions in groups.values():
        call = requests[positions[0]]
        try:
            outputs = call.run([requests[i].payload for i in positions])
            if len(outputs) != len(positions):
                raise ConfigurationError("a batched call returns one result per payload")
            for i, value in zip(positions, outputs):
                results[i] = value
        except Exception as exc:  # noqa: BLE001 - thrown into each routine of the group
            for i in positions:
                raised[i] = exc
    return results, raised


def run_lockstep(routines: Iterable[Routine]) -> list:
    """Run routines in lockstep (one batched read per round); results in order. Exceptions behave as if the
    routines ran one after another: the lowest failing index raises, later routines are closed."""
    routines = list(routines)
    results: list = [None] * len(routines)
    errors: dict[int, BaseException] = {}
    sends: dict[int, Any] = {i: None for i in range(len(routines))}
    throws: dict[int, BaseException] = {}
    active = list(range(len(routines)))
    try:
        while active:
            requests, waiting = [], []
            for i in active:
                if errors and i > min(errors):
                    routines[i].close()
                    continue
                try:
                    request = routines[i].throw(throws.pop(i)) if i in throws else routines[i].send(sends[i])
                except StopIteration as stop:
                    results[i] = stop.value
                    continue
                except Exception as exc:  # noqa: BLE001 - re-raised in sequential order
                    errors[i] = exc
                    continue
                requests.append(request if isinstance(request, BatchedCall) else tuple(request))
                waiting.append(i)
            if errors:
                first = min(errors)
                for i in [w for w in waiting if w > first]:
                    routines[i].close()
                kept = [(i, r) for i, r in zip(waiting, requests) if i < first]
                waiting = [i for i, _ in kept]
                requests = [r for _, r in kept]
            if not waiting:
                break
            hook = getattr(_STEP, "hook", None)
            if hook is not None:
                hook()
            with _STATS_LOCK:
                STATS["rounds"] += 1
            served, raised = _serve(requests)
            sends = dict(zip(waiting, served))
            throws = {waiting[p]: exc for p, exc in raised.items()}
            active = waiting
    except BaseException:
        for routine in routines:
            routine.close()
        raise
    if errors:
        raise errors[min(errors)]
    return results


def run_one(routine: Routine) -> Any:
    return run_lockstep([routine])[0]


def upload(tensors: Sequence[torch.Tensor], device: Any) -> list[torch.Tensor]:
    """Host tensors to ``device`` in one transfer: packed into one pinned staging buffer (bytes), copied once,
    split into views of their own dtypes and shapes on the device."""
    device = torch.device(device)
    if device.type != "cuda" or not tensors:
        return [t.to(device) for t in tensors]
    parts = [t.detach().contiguous().view(-1).view(torch.uint8) for t in tensors]
    sizes = [p.numel() for p in parts]
    aligned = [(n + 15) // 16 * 16 for n in sizes]
    staging = torch.empty(sum(aligned), dtype=torch.uint8, pin_memory=True)
    offset = 0
    for part, width in zip(parts, aligned):
        staging[offset:offset + part.numel()].copy_(part)
        offset += width
    flat = staging.to(device, non_blocking=True)
    out, offset = [], 0
    for t, n, width in zip(tensors, sizes, aligned):
        out.append(flat[offset:offset + n].view(t.dtype).view(t.shape))
        offset += width
    return out


def download(tensors: Sequence[torch.Tensor]) -> list[torch.Tensor]:
    """Device tensors to the host in one transfer per device (byte-packed, then split into their own dtypes)."""
    out: list = [None] * len(tensors)
    by_device: dict = {}
    for i, t in enumerate(tensors):
        if t.device.type == "cpu":
            out[i] = t
        else:
            by_device.setdefault(t.device, []).append(i)
    for device, indices in by_device.items():
        parts = [tensors[i].detach().contiguous().view(-1).view(torch.uint8) for i in indices]
        host = torch.cat(parts).cpu()
        offset = 0
        for i, part in zip(indices, parts):
            n = part.numel()
            out[i] = host[offset:offset + n].view(tensors[i].dtype).view(tensors[i].shape)
            offset += n
        with _STATS_LOCK:
            STATS["transfers"] += 1
    return out


def finite_flag(tensor: torch.Tensor) -> torch.Tensor:
    """Device 0-d boolean: every element of ``tensor`` is finite."""
    return torch.isfinite(tensor).all()


def condition_terms(basis: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
    """Device terms of the conditioning of stored rows ``basis[k, C]`` (FP16 or FP32): ``eta = ||Q Q^T - I||_F``
    from an FP32-accurate Gram, and the largest row norm."""
    from .exact_blas import gram
    q = basis.float()
    g = gram(q.t())
    eta = (g - torch.eye(g.shape[0], dtype=g.dtype, device=g.device)).norm()
    return eta, q.norm(dim=1).max()


def finish_condition(basis: torch.Tensor, eta: float, norm: float) -> float:
    """An upper bound on the 2-norm condition number of the rows: with ``||Q Q^T - I|| <= eta < 1`` the singular
    values lie in ``[sqrt(1 - eta), sqrt(1 + eta)]``; ``inf`` otherwise."""
    if not math.isfinite(eta) or eta >= 1.0 or basis.shape[0] == 0:
        return math.inf
    return math.sqrt((1.0 + eta) / (1.0 - eta))


def condition_routine(basis: torch.Tensor):
    """Yields once; returns the condition bound of :func:`finish_condition`."""
    eta, norm = condition_terms(basis)
    (eta_value, norm_value) = yield (eta, norm)
    return finish_condition(basis, eta_value, norm_value)


class TileWorkspace:
    """Reusable named buffers (one allocation per name, shape class, dtype and device)."""

    def __init__(self):
        self._buffers: dict = {}

    def get(self, name: str, shape, dtype: torch.dtype, device) -> torch.Tensor:
        shape = tuple(int(s) for s in shape)
        device = torch.device(device)
        numel = math.prod(shape)
        key = (name, dtype, device)
        buffer = self._buffers.get(key)
        if buffer is None or buffer.numel() < numel:
            buffer = torch.empty(max(numel, 1), dtype=dtype, device=device)
            self._buffers[key] = buffer
        return buffer[:numel].view(shape)

    def clear(self) -> None:
        self._buffers.clear()

    @property
    def nbytes(self) -> int:
        return sum(b.numel() * b.element_size() for b in self._buffers.values())


# ---------------------------------------------------------------------------------------------------------
# routines
# ---------------------------------------------------------------------------------------------------------

def _sums(x: torch.Tensor, r: torch.Tensor | None) -> torch.Tensor:
    """Device ``[3]`` FP64: sum x^2, sum (x - r)^2, non-finite flag (fused kernel on CUDA)."""
    if x.is_cuda:
        from .ops import _ext
        if _ext.available():
            from .ops.fitter import sq_partials
            return sq_partials(x, r).sum(0)
    xf = x.double()
    bad = (~torch.isfinite(x)).any().double()
    resid = (xf - r.double()).square().sum() if r is not None else torch.zeros((), dtype=torch.float64)
    return torch.stack([xf.square().sum(), resid, bad])


def source_energy_routine(tensor: torch.Tensor, *, tile_rows: int = 4096):
    """Yields once; returns (energy, finite)."""
    totals = sum(_sums(tensor[s:s + tile_rows], None) for s in range(0, tensor.shape[0], tile_rows))
    (values,) = yield (totals,)
    return float(values[0]), float(values[2]) == 0.0


def projection_routine(tensor: torch.Tensor, rows16: torch.Tensor, *, tile_rows: int = 4096):
    """Coefficients ``P = X Q^T`` (FP32-accurate) and the direct residual of the stored FP16 rows; yields
    once; returns (stored energy, coefficients, source energy)."""
    from .exact_blas import mm
    q = rows16.to(tensor.device).float()
    coefficients = torch.empty((tensor.shape[0], q.shape[0]), dtype=torch.float32, device=tensor.device)
    totals = None
    for start in range(0, tensor.shape[0], tile_rows):
        a = tensor[start:start + tile_rows]
        p = mm(a, q.t())
        coefficients[start:start + a.shape[0]] = p
        part = _sums(a, mm(p, q))
        totals = part if totals is None else totals + part
    (values,) = yield (totals,)
    source, residual, bad = float(values[0]), float(values[1]), float(values[2])
    if bad:
        raise IntegrityError("projection source is not finite")
    energy = 1.0 if source <= 0 else 1.0 - residual / source
    return energy, coefficients, source


def stored_energy_routine(tensor: torch.Tensor, rows16: torch.Tensor, total: float, *, tile_rows: int = 4096):
    """The planner's verification on stored factors: returns (energy, coefficients)."""
    _, coefficients, source = yield from projection_routine(tensor, rows16, tile_rows=tile_rows)
    residual_fraction = 1.0 - _  # residual / measured source energy
    if total <= 0:
        return 1.0, coefficients
    return 1.0 - residual_fraction * source / total, coefficients


def span_energy_routine(gram: torch.Tensor, directions: torch.Tensor, total: float):
    """``trace(S^T G S) / total`` for column-orthonormal ``S``; yields once."""
    from .exact_blas import mm
    value = (mm(gram, directions) * directions).sum(dtype=torch.float64)
    (values,) = yield (value,)
    return 1.0 if total <= 0 else float(values[0]) / total


__all__ = ["BatchedCall", "Routine", "STATS", "TileWorkspace", "blocked_wait", "condition_routine", "condition_terms",
           "current_phase", "download", "finish_condition", "finite_flag", "projection_routine", "read_host",
           "run_lockstep", "run_one", "set_step_hook", "step_phase", "upload", "yield_point", "source_energy_routine", "span_energy_routine", "stored_energy_routine"]
