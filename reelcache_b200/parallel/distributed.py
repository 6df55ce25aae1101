"""Transport and failure agreement for storage collectives (the counterpart of reference
reelcache/distributed.py:26-412; protocol kept: checkpoint records ``{sequence, operation, rank,
error, cancelled, details}`` gathered from every rank before any payload moves).

The framework never creates process groups: a :class:`DistributedOwner` runs on groups the engine
made. Control messages (bounded canonical JSON, at most 1 MiB, no pickle) travel on a ``control``
group (Gloo, CPU); payloads on a ``data`` group (NCCL on CUDA -- NVLink / NVSwitch on one node -- or
Gloo on CPU) in bounded point-to-point pieces (``max_wire_bytes``).

* ``checkpoint(op, error=...)``: every rank reports; a local failure or cancellation on any rank is
  raised on *every* rank (:class:`PeerFailure`, :class:`CollectiveCancelled`) before the next payload
  collective, so no rank is left blocked in a transfer its peer will never join. Ranks that disagree on
  the collective order fail the same way.
* ``gather_matrix``: a ``rows`` or ``heads`` shard of a matrix from every rank -> canonical
  ``[tokens, channels]`` on the storage owner.
* ``acquire_columns`` / ``local_columns``: the owner decodes one rank's head columns at a time and
  sends them; each rank receives only its own columns.
* ``transfer_tensor``, ``broadcast_json``, ``owner_call``.
"""

from __future__ import annotations

import json
import threading
from contextlib import ExitStack, contextmanager, nullcontext
from dataclasses import asdict, dataclass
from typing import Any, Callable

import torch

from ..errors import ConfigurationError, StateError
from ..telemetry import span

MAX_CONTROL_BYTES = 1 << 20


class PeerFailure(StateError):
    """A rank failed (or the transport did); raised on every rank of the collective."""


class CollectiveCancelled(PeerFailure):
    """A rank cancelled the collective."""


@dataclass(frozen=True)
class KVLayout:
    """Ulysses geometry of one matrix: ``rows`` shards split tokens, ``heads`` shards split KV heads."""

    tokens: int
    kv_heads: int
    head_dim: int
    world_size: int = 2

    def __post_init__(self):
        if any(type(v) is not int or v <= 0 for v in (self.tokens, self.kv_heads, self.head_dim, self.world_size)):
            raise ConfigurationError("KV layout dimensions must be positive integers")
        if self.kv_heads % self.world_size:
            raise ConfigurationError("KV heads must divide evenly across ranks")
        if self.tokens < self.world_size:
            raise ConfigurationError("every row owner needs at least one token")

    @property
    def channels(self) -> int:
        return self.kv_heads * self.head_dim

    @property
    def local_channels(self) -> int:
        return self.kv_heads // self.world_size * self.head_dim

    def _rank(self, rank: int) -> None:
        if type(rank) is not int or not 0 <= rank < self.world_size:
            raise ConfigurationError("rank is outside the KV layout")

    def rows(self, rank: int) -> slice:
        self._rank(rank)
        count, extra = divmod(self.tokens, self.world_size)
        start = rank * count + min(rank, extra)
        return slice(start, start + count + int(rank < extra))

    def columns(self, rank: int) -> slice:
        self._rank(rank)
        return slice(rank * self.local_channels, (rank + 1) * self.local_channels)

    def shape(self, rank: int, layout: str) -> tuple[int, int]:
        if layout == "rows":
            rows = self.rows(rank)
            return (rows.stop - rows.start, self.channels)
        if layout == "heads":
            self._rank(rank)
            return (self.tokens, self.local_channels)
        raise ConfigurationError("layout must be 'rows' or 'heads'")


@dataclass
class WireCounters:
    payload_sent_bytes: int = 0
    payload_received_bytes: int = 0
    control_sent_bytes: int = 0
    control_received_bytes: int = 0
    payload_messages_sent: int = 0
    payload_messages_received: int = 0
    checkpoints: int = 0

    def to_dict(self) -> dict:
        return {**asdict(self), "accounting": "application tensor bytes; control includes lengths and padding",
                "transport_protocol_overhead_included": False}


class DistributedOwner:
    def __init__(self, group=None, *, control_group=None, owner_rank: int = 0, max_wire_bytes: int = 16 << 20,
                 device="cpu", expected_world_size: int | None = None):
        import torch.distributed as dist

        self.dist = dist
        self.group = group
        self.control_group = control_group if control_group is not None else group
        self.initialized = dist.is_available() and dist.is_initialized()
        self.world_size = dist.get_world_size(group) if self.initialized else 1
        self.rank = dist.get_rank(group) if self.initialized else 0
        if not 0 <= owner_rank < self.world_size:
            raise ConfigurationError("invalid storage owner rank")
        if expected_world_size is not None and expected_world_size != self.world_size:
            raise ConfigurationError("storage and native sequence-parallel world sizes differ")
        if type(max_wire_bytes) is not int or max_wire_bytes < 8:
            raise ConfigurationError("max_wire_bytes must be at least eight")
        self.owner_rank = owner_rank
        self.max_wire_bytes = max_wire_bytes
        self.device = torch.device(device)
        if self.initialized:
            backend = str(dist.get_backend(group))
            if backend == "gloo" and self.device.type != "cpu":
                raise ConfigurationError("a Gloo data group moves CPU tensors")
            if backend == "nccl" and self.device.type != "cuda":
                raise ConfigurationError("an NCCL data group moves CUDA tensors")
            if str(dist.get_backend(self.control_group)) != "gloo":
                raise ConfigurationError("the control group must be a Gloo (CPU) group")
        self.counters = WireCounters()
        self.sequence = 0
        self._thread = threading.get_ident()
        self._broken = False

    @property
    def is_owner(self) -> bool:
        return self.rank == self.owner_rank

    def _guard(self) -> None:
        if self._thread != threading.get_ident():
            raise StateError("collectives must stay on the ordered execution thread")
        if self._broken:
            raise PeerFailure("the storage transport failed; create a new session")

    def _global(self, rank: int) -> int:
        return self.dist.get_global_rank(self.group, rank) if self.group is not None else rank

    def _run(self, fn, *args, **kwargs):
        try:
            with span("transport.collective"):
                return fn(*args, **kwargs)
        except Exception as error:
            self._broken = True
            raise PeerFailure(f"storage transport failed: {type(error).__name__}: {error}") from error

    # -- control ----------------------------------------------------------------------------------------------

    def _all_json(self, value: Any) -> list:
        self._guard()
        raw = json.dumps(value, sort_keys=True, separators=(",", ":"), allow_nan=False).encode()
        if len(raw) > MAX_CONTROL_BYTES:
            raise ConfigurationError("control messages are bounded to one MiB")
        if self.world_size == 1:
            return [json.loads(raw)]
        length = torch.tensor([len(raw)], dtype=torch.int64)
        lengths = [torch.zeros_like(length) for _ in range(self.world_size)]
        self._run(self.dist.all_gather, lengths, length, group=self.control_group)
        counts = [int(t.item()) for t in lengths]
        size = max(counts)
        if min(counts) < 0 or size > MAX_CONTROL_BYTES:
            self._broken = True
            raise PeerFailure("a peer sent an invalid control message length")
        buffer = torch.zeros(size, dtype=torch.uint8)
        buffer[:len(raw)] = torch.frombuffer(bytearray(raw), dtype=torch.uint8)
        gathered = [torch.empty_like(buffer) for _ in range(self.world_size)]
        self._run(self.dist.all_gather, gathered, buffer, group=self.control_group)
        wire = (8 + size) * (self.world_size - 1)
        self.counters.control_sent_bytes += wire
        self.counters.control_received_bytes += wire
        return [json.loads(bytes(t[:n].tolist())) for t, n in zip(gathered, counts)]

    def checkpoint(self, operation: str, *, error=None, cancelled: bool = False, details=None) -> list:
        """Every rank reports; raises on every rank if any failed or cancelled. Returns all details."""
        self._guard()
        if isinstance(error, BaseException):
            error = f"{type(error).__name__}: {error}"
        elif error is not None:
            error = str(error)
        try:
            if len(json.dumps(details, allow_nan=False).encode()) > MAX_CONTROL_BYTES // 2:
                raise ConfigurationError("checkpoint details exceed 512 KiB")
        except Exception as exc:  # noqa: BLE001 - reported through the checkpoint itself
            error, details = f"invalid checkpoint details: {exc}", None
        rows = self._all_json({"sequence": self.sequence, "operation": str(operation), "rank": self.rank,
                               "error": error, "cancelled": bool(cancelled), "details": details})
        self.sequence += 1
        self.counters.checkpoints += 1
        if len({(r["sequence"], r["operation"]) for r in rows}) != 1:
            raise PeerFailure(f"collective order mismatch: {rows}")
        if any(r["cancelled"] for r in rows):
            raise CollectiveCancelled(f"collective cancelled: {operation}")
        failures = [f"rank {r['rank']}: {r['error']}" for r in rows if r["error"] is not None]
        if failures:
            raise PeerFailure(f"{operation}: " + "; ".join(failures))
        return [r["details"] for r in rows]

    def owner_call(self, operation: str, function: Callable):
        """Run ``function`` on the owner; its failure is raised on every rank."""
        self.checkpoint(f"{operation}:begin")
        result, error = None, None
        if self.is_owner:
            try:
                result = function()
            except BaseException as exc:  # noqa: BLE001
                error = exc
        try:
            self.checkpoint(f"{operation}:complete", error=error)
        except PeerFailure as failure:
            if error is not None:
                raise failure from error
            raise
        return result

    def broadcast_json(self, value, *, operation: str = "broadcast_json", source: int | None = None):
        source = self.owner_rank if source is None else source
        error = None
        try:
            if not 0 <= source < self.world_size:
                raise ConfigurationError("invalid JSON source")
            if self.rank == source:
                json.dumps(value, allow_nan=False)
        except Exception as exc:  # noqa: BLE001
            error = exc
        self.checkpoint(operation, error=error)
        return self._all_json(value if self.rank == source else None)[source]

    # -- payloads ---------------------------------------------------------------------------------------------

    def _move(self, tensor: torch.Tensor, source: int, destination: int) -> None:
        """Point-to-point move of a contiguous tensor in bounded pieces (already allocated on both ends)."""
        self._guard()
        if source == destination or self.world_size == 1:
            return
        flat = tensor.reshape(-1)
        step = max(1, self.max_wire_bytes // tensor.element_size())
        for start in range(0, flat.numel(), step):
            block = flat[start:start + step]
            if self.rank == source:
                self._run(self.dist.send, block, dst=self._global(destination), group=self.group)
                self.counters.payload_sent_bytes += block.numel() * block.element_size()
                self.counters.payload_messages_sent += 1
            elif self.rank == destination:
                self._run(self.dist.recv, block, src=self._global(source), group=self.group)
                self.counters.payload_received_bytes += block.numel() * block.element_size()
                self.counters.payload_messages_received += 1

    def gather_matrix(self, local: torch.Tensor, layout: KVLayout, *, source_layout: str,
                      operation: str = "gather_matrix") -> torch.Tensor | None:
        """Canonical ``[tokens, channels]`` on the owner (``None`` elsewhere)."""
        error, details = None, None
        try:
            if layout.world_size != self.world_size:
                raise ConfigurationError("layout and group world sizes differ")
            if tuple(local.shape) != layout.shape(self.rank, source_layout):
                raise ConfigurationError("local shard shape does not match its declared layout")
            if local.device.type != self.device.type:
                raise ConfigurationError("transfer tensor is on the wrong device")
            if not local.dtype.is_floating_point:
                raise ConfigurationError("KV transfers require a floating point tensor")
            details = {"dtype": str(local.dtype), "layout": source_layout, "geometry": asdict(layout)}
        except Exception as exc:  # noqa: BLE001
            error = exc
        rows = self.checkpoint(operation, error=error, details=details)
        if any(r != rows[0] for r in rows):
            raise PeerFailure("peers disagree on the KV layout or dtype")
        local = local.detach().contiguous()
        canonical = torch.empty((layout.tokens, layout.channels), dtype=local.dtype, device=self.device) \
            if self.is_owner else None
        for source in range(self.world_size):
            value = None
            if self.rank == source:
                value = local
            elif self.is_owner:
                value = torch.empty(layout.shape(source, source_layout), dtype=local.dtype, device=self.device)
            self.checkpoint(f"{operation}:rank{source}")
            if self.rank in (source, self.owner_rank):
                self._move(value, source, self.owner_rank)
            if self.is_owner:
                target = canonical[layout.rows(source)] if source_layout == "rows" else \
                    canonical[:, layout.columns(source)]
                target.copy_(value)
        return canonical

    @contextmanager
    def acquire_columns(self, layout: KVLayout, loader: Callable, *, dtype, operation: str = "acquire_columns"):
        """The owner decodes each rank's head columns in turn (``loader(columns)`` -> tensor or context
        manager yielding one) and sends them; every rank yields only its own ``[tokens, local]`` view."""
        rows = self.checkpoint(operation, error=None if layout.world_size == self.world_size else
                               "layout and group world sizes differ",
                               details={"layout": asdict(layout), "dtype": str(dtype)})
        if any(r != rows[0] for r in rows):
            raise PeerFailure("peers disagree on the restore layout or dtype")
        with ExitStack() as keep:
            mine = None
            for destination in range(self.world_size):
                with ExitStack() as transient:
                    value, error = None, None
                    try:
                        if self.is_owner:
                            loaded = loader(layout.columns(destination))
                            stack = keep if destination == self.rank else transient
                            value = stack.enter_context(loaded if hasattr(loaded, "__enter__") else nullcontext(loaded))
                            if tuple(value.shape) != layout.shape(destination, "heads") or value.dtype != dtype \
                                    or not value.is_contiguous():
                                raise ConfigurationError("loader returned a wrong column view")
                        elif self.rank == destination:
                            value = torch.empty(layout.shape(destination, "heads"), dtype=dtype, device=self.device)
                    except BaseException as exc:  # noqa: BLE001
                        error = exc
                    self.checkpoint(f"{operation}:rank{destination}", error=error)
                    if self.rank in (self.owner_rank, destination):
                        self._move(value, self.owner_rank, destination)
                    if self.rank == destination:
                        mine = value
            yield mine

    def local_columns(self, layout: KVLayout, loader: Callable, *, dtype, operation: str = "local_columns"):
        with self.acquire_columns(layout, loader, dtype=dtype, operation=operation) as local:
            return local.clone()

    def transfer_tensor(self, value, *, source: int, destination: int, operation: str = "transfer_tensor"):
        """Move a tensor from ``source`` to ``destination`` (shape and dtype travel as JSON)."""
        error, description = None, None
        try:
            if not (0 <= source < self.world_size and 0 <= destination < self.world_size):
                raise ConfigurationError("invalid tensor source/destination")
            if self.rank == source:
                value = value.detach().to(self.device).contiguous()
                description = {"shape": list(value.shape), "dtype": str(value.dtype).split(".")[-1]}
        except Exception as exc:  # noqa: BLE001
            error = exc
        described = self.checkpoint(operation, error=error, details=description)[source]
        received = None
        if self.rank == source:
            received = value
        elif self.rank == destination:
            received = torch.empty(described["shape"], dtype=getattr(torch, described["dtype"]), device=self.device)
        self.checkpoint(f"{operation}:allocated")
        if self.rank in (source, destination):
            self._move(received, source, destination)
        return received if self.rank == destination else None
