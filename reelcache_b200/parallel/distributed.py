"""Storage collectives with failure agreement (the behaviour of reference reelcache/distributed.py: a control
round in which every rank reports before any payload moves).

The framework never creates the process groups itself; a :class:`DistributedOwner` runs on groups the engine
made. Two channels:

* **control** (a Gloo group, CPU): bounded canonical JSON (at most 1 MiB per message, never pickled), gathered
  from every rank by :class:`_ControlChannel` (a length round, then a padded byte round);
* **payload** (the data group: NCCL with CUDA tensors -- NVLink / NVSwitch on one node -- or Gloo with CPU
  tensors): point-to-point moves in pieces of at most ``max_wire_bytes``.

``checkpoint(operation, error=..., cancelled=...)`` is the agreement: every rank contributes one record
``{sequence, operation, rank, error, cancelled, details}``; if any rank failed or cancelled, or the ranks are
not at the same step, every rank raises (:class:`PeerFailure`, :class:`CollectiveCancelled`) before the next
payload collective -- so no rank is ever left waiting in a transfer a peer will not join.
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
MAX_DETAIL_BYTES = MAX_CONTROL_BYTES // 2


class PeerFailure(StateError):
    """Some rank of the collective failed (or the transport did); raised on every rank."""


class CollectiveCancelled(PeerFailure):
    """Some rank cancelled the collective; raised on every rank."""


@dataclass(frozen=True)
class KVLayout:
    """How one ``[tokens, kv_heads * head_dim]`` matrix is split over ranks: ``rows`` shards take contiguous
    token ranges (earlier ranks one extra token when uneven), ``heads`` shards take equal head groups."""

    tokens: int
    kv_heads: int
    head_dim: int
    world_size: int = 2

    def __post_init__(self):
        for name in ("tokens", "kv_heads", "head_dim", "world_size"):
            value = getattr(self, name)
            if type(value) is not int or value < 1:
                raise ConfigurationError(f"KV layout {name} must be a positive integer, got {value!r}")
        if self.kv_heads % self.world_size:
            raise ConfigurationError(f"{self.kv_heads} KV heads do not split evenly over {self.world_size} ranks")
        if self.tokens < self.world_size:
            raise ConfigurationError(f"{self.tokens} tokens cannot give each of {self.world_size} ranks a row")

    @property
    def channels(self) -> int:
        return self.kv_heads * self.head_dim

    @property
    def local_channels(self) -> int:
        return self.channels // self.world_size

    def _valid(self, rank: int) -> int:
        if type(rank) is not int or not 0 <= rank < self.world_size:
            raise ConfigurationError(f"rank {rank!r} is not in this {self.world_size}-rank layout")
        return rank

    def rows(self, rank: int) -> slice:
        base, extra = divmod(self.tokens, self.world_size)
        first = self._valid(rank) * base + min(rank, extra)
        return slice(first, first + base + (1 if rank < extra else 0))

    def columns(self, rank: int) -> slice:
        width = self.local_channels
        return slice(self._valid(rank) * width, (rank + 1) * width)

    def shape(self, rank: int, layout: str) -> tuple[int, int]:
        if layout == "rows":
            span_ = self.rows(rank)
            return span_.stop - span_.start, self.channels
        if layout == "heads":
            self._valid(rank)
            return self.tokens, self.local_channels
        raise ConfigurationError(f"layout {layout!r} is neither 'rows' nor 'heads'")


@dataclass
class WireCounters:
    """Application bytes and messages moved by one transport (protocol overheads excluded)."""

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


class _ControlChannel:
    """Gathers one bounded JSON value from every rank over the control group."""

    def __init__(self, owner: "DistributedOwner"):
        self.owner = owner

    def gather(self, value: Any) -> list:
        o = self.owner
        encoded = json.dumps(value, sort_keys=True, separators=(",", ":"), allow_nan=False).encode()
        if len(encoded) > MAX_CONTROL_BYTES:
            raise ConfigurationError(f"a control message of {len(encoded)} bytes exceeds {MAX_CONTROL_BYTES}")
        if o.world_size == 1:
            return [json.loads(encoded)]
        mine = torch.tensor([len(encoded)], dtype=torch.int64)
        sizes = [torch.empty_like(mine) for _ in range(o.world_size)]
        o._run(o.dist.all_gather, sizes, mine, group=o.control_group)
        lengths = [int(s.item()) for s in sizes]
        width = max(lengths)
        if min(lengths) < 0 or width > MAX_CONTROL_BYTES:
            o._broken = True
            raise PeerFailure(f"a peer announced a control message of {width} bytes")
        padded = torch.zeros(width, dtype=torch.uint8)
        padded[:len(encoded)] = torch.frombuffer(bytearray(encoded), dtype=torch.uint8)
        received = [torch.empty_like(padded) for _ in range(o.world_size)]
        o._run(o.dist.all_gather, received, padded, group=o.control_group)
        moved = (8 + width) * (o.world_size - 1)
        o.counters.control_sent_bytes += moved
        o.counters.control_received_bytes += moved
        return [json.loads(bytes(buf[:n].tolist())) for buf, n in zip(received, lengths)]


def _describe(error) -> str | None:
    if error is None:
        return None
    return f"{type(error).__name__}: {error}" if isinstance(error, BaseException) else str(error)


class DistributedOwner:
    """One rank's side of a storage collective domain whose canonical store lives on ``owner_rank``."""

    def __init__(self, group=None, *, control_group=None, owner_rank: int = 0, max_wire_bytes: int = 16 << 20,
                 device="cpu", expected_world_size: int | None = None):
        import torch.distributed as dist

        self.dist = dist
        self.group = group
        self.control_group = group if control_group is None else control_group
        self.initialized = dist.is_available() and dist.is_initialized()
        self.world_size = dist.get_world_size(group) if self.initialized else 1
        self.rank = dist.get_rank(group) if self.initialized else 0
        if type(owner_rank) is not int or not 0 <= owner_rank < self.world_size:
            raise ConfigurationError(f"owner rank {owner_rank!r} is not a rank of the {self.world_size}-rank group")
        if expected_world_size is not None and expected_world_size != self.world_size:
            raise ConfigurationError(f"the storage group has {self.world_size} ranks, the engine's sequence-parallel "
                                     f"group {expected_world_size}")
        if type(max_wire_bytes) is not int or max_wire_bytes < 8:
            raise ConfigurationError("max_wire_bytes is an integer of at least 8")
        self.owner_rank = owner_rank
        self.max_wire_bytes = max_wire_bytes
        self.device = torch.device(device)
        if self.initialized:
            data_backend = str(dist.get_backend(group))
            expected = {"gloo": "cpu", "nccl": "cuda"}.get(data_backend)
            if expected is not None and self.device.type != expected:
                raise ConfigurationError(f"a {data_backend} data group moves {expected} tensors, not "
                                         f"{self.device.type} ones")
            if str(dist.get_backend(self.control_group)) != "gloo":
                raise ConfigurationError("the control group must be a Gloo (CPU) group")
        self.counters = WireCounters()
        self.sequence = 0
        self._thread = threading.get_ident()
        self._broken = False
        self._control = _ControlChannel(self)

    @property
    def is_owner(self) -> bool:
        return self.rank == self.owner_rank

    def _guard(self) -> None:
        if threading.get_ident() != self._thread:
            raise StateError("storage collectives run on the thread that created the transport")
        if self._broken:
            raise PeerFailure("the storage transport failed earlier; open a new session")

    def _global(self, rank: int) -> int:
        return rank if self.group is None else self.dist.get_global_rank(self.group, rank)

    def _run(self, fn, *args, **kwargs):
        """Run one transport call; any failure breaks the domain for good."""
        try:
            with span("transport.collective"):
                return fn(*args, **kwargs)
        except Exception as exc:
            self._broken = True
            raise PeerFailure(f"the storage transport failed in {getattr(fn, '__name__', fn)}: "
                              f"{type(exc).__name__}: {exc}") from exc

    def _all_json(self, value: Any) -> list:
        self._guard()
        return self._control.gather(value)

    # -- agreement ----------------------------------------------------------------------------------------

    def checkpoint(self, operation: str, *, error=None, cancelled: bool = False, details=None) -> list:
        """Every rank reports; a failure, a cancellation or a step mismatch anywhere raises on every rank.
        Returns every rank's ``details``."""
        self._guard()
        message = _describe(error)
        try:
            if len(json.dumps(details, allow_nan=False).encode()) > MAX_DETAIL_BYTES:
                raise ConfigurationError(f"checkpoint details exceed {MAX_DETAIL_BYTES} bytes")
        except Exception as exc:  # noqa: BLE001 - reported through the checkpoint itself
            message, details = f"checkpoint details are not bounded JSON: {exc}", None
        records = self._all_json({"sequence": self.sequence, "operation": str(operation), "rank": self.rank,
                                  "error": message, "cancelled": bool(cancelled), "details": details})
        self.sequence += 1
        self.counters.checkpoints += 1
        steps = {(r["sequence"], r["operation"]) for r in records}
        if len(steps) > 1:
            raise PeerFailure(f"ranks reached different collective steps: {sorted(steps)}")
        if any(r["cancelled"] for r in records):
            raise CollectiveCancelled(f"{operation} was cancelled by rank(s) "
                                      f"{[r['rank'] for r in records if r['cancelled']]}")
        failed = [f"rank {r['rank']}: {r['error']}" for r in records if r["error"] is not None]
        if failed:
            raise PeerFailure(f"{operation} failed -- " + "; ".join(failed))
        return [r["details"] for r in records]

    def owner_call(self, operation: str, function: Callable):
        """Run ``function`` on the owner only; its failure surfaces on every rank."""
        self.checkpoint(f"{operation}:begin")
        result = error = None
        if self.is_owner:
            try:
                result = function()
            except BaseException as exc:  # noqa: BLE001 - agreed below
                error = exc
        try:
            self.checkpoint(f"{operation}:complete", error=error)
        except PeerFailure as failure:
            if error is not None:
                raise failure from error
            raise
        return result

    def broadcast_json(self, value, *, operation: str = "broadcast_json", source: int | None = None):
        """``source``'s JSON value on every rank."""
        source = self.owner_rank if source is None else source
        problem = None
        if not 0 <= source < self.world_size:
            problem = f"JSON source {source} is not a rank"
        elif self.rank == source:
            try:
                json.dumps(value, allow_nan=False)
            except (TypeError, ValueError) as exc:
                problem = exc
        self.checkpoint(operation, error=problem)
        return self._all_json(value if self.rank == source else None)[source]

    # -- payloads -----------------------------------------------------------------------------------------

    def _move(self, tensor: torch.Tensor, source: int, destination: int) -> None:
        """Point-to-point move of a contiguous tensor allocated on both ends, in bounded pieces."""
        self._guard()
        if self.world_size == 1 or source == destination:
            return
        flat = tensor.reshape(-1)
        step = max(1, self.max_wire_bytes // tensor.element_size())
        sending = self.rank == source
        peer = self._global(destination if sending else source)
        for first in range(0, flat.numel(), step):
            piece = flat[first:first + step]
            nbytes = piece.numel() * piece.element_size()
            if sending:
                self._run(self.dist.send, piece, dst=peer, group=self.group)
                self.counters.payload_sent_bytes += nbytes
                self.counters.payload_messages_sent += 1
            elif self.rank == destination:
                self._run(self.dist.recv, piece, src=peer, group=self.group)
                self.counters.payload_received_bytes += nbytes
                self.counters.payload_messages_received += 1

    def gather_matrix(self, local: torch.Tensor, layout: KVLayout, *, source_layout: str,
                      operation: str = "gather_matrix") -> torch.Tensor | None:
        """Every rank's ``rows`` or ``heads`` shard assembled into the canonical ``[tokens, channels]`` matrix
        on the owner (``None`` on the other ranks)."""
        problem = summary = None
        try:
            if layout.world_size != self.world_size:
                raise ConfigurationError(f"a {layout.world_size}-rank layout on a {self.world_size}-rank group")
            if tuple(local.shape) != layout.shape(self.rank, source_layout):
                raise ConfigurationError(f"local shard {tuple(local.shape)} is not this rank's {source_layout} "
                                         f"shard {layout.shape(self.rank, source_layout)}")
            if local.device.type != self.device.type:
                raise ConfigurationError(f"the shard is on {local.device.type}, the transport moves "
                                         f"{self.device.type} tensors")
            if not local.dtype.is_floating_point:
                raise ConfigurationError("KV shards are floating-point tensors")
            summary = {"dtype": str(local.dtype), "layout": source_layout, "geometry": asdict(layout)}
        except Exception as exc:  # noqa: BLE001
            problem = exc
        summaries = self.checkpoint(operation, error=problem, details=summary)
        if any(s != summaries[0] for s in summaries):
            raise PeerFailure("ranks describe their KV shards differently")
        local = local.detach().contiguous()
        canonical = torch.empty((layout.tokens, layout.channels), dtype=local.dtype, device=self.device) \
            if self.is_owner else None
        for source in range(self.world_size):
            if self.rank == source:
                shard = local
            elif self.is_owner:
                shard = torch.empty(layout.shape(source, source_layout), dtype=local.dtype, device=self.device)
            else:
                shard = None
            self.checkpoint(f"{operation}:rank{source}")
            if self.rank in (source, self.owner_rank):
                self._move(shard, source, self.owner_rank)
            if self.is_owner:
                region = canonical[layout.rows(source)] if source_layout == "rows" else \
                    canonical[:, layout.columns(source)]
                region.copy_(shard)
        return canonical

    @contextmanager
    def acquire_columns(self, layout: KVLayout, loader: Callable, *, dtype, operation: str = "acquire_columns"):
        """The owner loads each rank's head columns in turn (``loader(columns)`` returns a tensor or a context
        manager yielding one) and sends them; each rank yields only its own ``[tokens, local_channels]``."""
        problem = None if layout.world_size == self.world_size else "the layout describes another group size"
        plans = self.checkpoint(operation, error=problem, details={"layout": asdict(layout), "dtype": str(dtype)})
        if any(p != plans[0] for p in plans):
            raise PeerFailure("ranks asked for different column layouts or dtypes")
        with ExitStack() as kept:
            mine = None
            for destination in range(self.world_size):
                with ExitStack() as scratch:
                    buffer = failure = None
                    try:
                        if self.is_owner:
                            loaded = loader(layout.columns(destination))
                            holder = kept if destination == self.rank else scratch
                            buffer = holder.enter_context(loaded if hasattr(loaded, "__enter__") else nullcontext(loaded))
                            wanted = layout.shape(destination, "heads")
                            if tuple(buffer.shape) != wanted or buffer.dtype != dtype or not buffer.is_contiguous():
                                raise ConfigurationError(f"the loader returned {tuple(buffer.shape)} {buffer.dtype}, "
                                                         f"not contiguous {wanted} {dtype}")
                        elif self.rank == destination:
                            buffer = torch.empty(layout.shape(destination, "heads"), dtype=dtype, device=self.device)
                    except BaseException as exc:  # noqa: BLE001 - agreed below
                        failure = exc
                    self.checkpoint(f"{operation}:rank{destination}", error=failure)
                    if self.rank in (self.owner_rank, destination):
                        self._move(buffer, self.owner_rank, destination)
                    if self.rank == destination:
                        mine = buffer
            yield mine

    def local_columns(self, layout: KVLayout, loader: Callable, *, dtype, operation: str = "local_columns"):
        with self.acquire_columns(layout, loader, dtype=dtype, operation=operation) as columns:
            return columns.clone()

    def transfer_tensor(self, value, *, source: int, destination: int, operation: str = "transfer_tensor"):
        """``value`` moved from ``source`` to ``destination`` (its shape and dtype travel in the agreement);
        ``None`` on every other rank."""
        problem = description = None
        try:
            if not (0 <= source < self.world_size and 0 <= destination < self.world_size):
                raise ConfigurationError(f"transfer {source} -> {destination} names a rank outside the group")
            if self.rank == source:
                value = value.detach().to(self.device).contiguous()
                description = {"shape": list(value.shape), "dtype": str(value.dtype).rpartition(".")[2]}
        except Exception as exc:  # noqa: BLE001
            problem = exc
        described = self.checkpoint(operation, error=problem, details=description)[source]
        buffer = None
        if self.rank == source:
            buffer = value
        elif self.rank == destination:
            buffer = torch.empty(described["shape"], dtype=getattr(torch, described["dtype"]), device=self.device)
        self.checkpoint(f"{operation}:allocated")
        if self.rank in (source, destination):
            self._move(buffer, source, destination)
        return buffer if self.rank == destination else None


__all__ = ["MAX_CONTROL_BYTES", "CollectiveCancelled", "DistributedOwner", "KVLayout", "PeerFailure", "WireCounters"]
