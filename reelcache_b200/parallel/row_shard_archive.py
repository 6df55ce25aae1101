"""Context-parallel conditioning-cache archive with row-sharded factor ownership and per-rank raw tiers (the
counterpart of reference reelcache/integrations/longcat_factor_shard.py:1-30 ``RowShardedCacheArchive`` and
reelcache_sglang_models/longcat_video/cp_tiers.py:1-30 ``TieredRowArchive``).

Under context parallelism every rank holds only its token rows of each matrix of a cache epoch (LongCat: 48 layers
x K/V of ``[T, 4096]``).

* :class:`RowShardedCacheArchive`: **capture** keeps the rank's rows on the host; **flush** (collective) archives
  every pending epoch matrix by matrix -- the rows are gathered to the fit owner, which fits the rank reaching the
  energy target (FP64 Gram eigh) and scatters the factor blocks to their owners (whole-matrix owners alternating
  by layer and target, :class:`~.factor_sharding.FactorShardSpec`); each owner writes its blocks as one fragment
  pack into its own store (:class:`~.factor_sharding.OwnerFactorStore`). Publication is two-phase: every rank stages its fragment, a checkpoint agrees,
  then every rank sets its epoch ref; a failure anywhere discards every staged fragment. **restore** (collective)
  loads the fragments and delivers every rank its native rows (``P[rows] @ Q`` with the pieces moved to the
  native owner).
* :class:`TieredRowArchive`: keeps each rank's host copy of its rows as a ``host_raw`` entry (evictable, least
  recently used first within a byte budget, only after its epoch is published); **install** agrees on one tier
  for the whole epoch: all ranks report the tiers they hold, take the best tier available on every rank, stage and
  verify it (preflight), agree again and install -- or all roll back to the compressed archive together. A rank
  can neither block in a collective its peers skip nor install a tier its peers do not.
"""

from __future__ import annotations

import threading
import time
from collections import OrderedDict
from dataclasses import dataclass, field
from typing import Any, Mapping

import torch

from ..errors import ConfigurationError, IntegrityError, StateError
from ..types import MatrixKey, ModelIdentity, TensorContext
from .distributed import DistributedOwner, KVLayout, PeerFailure
from .factor_sharding import FactorShardDomain, NativeOwners, OwnerFactorStore, OwnershipPolicy

TIERS = ("host_raw", "compressed")
DOMAIN = "cp_cache"


def _label(key: MatrixKey) -> str:
    return f"{key.layer}:{key.target}"


@dataclass
class _Pending:
    epoch_id: str
    rows: dict            # key -> this rank's host rows [local_tokens, C]


class RowShardedCacheArchive:
    """Row-sharded CP cache archive (see the module docstring). ``token_indices[r]`` lists rank ``r``'s token
    rows of the canonical ``[tokens, channels]`` matrices; ``store`` is this rank's own object store, which
    holds this rank's fragment packs (``svd``: exact FP32 coefficients) and basis segments under
    ``factor_shard/cp_cache/<epoch>/...``."""

    def __init__(self, transport: DistributedOwner, store, token_indices: list[torch.Tensor], *, tokens: int,
                 channels: int, energy_target: float = 0.98, max_rank: int | None = None, fit_owner: int = 0,
                 policy: OwnershipPolicy | None = None, kind: str = "svd", model: ModelIdentity | None = None):
        world = transport.world_size
        if len(token_indices) != world:
            raise ConfigurationError("one token index list per rank")
        if not 0.0 < energy_target <= 1.0:
            raise ConfigurationError("energy_target must lie in (0, 1]")
        if channels % world:
            raise ConfigurationError("row shards describe channels divisible by the ranks")
        self.transport = transport
        self.tokens, self.channels = tokens, channels
        # the head split of this layout is bookkeeping only: row owners keep every channel
        layout = KVLayout(tokens=tokens, kv_heads=world, head_dim=channels // world, world_size=world)
        self.natives = NativeOwners(layout, "rows", [idx.long().tolist() for idx in token_indices])
        self.energy_target = energy_target
        self.max_rank = max_rank
        self.fit_owner = fit_owner
        self.kind = kind
        self.model = model or ModelIdentity("cp-row-cache", "row-shards", 4096, channels, "BTHD", "float32")
        self.fragments = OwnerFactorStore(store, transport.rank, world, domain=DOMAIN)
        self.domain = FactorShardDomain(transport, device=transport.device, store=self.fragments,
                                        policy=policy or OwnershipPolicy(world))
        self.pending: OrderedDict[str, _Pending] = OrderedDict()
        self.archived: set[str] = set()
        self.records: list[dict] = []

    def _context(self, key: MatrixKey) -> TensorContext:
        return TensorContext(self.model, key, 0, 1, 1, self.tokens, "pre_rope" if key.target == "K" else "none")

    def capture(self, epoch_id: str, rows: Mapping[MatrixKey, torch.Tensor]) -> None:
        """Keep this rank's rows of one epoch (host copies) for the next :meth:`flush`."""
        local = self.natives.rows(self.transport.rank).numel()
        for key, value in rows.items():
            if tuple(value.shape) != (local, self.channels):
                raise ConfigurationError(f"{key}: expected this rank's [{local}, {self.channels}] rows")
        self.pending[epoch_id] = _Pending(epoch_id, {k: v.detach().to("cpu", copy=True) for k, v in rows.items()})

    def _gather(self, key: MatrixKey, local: torch.Tensor, operation: str) -> torch.Tensor | None:
        t = self.transport
        canonical = torch.empty((self.tokens, self.channels), dtype=local.dtype) if t.rank == self.fit_owner else None
        for source in range(t.world_size):
            piece = local if t.rank == source else None
            piece = t.transfer_tensor(piece, source=source, destination=self.fit_owner,
                                      operation=f"{operation}:{_label(key)}:{source}")
            if t.rank == self.fit_owner:
                canonical[self.natives.rows(source)] = piece
        return canonical

    def flush(self) -> list[str]:
        """Collective: archive every pending epoch -- gather each matrix to the fit owner, fit it there (the
        smallest rank reaching the energy target), scatter the blocks to their owners, then publish the epoch's
        fragments in two phases (all owners or none). Returns the epochs archived by this call."""
        t = self.transport
        done = []
        epochs = t.broadcast_json(list(self.pending), operation="row_archive:epochs", source=self.fit_owner)
        for epoch_id in epochs:
            started = time.perf_counter()
            pending = self.pending.get(epoch_id)
            error = None if pending is not None else f"epoch {epoch_id} was not captured on rank {t.rank}"
            keys = t.broadcast_json(sorted(_label(k) for k in pending.rows) if pending else [],
                                    operation=f"row_archive:{epoch_id}:keys", source=self.fit_owner)
            t.checkpoint(f"row_archive:{epoch_id}:captured", error=error)
            shards = {}
            for label in keys:
                layer, target = label.split(":")
                key = MatrixKey(int(layer), target)
                canonical = self._gather(key, pending.rows[key], f"row_archive:{epoch_id}")
                shards.update(self.domain.fit_and_scatter(
                    [key], {key: canonical} if canonical is not None else None, {key: self._context(key)},
                    energy=self.energy_target, fit_owner=self.fit_owner, max_rank=self.max_rank,
                    operation=f"row_archive:{epoch_id}:{label}"))
            self.domain.publish_node(epoch_id, shards, kind=self.kind)
            self.pending.pop(epoch_id, None)
            self.archived.add(epoch_id)
            self.records.append({"epoch": epoch_id, "matrices": len(keys), "seconds": time.perf_counter() - started,
                                 "ranks": {_label(k): s.spec.rank_view for k, s in shards.items()}})
            done.append(epoch_id)
        return done

    def restore(self, epoch_id: str, *, dtype=torch.float32) -> dict[MatrixKey, torch.Tensor]:
        """Collective: this rank's native rows of every matrix of an archived epoch (owners send their
        coefficient rows and basis rows to each native owner, which multiplies)."""
        error, shards = None, {}
        try:
            node_map = self.domain.node_map(epoch_id)
            shards = self.domain.load_node(node_map, quantized=False)
        except Exception as exc:  # noqa: BLE001 - agreed before the reconstruction's payloads
            error = exc
        self.transport.checkpoint(f"row_restore:{epoch_id}:loaded", error=error)
        return self.domain.reconstruct(shards, self.natives, mode="factors", dtype=dtype,
                                       operation=f"row_restore:{epoch_id}")


@dataclass(eq=False)
class RowEntry:
    epoch_id: str
    rows: dict
    nbytes: int
    published: bool = False
    last_used: float = field(default_factory=time.monotonic)


class TieredRowArchive:
    """Per-rank ``host_raw`` entries in front of a :class:`RowShardedCacheArchive` (module docstring)."""

    def __init__(self, archive: RowShardedCacheArchive, *, host_raw_budget_bytes: int = 8 << 30):
        self.archive = archive
        self.budget = host_raw_budget_bytes
        self.entries: OrderedDict[str, RowEntry] = OrderedDict()
        self.last_restore_tier: dict | None = None
        self._lock = threading.Lock()

    def capture(self, epoch_id: str, rows: Mapping[MatrixKey, torch.Tensor]) -> None:
        self.archive.capture(epoch_id, rows)
        host = self.archive.pending[epoch_id].rows  # the archive's host copy: no second copy
        with self._lock:
            self.entries[epoch_id] = RowEntry(epoch_id, host, sum(v.numel() * v.element_size() for v in host.values()))

    def flush(self) -> list[str]:
        done = self.archive.flush()
        with self._lock:
            for epoch_id in done:
                if epoch_id in self.entries:
                    self.entries[epoch_id].published = True
            self._evict()
        return done

    def _evict(self) -> None:
        total = sum(e.nbytes for e in self.entries.values())
        for epoch_id in sorted(self.entries, key=lambda e: self.entries[e].last_used):
            if total <= self.budget:
                break
            entry = self.entries[epoch_id]
            if entry.published:                       # unpublished entries are flush sources: never evicted
                total -= entry.nbytes
                del self.entries[epoch_id]

    def install(self, epoch_id: str, *, fail_preflight: bool = False) -> tuple[str, dict[MatrixKey, torch.Tensor]]:
        """Collective: one tier for the whole epoch on every rank (``fail_preflight`` injects a local staging
        failure on this rank, which rolls every rank back)."""
        t = self.archive.transport
        started = time.perf_counter()
        with self._lock:
            entry = self.entries.get(epoch_id)
        mine = ["host_raw"] if entry is not None else []
        if epoch_id in self.archive.archived:
            mine.append("compressed")
        offered = t.checkpoint(f"tier:{epoch_id}:offer", details=mine)
        common = [tier for tier in TIERS if all(tier in rows for rows in offered)]
        rollback = False
        if common and common[0] == "host_raw":
            staged, error = None, None
            try:
                if fail_preflight:
                    raise IntegrityError("injected preflight failure")
                staged = {k: v.clone() for k, v in entry.rows.items()}
                local = self.archive.natives.rows(t.rank).numel()
                if any(tuple(v.shape) != (local, self.archive.channels) for v in staged.values()):
                    raise IntegrityError("staged rows differ from this rank's native rows")
            except Exception as exc:  # noqa: BLE001 - agreed below; every rank falls back together
                error = exc
            try:
                t.checkpoint(f"tier:{epoch_id}:preflight", error=error)
                entry.last_used = time.monotonic()
                self.last_restore_tier = {"tier": "host_raw", "rollback": False,
                                          "bytes": entry.nbytes, "seconds": time.perf_counter() - started}
                return "host_raw", staged
            except PeerFailure:
                rollback = True
                common = [tier for tier in common if tier != "host_raw"]
        if not common:
            raise StateError(f"epoch {epoch_id} is held by no tier on every rank")
        rows = self.archive.restore(epoch_id)
        self.last_restore_tier = {"tier": "compressed_cold", "rollback": rollback,
                                  "bytes": sum(v.numel() * v.element_size() for v in rows.values()),
                                  "seconds": time.perf_counter() - started}
        return "compressed", rows


__all__ = ["RowEntry", "RowShardedCacheArchive", "TieredRowArchive"]
