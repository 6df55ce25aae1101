"""Context-parallel conditioning-cache archive with row-sharded factor ownership and per-rank raw tiers (the
counterpart of reference reelcache/integrations/longcat_factor_shard.py:1-30 ``RowShardedCacheArchive`` and
reelcache_sglang_models/longcat_video/cp_tiers.py:1-30 ``TieredRowArchive``).

Under context parallelism every rank holds only its token rows of each matrix of a cache epoch (LongCat: 48 layers
x K/V of ``[T, 4096]``).

* :class:`RowShardedCacheArchive`: **capture** keeps the rank's rows on the host; **flush** (collective) archives
  every pending epoch matrix by matrix -- the rows are gathered to the fit owner, which fits the rank reaching the
  energy target (FP64 Gram eigh) and scatters the factor blocks to their owners (whole-matrix owners alternating
  by layer and target, :class:`FactorShardSpec`); each owner writes its blocks as one fragment pack into its own
  store (:class:`OwnerFactorStore`). Publication is two-phase: every rank stages its fragment, a checkpoint agrees,
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
from ..serialization import deserialize_tensors, serialize_tensors
from ..types import MatrixKey
from .distributed import DistributedOwner, PeerFailure
from .factor_sharding import FactorShardDomain, FactorShardSpec

FRAGMENT_SCHEMA = "reelcache.row_shard_fragment.v1"
REF_PREFIX = "cp_cache/epochs/"
TIERS = ("host_raw", "compressed")


def _label(key: MatrixKey) -> str:
    return f"{key.layer}:{key.target}"


class IndexedNativeOwners:
    """Native owners by explicit token indices (a CP rank's spatial block of every frame)."""

    kind = "rows"

    def __init__(self, token_indices: list[torch.Tensor], channels: int):
        self.token_indices = [idx.long() for idx in token_indices]
        self.channels = channels

    def rows(self, rank: int) -> torch.Tensor:
        return self.token_indices[rank]

    def columns(self, rank: int) -> slice:
        return slice(0, self.channels)


class OwnerFactorStore:
    """One rank's factor fragments, one pack per epoch, published by ref (two-phase)."""

    def __init__(self, store, rank: int):
        self.store, self.rank = store, rank

    def ref(self, epoch_id: str) -> str:
        return f"{REF_PREFIX}{epoch_id}/rank{self.rank}"

    def stage(self, epoch_id: str, blocks: Mapping[MatrixKey, list], ranks: Mapping[MatrixKey, int]) -> str:
        tensors = {}
        for key, items in blocks.items():
            for rows, p, q in items:
                tensors[f"{_label(key)}:{rows.start}:{rows.stop}:P"] = p.detach().cpu().contiguous()
                tensors[f"{_label(key)}:{rows.start}:{rows.stop}:Q"] = q.detach().cpu().contiguous()
        pack = self.store.put(serialize_tensors(tensors))
        return self.store.put_manifest({"schema": FRAGMENT_SCHEMA, "epoch": epoch_id, "rank": self.rank,
                                        "ranks": {_label(k): int(v) for k, v in ranks.items()}, "pack": pack},
                                       references=[pack])

    def publish(self, epoch_id: str, manifest: str) -> None:
        self.store.set_ref(self.ref(epoch_id), manifest)

    def load(self, epoch_id: str, device) -> tuple[dict, dict]:
        manifest_ref = self.store.get_ref(self.ref(epoch_id))
        if manifest_ref is None:
            raise StateError(f"epoch {epoch_id} has no fragment on rank {self.rank}")
        manifest = self.store.get_manifest(manifest_ref)
        if manifest.get("schema") != FRAGMENT_SCHEMA:
            raise IntegrityError("not a row-shard fragment")
        tensors = deserialize_tensors(self.store.get(manifest["pack"]), device=device)
        blocks: dict[MatrixKey, list] = {}
        for name, value in tensors.items():
            layer, target, start, stop, which = name.split(":")
            if which != "P":
                continue
            key = MatrixKey(int(layer), target)
            q = tensors[f"{layer}:{target}:{start}:{stop}:Q"]
            blocks.setdefault(key, []).append((slice(int(start), int(stop)), value, q))
        ranks = {MatrixKey(int(k.split(":")[0]), k.split(":")[1]): v for k, v in manifest["ranks"].items()}
        return blocks, ranks


@dataclass
class _Pending:
    epoch_id: str
    rows: dict            # key -> this rank's host rows [local_tokens, C]


class RowShardedCacheArchive:
    """Row-sharded CP cache archive (see the module docstring). ``token_indices[r]`` lists rank ``r``'s token
    rows of the canonical ``[tokens, channels]`` matrices; ``store`` is this rank's own object store."""

    def __init__(self, transport: DistributedOwner, store, token_indices: list[torch.Tensor], *, tokens: int,
                 channels: int, energy_target: float = 0.98, max_rank: int | None = None, fit_owner: int = 0,
                 spec: FactorShardSpec | None = None):
        if len(token_indices) != transport.world_size:
            raise ConfigurationError("one token index list per rank")
        covered = torch.cat([idx.long() for idx in token_indices]).sort().values
        if covered.numel() != tokens or not torch.equal(covered, torch.arange(tokens)):
            raise ConfigurationError("the ranks' token rows must partition the matrix rows")
        if not 0.0 < energy_target <= 1.0:
            raise ConfigurationError("energy_target must lie in (0, 1]")
        self.transport = transport
        self.tokens, self.channels = tokens, channels
        self.natives = IndexedNativeOwners(token_indices, channels)
        self.spec = spec or FactorShardSpec(transport.world_size)
        self.energy_target = energy_target
        self.max_rank = max_rank
        self.fit_owner = fit_owner
        self.fragments = OwnerFactorStore(store, transport.rank)
        self.pending: OrderedDict[str, _Pending] = OrderedDict()
        self.archived: set[str] = set()
        self.records: list[dict] = []

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

    def _rank_for(self, canonical: torch.Tensor) -> int:
        x = canonical.double()
        values = torch.linalg.eigvalsh(x.t() @ x).flip(0).clamp_min(0)
        total = float(values.sum())
        if total == 0.0:
            return 1
        cumulative = torch.cumsum(values, 0) / total
        rank = int(torch.searchsorted(cumulative, torch.tensor(self.energy_target, dtype=torch.float64))) + 1
        rank = min(rank, self.channels, self.tokens)
        return min(rank, self.max_rank) if self.max_rank else rank

    def flush(self) -> list[str]:
        """Collective: archive every pending epoch (two-phase); returns the epochs archived by this call."""
        t = self.transport
        done = []
        epochs = t.broadcast_json(list(self.pending), operation="row_archive:epochs", source=self.fit_owner)
        for epoch_id in epochs:
            started = time.perf_counter()
            domain = FactorShardDomain(t, self.spec, self.natives)
            pending = self.pending.get(epoch_id)
            error = None if pending is not None else f"epoch {epoch_id} was not captured on rank {t.rank}"
            keys = t.broadcast_json(sorted(_label(k) for k in pending.rows) if pending else [],
                                    operation=f"row_archive:{epoch_id}:keys", source=self.fit_owner)
            t.checkpoint(f"row_archive:{epoch_id}:captured", error=error)
            for label in keys:
                layer, target = label.split(":")
                key = MatrixKey(int(layer), target)
                canonical = self._gather(key, pending.rows[key], f"row_archive:{epoch_id}")
                rank = self._rank_for(canonical) if t.rank == self.fit_owner else 0
                domain.fit_and_scatter(key, canonical, rank, fit_owner=self.fit_owner,
                                       operation=f"row_archive:{epoch_id}:{label}")
            staged, error = None, None
            try:
                staged = self.fragments.stage(epoch_id, domain.factors, domain.ranks)
            except Exception as exc:  # noqa: BLE001 - phase one failed here: every rank discards
                error = exc
            t.checkpoint(f"row_archive:{epoch_id}:staged", error=error)   # raises on every rank on failure
            self.fragments.publish(epoch_id, staged)
            t.checkpoint(f"row_archive:{epoch_id}:published")
            self.pending.pop(epoch_id, None)
            self.archived.add(epoch_id)
            self.records.append({"epoch": epoch_id, "matrices": len(keys), "seconds": time.perf_counter() - started,
                                 "ranks": {_label(k): v for k, v in domain.ranks.items()}})
            done.append(epoch_id)
        return done

    def restore(self, epoch_id: str, *, dtype=torch.float32) -> dict[MatrixKey, torch.Tensor]:
        """Collective: this rank's native rows of every matrix of an archived epoch."""
        t = self.transport
        error = None
        blocks, ranks = {}, {}
        try:
            blocks, ranks = self.fragments.load(epoch_id, t.device)
        except Exception as exc:  # noqa: BLE001
            error = exc
        t.checkpoint(f"row_restore:{epoch_id}:loaded", error=error)
        all_ranks = t.broadcast_json({_label(k): v for k, v in ranks.items()},
                                     operation=f"row_restore:{epoch_id}:ranks", source=self.fit_owner)
        domain = FactorShardDomain(t, self.spec, self.natives)
        domain.factors = blocks
        out = {}
        for label in sorted(all_ranks):
            layer, target = label.split(":")
            key = MatrixKey(int(layer), target)
            domain.ranks[key] = all_ranks[label]
            out[key] = domain.reconstruct(key, mode="factors", dtype=dtype)
        return out


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


__all__ = ["IndexedNativeOwners", "OwnerFactorStore", "RowEntry", "RowShardedCacheArchive", "TieredRowArchive"]
