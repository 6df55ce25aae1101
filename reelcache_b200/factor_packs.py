"""FP16 factor packs of the SVD-only baseline representation (the counterpart of reference
reelcache/factor_packs.py:68-720: ``FactorRestorer`` :462, ``FactorLineageRestorer`` :673).

A ``svd`` node stores, per matrix, its FP16 coefficients ``P[N, r]`` in one ``reelcache.factor_pack.v1``
packet (tiles with offsets and SHA-256 digests; :class:`reelcache_b200.codecs.FactorPack`) and its basis rows
in the shared basis-version store. Reconstruction is ``P @ Q``: :class:`FactorRestorer` gives dense matrices
(FP32-accurate products on CUDA), :class:`FactorLineageRestorer` restores a node's attended history into
native caches through the fused sm_100a restore kernel (float coefficients: the hi/lo-split FP16 operand,
RoPE and the cast in the epilogue), with the :class:`~reelcache_b200.archive_restore.LineageRestorer`
contract.
"""

from __future__ import annotations

from collections import OrderedDict
from typing import Any

import numpy as np
import torch

from .archive_restore import JobLineageRestorer
from .errors import UnsupportedError
from .lineage import LineageRuntime
from .types import MatrixKey


COEFFICIENT_DTYPE = "float16"


def factor_codec(spec) -> dict[str, Any]:
    """The codec header a factor pack records for an ``svd`` spec (the run-local encoder path dropped)."""
    if spec.kind != "svd":
        raise UnsupportedError("factor packs hold svd (SVD-only) matrices")
    codec = spec.to_dict()
    codec.pop("ffmpeg_path", None)
    return codec


def is_factor_pack(value: Any) -> bool:
    """Whether ``value`` (an encoded packet or its metadata) is a ``reelcache.factor_pack.v1`` pack."""
    from .codecs import FACTOR_PACK_SCHEMA
    metadata = getattr(value, "metadata", value)
    return isinstance(metadata, dict) and metadata.get("schema") == FACTOR_PACK_SCHEMA


def validate_factor_pack(encoded, *, verify: bool = False) -> list[dict]:
    """The tile table of a factor pack after checking its layout (contiguous, non-overlapping tiles whose byte
    counts match ``tokens x rank`` FP16 values) and, with ``verify``, each tile's SHA-256."""
    import hashlib

    from .errors import IntegrityError
    if not is_factor_pack(encoded):
        raise IntegrityError("not a factor pack")
    factors = encoded.payloads["factors"]
    metadata = encoded.metadata
    cursor = 0
    for index, tile in enumerate(metadata["tiles"]):
        tokens = tile["context"]["frames"] * tile["context"]["height"] * tile["context"]["width"]
        if (tile["tile"] != index or tile["offset"] != cursor or tile["bytes"] != tokens * int(tile["rank"]) * 2):
            raise IntegrityError(f"factor pack tile {index} is inconsistent with its table")
        if verify and hashlib.sha256(factors[cursor:cursor + tile["bytes"]]).hexdigest() != tile["sha256"]:
            raise IntegrityError(f"factor pack tile {index} fails its hash")
        cursor += tile["bytes"]
    if cursor != int(metadata["bytes"]) or len(factors) != cursor:
        raise IntegrityError("factor pack size differs from its tiles")
    return list(metadata["tiles"])


class FactorTile:
    """One prepared tile of a factor pack: its entry, rank, and FP16 coefficients ``[tokens, rank]`` (a view of the
    packet's staging buffer)."""

    __slots__ = ("entry", "rank", "values", "basis")

    def __init__(self, entry, rank: int, values: torch.Tensor, basis: dict):
        self.entry, self.rank, self.values, self.basis = entry, rank, values, basis


def prepare_factor_packet(encoded, *, verify: bool = False, pin_memory: bool = False,
                          device: Any = None) -> list[FactorTile]:
    """Every tile of a factor pack as a view of ONE buffer holding the packet's coefficients (pinned host memory,
    or copied once to ``device``)."""
    from .codecs import _entry_of
    tiles = validate_factor_pack(encoded, verify=verify)
    raw = torch.frombuffer(bytearray(encoded.payloads["factors"]), dtype=torch.uint8)
    if pin_memory:
        raw = raw.pin_memory()
    if device is not None:
        raw = raw.to(device, non_blocking=pin_memory)
    out = []
    for tile in tiles:
        rank = int(tile["rank"])
        values = raw[tile["offset"]:tile["offset"] + tile["bytes"]].view(torch.float16).view(-1, rank)
        out.append(FactorTile(_entry_of(tile["entry"]), rank, values, tile["basis"]))
    return out


def decode_factor_pack(encoded, bases: dict, *, keys=None, device: Any = "cpu",
                       dtype: torch.dtype = torch.float32) -> dict:
    """``{entry: P @ Q}`` of the selected tiles (default: all); ``bases[entry]`` gives each tile's FP16 rows
    (the record's basis-version prefix), checked against the tile's basis digest."""
    import hashlib

    from .errors import IntegrityError
    wanted = None if keys is None else set(keys)
    out = {}
    for tile in prepare_factor_packet(encoded, verify=True, device=device):
        if wanted is not None and tile.entry not in wanted:
            continue
        rows = bases[tile.entry].to(torch.float16).contiguous()
        if rows.shape[0] != tile.rank:
            raise IntegrityError(f"basis of {tile.entry} has {rows.shape[0]} rows, the tile rank is {tile.rank}")
        if "sha256" in tile.basis and hashlib.sha256(rows.cpu().numpy().tobytes()).hexdigest() != tile.basis["sha256"]:
            raise IntegrityError(f"basis of {tile.entry} differs from the tile's digest")
        out[tile.entry] = (tile.values.float() @ rows.to(tile.values.device).float()).to(dtype)
    return out


class FactorRestorer:
    """Dense reconstructions of ``svd`` records (decoded packs cached LRU under a byte budget)."""

    def __init__(self, runtime: LineageRuntime, device="cpu", *, budget_bytes: int = 4 << 30):
        self.runtime = runtime
        self.device = torch.device(device)
        self.budget = budget_bytes
        self._packs: OrderedDict = OrderedDict()
        self._bytes = 0

    def pack(self, packet_ref: str):
        hit = self._packs.get(packet_ref)
        if hit is not None:
            self._packs.move_to_end(packet_ref)
            return hit
        _, pack = self.runtime.factor_pack(packet_ref)
        self._packs[packet_ref] = pack
        self._bytes += pack.raw.nbytes
        while self._bytes > self.budget and len(self._packs) > 1:
            _, old = self._packs.popitem(last=False)
            self._bytes -= old.raw.nbytes
        return pack

    def factors(self, record) -> np.ndarray:
        """FP16 ``[tokens, rank]`` coefficients of one record."""
        if record.codec.kind != "svd":
            raise UnsupportedError("factor restores take svd records")
        return self.pack(record.packet_ref).factors(record.decision["packet"]["tile"])

    def reconstruct(self, record_ref: str, *, dtype: torch.dtype = torch.float32) -> torch.Tensor:
        """Dense ``[tokens, C]`` pre-RoPE matrix ``P @ Q`` of one record."""
        from .exact_blas import mm
        record = self.runtime.load_record(record_ref)
        p = torch.from_numpy(self.factors(record).astype(np.float32)).to(self.device)
        q = self.runtime.basis.assemble(record.basis_version_ref, record.rank_view).to(self.device).float()
        return mm(p, q).to(dtype)

    def history(self, node_ref: str, key: MatrixKey, *, stream: str | None = None, ranges=None) -> torch.Tensor:
        """Dense history of one matrix over the node's attended ranges."""
        parts = []
        for piece in self.runtime.resolve_history(node_ref, ranges):
            full = self.reconstruct(piece.record(key, stream))
            parts.append(full[piece.offset:piece.offset + piece.token_end - piece.token_start])
        if not parts:
            return torch.zeros((0, self.runtime.model.channels_for(key)), device=self.device)
        return torch.cat(parts)


class FactorLineageRestorer(JobLineageRestorer):
    """Restores ``svd`` node histories into native caches with the fused restore kernel."""

    kinds = ("svd",)

    def __init__(self, runtime: LineageRuntime, device, *, budget_bytes: int = 4 << 30):
        super().__init__(runtime, device)
        self.factors = FactorRestorer(runtime, device, budget_bytes=budget_bytes)
        self._device_packs: dict = {}
        self._bounds: dict = {}

    def _prepare(self, pieces) -> None:
        """Each factor pack the history needs goes to the device once per restore (one pinned H2D copy)."""
        self._device_packs = {}
        for piece in pieces:
            for _, record_ref in piece.entry.records:
                record = self.runtime.load_record(record_ref)
                if record.packet_ref in self._device_packs:
                    continue
                pack = self.factors.pack(record.packet_ref)
                raw = torch.from_numpy(np.array(pack.raw, copy=True))
                if self.device.type == "cuda":
                    raw = raw.pin_memory().to(self.device, non_blocking=True)
                    self.stats_["h2d_bytes"] += raw.numel()
                self._device_packs[record.packet_ref] = raw

    def _source(self, piece, record, rows: slice):
        from . import restore_kernels as rk
        pack = self.factors.pack(record.packet_ref)
        index = record.decision["packet"]["tile"]
        tile = pack.tiles[index]
        rank = int(tile["rank"])
        raw = self._device_packs[record.packet_ref]
        values = raw[tile["offset"]:tile["offset"] + tile["bytes"]].view(torch.float16).view(-1, rank)[rows]
        key = (record.packet_ref, index)
        if key not in self._bounds:  # bound of the whole tile (covers every row range), computed once on the host
            self._bounds[key] = float(np.abs(pack.factors(index).astype(np.float32)).max(initial=0.0))
        return rk.CoefficientSource(values, bound=self._bounds[key]), self._basis(record)

    def stats(self) -> dict[str, Any]:
        return {**self.stats_, "packs": len(self.factors._packs), "pack_bytes": self.factors._bytes}


__all__ = ["FactorLineageRestorer", "FactorRestorer"]
