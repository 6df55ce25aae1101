"""Factor sharding: non-replicated ownership of the low-rank factors of archived matrices (the counterpart of
reference reelcache/factor_sharding.py; behaviour from its design notes, lines 1-66).

A restored matrix is ``A = P Q = sum_s P_s Q_s`` over blocks of basis rows ``s``. Every block has one owner
rank that stores (and decodes) only its coefficient columns ``P_s`` and basis rows ``Q_s``; nothing is
permanently replicated. Three pieces of state describe it:

* :class:`FactorShardSpec` -- per matrix: the basis version's cumulative row boundaries, the owner of every
  ``block_rows``-row block (``block_rows >= channels``: one block, the default whole-matrix ownership), and the
  rank view the coefficients use. Appended rows (augmentation) keep every existing row's owner.
* :class:`NativeOwners` -- the restore target: head (column) shards as under Ulysses, or token-row shards
  (context parallelism, explicit row sets such as a 2-D spatial split).
* :class:`ShardedNodeMap` -- per node: every matrix's spec and context, each owner's fragment pack and the
  content-addressed basis segments it stores (:class:`OwnerFactorStore`).

:class:`FactorShardDomain` runs the collective operations over a control transport
(:class:`~.distributed.DistributedOwner`, Gloo) and a payload group: the owner-fit archival path
(``fit_and_scatter``), two-phase publication (``publish_node``), ``load_node`` and ``reconstruct``.
``reconstruct`` has three modes: ``"factors"`` (point-to-point rounds ship coefficient rows and basis columns to
each native owner, which multiplies), ``"partials"`` (each owner multiplies its block for every destination;
a reduce-scatter sums them) and -- on CUDA, for 8-bit coefficient shards -- ``"fused"``: the owners' factors sit
in symmetric memory and each native owner's restore kernels load them over NVLink
(:mod:`.sp_restore`), with no collective call at all. Every payload phase is preceded by an agreed
checkpoint, so a failure on one rank surfaces on all of them before any payload moves.

Gram accumulation over token-row shards is exact (:func:`row_shard_gram`); over head/channel shards it drops the
cross-channel blocks and is rejected.
"""

from __future__ import annotations

import hashlib
import json
import math
from dataclasses import dataclass, field
from typing import Any, Callable, Iterable, Mapping, Sequence

import numpy as np
import torch

from ..errors import ConfigurationError, IntegrityError, StateError, UnsupportedError
from ..types import MatrixKey, TensorContext, canonical_digest, entry_key, entry_parts
from .distributed import CollectiveCancelled, DistributedOwner, KVLayout, PeerFailure

SPEC_SCHEMA = "reelcache.factor_shard_spec.v1"
FRAGMENT_SCHEMA = "reelcache.factor_fragment_pack.v1"
NODE_MAP_SCHEMA = "reelcache.factor_shard_node_map.v1"
REF_PREFIX = "factor_shard/"
PLAN_BLOCK_ROWS = 32             # the rank method's bucket: the finer ownership grid (an ablation)
MODES = ("factors", "partials", "fused")
FRAGMENT_KINDS = ("svd", "svd_hevc")
EXCHANGE_BYTES = 64 << 20        # coefficient bytes one "factors" round may carry per peer and matrix


def _check(condition: bool, message: str, error=ConfigurationError) -> None:
    if not condition:
        raise error(message)


def _count(value, name: str, minimum: int = 0) -> int:
    _check(type(value) is int and value >= minimum, f"{name}: expected an int >= {minimum}, got {value!r}")
    return value


def entry_json(entry) -> dict:
    key, stream = entry_parts(entry)
    out = {"key": key.to_dict()}
    if stream is not None:
        out["stream"] = stream
    return out


def entry_from_json(data: Mapping[str, Any]):
    try:
        key = MatrixKey.from_dict(data["key"])
    except (KeyError, TypeError) as exc:
        raise ConfigurationError("a factor-shard entry names a matrix key") from exc
    stream = data.get("stream")
    return key if stream is None else entry_key((key, stream))


def entry_name(entry) -> str:
    key, stream = entry_parts(entry)
    return f"{key.layer}:{key.target}" if stream is None else f"{key.layer}:{key.target}:{stream}"


def entry_sort_key(entry):
    key, stream = entry_parts(entry)
    return (stream or "", key.layer, key.target)


def rotation_of(entry, world: int) -> int:
    """First owner of a matrix: whole matrices alternate over layers, V one rank after K."""
    key, _ = entry_parts(entry)
    return (key.layer + (1 if key.target == "V" else 0)) % world


def _join(spans: Iterable[tuple[int, int]]) -> tuple[tuple[int, int], ...]:
    out: list[list[int]] = []
    for a, b in sorted(s for s in spans if s[0] < s[1]):
        if out and out[-1][1] == a:
            out[-1][1] = b
        else:
            out.append([a, b])
    return tuple((a, b) for a, b in out)


def span_rows(spans) -> int:
    return sum(b - a for a, b in spans)


def span_index(spans, device=None) -> torch.Tensor:
    parts = [torch.arange(a, b, dtype=torch.long, device=device) for a, b in spans]
    return torch.cat(parts) if parts else torch.empty(0, dtype=torch.long, device=device)


# ---------------------------------------------------------------------------------------------------------
# Ownership of one matrix's basis rows
# ---------------------------------------------------------------------------------------------------------

@dataclass(frozen=True)
class FactorShardSpec:
    """Who owns which basis rows of one matrix's basis version (and which prefix its coefficients use)."""

    key: MatrixKey
    channels: int
    world_size: int
    version_rows: tuple[int, ...]
    block_owners: tuple[int, ...]
    rank_view: int
    rotation: int = 0
    block_rows: int = PLAN_BLOCK_ROWS
    stream: str | None = None
    basis_group_id: str | None = None
    basis_version_ref: str | None = None

    def __post_init__(self):
        _check(isinstance(self.key, MatrixKey), "a spec describes one MatrixKey")
        for name in ("channels", "world_size", "block_rows", "rank_view"):
            _count(getattr(self, name), name, 1)
        _count(self.rotation, "rotation")
        _check(self.rotation < self.world_size, "rotation names a rank outside the group")
        rows = tuple(self.version_rows)
        _check(len(rows) > 0 and all(type(r) is int for r in rows), "version_rows: a list of row counts")
        _check(rows[0] >= 1 and all(b > a for a, b in zip(rows, rows[1:])), "version_rows must grow strictly")
        _check(rows[-1] <= self.channels, "a basis has at most `channels` rows")
        owners = tuple(self.block_owners)
        _check(len(owners) == -(-rows[-1] // self.block_rows), "one owner per block of basis rows")
        _check(all(type(o) is int and 0 <= o < self.world_size for o in owners), "block owners must be ranks")
        _check(self.rank_view <= rows[-1], "the rank view lies inside the basis version")
        if self.stream is not None:
            entry_key((self.key, self.stream))
        if self.basis_group_id is not None:
            _check(isinstance(self.basis_group_id, str) and len(self.basis_group_id) == 64
                   and all(ch in "0123456789abcdef" for ch in self.basis_group_id),
                   "basis_group_id is a lowercase SHA-256 hex digest")
        object.__setattr__(self, "version_rows", rows)
        object.__setattr__(self, "block_owners", owners)

    @classmethod
    def fresh(cls, entry, *, channels: int, rank: int, world_size: int, rotation: int | None = None,
              block_rows: int | None = None, basis_group_id: str | None = None,
              basis_version_ref: str | None = None) -> "FactorShardSpec":
        """Ownership of a freshly fitted basis (one block of ``channels`` rows unless ``block_rows``)."""
        key, stream = entry_parts(entry)
        _count(rank, "rank", 1)
        rot = rotation_of(entry, world_size) if rotation is None else rotation
        size = channels if block_rows is None else _count(block_rows, "block_rows", 1)
        owners = tuple((b + rot) % world_size for b in range(-(-rank // size)))
        return cls(key, channels, world_size, (rank,), owners, rank, rot, size, stream, basis_group_id,
                   basis_version_ref)

    def extend(self, added_rows: int, *, rank_view: int | None = None,
               basis_version_ref: str | None = None) -> "FactorShardSpec":
        """Append ``added_rows`` rows (augmentation): existing rows keep their owners."""
        total = self.total_rank + _count(added_rows, "added_rows", 1)
        _check(total <= self.channels, "an extension would exceed the channel count")
        owners = self.block_owners + tuple((b + self.rotation) % self.world_size
                                           for b in range(len(self.block_owners), -(-total // self.block_rows)))
        return FactorShardSpec(self.key, self.channels, self.world_size, self.version_rows + (total,), owners,
                               total if rank_view is None else rank_view, self.rotation, self.block_rows,
                               self.stream, self.basis_group_id, basis_version_ref)

    def with_view(self, rank_view: int) -> "FactorShardSpec":
        return FactorShardSpec(self.key, self.channels, self.world_size, self.version_rows, self.block_owners,
                               rank_view, self.rotation, self.block_rows, self.stream, self.basis_group_id,
                               self.basis_version_ref)

    @property
    def entry(self):
        return self.key if self.stream is None else (self.key, self.stream)

    @property
    def total_rank(self) -> int:
        return self.version_rows[-1]

    @property
    def whole_matrix(self) -> bool:
        return self.block_rows >= self.channels

    def owner_of(self, row: int) -> int:
        _check(0 <= row < self.total_rank, "row outside the basis version")
        return self.block_owners[row // self.block_rows]

    def basis_ranges(self, owner: int) -> tuple[tuple[int, int], ...]:
        """Rows ``[a, b)`` of the whole version that ``owner`` stores."""
        _check(type(owner) is int and 0 <= owner < self.world_size, "owner outside the group")
        return _join((b * self.block_rows, min((b + 1) * self.block_rows, self.total_rank))
                     for b, o in enumerate(self.block_owners) if o == owner)

    def view_ranges(self, owner: int) -> tuple[tuple[int, int], ...]:
        """Rows of the rank view owned by ``owner``: its coefficient columns, in global order."""
        return tuple((a, min(b, self.rank_view)) for a, b in self.basis_ranges(owner) if a < self.rank_view)

    def view_rows(self, owner: int) -> int:
        return span_rows(self.view_ranges(owner))

    @property
    def view_loads(self) -> tuple[int, ...]:
        return tuple(self.view_rows(o) for o in range(self.world_size))

    def segments(self) -> tuple[tuple[int, int, int], ...]:
        """Immutable basis segments ``(start, stop, owner)``: blocks cut at the version boundaries."""
        cuts = sorted({0, *self.version_rows, *range(0, self.total_rank, self.block_rows)})
        return tuple((a, b, self.owner_of(a)) for a, b in zip(cuts, cuts[1:]))

    def owner_segments(self, owner: int) -> tuple[tuple[int, int], ...]:
        return tuple((a, b) for a, b, o in self.segments() if o == owner)

    def check_partition(self) -> None:
        spans = sorted(s for o in range(self.world_size) for s in self.view_ranges(o))
        cursor = 0
        for a, b in spans:
            _check(a == cursor and b > a, "owner view ranges leave a gap or overlap", IntegrityError)
            cursor = b
        _check(cursor == self.rank_view, "owner view ranges do not cover the rank view", IntegrityError)

    def check_stable(self, parent: "FactorShardSpec") -> None:
        same = (parent.key, parent.stream, parent.channels, parent.world_size, parent.block_rows)
        _check(same == (self.key, self.stream, self.channels, self.world_size, self.block_rows),
               "the specs describe different matrices or groups", IntegrityError)
        shared = min(parent.total_rank, self.total_rank)
        for b in range(-(-shared // self.block_rows)):
            _check(parent.block_owners[b] == self.block_owners[b],
                   f"row block {b} changed owner ({parent.block_owners[b]} -> {self.block_owners[b]})", IntegrityError)

    def to_dict(self) -> dict[str, Any]:
        return {"schema": SPEC_SCHEMA, "entry": entry_json(self.entry), "channels": self.channels,
                "world_size": self.world_size, "version_rows": list(self.version_rows),
                "block_owners": list(self.block_owners), "rank_view": self.rank_view, "rotation": self.rotation,
                "block_rows": self.block_rows, "basis_group_id": self.basis_group_id,
                "basis_version_ref": self.basis_version_ref}

    @classmethod
    def from_dict(cls, data: Mapping[str, Any]) -> "FactorShardSpec":
        _check(isinstance(data, Mapping) and data.get("schema") == SPEC_SCHEMA, "not a factor-shard spec")
        try:
            key, stream = entry_parts(entry_from_json(data["entry"]))
            spec = cls(key, data["channels"], data["world_size"], tuple(data["version_rows"]),
                       tuple(data["block_owners"]), data["rank_view"], data["rotation"], data["block_rows"], stream,
                       data["basis_group_id"], data["basis_version_ref"])
        except (KeyError, TypeError) as exc:
            raise ConfigurationError("factor-shard spec is missing fields") from exc
        spec.check_partition()
        return spec

    @property
    def digest(self) -> str:
        return canonical_digest(self.to_dict())


def split_factors(spec: FactorShardSpec, coefficients: torch.Tensor, basis: torch.Tensor) -> dict:
    """``{owner: (P_s, Q_s)}``: each owner's coefficient columns and basis rows of the rank view."""
    _check(coefficients.dim() == 2 and coefficients.shape[1] == spec.rank_view, "coefficients: [tokens, rank_view]")
    _check(basis.dim() == 2 and basis.shape[0] >= spec.rank_view and basis.shape[1] == spec.channels,
           "basis: [>= rank_view, channels]")
    out = {}
    for owner in range(spec.world_size):
        index = span_index(spec.view_ranges(owner), coefficients.device)
        out[owner] = (coefficients.index_select(1, index).contiguous(),
                      basis.index_select(0, index.to(basis.device)).contiguous())
    return out


@dataclass(frozen=True)
class OwnershipPolicy:
    """How a group assigns owners to new bases: whole matrices (``block_rows=None``) or ``block_rows``-row
    blocks, starting at :func:`rotation_of`."""

    world_size: int
    block_rows: int | None = None

    def __post_init__(self):
        _count(self.world_size, "world_size", 1)
        if self.block_rows is not None:
            _count(self.block_rows, "block_rows", 1)

    def spec(self, entry, channels: int, rank: int, **kwargs) -> FactorShardSpec:
        return FactorShardSpec.fresh(entry, channels=channels, rank=rank, world_size=self.world_size,
                                     block_rows=self.block_rows, **kwargs)

    def owner(self, key) -> int:
        return rotation_of(key, self.world_size)

    def blocks(self, key, rank_count: int) -> list[tuple[int, slice]]:
        """``(owner, basis-row slice)`` of every block of a fresh ``rank_count``-row basis."""
        size = rank_count if self.block_rows is None else self.block_rows
        first = self.owner(key)
        return [((first + b) % self.world_size, slice(start, min(rank_count, start + size)))
                for b, start in enumerate(range(0, rank_count, size))]

    def to_dict(self) -> dict:
        return {"world_size": self.world_size, "block_rows": self.block_rows}


# ---------------------------------------------------------------------------------------------------------
# Native ownership of restored KV
# ---------------------------------------------------------------------------------------------------------

class NativeOwners:
    """The restore target: ``"heads"`` (rank ``r`` keeps channels ``layout.columns(r)`` of every token) or
    ``"rows"`` (rank ``r`` keeps token rows ``row_index[r]`` of every channel; contiguous by default)."""

    KINDS = ("heads", "rows")

    def __init__(self, layout: KVLayout, kind: str = "heads", row_index: Sequence[Sequence[int]] | None = None):
        _check(isinstance(layout, KVLayout), "native owners need a KVLayout")
        _check(kind in self.KINDS, f"native owner kind is one of {self.KINDS}")
        _check(kind == "rows" or row_index is None, "head shards hold every token row")
        self.layout, self.kind = layout, kind
        self.row_index = None
        if kind == "rows":
            if row_index is None:
                row_index = [range(layout.rows(r).start, layout.rows(r).stop) for r in range(layout.world_size)]
            rows = tuple(torch.as_tensor(list(r), dtype=torch.long) for r in row_index)
            _check(len(rows) == layout.world_size, "one row set per rank")
            _check(all(r.numel() > 0 for r in rows), "every rank owns at least one row")
            flat = torch.cat(rows)
            _check(flat.numel() == layout.tokens and torch.equal(flat.sort().values, torch.arange(layout.tokens)),
                   "the row sets must partition the tokens")
            self.row_index = rows

    @classmethod
    def spatial_rows(cls, *, frames: int, height: int, width: int, split_h: int, split_w: int, kv_heads: int,
                     head_dim: int) -> "NativeOwners":
        """Context-parallel 2-D split: rank ``i * split_w + j`` keeps spatial block ``(i, j)`` of every frame."""
        _check(height % split_h == 0 and width % split_w == 0, "the split must divide the latent grid")
        grid = torch.arange(frames * height * width).reshape(frames, height, width)
        bh, bw = height // split_h, width // split_w
        rows = [grid[:, i * bh:(i + 1) * bh, j * bw:(j + 1) * bw].reshape(-1).tolist()
                for i in range(split_h) for j in range(split_w)]
        layout = KVLayout(tokens=frames * height * width, kv_heads=kv_heads, head_dim=head_dim,
                          world_size=split_h * split_w)
        return cls(layout, "rows", rows)

    @property
    def world_size(self) -> int:
        return self.layout.world_size

    @property
    def tokens(self) -> int:
        return self.layout.tokens

    @property
    def channels(self) -> int:
        return self.layout.channels

    def rows(self, rank: int) -> torch.Tensor:
        return self.row_index[rank] if self.kind == "rows" else torch.arange(self.tokens)

    def columns(self, rank: int) -> slice:
        return self.layout.columns(rank) if self.kind == "heads" else slice(0, self.channels)

    def shape(self, rank: int) -> tuple[int, int]:
        if self.kind == "rows":
            return int(self.row_index[rank].numel()), self.channels
        return self.tokens, self.layout.local_channels

    def to_dict(self) -> dict:
        out = {"kind": self.kind, "tokens": self.tokens, "kv_heads": self.layout.kv_heads,
               "head_dim": self.layout.head_dim, "world_size": self.world_size}
        if self.kind == "rows":
            out["rows_sha256"] = [hashlib.sha256(r.numpy().astype("<i8").tobytes()).hexdigest()
                                  for r in self.row_index]
        return out


def row_shard_gram(local_rows: torch.Tensor, group=None, *, fused=None, owner: int = 0, layout: str = "rows"):
    """``X^T X`` of a matrix whose token rows are spread over the ranks.

    Default: the local FP64 Gram, all-reduced when a process group is up (every rank gets the sum).
    ``fused``: a :class:`~.gram_rs.GramReduceScatter` -- the partial Grams go straight from the Gram kernel into
    ``owner``'s buffer over NVLink; ``owner`` gets the FP32-accurate Gram, the others ``None``. Channel shards
    are rejected: their Grams miss the cross-channel blocks."""
    import torch.distributed as dist

    _check(layout == "rows", "per-shard Grams sum to X^T X only for token-row shards; gather channel shards first")
    if fused is not None:
        from .gram_rs import stacked_transpose
        return fused.run(stacked_transpose([local_rows.to(torch.bfloat16)]), [owner]).get(0)
    x = local_rows.detach().double()
    gram = x.t() @ x
    if dist.is_available() and dist.is_initialized():
        dist.all_reduce(gram, op=dist.ReduceOp.SUM, group=group)
    return gram


def channel_shard_gram(*_args, **_kwargs):
    raise ConfigurationError("a Gram matrix does not sum over channel shards; gather rows or use row shards")


# ---------------------------------------------------------------------------------------------------------
# Owner storage: fragment packs and basis segments
# ---------------------------------------------------------------------------------------------------------

@dataclass(frozen=True)
class FragmentInput:
    """One matrix's part of an owner's fragment: its view coefficient columns (FP32 ``[tokens, rows]``) and the
    matching basis rows (FP16 ``[rows, channels]``)."""

    entry: Any
    spec: FactorShardSpec
    context: TensorContext
    coefficients: torch.Tensor
    basis: torch.Tensor

    def __post_init__(self):
        entry_key(self.entry)
        _check(isinstance(self.spec, FactorShardSpec) and self.spec.entry == self.entry,
               "the spec describes another entry")
        _check(isinstance(self.context, TensorContext) and self.context.key == self.spec.key,
               "the context describes another matrix")
        c = self.coefficients
        _check(c.dtype == torch.float32 and c.dim() == 2 and c.shape[0] == self.context.token_count and c.shape[1] >= 1,
               "fragment coefficients: FP32 [tokens, owned rows >= 1]")
        _check(self.basis.dtype == torch.float16 and tuple(self.basis.shape) == (c.shape[1], self.spec.channels),
               "fragment basis: FP16 [owned rows, channels]")


def encode_fragment_pack(node_id: str, owner: int, world_size: int, fragments: Sequence[FragmentInput], *,
                         kind: str = "svd_hevc", stream_codec: str | None = None,
                         normalization: str = "per_channel"):
    """ONE owner's coefficient columns of the matrices of ONE node as an independently decodable pack.

    ``svd``: exact FP32 coefficients. ``svd_hevc``: the 8-bit covering-affine quantization of exactly these
    columns (per column), stored through the node-pack stream codecs (HEVC where an encoder exists, else the
    uncompressed 8-bit stream). Basis rows are not embedded: every tile records the SHA-256 of its rows, which
    the owner keeps as content-addressed segments."""
    from .. import _hevc
    from ..codecs import default_stream_codec
    from ..types import EncodedTensor

    _check(isinstance(node_id, str) and node_id.strip() != "", "node_id is a nonempty string")
    _check(type(owner) is int and 0 <= owner < world_size, "owner outside the group")
    _check(kind in FRAGMENT_KINDS, f"fragment kind is one of {FRAGMENT_KINDS}")
    items = sorted(fragments, key=lambda f: entry_sort_key(f.entry))
    tiles, blobs, affines = [], [], []
    cursor = records = 0
    codec = None
    if kind == "svd_hevc":
        codec = stream_codec or default_stream_codec()
        _check(codec in ("raw8", "raw8+zlib"), "fragment streams are raw8 or raw8+zlib where no HEVC encoder exists",
               UnsupportedError)
    for index, item in enumerate(items):
        _check(item.spec.view_rows(owner) == item.coefficients.shape[1], "fragment columns differ from the spec's view")
        coeff = item.coefficients.detach().cpu().contiguous()
        tile = {"tile": index, "entry": entry_json(item.entry), "spec": item.spec.digest,
                "context": item.context.to_dict(), "rows": int(coeff.shape[1]),
                "basis_sha256": hashlib.sha256(item.basis.detach().cpu().contiguous().numpy().tobytes()).hexdigest()}
        if kind == "svd":
            data = coeff.numpy().astype("<f4").tobytes()
        else:
            pixels, affine, layout = _hevc.quantize_coefficients(coeff.numpy(), normalization)
            data = np.ascontiguousarray(pixels).tobytes()
            affine = np.ascontiguousarray(affine, dtype="<f4")
            tile["normalization"] = layout
            tile["affine"] = {"record": records, "records": int(affine.shape[1])}
            affines.append(affine)
            records += int(affine.shape[1])
        tile["coefficients"] = {"offset": cursor, "bytes": len(data), "shape": [int(coeff.shape[0]), int(coeff.shape[1])],
                                "sha256": hashlib.sha256(data).hexdigest()}
        cursor += len(data)
        blobs.append(data)
        tiles.append(tile)
    raw = b"".join(blobs)
    payloads = {}
    if kind == "svd":
        payloads["coefficients"] = raw if raw else b"\0"
    else:
        import zlib
        payloads["stream"] = (zlib.compress(raw, 1) if codec == "raw8+zlib" else raw) or b"\0"
        payloads["affines"] = (np.concatenate(affines, axis=1) if affines else np.zeros((2, 0), "<f4")).tobytes() \
            or b"\0"
    metadata = {"schema": FRAGMENT_SCHEMA, "node_id": node_id, "owner": owner, "world_size": world_size,
                "kind": kind, "stream_codec": codec, "tiles": tiles, "raw_bytes": cursor}
    return EncodedTensor(metadata, payloads, metrics={"bytes": sum(len(p) for p in payloads.values())})


class FragmentPack:
    """Decoded view of one owner's fragment pack: per entry, FP32 coefficients (``svd``) or 8-bit coefficients
    with their per-column scale and offset (``svd_hevc``)."""

    def __init__(self, metadata: Mapping[str, Any], payloads: Mapping[str, bytes], *, verify: bool = True):
        _check(metadata.get("schema") == FRAGMENT_SCHEMA, "not a factor fragment pack", IntegrityError)
        self.metadata = metadata
        self.kind = metadata["kind"]
        if self.kind == "svd":
            raw = payloads["coefficients"]
        else:
            import zlib
            raw = payloads["stream"]
            if metadata.get("stream_codec") == "raw8+zlib":
                raw = zlib.decompress(raw)
            records = sum(t["affine"]["records"] for t in metadata["tiles"])
            self.affines = np.frombuffer(payloads["affines"][:8 * records], dtype="<f4").reshape(2, records)
        raw = raw[:metadata["raw_bytes"]]
        _check(len(raw) == metadata["raw_bytes"], "fragment stream is shorter than its tiles", IntegrityError)
        self.raw = raw
        self.by_entry = {}
        for tile in metadata["tiles"]:
            c = tile["coefficients"]
            chunk = raw[c["offset"]:c["offset"] + c["bytes"]]
            if verify:
                _check(hashlib.sha256(chunk).hexdigest() == c["sha256"],
                       f"fragment tile {tile['tile']} differs from its digest", IntegrityError)
            self.by_entry[entry_from_json(tile["entry"])] = tile

    def coefficients(self, entry) -> torch.Tensor:
        """FP32 ``[tokens, rows]`` (dequantized for ``svd_hevc``)."""
        from .. import _hevc
        tile = self.by_entry[entry]
        c = tile["coefficients"]
        chunk = self.raw[c["offset"]:c["offset"] + c["bytes"]]
        if self.kind == "svd":
            return torch.from_numpy(np.frombuffer(chunk, dtype="<f4").reshape(c["shape"]).copy())
        pixels = np.frombuffer(chunk, dtype=np.uint8).reshape(c["shape"])
        return torch.from_numpy(np.ascontiguousarray(_hevc.dequantize_coefficients(pixels, self.affine(entry),
                                                                                   tile["normalization"]),
                                                     dtype=np.float32))

    def pixels(self, entry) -> tuple[np.ndarray, np.ndarray, np.ndarray]:
        """``svd_hevc``: ``(uint8 [tokens, rows], scale [rows], offset [rows])``."""
        from .. import _hevc
        _check(self.kind == "svd_hevc", "exact FP32 fragments hold no 8-bit coefficients")
        tile = self.by_entry[entry]
        c = tile["coefficients"]
        pixels = np.frombuffer(self.raw[c["offset"]:c["offset"] + c["bytes"]], dtype=np.uint8).reshape(c["shape"])
        scale, offset = _hevc.expanded_affine(self.affine(entry), tile["normalization"], c["shape"][1])
        return pixels, np.asarray(scale, dtype=np.float32), np.asarray(offset, dtype=np.float32)

    def affine(self, entry) -> np.ndarray:
        record = self.by_entry[entry]["affine"]
        return np.ascontiguousarray(self.affines[:, record["record"]:record["record"] + record["records"]])


class OwnerFactorStore:
    """One owner's factor storage inside an :class:`~reelcache_b200.store.ObjectStore`: content-addressed basis
    segments (stored once, shared by forks and later nodes) and one fragment pack per published node, named by
    refs ``factor_shard/<domain>/<node>/owner<r>``."""

    def __init__(self, store, owner: int, world_size: int, *, domain: str = "default"):
        _check(type(owner) is int and 0 <= owner < world_size, "owner outside the group")
        self.store, self.owner, self.world_size, self.domain = store, owner, world_size, domain
        self.counters = {"segments_written": 0, "segment_bytes": 0, "fragments_written": 0, "fragment_bytes": 0}

    def ref(self, node_id: str) -> str:
        return f"{REF_PREFIX}{self.domain}/{node_id}/owner{self.owner}"

    def put_segment(self, rows: torch.Tensor) -> str:
        _check(rows.dtype == torch.float16 and rows.dim() == 2, "basis segments are FP16 [rows, channels]")
        data = rows.detach().cpu().contiguous().numpy().astype("<f2").tobytes()
        ref = self.store.put(data, kind="basis")
        self.counters["segments_written"] += 1
        self.counters["segment_bytes"] += len(data)
        return ref

    def get_segment(self, ref: str, channels: int, device="cpu") -> torch.Tensor:
        raw = self.store.get(ref)
        return torch.from_numpy(np.frombuffer(raw, dtype="<f2").reshape(-1, channels).copy()).to(device)

    def put_fragment(self, encoded, segments: Mapping[str, list]) -> str:
        """Stage one fragment pack (payload blobs + manifest); returns the manifest id (not yet published)."""
        refs = {name: self.store.put(payload) for name, payload in encoded.payloads.items()}
        data = {"fragment": dict(encoded.metadata), "payloads": refs, "segments": segments}
        manifest = self.store.put_manifest(data, references=sorted(set(refs.values()) | {
            ref for items in segments.values() for _, _, ref in items}))
        self.counters["fragments_written"] += 1
        self.counters["fragment_bytes"] += sum(len(p) for p in encoded.payloads.values())
        return manifest

    def load_fragment(self, manifest: str, *, verify: bool = True) -> tuple[FragmentPack, dict]:
        data = self.store.get_manifest(manifest)
        payloads = {name: self.store.get(ref) for name, ref in data["payloads"].items()}
        return FragmentPack(data["fragment"], payloads, verify=verify), data["segments"]

    def publish(self, node_id: str, manifest: str) -> None:
        self.store.set_ref(self.ref(node_id), manifest)

    def retract(self, node_id: str) -> None:
        if self.store.get_ref(self.ref(node_id)) is not None:
            self.store.delete_ref(self.ref(node_id))

    def published(self, node_id: str) -> str | None:
        return self.store.get_ref(self.ref(node_id))

    def stats(self) -> dict[str, int]:
        return dict(self.counters)


@dataclass(frozen=True)
class ShardedNodeMap:
    """The distributed layout of one published node: every entry's spec and context, and per owner its fragment
    pack manifest. Identical on every rank; its digest is what the owners agree on before publishing."""

    node_id: str
    world_size: int
    specs: Mapping[Any, FactorShardSpec]
    contexts: Mapping[Any, TensorContext]
    fragments: tuple[str | None, ...]     # owner -> fragment manifest (None: the owner holds no rows)
    kind: str = "svd_hevc"

    def __post_init__(self):
        _check(len(self.fragments) == self.world_size, "one fragment slot per owner")
        _check(set(self.specs) == set(self.contexts), "specs and contexts cover the same entries")
        for entry, spec in self.specs.items():
            _check(spec.world_size == self.world_size, f"{entry_name(entry)}: spec of another group")

    @property
    def entries(self) -> list:
        return sorted(self.specs, key=entry_sort_key)

    def to_dict(self) -> dict[str, Any]:
        return {"schema": NODE_MAP_SCHEMA, "node_id": self.node_id, "world_size": self.world_size, "kind": self.kind,
                "entries": [{"entry": entry_json(e), "spec": self.specs[e].to_dict(),
                             "context": self.contexts[e].to_dict()} for e in self.entries],
                "fragments": list(self.fragments)}

    @classmethod
    def from_dict(cls, data: Mapping[str, Any]) -> "ShardedNodeMap":
        _check(data.get("schema") == NODE_MAP_SCHEMA, "not a factor-shard node map", IntegrityError)
        specs, contexts = {}, {}
        for item in data["entries"]:
            entry = entry_from_json(item["entry"])
            specs[entry] = FactorShardSpec.from_dict(item["spec"])
            contexts[entry] = TensorContext.from_dict(item["context"])
        return cls(data["node_id"], data["world_size"], specs, contexts, tuple(data["fragments"]), data["kind"])

    @property
    def digest(self) -> str:
        return canonical_digest(self.to_dict())


@dataclass
class OwnerShard:
    """This rank's factors of one matrix: its view coefficient columns (FP32, or 8-bit with ``scale``/``offset``)
    and every basis row it owns (global row order). An owner without rows holds ``None``."""

    entry: Any
    spec: FactorShardSpec
    context: TensorContext
    owner: int
    coefficients: torch.Tensor | None
    basis: torch.Tensor | None
    scale: np.ndarray | None = None
    offset: np.ndarray | None = None

    def __post_init__(self):
        rows = self.spec.view_rows(self.owner)
        if rows == 0:
            _check(self.coefficients is None, "an owner without rows holds no coefficients")
        else:
            c = self.coefficients
            _check(c is not None and c.dim() == 2 and tuple(c.shape) == (self.context.token_count, rows),
                   "owner coefficients: [tokens, owned view rows]")
            _check(c.dtype == torch.float32 or (c.dtype == torch.uint8 and self.scale is not None
                                                 and self.offset is not None),
                   "owner coefficients are FP32, or uint8 with a per-column scale and offset")
        owned = span_rows(self.spec.basis_ranges(self.owner))
        if owned == 0:
            _check(self.basis is None, "an owner without basis rows holds no basis")
        else:
            _check(self.basis is not None and self.basis.dtype == torch.float16
                   and tuple(self.basis.shape) == (owned, self.spec.channels), "owner basis: FP16 [owned rows, channels]")

    @property
    def quantized(self) -> bool:
        return self.coefficients is not None and self.coefficients.dtype == torch.uint8

    def view_basis(self) -> torch.Tensor | None:
        rows = self.spec.view_rows(self.owner)
        return None if rows == 0 else self.basis[:rows]

    def dense_coefficients(self) -> torch.Tensor | None:
        """FP32 coefficients (8-bit ones dequantized: ``p * scale + offset``)."""
        if self.coefficients is None or not self.quantized:
            return self.coefficients
        device = self.coefficients.device
        scale = torch.as_tensor(self.scale, dtype=torch.float32, device=device)
        offset = torch.as_tensor(self.offset, dtype=torch.float32, device=device)
        return self.coefficients.float() * scale + offset


# ---------------------------------------------------------------------------------------------------------
# The collective domain
# ---------------------------------------------------------------------------------------------------------

class FactorShardDomain:
    """One rank's side of a factor-sharded group; construct it identically on every rank.

    ``transport``: the :class:`~.distributed.DistributedOwner` whose ``control_group`` orders the agreed
    checkpoints and whose ``group`` carries payloads. ``store``: this rank's :class:`OwnerFactorStore`
    (publication and ``load_node``). ``policy``: owners of fresh fits. ``mode``: the default reconstruction."""

    def __init__(self, transport: DistributedOwner, *, device="cpu", store: OwnerFactorStore | None = None,
                 policy: OwnershipPolicy | None = None, mode: str = "factors", tile_tokens: int = 4096):
        _check(isinstance(transport, DistributedOwner), "the domain runs over a DistributedOwner")
        _check(mode in MODES, f"reconstruction mode is one of {MODES}")
        self.t = transport
        self.rank, self.world_size = transport.rank, transport.world_size
        self.device = torch.device(device)
        _check(store is None or (store.owner == self.rank and store.world_size == self.world_size),
               "store must be this rank's OwnerFactorStore")
        self.store = store
        self.policy = policy or OwnershipPolicy(self.world_size)
        _check(self.policy.world_size == self.world_size, "the ownership policy describes another group")
        self.mode = mode
        self.tile_tokens = _count(tile_tokens, "tile_tokens", 1)
        self.counters = {"fits": 0, "published": 0, "rolled_back": 0, "restored": 0, "p2p_bytes_sent": 0,
                         "p2p_bytes_received": 0, "reduce_scatter_bytes": 0, "fused_restores": 0}
        rows = self.t.checkpoint("factor_domain:config", details={"mode": mode, "tile_tokens": tile_tokens,
                                                                  "policy": self.policy.to_dict(),
                                                                  "device": self.device.type})
        if any(r != rows[0] for r in rows):
            raise PeerFailure(f"ranks configured the factor domain differently: {rows}")

    # -- archival: owner fit, then scatter ------------------------------------------------------------------

    def fit_and_scatter(self, entries: Sequence[Any], canonical: Mapping[Any, torch.Tensor] | None,
                        contexts: Mapping[Any, TensorContext], *, ranks: Mapping[Any, int] | None = None,
                        energy: float = 0.98, fit_owner: int = 0, max_rank: int | None = None,
                        operation: str = "fit_and_scatter") -> dict[Any, OwnerShard]:
        """The fit owner (holding every canonical ``[tokens, channels]`` matrix) fits each entry -- the
        smallest rank reaching ``energy`` of the FP64 Gram spectrum, or ``ranks[entry]`` -- and sends every
        block's coefficient columns (FP32) and basis rows (FP16) to its owner. Collective; returns this rank's
        :class:`OwnerShard` of every entry."""
        t = self.t
        result = {}
        for entry in sorted(entries, key=entry_sort_key):
            p = q = None
            error, rank_count = None, None
            if t.rank == fit_owner:
                try:
                    x = canonical[entry].detach().to(self.device).double()
                    values, vectors = torch.linalg.eigh(x.t() @ x)
                    values, vectors = values.flip(0).clamp_min(0), vectors.flip(1)
                    if ranks is not None and entry in ranks:
                        rank_count = int(ranks[entry])
                    else:
                        total = float(values.sum())
                        share = torch.cumsum(values, 0) / max(total, 1e-300)
                        rank_count = int(torch.searchsorted(share, torch.tensor(energy, dtype=share.dtype,
                                                                                  device=share.device)).item()) + 1
                    rank_count = max(1, min(rank_count, x.shape[1], max_rank or x.shape[1]))
                    q = vectors[:, :rank_count].t().contiguous().to(torch.float16)
                    p = (x @ q.double().t()).float().contiguous()
                except Exception as exc:  # noqa: BLE001 - agreed before any payload moves
                    error = exc
            t.checkpoint(f"{operation}:fitted", error=error)   # a failed fit is raised on every rank here
            rank_count = t.broadcast_json(rank_count, operation=f"{operation}:rank", source=fit_owner)
            channels = contexts[entry].channels
            spec = self.policy.spec(entry, channels, rank_count)
            p_mine = q_mine = None
            for owner in range(self.world_size):
                spans = spec.view_ranges(owner)
                if not spans:
                    continue
                index = span_index(spans)
                p_s = p.index_select(1, index.to(p.device)).contiguous() if p is not None else None
                q_s = q.index_select(0, index.to(q.device)).contiguous() if q is not None else None
                if owner != fit_owner:
                    p_s = t.transfer_tensor(p_s, source=fit_owner, destination=owner, operation=f"{operation}:p")
                    q_s = t.transfer_tensor(q_s, source=fit_owner, destination=owner, operation=f"{operation}:q")
                if owner == self.rank:
                    p_mine, q_mine = p_s.to(self.device), q_s.to(self.device)
            result[entry] = OwnerShard(entry, spec, contexts[entry], self.rank, p_mine, q_mine)
            self.counters["fits"] += 1
        return result

    # -- two-phase publication ------------------------------------------------------------------------------

    def publish_node(self, node_id: str, shards: Mapping[Any, OwnerShard], *, kind: str = "svd_hevc",
                     fail: Callable[[str], None] | None = None) -> ShardedNodeMap:
        """Collective two-phase publication: every owner stages its fragment pack and basis segments, all
        ranks agree on one node map, every owner sets its ref; if any rank fails to commit, every owner
        retracts its ref and the failure is raised everywhere. ``fail(phase)`` (tests) may raise inside a
        phase to exercise the rollback."""
        _check(self.store is not None, "publication needs this rank's OwnerFactorStore")
        t = self.t
        op = f"factor_publish:{node_id}"
        manifest, error = None, None
        try:
            if fail is not None:
                fail("prepare")
            fragments = [FragmentInput(e, s.spec, s.context, s.dense_coefficients().float().cpu(),
                                       s.view_basis().cpu())
                         for e, s in sorted(shards.items(), key=lambda kv: entry_sort_key(kv[0]))
                         if s.coefficients is not None]
            if fragments:
                encoded = encode_fragment_pack(node_id, self.rank, self.world_size, fragments, kind=kind)
                segments = {}
                for e, s in shards.items():
                    if s.basis is None:
                        continue
                    rows, cursor = [], 0
                    for a, b in s.spec.owner_segments(self.rank):
                        rows.append([a, b, self.store.put_segment(s.basis[cursor:cursor + b - a])])
                        cursor += b - a
                    segments[entry_name(e)] = rows
                manifest = self.store.put_fragment(encoded, segments)
        except Exception as exc:  # noqa: BLE001 - agreed in the next checkpoint
            error = exc
        manifests = t.checkpoint(f"{op}:prepared", error=error, details=manifest)
        entries = sorted(shards, key=entry_sort_key)
        node_map = ShardedNodeMap(node_id, self.world_size, {e: shards[e].spec for e in entries},
                                  {e: shards[e].context for e in entries}, tuple(manifests), kind)
        digests = t.checkpoint(f"{op}:agree", details=node_map.digest)
        if any(d != digests[0] for d in digests):
            raise PeerFailure(f"{op}: ranks built different node maps")
        error = None
        try:
            if fail is not None:
                fail("commit")
            if manifest is not None:
                self.store.publish(node_id, manifest)
            # other owners' fragments may live in other stores: only this owner's is a reference here
            map_ref = self.store.store.put_manifest(node_map.to_dict(), references=[manifest] if manifest else [])
            self.store.store.set_ref(f"{REF_PREFIX}{self.store.domain}/{node_id}/map", map_ref)
        except Exception as exc:  # noqa: BLE001
            error = exc
        try:
            t.checkpoint(f"{op}:committed", error=error)
        except PeerFailure:
            self.store.retract(node_id)
            name = f"{REF_PREFIX}{self.store.domain}/{node_id}/map"
            if self.store.store.get_ref(name) is not None:
                self.store.store.delete_ref(name)
            self.counters["rolled_back"] += 1
            raise
        self.counters["published"] += 1
        return node_map

    def node_map(self, node_id: str) -> ShardedNodeMap:
        _check(self.store is not None, "reading node maps needs this rank's OwnerFactorStore")
        ref = self.store.store.get_ref(f"{REF_PREFIX}{self.store.domain}/{node_id}/map")
        if ref is None:
            raise StateError(f"node {node_id} is not published")
        return ShardedNodeMap.from_dict(self.store.store.get_manifest(ref))

    def load_node(self, node_map: ShardedNodeMap, *, entries: Iterable[Any] | None = None, device=None,
                  quantized: bool = True, verify: bool = True) -> dict[Any, OwnerShard]:
        """This rank's shards of a published node (its own fragment and segments only). ``quantized``: keep
        8-bit coefficients with their affine (what the fused restore consumes) instead of FP32."""
        _check(self.store is not None, "loading needs this rank's OwnerFactorStore")
        device = self.device if device is None else torch.device(device)
        wanted = node_map.entries if entries is None else [entry_key(e) for e in entries]
        manifest = node_map.fragments[self.rank]
        pack, segments = (None, {}) if manifest is None else self.store.load_fragment(manifest, verify=verify)
        out = {}
        for entry in wanted:
            spec, context = node_map.specs[entry], node_map.contexts[entry]
            coeff = basis = scale = offset = None
            if spec.view_rows(self.rank):
                _check(pack is not None and entry in pack.by_entry, f"owner {self.rank} lost {entry_name(entry)}",
                       IntegrityError)
                if quantized and pack.kind == "svd_hevc":
                    pixels, scale, offset = pack.pixels(entry)
                    coeff = torch.from_numpy(pixels.copy()).to(device)
                else:
                    coeff = pack.coefficients(entry).to(device)
            parts = [self.store.get_segment(ref, spec.channels, device)
                     for _, _, ref in segments.get(entry_name(entry), [])]
            if parts:
                basis = torch.cat(parts)
            out[entry] = OwnerShard(entry, spec, context, self.rank, coeff, basis, scale, offset)
        return out

    # -- reconstruction -------------------------------------------------------------------------------------

    def reconstruct(self, shards: Mapping[Any, OwnerShard], native: NativeOwners, *, mode: str | None = None,
                    dtype=torch.bfloat16, rope: Callable | None = None, rope_positions: Callable | None = None,
                    out: Mapping[Any, torch.Tensor] | None = None,
                    operation: str = "factor_reconstruct") -> dict[Any, torch.Tensor]:
        """Collective: every rank's native part ``[native rows, native columns]`` of every entry.

        ``rope(entry, values, positions, columns)`` rotates FP32 values of K entries on the native owner
        (``factors`` / ``partials``); the ``fused`` mode takes ``rope_positions(entry)`` (a ``RopePositions``)
        and applies RoPE in the restore kernel's epilogue."""
        mode = self.mode if mode is None else mode
        _check(mode in MODES, f"reconstruction mode is one of {MODES}")
        _check(isinstance(native, NativeOwners) and native.world_size == self.world_size,
               "native owners must describe this group")
        items = sorted(shards.items(), key=lambda kv: entry_sort_key(kv[0]))
        error = None
        try:
            for entry, shard in items:
                _check(isinstance(shard, OwnerShard) and shard.owner == self.rank, "pass this rank's OwnerShards")
                _check(shard.spec.channels == native.channels and shard.context.token_count == native.tokens,
                       f"{entry_name(entry)}: shard geometry differs from the native layout")
            if mode == "fused":
                self._check_fused(items, native, rope)
        except Exception as exc:  # noqa: BLE001 - agreed before any payload moves
            error = exc
        plan = [(entry_name(e), s.spec.digest) for e, s in items]
        rows = self.t.checkpoint(f"{operation}:plan", error=error, details={"mode": mode, "entries": plan,
                                                                            "native": native.to_dict()})
        if any(r != rows[0] for r in rows):
            raise PeerFailure(f"{operation}: ranks planned different reconstructions")
        outputs = {}
        for entry, _ in items:
            target = None if out is None else out.get(entry)
            if target is None:
                target = torch.empty(native.shape(self.rank), dtype=dtype, device=self.device)
            _check(tuple(target.shape) == native.shape(self.rank) and target.is_contiguous(),
                   "output buffers hold exactly this rank's native part")
            outputs[entry] = target
        if mode == "fused":
            self._reconstruct_fused(items, native, outputs, rope_positions)
        else:
            for entry, shard in items:
                part = self._factors_one(shard, native) if mode == "factors" else self._partials_one(shard, native)
                if rope is not None and shard.spec.key.target == "K":
                    part = rope(entry, part, native.rows(self.rank).to(part.device), native.columns(self.rank))
                outputs[entry].copy_(part)
        self.t.checkpoint(f"{operation}:complete")
        self.counters["restored"] += len(items)
        return outputs

    def _exchange(self, sends, receives) -> None:
        """One batched point-to-point round on the data group (``(tensor, peer, tag)`` lists)."""
        import torch.distributed as dist
        if self.world_size == 1 or (not sends and not receives):
            return
        ops = [dist.P2POp(dist.isend, x, self.t._global(p), self.t.group, tag) for x, p, tag in sends]
        ops += [dist.P2POp(dist.irecv, x, self.t._global(p), self.t.group, tag) for x, p, tag in receives]
        for work in self.t._run(dist.batch_isend_irecv, ops):
            self.t._run(work.wait)
        self.counters["p2p_bytes_sent"] += sum(x.numel() * x.element_size() for x, _, _ in sends)
        self.counters["p2p_bytes_received"] += sum(x.numel() * x.element_size() for x, _, _ in receives)

    def _factors_one(self, shard: OwnerShard, native: NativeOwners) -> torch.Tensor:
        """Owners ship coefficient rows and basis columns to every native owner, which multiplies in FP32."""
        spec, me = shard.spec, self.rank
        owners = [o for o in range(self.world_size) if spec.view_rows(o)]
        p_local = shard.dense_coefficients()
        q_local = shard.view_basis()
        sends, receives, parts = [], [], {}
        for dest in range(self.world_size):
            rows_d, cols_d = native.rows(dest), native.columns(dest)
            if me in owners:
                p_d = p_local.index_select(0, rows_d.to(p_local.device)).contiguous()
                q_d = q_local[:, cols_d].contiguous()
                if dest == me:
                    parts[me] = (p_d, q_d)
                else:
                    sends += [(p_d, dest, 1), (q_d, dest, 2)]
        n_me, c_me = native.shape(me)
        for owner in owners:
            if owner == me:
                continue
            r = spec.view_rows(owner)
            p_r = torch.empty((n_me, r), dtype=torch.float32, device=self.device)
            q_r = torch.empty((r, c_me), dtype=torch.float16, device=self.device)
            receives += [(p_r, owner, 1), (q_r, owner, 2)]
            parts[owner] = (p_r, q_r)
        self._exchange(sends, receives)
        coefficients = torch.zeros((n_me, spec.rank_view), dtype=torch.float32, device=self.device)
        basis = torch.zeros((spec.rank_view, c_me), dtype=torch.float32, device=self.device)
        for owner, (p_o, q_o) in parts.items():
            index = span_index(spec.view_ranges(owner), self.device)
            coefficients.index_copy_(1, index, p_o.float())
            basis.index_copy_(0, index, q_o.float())
        return coefficients @ basis

    def _partials_one(self, shard: OwnerShard, native: NativeOwners) -> torch.Tensor:
        """Each owner multiplies its block for every destination; one reduction per destination sums them."""
        import torch.distributed as dist
        me = self.rank
        p_local = shard.dense_coefficients()
        q_local = shard.view_basis()
        mine = None
        for dest in range(self.world_size):
            shape = native.shape(dest)
            if p_local is None:
                part = torch.zeros(shape, dtype=torch.float32, device=self.device)
            else:
                part = p_local.index_select(0, native.rows(dest).to(p_local.device)) @ \
                    q_local[:, native.columns(dest)].float()
            if self.world_size > 1:
                self.t._run(dist.reduce, part, dst=self.t._global(dest), op=dist.ReduceOp.SUM, group=self.t.group)
                self.counters["reduce_scatter_bytes"] += part.numel() * 4
            if dest == me:
                mine = part
        return mine

    # -- fused restore over symmetric memory -----------------------------------------------------------------

    def _check_fused(self, items, native: NativeOwners, rope) -> None:
        _check(self.device.type == "cuda", "the fused reconstruction runs on CUDA devices", UnsupportedError)
        _check(rope is None, "the fused reconstruction applies RoPE in its kernel: pass rope_positions")
        if native.kind == "rows":
            layout = KVLayout(native.tokens, native.layout.kv_heads, native.layout.head_dim, self.world_size)
            for r in range(self.world_size):
                span = layout.rows(r)
                _check(torch.equal(native.rows(r), torch.arange(span.start, span.stop)),
                       "the fused reconstruction takes contiguous row shards", UnsupportedError)
        for entry, shard in items:
            _check(shard.spec.whole_matrix, "the fused reconstruction needs whole-matrix owners", UnsupportedError)
            _check(shard.coefficients is None or shard.quantized,
                   "the fused reconstruction reads 8-bit coefficients (load_node(quantized=True))", UnsupportedError)

    def prepare_history(self, nodes: Sequence[Mapping[Any, OwnerShard]], *, kind: str = "sequence", heads: int,
                        head_dim: int, destination: Callable[[int, str], torch.Tensor],
                        rope_positions: Callable | None = None, stream=None, precision: str = "fp16x2"):
        """Stage a history of nodes (chunk order) for repeated fused restores: returns a
        :class:`~.sp_restore.FusedHistoryRestore` whose ``restore()`` writes every rank's native part of every
        node into ``destination(layer, target)`` (``kind``: ``sequence`` / ``heads`` / ``rows``).
        ``rope_positions(chunk, entry)`` gives the ``RopePositions`` of a K matrix."""
        from .sp_restore import FusedHistoryRestore, HistoryLayout, plan_history

        _check(len(nodes) > 0, "a history holds at least one node")
        first = nodes[0]
        context = next(iter(first.values())).context
        grid = (context.frames, context.height, context.width)
        shapes, owners_of, lookup = [], {}, {}
        for chunk, node in enumerate(nodes):
            for entry, shard in sorted(node.items(), key=lambda kv: entry_sort_key(kv[0])):
                key, _ = entry_parts(entry)
                _check(shard.spec.whole_matrix, "fused histories need whole-matrix owners", UnsupportedError)
                shapes.append((chunk, key.layer, key.target, shard.context.token_count, shard.spec.rank_view))
                owners_of[(chunk, key.layer, key.target)] = shard.spec.block_owners[0]
                lookup[len(shapes) - 1] = shard
        plan = plan_history(shapes, self.world_size, heads * head_dim,
                            owners=[owners_of[(c, l, t)] for c, l, t, _, _ in shapes])
        layout = HistoryLayout(kind, self.world_size, chunks=len(nodes), tokens=shapes[0][3], heads=heads,
                               head_dim=head_dim)
        group = self.t.group if self.world_size > 1 else None
        fused = FusedHistoryRestore.create(plan, layout, grid, self.device, group=group, precision=precision)
        factors = {}
        for tile in plan.owned(self.rank):
            shard = lookup[tile.index]
            factors[tile.index] = (shard.coefficients, shard.view_basis(), shard.scale, shard.offset)
        fused.stage(factors)
        rope = None
        if rope_positions is not None:
            def rope(tile):
                return rope_positions(tile.chunk, MatrixKey(tile.layer, tile.target))
        fused.build(destination, rope, stream=stream)
        self.counters["fused_restores"] += 1
        return fused

    def _reconstruct_fused(self, items, native: NativeOwners, outputs, rope_positions) -> None:
        heads = native.layout.kv_heads
        head_dim = native.layout.head_dim
        node = {entry: shard for entry, shard in items}
        by_key = {entry_parts(e)[0]: outputs[e] for e in node}
        n, c = native.shape(self.rank)

        def destination(layer, target):
            return by_key[MatrixKey(layer, target)].view(1, n, c // head_dim, head_dim)

        positions = None if rope_positions is None else (lambda chunk, key: rope_positions(key))
        fused = self.prepare_history([node], kind=native.kind, heads=heads, head_dim=head_dim,
                                     destination=destination, rope_positions=positions)
        fused.restore()
        torch.cuda.synchronize(self.device)
        fused.check()
        fused.close()

    def report(self) -> dict[str, Any]:
        return {**self.counters, "rank": self.rank, "world_size": self.world_size, "mode": self.mode,
                "store": None if self.store is None else self.store.stats()}


__all__ = ["EXCHANGE_BYTES", "FRAGMENT_KINDS", "FRAGMENT_SCHEMA", "MODES", "NODE_MAP_SCHEMA", "PLAN_BLOCK_ROWS",
           "SPEC_SCHEMA", "FactorShardDomain", "FactorShardSpec", "FragmentInput", "FragmentPack", "NativeOwners",
           "OwnerFactorStore", "OwnerShard", "OwnershipPolicy", "ShardedNodeMap", "channel_shard_gram",
           "encode_fragment_pack", "entry_from_json", "entry_json", "rotation_of", "row_shard_gram", "split_factors"]
