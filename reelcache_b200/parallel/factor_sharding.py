"""Factor sharding: non-replicated ownership of the low-rank factors of every archived matrix (the
counterpart of reference reelcache/factor_sharding.py:1-2226; design from its docstring, lines 1-66).

``A ~ P Q = sum_s P_s Q_s`` over rank-direction blocks ``s`` (coefficient columns ``P_s`` and basis
rows ``Q_s``). Each block has one **owner** rank that stores and decodes only that block; by default
whole matrices are owned alternately by (layer, target) (``FactorShardSpec.owner``), optionally split
into 32-row blocks. Reconstruction delivers every **native owner** (the rank whose attention needs
them: Ulysses head columns or CP token rows) its slice of ``A``:

* ``mode="factors"`` (default): one batched point-to-point round sends each native owner the factor
  pieces it needs (all coefficient rows of its tokens, the basis columns of its heads) and the native
  owner runs the GEMM itself. On B200 the GEMM reads the owner's coefficients straight out of peer
  memory (``ops.restore`` fused restore with peer A operands), so the "gather" is the GEMM's own loads.
* ``mode="partials"``: every block owner computes FP32 partials ``P_s Q_s`` for all destinations and one
  ``reduce_scatter`` (SUM) per tile delivers each native owner its sums.

Gram fitting over **row** shards is exact (``row_shard_gram``: the all-reduced sum of local Grams);
over channel shards it is not (rejected).
"""

from __future__ import annotations

from dataclasses import dataclass

import torch

from ..errors import ConfigurationError
from ..types import MatrixKey
from .distributed import DistributedOwner, KVLayout

SPEC_SCHEMA = "reelcache.factor_shard_spec.v1"
FRAGMENT_SCHEMA = "reelcache.factor_fragment_pack.v1"
NODE_MAP_SCHEMA = "reelcache.factor_shard_node_map.v1"
MODES = ("factors", "partials")


@dataclass(frozen=True)
class FactorShardSpec:
    world_size: int
    granularity: str = "matrix"     # "matrix": whole-matrix owners; "rows": blocks of block_rows basis rows
    block_rows: int = 32

    def __post_init__(self):
        if type(self.world_size) is not int or self.world_size < 1:
            raise ConfigurationError("world_size must be a positive integer")
        if self.granularity not in ("matrix", "rows") or self.block_rows < 1:
            raise ConfigurationError("granularity is matrix|rows with positive block_rows")

    def owner(self, key: MatrixKey) -> int:
        """Whole-matrix owner: alternating by (layer, target)."""
        return (2 * key.layer + (key.target == "V")) % self.world_size

    def blocks(self, key: MatrixKey, rank_count: int) -> list[tuple[int, slice]]:
        """``(owner rank, basis-row slice)`` of every block of one matrix with ``rank_count`` rows."""
        if self.granularity == "matrix":
            return [(self.owner(key), slice(0, rank_count))]
        out = []
        for i, start in enumerate(range(0, rank_count, self.block_rows)):
            out.append(((self.owner(key) + i) % self.world_size, slice(start, min(rank_count, start + self.block_rows))))
        return out

    def to_dict(self) -> dict:
        return {"schema": SPEC_SCHEMA, "world_size": self.world_size, "granularity": self.granularity,
                "block_rows": self.block_rows}


def row_shard_gram(local_rows: torch.Tensor, group=None, *, fused=None, owner: int = 0) -> torch.Tensor | None:
    """``X^T X`` of a matrix whose token rows are sharded across ranks.

    Default: all-reduce of the local FP64 Grams (every rank gets it). ``fused``: a
    :class:`~reelcache_b200.parallel.gram_rs.GramReduceScatter` -- the partial Grams (bf16 rows, FP32-accurate)
    travel straight from the Gram kernel into ``owner``'s buffer over NVLink; ``owner`` gets the FP32 Gram and
    the other ranks ``None``."""
    import torch.distributed as dist
    if fused is not None:
        from .gram_rs import stacked_transpose
        grams = fused.run(stacked_transpose([local_rows.to(torch.bfloat16)]), [owner])
        return grams.get(0)
    x = local_rows.double()
    g = x.t() @ x
    if dist.is_available() and dist.is_initialized():
        dist.all_reduce(g, op=dist.ReduceOp.SUM, group=group)
    return g


def channel_shard_gram(*_args, **_kwargs):
    raise ConfigurationError("a Gram matrix does not sum over channel shards; gather rows or use row shards")


@dataclass(frozen=True)
class NativeOwners:
    """Which slice of ``A [tokens, channels]`` each rank needs: ``heads`` (Ulysses: column blocks) or
    ``rows`` (context parallel: token blocks)."""

    layout: KVLayout
    kind: str = "heads"

    def __post_init__(self):
        if self.kind not in ("heads", "rows"):
            raise ConfigurationError("native owners hold heads or rows")

    def rows(self, rank: int) -> slice:
        return slice(0, self.layout.tokens) if self.kind == "heads" else self.layout.rows(rank)

    def columns(self, rank: int) -> slice:
        return self.layout.columns(rank) if self.kind == "heads" else slice(0, self.layout.channels)


class FactorShardDomain:
    """Owner-side factor storage and native-owner reconstruction over one :class:`DistributedOwner`."""

    def __init__(self, transport: DistributedOwner, spec: FactorShardSpec, natives: NativeOwners):
        if spec.world_size != transport.world_size:
            raise ConfigurationError("factor shard spec and transport world sizes differ")
        self.transport = transport
        self.spec = spec
        self.natives = natives
        self.factors: dict[MatrixKey, list[tuple[slice, torch.Tensor, torch.Tensor]]] = {}  # this rank's blocks
        self.ranks: dict[MatrixKey, int] = {}

    # -- archival: owner fit then scatter --------------------------------------------------------------------

    def fit_and_scatter(self, key: MatrixKey, canonical: torch.Tensor | None, rank: int, *,
                        fit_owner: int = 0, operation: str = "fit_and_scatter") -> None:
        """The fit owner (holding the canonical matrix) fits ``rank`` directions (FP64 Gram eigh) and
        sends every block to its owner, which keeps ``(rows, P_s, Q_s)``."""
        t = self.transport
        rank_count = t.broadcast_json(rank, operation=f"{operation}:rank", source=fit_owner)
        p = q = None
        if t.rank == fit_owner:
            x = canonical.double()
            values, vectors = torch.linalg.eigh(x.t() @ x)
            order = torch.argsort(values, descending=True)[:rank_count]
            q = vectors[:, order].t().contiguous()            # [r, C]
            p = (x @ q.t()).contiguous()                      # [N, r]
        self.ranks[key] = rank_count
        mine = []
        for owner, rows in self.spec.blocks(key, rank_count):
            p_s = p[:, rows].float().contiguous() if p is not None else None
            q_s = q[rows].float().contiguous() if q is not None else None
            if owner == fit_owner:
                if t.rank == owner:
                    mine.append((rows, p_s, q_s))
                continue
            p_r = t.transfer_tensor(p_s, source=fit_owner, destination=owner, operation=f"{operation}:p")
            q_r = t.transfer_tensor(q_s, source=fit_owner, destination=owner, operation=f"{operation}:q")
            if t.rank == owner:
                mine.append((rows, p_r, q_r))
        self.factors[key] = mine

    # -- restore ------------------------------------------------------------------------------------------------

    def reconstruct(self, key: MatrixKey, *, mode: str = "factors", dtype=torch.float32) -> torch.Tensor:
        """This rank's native slice of ``A`` (``natives.rows(rank) x natives.columns(rank)``)."""
        if mode not in MODES:
            raise ConfigurationError(f"mode must be one of {MODES}")
        return self._factors(key, dtype) if mode == "factors" else self._partials(key, dtype)

    def _factors(self, key: MatrixKey, dtype) -> torch.Tensor:
        t = self.transport
        out = None
        for owner, rows in self.spec.blocks(key, self.ranks[key]):
            block = next(((p, q) for r, p, q in self.factors.get(key, []) if r == rows), None)
            for destination in range(t.world_size):
                need_rows, need_cols = self.natives.rows(destination), self.natives.columns(destination)
                p_piece = q_piece = None
                if t.rank == owner:
                    p_piece = block[0][need_rows].contiguous()
                    q_piece = block[1][:, need_cols].contiguous()
                if owner != destination:
                    p_piece = t.transfer_tensor(p_piece, source=owner, destination=destination,
                                                operation="factors:p")
                    q_piece = t.transfer_tensor(q_piece, source=owner, destination=destination,
                                                operation="factors:q")
                if t.rank == destination:
                    partial = p_piece @ q_piece
                    out = partial if out is None else out + partial
        return out.to(dtype)

    def _partials(self, key: MatrixKey, dtype) -> torch.Tensor:
        import torch.distributed as dist
        t = self.transport
        layout = self.natives.layout
        total = torch.zeros((layout.tokens, layout.channels), dtype=torch.float32, device=t.device)
        for rows, p, q in self.factors.get(key, []):
            total += p @ q
        if t.world_size == 1:
            return total.to(dtype)
        t.checkpoint("partials:reduce_scatter")
        if self.natives.kind == "heads":
            chunks = [total[:, self.natives.columns(r)].contiguous() for r in range(t.world_size)]
        else:
            chunks = [total[self.natives.rows(r)].contiguous() for r in range(t.world_size)]
        out = torch.empty_like(chunks[t.rank])
        if dist.get_backend(t.group) == "gloo":  # Gloo has no reduce_scatter: reduce to each owner in turn
            for r in range(t.world_size):
                buf = chunks[r].clone()
                dist.reduce(buf, dst=t._global(r), op=dist.ReduceOp.SUM, group=t.group)
                if r == t.rank:
                    out = buf
        else:
            dist.reduce_scatter(out, chunks, op=dist.ReduceOp.SUM, group=t.group)
        return out.to(dtype)

    def node_map(self) -> dict:
        return {"schema": NODE_MAP_SCHEMA, "spec": self.spec.to_dict(),
                "owners": {f"{k.layer}:{k.target}": [o for o, _ in self.spec.blocks(k, self.ranks[k])]
                           for k in self.ranks}}
