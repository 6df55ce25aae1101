"""MAGI Ulysses clean-history adapter (sequence parallel 2 in the reference's runs; any world size whose ranks
split the KV heads evenly). Reference: reelcache/adapters/magi.py:1-60 (MagiGeometry :36), :523-930 (the seam),
:1832-1980 (sealing a chunk).

Execution mode: serial, batch-one clean history. Every rank wraps its own copy of the model; only the storage
owner holds a lineage runtime. During a chunk's clean forward each rank captures, for every layer, the
normalized pre-RoPE K and the V of *its token rows* -- the layout before MAGI's Ulysses all-to-all scatters heads
-- through wrappers around the attention's ``get_k`` / ``get_v`` (the native functions stay in place and keep
their results; the wrappers only observe). :meth:`MagiAdapter.seal_chunk` first agrees that every rank captured
every layer (a rank that failed makes the seal fail on every rank, before any bytes move), gathers each matrix's
row shards into the canonical ``[tokens, kv_heads * head_dim]`` matrix on the owner, commits one lineage node
there and broadcasts its reference, so every rank knows the session head.

:meth:`MagiAdapter.restore_history` is the inverse for the native cache after Ulysses: the owner resolves the
head's history and sends each rank only its KV-head columns; the rank applies the model's rotary embedding at the
global token positions and returns per-layer ``K, V [history_tokens, local_heads, head_dim]``.
"""

from __future__ import annotations

from contextlib import contextmanager
from dataclasses import dataclass
from typing import Any, Callable

import torch

from ..errors import ConfigurationError, StateError
from ..parallel.distributed import DistributedOwner, KVLayout
from ..rank_method import RankMethodConfig
from ..types import CodecSpec, MatrixKey, ModelIdentity, TensorContext, energy_targets

REPRESENTATIONS = ("raw", "svd_hevc")


@dataclass(frozen=True)
class MagiGeometry:
    """MAGI-1 distill: 48 layers, 8 KV heads of 128 channels (grouped-query attention), chunks of 6 latent frames
    of 68 x 120 tokens, Ulysses over ``world_size`` ranks."""

    layers: int = 48
    kv_heads: int = 8
    head_dim: int = 128
    frames: int = 6
    height: int = 68
    width: int = 120
    world_size: int = 2
    name: str = "magi-1-distill"
    fingerprint: str = "magi-1-4.5b-distill"

    def __post_init__(self):
        for field in ("layers", "kv_heads", "head_dim", "frames", "height", "width", "world_size"):
            value = getattr(self, field)
            if type(value) is not int or value < 1:
                raise ConfigurationError(f"MAGI geometry: {field} must be a positive integer, got {value!r}")
        self.layout  # the heads must split evenly over the ranks

    @property
    def tokens(self) -> int:
        return self.frames * self.height * self.width

    @property
    def channels(self) -> int:
        return self.kv_heads * self.head_dim

    @property
    def layout(self) -> KVLayout:
        return KVLayout(self.tokens, self.kv_heads, self.head_dim, self.world_size)

    def identity(self) -> ModelIdentity:
        return ModelIdentity(self.name, self.fingerprint, self.layers, self.channels, "BTHD", "bfloat16")


class MagiAdapter:
    """A reversible seam around one rank's model (see the module docstring).

    ``model.layers[l].attention`` must provide ``get_k(mixed, *rope_args)`` (post-RoPE K of the rank's rows, after
    the key normalization module ``k_norm``) and ``get_v(mixed)``. ``rotary(k [tokens, heads, head_dim],
    first_token)`` applies the model's rotary embedding at global positions. ``runtime`` only on the owner."""

    mode = "serial_clean_history"

    def __init__(self, model, *, geometry: MagiGeometry, transport: DistributedOwner, branch_id: str,
                 rotary: Callable[[torch.Tensor, int], torch.Tensor], runtime=None, representation: str = "raw",
                 targets: str = "causvid", device: Any = "cpu"):
        if representation not in REPRESENTATIONS:
            raise ConfigurationError(f"representation must be one of {REPRESENTATIONS}, got {representation!r}")
        if transport.world_size != geometry.world_size:
            raise ConfigurationError(f"a {geometry.world_size}-rank MAGI geometry on a {transport.world_size}-rank "
                                     "transport")
        if transport.is_owner != (runtime is not None):
            raise ConfigurationError("exactly the storage owner holds the lineage runtime")
        self.model = model
        self.geometry = geometry
        self.transport = transport
        self.runtime = runtime
        self.branch_id = branch_id
        self.rotary = rotary
        self.representation = representation
        self.device = torch.device(device)
        self.method = (None if representation == "raw" else
                       RankMethodConfig(targets=energy_targets(targets), codec=CodecSpec("svd_hevc", 32),
                                        solver="gram_eigh"))
        self.rows = geometry.layout.rows(transport.rank)
        self.phase = "idle"
        self.chunk_index: int | None = None
        self.head_ref: str | None = None
        self.chunks = 0
        self._captured: dict[MatrixKey, torch.Tensor] = {}
        self._originals: list[tuple[Any, str, Any]] = []

    # -- the seam ---------------------------------------------------------------------------------------------------

    def attach(self) -> "MagiAdapter":
        if self._originals:
            raise StateError("the MAGI adapter is already attached")
        for layer, block in enumerate(self.model.layers):
            attention = block.attention
            self._wrap(attention, "get_k", self._k_wrapper(layer, attention, attention.get_k))
            self._wrap(attention, "get_v", self._v_wrapper(layer, attention.get_v))
        return self

    def _wrap(self, obj, name: str, function) -> None:
        self._originals.append((obj, name, obj.__dict__.get(name)))
        setattr(obj, name, function)

    def _k_wrapper(self, layer: int, attention, original):
        def get_k(mixed, *args, **kwargs):
            if self.phase != "clean":
                return original(mixed, *args, **kwargs)
            seen = []
            handle = attention.k_norm.register_forward_hook(lambda _m, _i, out: seen.append(out))
            try:
                result = original(mixed, *args, **kwargs)
            finally:
                handle.remove()
            if len(seen) != 1:
                raise StateError(f"layer {layer}: the key normalization ran {len(seen)} times in one get_k")
            self._store(MatrixKey(layer, "K"), seen[0])
            return result
        return get_k

    def _v_wrapper(self, layer: int, original):
        def get_v(mixed, *args, **kwargs):
            result = original(mixed, *args, **kwargs)
            if self.phase == "clean":
                self._store(MatrixKey(layer, "V"), result)
            return result
        return get_v

    def _store(self, key: MatrixKey, value: torch.Tensor) -> None:
        rows = self.rows.stop - self.rows.start
        flat = value.detach().reshape(-1, self.geometry.channels)
        if flat.shape[0] != rows:
            raise StateError(f"{key}: captured {flat.shape[0]} token rows, this rank owns {rows}")
        self._captured[key] = flat.float().clone()

    def detach(self) -> None:
        originals, self._originals = self._originals, []
        for obj, name, previous in reversed(originals):
            if previous is None:
                delattr(obj, name)
            else:
                setattr(obj, name, previous)

    def __enter__(self):
        return self.attach()

    def __exit__(self, *exc):
        self.detach()

    @contextmanager
    def execution(self, *, chunk_index: int, clean: bool):
        """Around one native forward: a clean forward captures this rank's K / V rows."""
        if self.phase != "idle":
            raise StateError(f"a {self.phase} execution is already running")
        self.phase = "clean" if clean else "denoise"
        self.chunk_index = chunk_index
        if clean:
            self._captured = {}
        try:
            yield self
        finally:
            self.phase = "idle"

    # -- archival -------------------------------------------------------------------------------------------------

    def seal_chunk(self, chunk_id: str | None = None) -> str:
        """Commit the captured clean chunk (collective; every rank calls it). Returns the new head node."""
        g = self.geometry
        expected = {MatrixKey(layer, target) for layer in range(g.layers) for target in ("K", "V")}
        problem = None
        if self.chunk_index is None:
            problem = StateError("no clean execution ran before seal_chunk")
        elif set(self._captured) != expected:
            missing = sorted(str(k) for k in expected - set(self._captured))
            problem = StateError(f"clean capture incomplete, missing {missing[:4]}{'...' if len(missing) > 4 else ''}")
        self.transport.checkpoint("magi_capture", error=problem)
        chunk = self.chunk_index
        layout = g.layout
        matrices: dict[MatrixKey, torch.Tensor] = {}
        for key in sorted(expected, key=lambda k: (k.layer, k.target)):
            canonical = self.transport.gather_matrix(self._captured[key].to(self.transport.device), layout,
                                                     source_layout="rows", operation=f"magi_gather:{key}")
            if canonical is not None:
                matrices[key] = canonical
        self._captured = {}
        chunk_id = chunk_id or f"chunk{chunk}"

        def commit():
            model = self.runtime.model
            contexts = {key: TensorContext(model, key, chunk * g.tokens, g.frames, g.height, g.width,
                                           "pre_rope" if key.target == "K" else "none") for key in matrices}
            if self.method is None:
                return self.runtime.commit_raw_node(self.branch_id, chunk_id, matrices, contexts).node_ref
            return self.runtime.commit_node(self.branch_id, chunk_id, matrices, contexts, method=self.method,
                                            device=self.device).node_ref

        node = self.transport.owner_call("magi_commit", commit)
        self.head_ref = self.transport.broadcast_json(node, operation="magi_head")
        self.chunks += 1
        return self.head_ref

    def fork(self, node_ref: str, branch_id: str) -> None:
        """Continue on a new branch at ``node_ref`` (collective)."""
        self.transport.owner_call("magi_fork", lambda: self.runtime.fork_lineage(node_ref, branch_id))
        self.branch_id = branch_id
        self.head_ref = node_ref

    # -- restore ------------------------------------------------------------------------------------------------

    def restore_history(self, node_ref: str | None = None, *, dtype=torch.bfloat16) -> list[tuple[torch.Tensor,
                                                                                                   torch.Tensor]]:
        """Per layer ``(K, V)`` of this rank's KV heads over the whole history of ``node_ref`` (default: the head),
        K rotated at global positions (collective)."""
        node_ref = node_ref or self.head_ref
        if node_ref is None:
            raise StateError("nothing to restore: no chunk was sealed and no node was given")
        g = self.geometry

        def plan():
            pieces = self.runtime.resolve_history(node_ref)
            return {"tokens": sum(p.token_end - p.token_start for p in pieces),
                    "first": min(p.token_start for p in pieces)}

        shape = self.transport.broadcast_json(self.transport.owner_call("magi_plan", plan), operation="magi_plan")
        layout = KVLayout(shape["tokens"], g.kv_heads, g.head_dim, g.world_size)
        local_heads = g.kv_heads // g.world_size
        out = []
        for layer in range(g.layers):
            pair = []
            for target in ("K", "V"):
                key = MatrixKey(layer, target)
                full = (self.runtime.acquire_node_history(node_ref, key).float().to(self.transport.device)
                        if self.transport.is_owner else None)
                columns = self.transport.local_columns(
                    layout, lambda cols, full=full: full[:, cols].contiguous(), dtype=torch.float32,
                    operation=f"magi_restore:{key}")
                values = columns.reshape(shape["tokens"], local_heads, g.head_dim)
                if target == "K":
                    values = self.rotary(values, shape["first"])
                pair.append(values.to(dtype))
            out.append(tuple(pair))
        return out
