"""Sequence-parallel restore with the all-gather fused into the restore GEMM over NVLink peer memory.

Under Ulysses every rank attends over all tokens with its own head slice, so each rank needs
``A[:, its heads] = P @ Q[:, its heads]`` for the whole history, while the coefficient tiles ``P`` of the
history are spread over the ranks that archived (or decoded) them. Instead of an all-gather of ``P``
followed by a GEMM, every owner unpacks its tiles once into a symmetric buffer (one allocation per rank,
mapped into every peer through NVLink / NVSwitch), and every rank runs the fused restore kernel with
its A operand's TMA tensor maps pointing straight into the owners' buffers: each CTA fetches the remote
A tiles it multiplies, so the transfer overlaps the tensor-core work tile by tile. The loads are plain
(non-multicast) TMA loads; B (the basis columns of this rank's heads, scaled per tile) and the
epilogue (bias, RoPE, cast, TMA store into the native cache) stay local.

Protocol per restore: (1) owners unpack their u8 tiles into their buffers, (2) a group barrier
(device work done before it), (3) every rank launches its restore, (4) a second barrier before any
owner reuses its buffer.
"""

from __future__ import annotations

from dataclasses import dataclass
from typing import Any

import numpy as np
import torch

from ..errors import CapacityError, ConfigurationError
from ._ext import ext
from .restore import RestoreProgram, k_pad_of


@dataclass(frozen=True)
class PeerTile:
    """One archived coefficient tile (one chunk's K or V of one layer) and where it is staged."""

    owner: int
    tokens: int
    rank: int
    offset: int     # byte offset in the owner's symmetric buffer

    @property
    def k_pad(self) -> int:
        return k_pad_of(self.rank)

    @property
    def nbytes(self) -> int:
        return self.tokens * self.k_pad * 2


def plan_tiles(shapes: list[tuple[int, int, int]]) -> list[PeerTile]:
    """``(owner, tokens, rank)`` of every tile -> staged tiles with per-owner 256-byte aligned offsets
    (the same on every rank: every rank computes the layout from the shared plan)."""
    cursors: dict[int, int] = {}
    out = []
    for owner, tokens, rank in shapes:
        offset = cursors.get(owner, 0)
        tile = PeerTile(owner, tokens, rank, offset)
        cursors[owner] = offset + (tile.nbytes + 255) // 256 * 256
        out.append(tile)
    return out


class PeerRestoreDomain:
    def __init__(self, group, device, capacity_bytes: int):
        import torch.distributed as dist
        import torch.distributed._symmetric_memory as symm

        self.dist = dist
        self.group = group
        self.device = torch.device(device)
        self.rank = dist.get_rank(group)
        self.world = dist.get_world_size(group)
        self.capacity = (capacity_bytes + 255) // 256 * 256
        name = group.group_name if group is not None else dist.group.WORLD.group_name
        if hasattr(symm, "enable_symm_mem_for_group"):
            try:
                symm.enable_symm_mem_for_group(name)
            except Exception:  # noqa: BLE001 - newer releases enable it implicitly
                pass
        self.buffer = symm.empty(self.capacity, dtype=torch.uint8, device=self.device)
        self.handle = symm.rendezvous(self.buffer, group if group is not None else name)
        self.stats = {"restores": 0, "remote_a_bytes": 0, "local_a_bytes": 0}

    def _barrier(self) -> None:
        torch.cuda.current_stream(self.device).synchronize()
        self.dist.barrier(group=self.group)

    def a_view(self, tile: PeerTile) -> torch.Tensor:
        """FP16 ``[tokens, k_pad]`` view of a staged tile (in a peer's buffer when it is not ours)."""
        if tile.offset + tile.nbytes > self.capacity:
            raise CapacityError("staged tiles exceed the symmetric buffer")
        if tile.owner == self.rank:
            return self.buffer[tile.offset:tile.offset + tile.nbytes].view(torch.float16).view(tile.tokens, tile.k_pad)
        return self.handle.get_buffer(tile.owner, (tile.tokens, tile.k_pad), torch.float16, tile.offset // 2)

    def stage(self, tiles: list[PeerTile], sources: dict[int, torch.Tensor]) -> None:
        """Unpack this rank's tiles (``sources[i]``: uint8 ``[tokens, >= rank]`` on this device) into its
        buffer, then wait until every rank has staged its tiles."""
        rows = []
        for index, tile in enumerate(tiles):
            if tile.owner != self.rank:
                continue
            if tile.offset + tile.nbytes > self.capacity:
                raise CapacityError("staged tiles exceed the symmetric buffer")
            values = sources[index]
            out = self.buffer[tile.offset:tile.offset + tile.nbytes]
            rows.append([-1, -1, -1, values.data_ptr(), out.data_ptr(), values.stride(0), tile.tokens, tile.k_pad,
                         tile.rank, 1, 1, tile.tokens])
        rows = [[0 if v == -1 else v for v in row] for row in rows]
        for i in range(0, len(rows), 48):
            ext().unpack_launch(torch.tensor(rows[i:i + 48], dtype=torch.int64), self.device.index)
        self._barrier()

    def restore(self, tiles: list[PeerTile], jobs: list[dict[str, Any]], *, precision: str = "fp16",
                stream=None) -> RestoreProgram:
        """One restore job per tile (``jobs[i]``: the RestoreProgram fields other than the A source --
        ``basis`` = this rank's head columns ``[>= rank, channels_local]`` FP16, ``scale``/``offset``,
        ``grid``, ``dest``, ``rope``, ``group``); every A operand is read from its owner's buffer."""
        if len(tiles) != len(jobs):
            raise ConfigurationError("one job per staged tile")
        stream = stream or torch.cuda.current_stream(self.device)
        program = RestoreProgram(self.device, stream, precision=precision)
        for tile, job in zip(tiles, jobs):
            item = dict(job)
            item.update(kind="a16", a=self.a_view(tile), tokens=tile.tokens, rank=tile.rank)
            program.add(item, group=item.pop("group", 0))
            key = "local_a_bytes" if tile.owner == self.rank else "remote_a_bytes"
            self.stats[key] += tile.nbytes
        program.prepare(run_aux=True)
        program.launch_all(stream)
        self.stats["restores"] += 1
        self._barrier()
        return program


def column_basis(basis: torch.Tensor, rank: int, columns: slice) -> torch.Tensor:
    """This rank's head columns of a basis ``[R, C]`` as a contiguous FP16 ``[rank, channels_local]``."""
    return basis[:rank, columns].to(torch.float16).contiguous()


def host_affine(scale, offset, rank: int) -> tuple[np.ndarray, np.ndarray]:
    return (np.ascontiguousarray(np.asarray(scale, dtype=np.float32)[:rank]),
            np.ascontiguousarray(np.asarray(offset, dtype=np.float32)[:rank]))
