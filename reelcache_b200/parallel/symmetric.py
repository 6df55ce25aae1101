"""Symmetric device memory shared by the ranks of one process group over NVLink / NVSwitch.

Every rank allocates one buffer of the same size through torch's symmetric-memory allocator; the
rendezvous maps each peer's buffer into this process, so a kernel on this GPU can load from or store
to any rank's buffer with ordinary (non-multicast) global-memory instructions or TMA loads. Regions
inside the buffer are carved by a plan that every rank computes from the same inputs, so an offset
names the same region on every rank.

The last 256 bytes hold the flag words of a bounded device-side barrier (``barrier``): every rank
stores the barrier's epoch into its slot of every peer's flag array (release, system scope) and spins,
with a wall-time limit, until every peer's store has reached its own array (acquire). The barrier is
a kernel on the caller's stream, so it orders the GPU work around it without a host synchronization;
a barrier that gives up records a status word (``check``) instead of trapping.
"""

from __future__ import annotations

import torch

from ..errors import CapacityError, ConfigurationError
from ..ops._ext import check_status, ext, status_word

FLAG_BYTES = 256
MAX_RANKS = 32  # the barrier kernel runs one thread per peer in one warp


def align(n: int, to: int = 256) -> int:
    return (n + to - 1) // to * to


class SymmetricArena:
    """One symmetric buffer of ``capacity`` bytes per rank of ``group`` (None: the default group)."""

    def __init__(self, group, device, capacity: int):
        import torch.distributed as dist
        import torch.distributed._symmetric_memory as symm

        self.group = group
        self.device = torch.device(device)
        self.rank = dist.get_rank(group)
        self.world = dist.get_world_size(group)
        if self.world > MAX_RANKS:
            raise ConfigurationError(f"a symmetric arena spans at most {MAX_RANKS} ranks")
        self.capacity = align(max(int(capacity), 256))
        name = group.group_name if group is not None else dist.group.WORLD.group_name
        if hasattr(symm, "enable_symm_mem_for_group"):
            try:
                symm.enable_symm_mem_for_group(name)
            except Exception:  # noqa: BLE001 - newer releases enable it implicitly
                pass
        self.buffer = symm.empty(self.capacity + FLAG_BYTES, dtype=torch.uint8, device=self.device)
        self.buffer[self.capacity:].zero_()
        self.handle = symm.rendezvous(self.buffer, group if group is not None else name)
        flags = [self._raw(peer, self.capacity, (self.world,), torch.int32) for peer in range(self.world)]
        self.flag_table = torch.tensor([f.data_ptr() for f in flags], dtype=torch.int64, device=self.device)
        self.epoch = 0
        self.status = status_word(self.device)
        torch.cuda.synchronize(self.device)
        dist.barrier(group=group)

    def _raw(self, peer: int, offset: int, shape, dtype) -> torch.Tensor:
        count = 1
        for s in shape:
            count *= int(s)
        itemsize = torch.empty((), dtype=dtype).element_size()
        if offset % itemsize:
            raise ConfigurationError("region offset is not aligned to its element size")
        if peer == self.rank:
            return self.buffer[offset:offset + count * itemsize].view(dtype).view(tuple(shape))
        return self.handle.get_buffer(peer, tuple(shape), dtype, offset // itemsize)

    def view(self, peer: int, offset: int, shape, dtype) -> torch.Tensor:
        """``shape``/``dtype`` view of bytes ``[offset, ...)`` of ``peer``'s buffer (this rank's own buffer
        when ``peer`` is this rank)."""
        itemsize = torch.empty((), dtype=dtype).element_size()
        count = 1
        for s in shape:
            count *= int(s)
        if offset < 0 or offset + count * itemsize > self.capacity:
            raise CapacityError("region lies outside the symmetric arena")
        return self._raw(peer, offset, shape, dtype)

    def barrier(self, stream=None) -> None:
        """Bounded device barrier of every rank on ``stream`` (default: the current stream)."""
        self.epoch += 1
        with torch.cuda.stream(stream or torch.cuda.current_stream(self.device)):
            ext().peer_barrier(self.flag_table, self.rank, self.epoch, self.status)

    def check(self) -> None:
        check_status(self.device)

    def close(self) -> None:
        import torch.distributed as dist
        torch.cuda.synchronize(self.device)
        dist.barrier(group=self.group)
        self.handle = None
        self.buffer = None


__all__ = ["SymmetricArena", "align"]
