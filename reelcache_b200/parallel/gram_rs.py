"""Sequence-parallel Gram fit with the reduce-scatter fused into the Gram GEMM over NVLink peer memory (the
B200 counterpart of reference reelcache/factor_sharding.py:445 ``row_shard_gram`` -- a local Gram and an
all-reduce over NCCL -- and of the owner-fit gather of factor_sharding.py:1501-1543).

Every rank holds a token shard of each captured matrix; the fit of matrix ``b`` runs on ``owners[b]`` and
needs ``G_b = sum_r X_{b,r}^T X_{b,r}``. One kernel per rank (csrc/dist/gram_rs.cu) computes the
upper-triangular 128 x 128 tiles of its partial Grams with FP32-level accuracy (tensor-core partials promoted
to IEEE adds every 256 tokens) and stores each tile into the owner's symmetric buffer
``partials[rank][slot]`` as it finishes (NVLink stores for a peer owner), so the transfer overlaps the GEMM and
only half of each symmetric Gram crosses NVLink. After a bounded device barrier the owner sums the ranks'
partials in rank order in FP32 and mirrors the upper triangle: deterministic, FP32-accurate Grams.

``nvls="auto"`` (default: where the GPUs share an NVLink multicast object) or ``True``: the in-switch variant. Each rank's
kernel stores its tiles into its *own* symmetric buffer, every matrix at the same offset on every rank; after the
barrier the owner reads the matrix through the buffer's multicast address with ``multimem.ld_reduce``
(csrc/dist/nvls_reduce.cu), so the NVSwitch adds the ranks' partials and returns one reduced stream. The sum's
order is the switch's (it may differ in the last bit from the rank-ordered one).
"""

from __future__ import annotations

import torch

from ..errors import ConfigurationError
from ..ops._ext import check_status, ext, status_word


class GramReduceScatter:
    def __init__(self, group, device, *, channels: int, max_slots: int, nvls="auto"):
        import torch.distributed as dist
        import torch.distributed._symmetric_memory as symm

        if channels % 128:
            raise ConfigurationError("channels must be a multiple of 128")
        self.group = group
        self.device = torch.device(device)
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        if self.world > 8:
            raise ConfigurationError("the fused Gram reduce-scatter addresses at most 8 ranks")
        self.channels, self.max_slots = channels, max_slots
        part_elems = self.world * max_slots * channels * channels
        self._flags_offset = part_elems * 4
        total = self._flags_offset + 256
        name = group.group_name if group is not None else dist.group.WORLD.group_name
        if hasattr(symm, "enable_symm_mem_for_group"):
            try:
                symm.enable_symm_mem_for_group(name)
            except Exception:  # noqa: BLE001 - newer releases enable it implicitly
                pass
        self.buffer = symm.empty(total, dtype=torch.uint8, device=self.device)
        self.buffer.zero_()
        self.handle = symm.rendezvous(self.buffer, group if group is not None else name)
        shape = (self.world, max_slots, channels, channels)
        self.partials = []
        flags = []
        for peer in range(self.world):
            if peer == self.rank:
                self.partials.append(self.buffer[:self._flags_offset].view(torch.float32).view(shape))
                flags.append(self.buffer[self._flags_offset:self._flags_offset + 4 * self.world].view(torch.int32))
            else:
                self.partials.append(self.handle.get_buffer(peer, shape, torch.float32, 0))
                flags.append(self.handle.get_buffer(peer, (self.world,), torch.int32, self._flags_offset // 4))
        self.flag_table = torch.tensor([f.data_ptr() for f in flags], dtype=torch.int64, device=self.device)
        self.mc_ptr = int(getattr(self.handle, "multicast_ptr", 0) or 0) if nvls else 0
        if nvls is True and not self.mc_ptr:
            raise ConfigurationError("NVLS was requested but these GPUs share no NVLink multicast object")
        self.nvls = bool(self.mc_ptr)
        # in-switch mode: this rank's buffer viewed as one slot per matrix of a call (world * max_slots of them)
        self._local_slots = self.buffer[:self._flags_offset].view(torch.float32).view(
            1, self.world * max_slots, channels, channels)
        self.epoch = 0
        self.status = status_word(self.device)
        torch.cuda.synchronize(self.device)
        dist.barrier(group=group)

    @staticmethod
    def slots_for(owners: list[int]) -> list[int]:
        """Slot of every matrix in its owner's buffer (order of appearance per owner)."""
        count: dict[int, int] = {}
        out = []
        for owner in owners:
            out.append(count.get(owner, 0))
            count[owner] = out[-1] + 1
        return out

    def run(self, xt: torch.Tensor, owners: list[int]) -> dict[int, torch.Tensor]:
        """``xt``: this rank's shards as X^T stacked ``[B * C, tokens]`` bf16; returns ``{b: G_b}`` (FP32
        ``[C, C]``) for the matrices this rank owns."""
        matrices = len(owners)
        if xt.shape[1] % 8:
            xt = torch.nn.functional.pad(xt, (0, -xt.shape[1] % 8))  # zero tokens add nothing to a Gram
        slots = self.slots_for(owners)
        if max(slots) >= self.max_slots:
            raise ConfigurationError("more matrices per owner than the buffer has slots")
        # Entry barrier: an owner sums the previous call's partials on its stream after that call's exit
        # barrier, so no rank may store this call's tiles into a peer's slots until every owner has passed
        # that sum (the sum precedes this barrier on the owner's stream).
        self.epoch += 1
        ext().peer_barrier(self.flag_table, self.rank, self.epoch, self.status)
        if self.nvls:
            return self._run_nvls(xt, owners)
        ext().gram_reduce_scatter(xt.contiguous(), matrices, self.partials,
                                  torch.tensor(owners, dtype=torch.int64), torch.tensor(slots, dtype=torch.int64),
                                  self.rank, self.status)
        self.epoch += 1
        ext().peer_barrier(self.flag_table, self.rank, self.epoch, self.status)
        owned = [b for b, owner in enumerate(owners) if owner == self.rank]
        if not owned:
            return {}
        # every owned matrix at once (an owner's slots are 0 .. n - 1): FP32 sum of the ranks' partials in rank
        # order, then the mirrored upper triangle
        local = self.partials[self.rank]
        count = len(owned)
        sums = local[0, :count].clone()
        for rank in range(1, self.world):
            sums += local[rank, :count]
        grams = symmetric_from_upper(sums)
        return {b: grams[slots[b]] for b in owned}

    def _run_nvls(self, xt: torch.Tensor, owners: list[int]) -> dict[int, torch.Tensor]:
        matrices = len(owners)
        if matrices > self._local_slots.shape[1]:
            raise ConfigurationError(f"{matrices} matrices exceed the {self._local_slots.shape[1]} slots of the buffer")
        ext().gram_reduce_scatter(xt.contiguous(), matrices, [self._local_slots],
                                  torch.tensor(owners, dtype=torch.int64), torch.arange(matrices, dtype=torch.int64),
                                  self.rank, self.status, to_local=True)
        self.epoch += 1
        ext().peer_barrier(self.flag_table, self.rank, self.epoch, self.status)
        owned = [b for b, owner in enumerate(owners) if owner == self.rank]
        if not owned:
            return {}
        c = self.channels
        out = torch.empty((len(owned), c, c), dtype=torch.float32, device=self.device)
        offsets = torch.tensor([b * c * c for b in owned], dtype=torch.int64)
        ext().nvls_reduce_upper(self.mc_ptr, self._flags_offset // 4, offsets, out, c)
        grams = symmetric_from_upper(out)
        return {b: grams[i] for i, b in enumerate(owned)}

    def check(self) -> None:
        check_status(self.device)

    def close(self) -> None:
        import torch.distributed as dist
        torch.cuda.synchronize(self.device)
        dist.barrier(group=self.group)
        self.partials = []
        self.handle = None
        self.buffer = None


def stacked_transpose(shards: list[torch.Tensor]) -> torch.Tensor:
    """This rank's token shards ``[tokens, C]`` of the batch's matrices as X^T stacked ``[B * C, tokens_pad]``
    bf16, the token count padded with zero columns to a multiple of 8 (zero tokens add nothing to a Gram)."""
    tokens = shards[0].shape[0]
    pad = -tokens % 8
    out = torch.zeros((len(shards) * shards[0].shape[1], tokens + pad), dtype=torch.bfloat16, device=shards[0].device)
    for b, x in enumerate(shards):
        c = x.shape[1]
        out[b * c:(b + 1) * c, :tokens].copy_(x.t())
    return out


def symmetric_from_upper(s: torch.Tensor) -> torch.Tensor:
    """The symmetric matrix (or batch of matrices) whose upper triangle (diagonal included) is that of ``s``."""
    return torch.triu(s) + torch.triu(s, 1).transpose(-1, -2)


__all__ = ["GramReduceScatter", "stacked_transpose", "symmetric_from_upper"]
