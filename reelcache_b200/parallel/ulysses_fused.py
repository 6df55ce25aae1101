"""Ulysses context parallelism with the all-to-alls fused into the projection GEMMs (the B200 counterpart of
reference reelcache_sglang_models/longcat_video/context_parallel.py:133-159 ``all_to_all`` /
:213-223 ``ulysses_in`` / ``ulysses_out``, which call NCCL ``all_to_all_single`` around the GEMMs).

One symmetric allocation per rank (mapped into every peer over NVLink / NVSwitch) holds, for this rank's
``Hp = heads / world`` heads:

* ``q``  ``[rows, Hp, d]``                    -- written by every rank's fused QKV kernel (remote stores),
* ``k``, ``v`` ``[cache_rows + rows, Hp, d]``   -- the conditioning-cache rows first (set once per epoch),
  then the current tokens, so attention reads one contiguous K/V without a concatenation,
* ``o``  ``[rows, Hp * d]``                    -- this rank's attention output, read by every rank's fused
  output projection (TMA loads of peer memory, never multicast),
* ``flags`` ``int32 [world]``                  -- the device-side barrier's epoch slots.

Per layer: ``qkv()`` (fused GEMM + scatter, then a barrier: every rank's stores have landed), local q/k norm
+ RoPE and attention into ``o``, ``out()`` (a barrier: every rank's ``o`` is complete, then the fused gather +
output projection with the FP32 residual update: each remote attention-output tile is copied over NVLink
once into a local staging buffer by the kernel itself, M tile by M tile, while earlier M tiles multiply).
The barrier kernel waits with a bound and reports a timeout in the status word instead of hanging.
"""

from __future__ import annotations

import torch

from ..errors import ConfigurationError
from ..ops._ext import check_status, ext, status_word


def _align(n: int) -> int:
    return (n + 255) // 256 * 256


class FusedUlysses:
    def __init__(self, group, device, *, heads: int, head_dim: int, rows: int, cache_rows: int = 0):
        import torch.distributed as dist
        import torch.distributed._symmetric_memory as symm

        self.group = group
        self.device = torch.device(device)
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        if heads % self.world:
            raise ConfigurationError("heads must divide evenly across the context-parallel ranks")
        if self.world > 8:
            raise ConfigurationError("the fused Ulysses kernels address at most 8 ranks")
        self.heads, self.head_dim, self.hp = heads, head_dim, heads // self.world
        self.rows, self.cache_rows = rows, cache_rows
        row_bytes = self.hp * head_dim * 2
        self._layout = {}
        cursor = 0
        for name, nrows in (("q", rows), ("k", cache_rows + rows), ("v", cache_rows + rows), ("o", rows)):
            self._layout[name] = (cursor, nrows)
            cursor += _align(nrows * row_bytes)
        self._flags_offset = cursor
        cursor += _align(4 * self.world)
        name = group.group_name if group is not None else dist.group.WORLD.group_name
        if hasattr(symm, "enable_symm_mem_for_group"):
            try:
                symm.enable_symm_mem_for_group(name)
            except Exception:  # noqa: BLE001 - newer releases enable it implicitly
                pass
        self.buffer = symm.empty(cursor, dtype=torch.uint8, device=self.device)
        self.buffer.zero_()
        self.handle = symm.rendezvous(self.buffer, group if group is not None else name)
        self.views = [self._views_of(p) for p in range(self.world)]
        self.flag_table = torch.tensor([v["flags"].data_ptr() for v in self.views], dtype=torch.int64,
                                       device=self.device)
        self.epoch = 0
        self.calls = 0
        # staging of the remote owners' columns of this rank's rows (the output projection's A operand)
        local_rows = (rows // self.world + 127) // 128 * 128 + 128
        self.stage = torch.empty(local_rows, heads * head_dim, dtype=torch.bfloat16, device=self.device)
        self.tile_flags = torch.zeros(local_rows // 128, dtype=torch.int32, device=self.device)
        self.status = status_word(self.device)
        torch.cuda.synchronize(self.device)
        dist.barrier(group=group)

    def _views_of(self, peer: int) -> dict:
        out = {}
        for name, (offset, nrows) in self._layout.items():
            shape = (nrows, self.hp * self.head_dim) if name == "o" else (nrows, self.hp, self.head_dim)
            if peer == self.rank:
                flat = self.buffer[offset:offset + nrows * self.hp * self.head_dim * 2].view(torch.bfloat16)
                out[name] = flat.view(shape)
            else:
                out[name] = self.handle.get_buffer(peer, shape, torch.bfloat16, offset // 2)
        if peer == self.rank:
            out["flags"] = self.buffer[self._flags_offset:self._flags_offset + 4 * self.world].view(torch.int32)
        else:
            out["flags"] = self.handle.get_buffer(peer, (self.world,), torch.int32, self._flags_offset // 4)
        return out

    @property
    def local(self) -> dict:
        return self.views[self.rank]

    def barrier(self) -> None:
        """Device-side barrier on the current stream: work issued before it on every rank is complete."""
        self.epoch += 1
        ext().peer_barrier(self.flag_table, self.rank, self.epoch, self.status)

    def set_cache(self, k_cache: torch.Tensor, v_cache: torch.Tensor) -> None:
        """Conditioning-cache rows already in Ulysses layout ``[cache_rows, Hp, d]`` (RoPE applied to K)."""
        if k_cache.shape[0] != self.cache_rows or v_cache.shape[0] != self.cache_rows:
            raise ConfigurationError("cache rows disagree with the buffer layout")
        self.local["k"][:self.cache_rows].copy_(k_cache)
        self.local["v"][:self.cache_rows].copy_(v_cache)

    def qkv(self, y: torch.Tensor, weight: torch.Tensor, bias: torch.Tensor | None):
        """Fused QKV projection of this rank's ``n_loc`` tokens; returns this rank's ``(q, k_cur, v_cur)``
        ``[world * n_loc, Hp, d]`` views (rank-major token order) once every rank's stores have landed."""
        n_loc = y.shape[0]
        rows = self.world * n_loc
        if rows > self.rows:
            raise ConfigurationError("more tokens than the buffers were sized for")
        c = self.cache_rows
        ext().ulysses_qkv(y.contiguous(), weight, bias, [v["q"] for v in self.views],
                          [v["k"][c:] for v in self.views], [v["v"][c:] for v in self.views], self.rank,
                          self.head_dim, self.status)
        self.barrier()
        local = self.local
        return local["q"][:rows], local["k"][c:c + rows], local["v"][c:c + rows]

    def kv_all(self, rows: int):
        """Cache rows followed by the current ``rows`` tokens (contiguous views)."""
        return self.local["k"][:self.cache_rows + rows], self.local["v"][:self.cache_rows + rows]

    def out(self, x: torch.Tensor, weight: torch.Tensor, bias: torch.Tensor | None, gate: torch.Tensor | None):
        """``x += gate * (O_gathered @ weight^T + bias)`` for this rank's tokens, reading every rank's ``o``
        (complete after the barrier) straight from its memory."""
        n_loc = x.shape[0]
        self.barrier()
        self.calls += 1
        ext().ulysses_out([v["o"] for v in self.views], weight, bias, gate, x, self.rank, n_loc, 1, self.stage,
                          self.tile_flags, self.calls, self.status)
        return x

    def check(self) -> None:
        check_status(self.device)

    def close(self) -> None:
        import torch.distributed as dist
        torch.cuda.synchronize(self.device)
        dist.barrier(group=self.group)
        self.views = []
        self.handle = None
        self.buffer = None


__all__ = ["FusedUlysses"]
