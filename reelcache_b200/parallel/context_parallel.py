"""Context parallelism for the LongCat-shaped DiT: Ulysses head/sequence all-to-all plus a 2-D spatial
split of every latent frame (the counterpart of reference
reelcache_sglang_models/longcat_video/context_parallel.py:1-239).

Each rank keeps a spatial block ``(split_h, split_w) = optimal_split(cp, H, W)`` of every frame
(:class:`RowShard`). Self-attention runs one all-to-all per q/k/v (heads scattered, sequence gathered,
:func:`ulysses_in`) and the inverse on its output (:func:`ulysses_out`); cross-attention and the FFN
stay on local tokens. RoPE uses the rank's rows of the angle tables (``RowShard.token_index``). The
last layer's output is gathered (:func:`gather_tokens`); prompt embeddings and initial latents are
broadcast from rank 0.
"""

from __future__ import annotations

from dataclasses import dataclass

import torch

from ..errors import ConfigurationError


def optimal_split(cp: int, height: int, width: int) -> tuple[int, int]:
    """``(split_h, split_w)`` with ``split_h * split_w = cp`` dividing the grid, minimizing the block
    perimeter (the halo a 2-D split exchanges), ties to more rows."""
    best = None
    for split_h in range(1, cp + 1):
        if cp % split_h:
            continue
        split_w = cp // split_h
        if height % split_h or width % split_w:
            continue
        perimeter = height // split_h + width // split_w
        key = (perimeter, -split_h)
        if best is None or key < best[0]:
            best = (key, (split_h, split_w))
    if best is None:
        raise ConfigurationError(f"no 2-D split of a {height} x {width} grid into {cp} blocks")
    return best[1]


@dataclass(frozen=True)
class RowShard:
    """The spatial block of rank ``rank`` in a ``cp``-way split of ``frames x height x width`` tokens."""

    rank: int
    cp: int
    frames: int
    height: int
    width: int

    @property
    def split(self) -> tuple[int, int]:
        return optimal_split(self.cp, self.height, self.width)

    @property
    def block(self) -> tuple[slice, slice]:
        split_h, split_w = self.split
        bh, bw = self.height // split_h, self.width // split_w
        r, c = divmod(self.rank, split_w)
        return slice(r * bh, (r + 1) * bh), slice(c * bw, (c + 1) * bw)

    @property
    def local_tokens(self) -> int:
        rows, cols = self.block
        return self.frames * (rows.stop - rows.start) * (cols.stop - cols.start)

    def token_index(self) -> torch.Tensor:
        """Global (frame-major) token indices of this rank's tokens, in local order."""
        rows, cols = self.block
        f = torch.arange(self.frames).view(-1, 1, 1)
        y = torch.arange(rows.start, rows.stop).view(1, -1, 1)
        x = torch.arange(cols.start, cols.stop).view(1, 1, -1)
        return (f * self.height * self.width + y * self.width + x).reshape(-1)

    def local(self, x: torch.Tensor) -> torch.Tensor:
        """This rank's tokens of a full ``[tokens, ...]`` tensor."""
        return x.index_select(0, self.token_index().to(x.device))


def _world(group):
    import torch.distributed as dist
    return dist.get_world_size(group), dist.get_rank(group)


def ulysses_in(x: torch.Tensor, group=None) -> torch.Tensor:
    """``[local_tokens, heads, d]`` (every rank's spatial block) -> ``[all_tokens, heads / cp, d]``
    (rank-major token order: rank 0's tokens first)."""
    import torch.distributed as dist
    cp, _ = _world(group)
    tokens, heads, d = x.shape
    if heads % cp:
        raise ConfigurationError("heads must divide evenly across context-parallel ranks")
    send = x.reshape(tokens, cp, heads // cp, d).transpose(0, 1).contiguous()  # [cp, tokens, h/cp, d]
    recv = torch.empty_like(send)
    dist.all_to_all_single(recv, send, group=group)
    return recv.reshape(cp * tokens, heads // cp, d)


def ulysses_out(y: torch.Tensor, group=None) -> torch.Tensor:
    """Inverse of :func:`ulysses_in`: ``[all_tokens, heads / cp, d]`` -> ``[local_tokens, heads, d]``."""
    import torch.distributed as dist
    cp, _ = _world(group)
    total, local_heads, d = y.shape
    tokens = total // cp
    send = y.reshape(cp, tokens, local_heads, d).contiguous()
    recv = torch.empty_like(send)
    dist.all_to_all_single(recv, send, group=group)
    return recv.transpose(0, 1).reshape(tokens, cp * local_heads, d)


def gather_tokens(x: torch.Tensor, shards: list[RowShard], group=None) -> torch.Tensor:
    """All ranks' local tokens reassembled into global frame-major order (every rank gets it)."""
    import torch.distributed as dist
    cp, _ = _world(group)
    parts = [torch.empty_like(x) for _ in range(cp)]
    dist.all_gather(parts, x.contiguous(), group=group)
    total = sum(s.local_tokens for s in shards)
    out = torch.empty((total, *x.shape[1:]), dtype=x.dtype, device=x.device)
    for shard, part in zip(shards, parts):
        out[shard.token_index().to(x.device)] = part
    return out


def broadcast(x: torch.Tensor, src: int = 0, group=None) -> torch.Tensor:
    import torch.distributed as dist
    dist.broadcast(x, src=dist.get_global_rank(group, src) if group is not None else src, group=group)
    return x
