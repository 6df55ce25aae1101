"""Sequence-parallel fused history restore (parallel/sp_restore.py) on one GPU: every rank of a 2- or 3-rank
group is emulated on one device (one arena buffer per rank, every rank's program launched in turn), so the
plan's offsets, the per-layout pieces, the peer-addressed operands and the row-slice RoPE run through the real
kernels. Each rank's restored pieces must equal, bitwise, the same matrix restored whole by the fused entry
point (``restore_kernels.reconstruct``), which is itself checked against its error bound elsewhere."""

import numpy as np
import pytest
import torch

from reelcache_b200 import restore_kernels as rk
from reelcache_b200.parallel.sp_restore import FusedHistoryRestore, HistoryLayout, LocalArena, plan_history

pytestmark = pytest.mark.gpu

GRID = (3, 6, 16)          # 288 tokens per chunk (not a multiple of 128: partial token tiles)
HEADS, HEAD_DIM = 3, 128


def _factors(device, chunks, layers, seed=0):
    rng = np.random.default_rng(seed)
    tokens = GRID[0] * GRID[1] * GRID[2]
    channels = HEADS * HEAD_DIM
    shapes, factors = [], {}
    for chunk in range(chunks):
        for layer in range(layers):
            for target in ("K", "V"):
                rank = int(rng.integers(20, 140))
                index = len(shapes)
                shapes.append((chunk, layer, target, tokens, rank))
                coeff = torch.from_numpy(rng.integers(0, 256, (tokens, rank), dtype=np.uint8)).to(device)
                basis = torch.from_numpy(rng.standard_normal((rank, channels)).astype(np.float32) / 30).half().to(device)
                scale = rng.uniform(0.002, 0.05, rank).astype(np.float32)
                offset = rng.uniform(-3, 3, rank).astype(np.float32)
                factors[index] = (coeff, basis, scale, offset)
    return shapes, factors, tokens, channels


@pytest.mark.parametrize("kind,world", [("sequence", 2), ("sequence", 3), ("heads", 2), ("heads", 3),
                                        ("rows", 2), ("rows", 3)])
def test_emulated_ranks_match_whole_restore(cuda_device, kind, world):
    chunks, layers = 3, 2
    shapes, factors, tokens, channels = _factors(cuda_device, chunks, layers, seed=world)
    plan = plan_history(shapes, world, channels)
    layout = HistoryLayout(kind, world, chunks=chunks, tokens=tokens, heads=HEADS, head_dim=HEAD_DIM)
    arena = LocalArena(cuda_device, plan.capacity, world)
    fused = FusedHistoryRestore(plan, layout, GRID, arena)
    fused.stage(factors)
    table = rk.RopeTable.wan(HEAD_DIM, 64, device=cuda_device)

    def rope(tile):
        return rk.RopePositions(table, (GRID[0] * tile.chunk, 0, 0))

    caches = {}
    for rank in range(world):
        local = {(layer, target): torch.full((1, layout.local_tokens(rank), layout.local_heads(rank), HEAD_DIM),
                                             float("nan"), dtype=torch.bfloat16, device=cuda_device)
                 for layer in range(layers) for target in ("K", "V")}
        caches[rank] = local
        fused.build(lambda layer, target, local=local: local[(layer, target)], rope, rank=rank)
    for _ in range(2):  # twice: the second run restores the same resident factors again
        for rank in range(world):
            fused.launch(rank=rank)
    torch.cuda.synchronize(cuda_device)
    fused.check()
    # the whole history restored matrix by matrix through the existing entry point
    whole = {}
    for tile in plan.tiles:
        coeff, basis, scale, offset = factors[tile.index]
        out = torch.zeros((1, tokens, HEADS, HEAD_DIM), dtype=torch.bfloat16, device=cuda_device)
        job = rk.ReconstructionJob(rk.CoefficientSource(coeff, scale, offset), rk.NativeView(out), GRID, basis,
                                   rope=rope(tile) if tile.target == "K" else None)
        rk.reconstruct([job], backend="fused", precision="fp16x2").synchronize()
        whole[tile.index] = out[0]
    for rank in range(world):
        for tile in plan.tiles:
            for piece in layout.pieces(rank, tile):
                got = caches[rank][(tile.layer, tile.target)][0, piece.dest_row:piece.dest_row + piece.rows]
                want = whole[tile.index][piece.row0:piece.row0 + piece.rows]
                want = want.reshape(piece.rows, -1)[:, piece.col0:piece.col0 + piece.cols]
                assert torch.equal(got.reshape(piece.rows, -1), want), (rank, tile, piece)
    # every native token of every rank was written exactly by its pieces
    for rank in range(world):
        for cache in caches[rank].values():
            assert not torch.isnan(cache.float()).any()
