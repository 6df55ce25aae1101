"""Sequence-parallel fused history restore on 2 GPUs (one process per GPU, symmetric arenas over NVLink):
every rank restores its native pieces reading the owners' coefficients and bases from peer memory; the result
equals, bitwise, the same matrices restored whole on one GPU. The resident restore runs twice, then the
end-to-end restore (host upload into alternating regions + one device barrier per call) three times with
different coefficients each call, each checked. Skipped unless the box has two GPUs."""

import os
import socket

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

GRID = (3, 6, 16)
HEADS, HEAD_DIM = 4, 128


def _free_port() -> int:
    with socket.socket() as sock:
        sock.bind(("127.0.0.1", 0))
        return sock.getsockname()[1]


def _shapes(chunks, layers, seed):
    rng = np.random.default_rng(seed)
    tokens = GRID[0] * GRID[1] * GRID[2]
    return [(c, l, t, tokens, int(rng.integers(20, 140))) for c in range(chunks) for l in range(layers)
            for t in ("K", "V")]


def _factor(tile, device, salt=0):
    rng = np.random.default_rng(1000 * tile.index + salt)
    channels = HEADS * HEAD_DIM
    coeff = torch.from_numpy(rng.integers(0, 256, (tile.tokens, tile.rank), dtype=np.uint8)).to(device)
    rng_b = np.random.default_rng(1000 * tile.index)  # basis and affine fixed across calls
    basis = torch.from_numpy(rng_b.standard_normal((tile.rank, channels)).astype(np.float32) / 30).half().to(device)
    scale = rng_b.uniform(0.002, 0.05, tile.rank).astype(np.float32)
    offset = rng_b.uniform(-3, 3, tile.rank).astype(np.float32)
    return coeff, basis, scale, offset


def _worker(rank, world, port, kind, result_path):
    import datetime

    import torch.distributed as dist

    from reelcache_b200 import restore_kernels as rk
    from reelcache_b200.parallel.sp_restore import FusedHistoryRestore, HistoryLayout, plan_history

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    torch.cuda.set_device(rank)
    device = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60),
                            device_id=device)
    failures = []
    try:
        chunks, layers = 4, 3
        shapes = _shapes(chunks, layers, 7)
        tokens = shapes[0][3]
        plan = plan_history(shapes, world, HEADS * HEAD_DIM)
        layout = HistoryLayout(kind, world, chunks=chunks, tokens=tokens, heads=HEADS, head_dim=HEAD_DIM)
        fused = FusedHistoryRestore.create(plan, layout, GRID, device)
        fused.stage({t.index: _factor(t, device) for t in plan.owned(rank)})
        table = rk.RopeTable.wan(HEAD_DIM, 64, device=device)

        def rope(tile):
            return rk.RopePositions(table, (GRID[0] * tile.chunk, 0, 0))

        local = {(l, t): torch.zeros((1, layout.local_tokens(rank), layout.local_heads(rank), HEAD_DIM),
                                     dtype=torch.bfloat16, device=device) for l in range(layers) for t in ("K", "V")}
        fused.build(lambda l, t: local[(l, t)], rope)

        def check(salt):
            for tile in plan.tiles:
                coeff, basis, scale, offset = _factor(tile, device, salt)
                out = torch.zeros((1, tokens, HEADS, HEAD_DIM), dtype=torch.bfloat16, device=device)
                job = rk.ReconstructionJob(rk.CoefficientSource(coeff, scale, offset), rk.NativeView(out), GRID,
                                           basis, rope=rope(tile) if tile.target == "K" else None)
                rk.reconstruct([job], backend="fused", precision="fp16x2").synchronize()
                for piece in layout.pieces(rank, tile):
                    got = local[(tile.layer, tile.target)][0, piece.dest_row:piece.dest_row + piece.rows]
                    want = out[0, piece.row0:piece.row0 + piece.rows].reshape(piece.rows, -1)
                    want = want[:, piece.col0:piece.col0 + piece.cols]
                    if not torch.equal(got.reshape(piece.rows, -1), want):
                        failures.append((salt, tile.index, piece.row0))

        for _ in range(2):
            fused.restore()
        torch.cuda.synchronize(device)
        fused.check()
        check(0)
        for call in range(1, 4):
            # new coefficients for this call: the owner rewrites its pinned mirror, then the public restore
            # uploads them, runs the device barrier and restores
            mirror = fused.host_mirror()
            base = fused.plan.basis_bytes[rank]
            base = (base + 255) // 256 * 256
            for tile in plan.owned(rank):
                coeff = _factor(tile, "cpu", call)[0].numpy()
                start = tile.coeff_offset - base
                view = mirror[start:start + tile.coeff_bytes].view(tile.tokens, tile.k_pad)
                view[:, :tile.rank].copy_(torch.from_numpy(coeff))
            fused.restore(from_host=True)
            torch.cuda.synchronize(device)
            fused.check()
            check(call)
        fused.close()
        flag = torch.tensor([len(failures)], device=device)
        dist.all_reduce(flag)
        if rank == 0:
            with open(result_path, "w") as handle:
                handle.write(str(int(flag.item())))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("kind", ["sequence", "rows", "heads"])
def test_fused_history_restore_two_gpus(tmp_path, kind):
    world = 2
    if not torch.cuda.is_available() or torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    import torch.multiprocessing as mp
    result = tmp_path / "failures.txt"
    mp.spawn(_worker, args=(world, _free_port(), kind, str(result)), nprocs=world, join=True)
    assert result.read_text() == "0"
