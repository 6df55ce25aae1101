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


def _domain_worker(rank, world, port, root, result_path):
    """FactorShardDomain.reconstruct(mode="fused") against the NCCL "factors" mode, and the SP tiered
    history's fused cold restore against its point-to-point load_layer, on real archived factors."""
    import datetime

    import torch.distributed as dist

    from reelcache_b200 import restore_kernels as rk
    from reelcache_b200.lineage import LineageRuntime
    from reelcache_b200.parallel.distributed import DistributedOwner, KVLayout
    from reelcache_b200.parallel.factor_sharding import FactorShardDomain, NativeOwners, OwnerFactorStore
    from reelcache_b200.parallel.sp_kv import SPTieredHistory
    from reelcache_b200.store import ObjectStore
    from reelcache_b200.types import MatrixKey, ModelIdentity, TensorContext
    from tests.lineage_support import FRAMES, HEIGHT, MODEL, TOKENS, WIDTH, chunk, method

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    torch.cuda.set_device(rank)
    device = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60),
                            device_id=device)
    errors = []
    try:
        control = dist.new_group(backend="gloo")
        t = DistributedOwner(None, control_group=control, device=device)
        # -- factor-sharded node: fused vs factors --------------------------------------------------------
        heads, head_dim = 4, 128
        channels, grid = heads * head_dim, GRID
        tokens = grid[0] * grid[1] * grid[2]
        model = ModelIdentity("tiny-cp", "fp", 2, channels, "BTHD", "bfloat16")
        gen = torch.Generator().manual_seed(5)
        keys = [MatrixKey(l, tg) for l in range(2) for tg in ("K", "V")]
        canon = {k: (torch.randn(tokens, 24, generator=gen) @ torch.randn(24, channels, generator=gen)) for k in keys}
        contexts = {k: TensorContext(model, k, 0, *grid, "pre_rope" if k.target == "K" else "none") for k in keys}
        store = ObjectStore(f"{root}/owner{rank}")
        domain = FactorShardDomain(t, device=device, store=OwnerFactorStore(store, rank, world))
        shards = domain.fit_and_scatter(keys, canon if rank == 0 else None, contexts, ranks={k: 24 for k in keys})
        node_map = domain.publish_node("n0", shards, kind="svd_hevc")
        loaded = domain.load_node(node_map, quantized=True)
        table = rk.RopeTable.wan(head_dim, 16, device=device)
        for kind in ("heads", "rows"):
            native = NativeOwners(KVLayout(tokens, heads, head_dim, world), kind)
            fused = domain.reconstruct(loaded, native, mode="fused", dtype=torch.float32,
                                       rope_positions=lambda key: rk.RopePositions(table, (0, 0, 0)))
            plain = domain.reconstruct(loaded, native, mode="factors", dtype=torch.float32)
            for key in keys:
                want = plain[key]
                if key.target == "K":  # the factors path leaves K pre-RoPE: rotate it the reference way
                    view = want.reshape(want.shape[0], -1, head_dim).double()
                    rows = native.rows(rank)
                    job_rows = rk.RopePositions(table, (0, 0, 0))
                    cos, sin = rk.rope_cos_sin(job_rows, grid, dtype=torch.float64, device=device)
                    cos, sin = cos[rows.to(device)][:, None, :], sin[rows.to(device)][:, None, :]
                    rot = torch.empty_like(view)
                    rot[..., 0::2] = view[..., 0::2] * cos - view[..., 1::2] * sin
                    rot[..., 1::2] = view[..., 0::2] * sin + view[..., 1::2] * cos
                    want = rot.reshape(want.shape).float()
                err = float((fused[key] - want).norm() / want.norm())
                if err > 1e-3:
                    errors.append(("domain", kind, str(key), err))
        store.close()
        # -- SP tiered history: fused cold restore vs point-to-point load_layer ----------------------------
        shared = ObjectStore(f"{root}/shared")
        runtime = LineageRuntime(shared, MODEL)
        if rank == 0:
            runtime.create_lineage("sp")
        t.checkpoint("created")
        hist_heads = 2
        hd = MODEL.channels_for("K") // hist_heads
        hist = SPTieredHistory(t, runtime, "sp", layers=MODEL.layers, kv_heads=hist_heads, head_dim=hd,
                               chunk_tokens=TOKENS, grid=(FRAMES, HEIGHT, WIDTH), hot_budget_bytes=0,
                               method=method(), device=device)
        cols = slice(rank * (MODEL.channels_for("K") // world), (rank + 1) * (MODEL.channels_for("K") // world))
        for index in range(3):
            matrices, _ = chunk(index)
            hist.capture(index, {(k.layer, k.target): v[:, cols].contiguous().to(device) for k, v in matrices.items()})
        local = {(l, tg): torch.zeros((1, 3 * TOKENS, hist_heads // world, hd), dtype=torch.float32, device=device)
                 for l in range(MODEL.layers) for tg in ("K", "V")}
        fused_hist = hist.prepare_fused(lambda l, tg: local[(l, tg)])
        fused_hist.restore()
        torch.cuda.synchronize(device)
        fused_hist.check()
        for layer in range(MODEL.layers):
            dense = hist.load_layer(layer)
            for target in ("K", "V"):
                got = local[(layer, target)][0].reshape(3 * TOKENS, -1)
                want = dense[target].to(device).float()
                err = float((got - want).norm() / want.norm())
                if err > 2e-3:
                    errors.append(("sp_history", layer, target, err))
        fused_hist.close()
        shared.close()
        flag = torch.tensor([len(errors)], device=device)
        dist.all_reduce(flag)
        if rank == 0:
            with open(result_path, "w") as handle:
                handle.write(f"{int(flag.item())} {errors}")
    finally:
        dist.destroy_process_group()


def test_factor_domain_and_sp_history_fused_two_gpus(tmp_path):
    world = 2
    if not torch.cuda.is_available() or torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    import torch.multiprocessing as mp
    result = tmp_path / "failures.txt"
    mp.spawn(_domain_worker, args=(world, _free_port(), str(tmp_path), str(result)), nprocs=world, join=True)
    text = result.read_text()
    assert text.startswith("0 "), text
