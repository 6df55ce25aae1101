"""Distributed components on CPU with Gloo process groups (world size 2 and 3): the failure-agreement
transport, Ulysses / context-parallel exchanges, factor sharding (both reconstruction modes) and the
tiered sequence-parallel history. Failures are made on the host: a rank that raises, a rank that
cancels."""

import os
import socket
import tempfile
import traceback

import pytest
import torch
import torch.multiprocessing as mp


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _entry(rank, world, port, fn_name, args, errors):
    import datetime
    import torch.distributed as dist
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    try:
        timeout = 5 if fn_name == "w_dead_peer" else 60
        dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=timeout))
        globals()[fn_name](rank, world, *args)
    except BaseException:  # noqa: BLE001
        errors.put((rank, traceback.format_exc()))
    finally:
        if dist.is_initialized():
            dist.destroy_process_group()


def run(fn_name, world=2, *args):
    ctx = mp.get_context("spawn")
    errors = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_entry, args=(r, world, port, fn_name, args, errors)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(180)
        if p.is_alive():
            p.kill()
            raise AssertionError("a rank hung")
    failures = []
    while not errors.empty():
        failures.append(errors.get())
    assert not failures, "\n".join(f"rank {r}:\n{tb}" for r, tb in failures)


# ---- workers (module level so spawn can pickle them by name) ----------------------------------------------------

def w_transport(rank, world):
    from reelcache_b200.parallel.distributed import CollectiveCancelled, DistributedOwner, KVLayout, PeerFailure
    t = DistributedOwner(device="cpu", max_wire_bytes=64)
    assert t.broadcast_json({"x": 1}) == {"x": 1}
    heads = 2 * world
    layout = KVLayout(tokens=10, kv_heads=heads, head_dim=3, world_size=world)
    full = torch.arange(10 * heads * 3, dtype=torch.float32).reshape(10, heads * 3)
    g = t.gather_matrix(full[layout.rows(rank)].clone(), layout, source_layout="rows")
    h = t.gather_matrix(full[:, layout.columns(rank)].clone(), layout, source_layout="heads")
    if rank == 0:
        assert torch.equal(g, full) and torch.equal(h, full)
    else:
        assert g is None and h is None
    mine = t.local_columns(layout, lambda cols: full[:, cols].contiguous(), dtype=torch.float32)
    assert torch.equal(mine, full[:, layout.columns(rank)])
    moved = t.transfer_tensor(full * 2 if rank == 1 else None, source=1, destination=0)
    assert (rank != 0) or torch.equal(moved, full * 2)
    assert t.counters.payload_messages_sent + t.counters.payload_messages_received > 0
    # a local failure on one rank is raised on every rank before any payload moves
    with pytest.raises(PeerFailure):
        t.checkpoint("step", error=ValueError("boom") if rank == 1 else None)
    with pytest.raises(CollectiveCancelled):
        t.checkpoint("cancel", cancelled=(rank == 0))
    with pytest.raises(PeerFailure):
        t.owner_call("owner", lambda: 1 / 0)


def w_ulysses(rank, world):
    from reelcache_b200.parallel.context_parallel import RowShard, gather_tokens, optimal_split, ulysses_in, ulysses_out
    assert optimal_split(4, 44, 82) == (2, 2)
    frames, height, width, heads, d = 2, 4, 6, 4, 3
    shards = [RowShard(r, world, frames, height, width) for r in range(world)]
    tokens = frames * height * width
    full = torch.arange(tokens * heads * d, dtype=torch.float32).reshape(tokens, heads, d)
    local = shards[rank].local(full)
    seq = ulysses_in(local, None)
    order = torch.cat([s.token_index() for s in shards])
    hw = heads // world
    assert torch.equal(seq, full[order][:, rank * hw:(rank + 1) * hw])
    back = ulysses_out(seq, None)
    assert torch.equal(back, local)
    assert torch.equal(gather_tokens(local, shards), full)


def w_factor(rank, world, mode, granularity, root):
    """Factor-sharded fit, two-phase publication (including a rollback), load and reconstruction on Gloo ranks."""
    from reelcache_b200.parallel.distributed import DistributedOwner, KVLayout, PeerFailure
    from reelcache_b200.parallel.factor_sharding import (FactorShardDomain, NativeOwners, OwnerFactorStore,
                                                         OwnershipPolicy, row_shard_gram)
    from reelcache_b200.store import ObjectStore
    from reelcache_b200.types import MatrixKey, ModelIdentity, TensorContext
    t = DistributedOwner(device="cpu")
    layout = KVLayout(tokens=24, kv_heads=4, head_dim=8, world_size=world)
    g = torch.Generator().manual_seed(3)
    full = torch.randn(24, 6, generator=g) @ torch.randn(6, 32, generator=g)
    gram = row_shard_gram(full[layout.rows(rank)])
    assert torch.allclose(gram, full.double().t() @ full.double(), atol=1e-8)
    model = ModelIdentity("tiny", "fp", 2, 32, "BTHD", "float32")
    keys = [MatrixKey(l, tg) for l in range(2) for tg in ("K", "V")]
    contexts = {k: TensorContext(model, k, 0, 1, 4, 6, "pre_rope" if k.target == "K" else "none") for k in keys}
    store = ObjectStore(f"{root}/rank{rank}")
    owner_store = OwnerFactorStore(store, rank, world)
    policy = OwnershipPolicy(world, block_rows=2 if granularity == "rows" else None)
    domain = FactorShardDomain(t, store=owner_store, policy=policy)
    shards = domain.fit_and_scatter(keys, {k: full for k in keys} if rank == 0 else None, contexts,
                                    ranks={k: 6 for k in keys})
    for key, shard in shards.items():
        assert shard.spec.rank_view == 6 and shard.spec.view_rows(rank) == (0 if shard.coefficients is None
                                                                            else shard.coefficients.shape[1])
    heads = NativeOwners(layout, "heads")
    rows = NativeOwners(layout, "rows")
    for native in (heads, rows):
        mine = domain.reconstruct(shards, native, mode=mode, dtype=torch.float32)
        for key in keys:
            want = full[native.rows(rank)][:, native.columns(rank)]
            # the stored basis is FP16 (the archive format): relative error ~2^-11
            assert float((mine[key] - want).norm() / want.norm()) < 2e-3, (mode, key, native.kind)
    # a commit failure on one rank retracts every owner's fragment
    def fail(phase):
        if phase == "commit" and rank == 1:
            raise OSError("injected commit failure")
    try:
        domain.publish_node("n-failed", shards, kind="svd", fail=fail)
        raise AssertionError("the failed publication must raise on every rank")
    except PeerFailure:
        pass
    assert owner_store.published("n-failed") is None
    node_map = domain.publish_node("n0", shards, kind="svd")
    assert domain.node_map("n0").digest == node_map.digest
    loaded = domain.load_node(node_map, quantized=False)
    again = domain.reconstruct(loaded, heads, mode=mode, dtype=torch.float32)
    for key in keys:
        want = full[:, layout.columns(rank)]
        assert float((again[key] - want).norm() / want.norm()) < 2e-3
    # the 8-bit fragment kind round-trips through its quantization
    map8 = domain.publish_node("n8", shards, kind="svd_hevc")
    loaded8 = domain.load_node(map8, quantized=True)
    got8 = domain.reconstruct(loaded8, heads, mode=mode, dtype=torch.float32)
    for key in keys:
        want = full[:, layout.columns(rank)]
        assert float((got8[key] - want).norm() / want.norm()) < 2e-2
    store.close()


def w_sp_history(rank, world, root):
    from reelcache_b200.lineage import LineageRuntime
    from reelcache_b200.parallel.distributed import DistributedOwner
    from reelcache_b200.parallel.sp_kv import SPTieredHistory
    from reelcache_b200.store import ObjectStore
    from tests.lineage_support import FRAMES, HEIGHT, MODEL, TOKENS, WIDTH, chunk, method, relative_error
    t = DistributedOwner(device="cpu")
    store = ObjectStore(root)
    runtime = LineageRuntime(store, MODEL)
    if rank == 0:
        runtime.create_lineage("sp")
    t.checkpoint("created")
    heads = 2
    head_dim = MODEL.channels_for("K") // heads
    per_chunk = 2 * MODEL.layers * TOKENS * (MODEL.channels_for("K") // world) * 4
    hist = SPTieredHistory(t, runtime, "sp", layers=MODEL.layers, kv_heads=heads, head_dim=head_dim,
                           chunk_tokens=TOKENS, grid=(FRAMES, HEIGHT, WIDTH), hot_budget_bytes=per_chunk,
                           method=method())
    sources = []
    for index in range(3):
        matrices, _ = chunk(index)
        sources.append(matrices)
        cols = slice(rank * (MODEL.channels_for("K") // world), (rank + 1) * (MODEL.channels_for("K") // world))
        local = {(k.layer, k.target): v[:, cols].contiguous() for k, v in matrices.items()}
        hist.capture(index, local)
    assert hist.hot_chunks() == [2]  # budget of one chunk: the two oldest went cold on every rank
    from reelcache_b200.types import MatrixKey
    for layer in range(MODEL.layers):
        got = hist.load_layer(layer)
        for target in ("K", "V"):
            expect = torch.cat([s[MatrixKey(layer, target)] for s in sources])[:, cols]
            assert relative_error(got[target], expect) < 0.1
    assert hist.stats["cold_decodes"] > 0
    store.close()


def w_dead_peer(rank, world):
    """Rank 1 leaves between steps (no collective in flight); rank 0's next checkpoint fails within the
    process group's short timeout instead of blocking."""
    from reelcache_b200.parallel.distributed import DistributedOwner, PeerFailure
    import torch.distributed as dist
    t = DistributedOwner(device="cpu")
    t.checkpoint("step0")
    if rank == 1:
        dist.destroy_process_group()
        os._exit(0)
    with pytest.raises(PeerFailure):
        t.checkpoint("step1")
    with pytest.raises(PeerFailure):  # the transport is marked broken for good
        t.checkpoint("step2")


def w_row_archive(rank, world, root):
    from reelcache_b200.errors import IntegrityError
    from reelcache_b200.parallel.context_parallel import RowShard
    from reelcache_b200.parallel.distributed import DistributedOwner
    from reelcache_b200.parallel.row_shard_archive import RowShardedCacheArchive, TieredRowArchive
    from reelcache_b200.store import ObjectStore
    from reelcache_b200.types import MatrixKey
    t = DistributedOwner(device="cpu")
    frames, height, width, channels = 2, 4, 6, 16
    shards = [RowShard(r, world, frames, height, width) for r in range(world)]
    indices = [s.token_index() for s in shards]
    tokens = frames * height * width
    g = torch.Generator().manual_seed(3)
    full = {MatrixKey(l, tg): (torch.randn(tokens, 4, generator=g) @ torch.randn(4, channels, generator=g))
            for l in range(2) for tg in ("K", "V")}
    store = ObjectStore(f"{root}/rank{rank}")
    archive = RowShardedCacheArchive(t, store, indices, tokens=tokens, channels=channels, energy_target=0.999)
    tiers = TieredRowArchive(archive, host_raw_budget_bytes=1 << 20)
    local = {k: v[indices[rank]] for k, v in full.items()}
    tiers.capture("e0", local)
    assert tiers.flush() == ["e0"]
    # every rank's fragment holds only the matrices it owns (whole-matrix owners alternate by layer/target)
    tier, rows = tiers.install("e0")
    assert tier == "host_raw" and torch.equal(rows[MatrixKey(1, "V")], local[MatrixKey(1, "V")])
    # a staging failure on one rank rolls every rank back to the compressed archive
    tier, rows = tiers.install("e0", fail_preflight=(rank == 1))
    assert tier == "compressed" and tiers.last_restore_tier["rollback"]
    for key, value in rows.items():
        assert float((value - local[key]).norm() / local[key].norm()) < 2e-3  # FP16 basis rows
    # after eviction of the host copy the tiers agree on the compressed archive
    tiers.entries.clear()
    tier, _ = tiers.install("e0")
    assert tier == "compressed"
    store.close()


def test_dead_peer_detected():
    run("w_dead_peer", 2)


@pytest.mark.parametrize("world", [2, 3])
def test_transport_failure_agreement(world):
    run("w_transport", world)


def test_ulysses_and_context_parallel():
    run("w_ulysses", 2)


@pytest.mark.parametrize("mode,granularity", [("factors", "matrix"), ("partials", "matrix"), ("factors", "rows")])
def test_factor_sharding(mode, granularity, tmp_path):
    run("w_factor", 2, mode, granularity, str(tmp_path))


def test_sp_tiered_history(tmp_path):
    run("w_sp_history", 2, str(tmp_path / "store"))


def test_row_sharded_cache_archive_and_tiers(tmp_path):
    run("w_row_archive", 2, str(tmp_path))


def test_gram_rs_host_helpers():
    """Slots per owner follow the order of appearance; the stacked X^T pads tokens with zero columns (which add
    nothing to a Gram); the mirrored upper triangle of a symmetric matrix's partial sum is the matrix."""
    from reelcache_b200.parallel.gram_rs import GramReduceScatter, stacked_transpose, symmetric_from_upper
    assert GramReduceScatter.slots_for([0, 1, 0, 2, 1, 0]) == [0, 0, 1, 0, 1, 2]
    torch.manual_seed(0)
    shards = [torch.randn(13, 4), torch.randn(13, 4)]
    xt = stacked_transpose(shards)
    assert xt.shape == (8, 16) and xt.dtype == torch.bfloat16
    assert torch.equal(xt[:4, :13], shards[0].t().bfloat16()) and not xt[:, 13:].any()
    x = xt[:4].double()
    gram = x @ x.t()
    upper_only = torch.triu(gram) + torch.tril(torch.full_like(gram, 7.0), -1)
    assert torch.allclose(symmetric_from_upper(upper_only), gram)


def test_history_plan_and_layouts():
    """Sequence-parallel restore plan (parallel/sp_restore.py): owners, aligned arena offsets, and layouts that
    partition the history exactly (every token and channel of every matrix restored by exactly one rank)."""
    from reelcache_b200.parallel.sp_restore import HistoryLayout, default_owner, plan_history
    shapes = [(c, l, t, 4680, 30 + 7 * (c + l)) for c in range(5) for l in range(3) for t in ("K", "V")]
    for world in (1, 2, 3, 4):
        plan = plan_history(shapes, world, 1536)
        for tile in plan.tiles:
            assert tile.owner == default_owner(tile.layer, tile.target, world)
            assert tile.coeff_offset % 256 == 0 and tile.basis_offset % 256 == 0
            assert tile.coeff_offset >= plan.basis_bytes[tile.owner]
            end = tile.coeff_offset + plan.region_shift(tile.owner) + tile.coeff_bytes
            assert end <= plan.capacity
        for owner in range(world):  # regions of one owner do not overlap
            spans = sorted((t.coeff_offset, t.coeff_offset + t.coeff_bytes) for t in plan.owned(owner))
            spans += sorted((t.basis_offset, t.basis_offset + t.basis_bytes) for t in plan.owned(owner))
            spans.sort()
            assert all(a[1] <= b[0] for a, b in zip(spans, spans[1:]))
        for kind in ("sequence", "heads", "rows"):
            if kind == "sequence" and world > 5:
                continue
            layout = HistoryLayout(kind, world, chunks=5, tokens=4680, heads=12, head_dim=128)
            for tile in plan.tiles:
                cover = torch.zeros((4680, 1536), dtype=torch.int32)
                for rank in range(world):
                    for piece in layout.pieces(rank, tile):
                        cover[piece.row0:piece.row0 + piece.rows, piece.col0:piece.col0 + piece.cols] += 1
                        assert piece.dest_row + piece.rows <= layout.local_tokens(rank)
                        assert piece.cols == layout.local_heads(rank) * 128
                assert bool((cover == 1).all()), (kind, world, tile)
