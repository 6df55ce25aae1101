"""Restore tiers on CPU: the staging engine (native parallel pread + hash checks), the decoder pool and
decoded tier behind the packed-decode restorer, archive eviction under a budget, device-pressure trims
and runtime telemetry."""

import numpy as np
import pytest
import torch

from reelcache_b200 import restore_kernels as rk
from reelcache_b200.decoded_tier import DecodedTier
from reelcache_b200.decoder_pool import DecoderPool
from reelcache_b200.device_pressure import DeviceTrimRegistry
from reelcache_b200.errors import CapacityError, ConfigurationError, IntegrityError
from reelcache_b200.integrations.sglang.archive_eviction import ArchiveEviction
from reelcache_b200.lineage import LineageRuntime
from reelcache_b200.packed_decode import PackedRestorer
from reelcache_b200.restore_staging import StagingEngine
from reelcache_b200.store import ObjectStore
from reelcache_b200.telemetry import RuntimeTelemetry, span
from reelcache_b200.types import MatrixKey

from .lineage_support import MODEL, TOKENS, chunk, method, relative_error


@pytest.fixture
def archived(tmp_path):
    store = ObjectStore(tmp_path / "store", verify_reads=True)
    runtime = LineageRuntime(store, MODEL)
    runtime.create_lineage("main")
    nodes, sources = [], []
    for index in range(3):
        m, c = chunk(index)
        sources.append(m)
        nodes.append(runtime.commit_node("main", f"c{index}", m, c, method=method()).node_ref)
    yield runtime, nodes, sources
    store.close()


def test_staging_engine_reads_and_verifies(archived, tmp_path):
    runtime, nodes, _ = archived
    ids = sorted({ref for ref in runtime.store.references(nodes[-1])})
    blobs = [i for i in ids if not i.startswith("manifest:")] or ids
    engine = StagingEngine(runtime.store, pinned_bytes=8 << 20, threads=4)
    staged = engine.stage(blobs)
    for object_id in blobs:
        assert staged.bytes(object_id) == runtime.store.get(object_id)
    staged.release()
    # corrupt one payload: the staged hash check refuses it
    victim = next(i for i in runtime.store.list_refs() and blobs)
    path = runtime.store.path_for(victim)
    data = bytearray(path.read_bytes())
    data[0] ^= 0xFF
    path.write_bytes(bytes(data))
    with pytest.raises(IntegrityError):
        engine.stage([victim])


def test_packed_restorer_with_decoder_pool_and_tier(archived):
    runtime, nodes, sources = archived
    pool = DecoderPool(2)
    tier = DecodedTier(64 << 20, route="all")
    restorer = PackedRestorer(runtime, pool, decoded_tier=tier, device="cpu")
    pieces = restorer.plan(nodes[-1])
    # warm the tier with one pack's decoded tiles (as an archival validation decode would)
    first = restorer.prepared(restorer.runtime.load_record(pieces[0].entry.records[0][1]).packet_ref)
    tier.offer(first.digest, [pool.decode_stream(first.stream, first.stream_codec, first.raw_shape).wait()])
    batch = restorer.submit(pieces, MODEL.layers)
    assert first.packet_ref in batch.routed
    heads, head_dim = 2, MODEL.channels_for("K") // 2
    caches = {(l, t): torch.zeros((1, 3 * TOKENS, heads, head_dim)) for l in range(MODEL.layers) for t in "KV"}
    table = rk.RopeTable.wan(head_dim, 32)
    for layer in range(MODEL.layers):
        handle = restorer.reconstruct(batch, pieces, layer, lambda l, w: caches[(l, w)],
                                      lambda piece: (table, (2 * (piece.token_start // TOKENS), 0, 0)))
        handle.synchronize()
    restorer.release(batch)
    for layer in range(MODEL.layers):
        got = caches[(layer, "V")].reshape(3 * TOKENS, -1)
        expect = torch.cat([s[MatrixKey(layer, "V")] for s in sources])
        assert relative_error(got, expect) < 0.1
    assert pool.stats()["decoded"] >= 2 and tier.stats()["routed"] == 1
    pool.close()


def test_decoded_tier_deficit_route():
    tier = DecodedTier(1 << 20, route="deficit", layer_ms=(1.5, 0.0, None), decode_gbps=1.0)
    for i in range(4):
        tier.bind(f"p{i}", f"d{i}")
        tier.offer(f"d{i}", [torch.zeros(1000, dtype=torch.uint8).numpy()])
    # 4 packs of 30 MB over 30 layers: 4 ms of decode per layer vs a 0.85 x 1.5 ms budget -> route the oldest 3
    routed = tier.route([(f"p{i}", 30_000_000) for i in range(4)], layers=30)
    assert routed == ["p0", "p1", "p2"]
    tier.release(routed)
    assert tier.forget_packets(["p0"]) == 1


def test_archive_eviction_budget(archived):
    runtime, nodes, _ = archived
    store = runtime.store
    sizes = {}
    objects = {}
    for ref in nodes:
        payload = [o for o in store.references(ref) if not o.startswith("manifest:")]
        packet = runtime.load_node(ref).packet_ref
        payload += [o for o in store.references(packet) if not o.startswith("manifest:")]
        objects[ref] = set(payload)
        sizes[ref] = sum(store.object_size(o) for o in objects[ref])
    budget = sum(sizes.values()) + 1
    evictor = ArchiveEviction(store, budget)
    for ref in nodes:
        evictor.published(ref, objects[ref])
    assert evictor.live_bytes <= budget
    evictor.touch([nodes[0]])  # node 0 is now the most recently used
    with evictor.pin([nodes[1]]):
        evictor.reserve(sizes[nodes[2]] // 2 + 1)  # evicts the least recently used unpinned node: node 2
    assert evictor.evicted(nodes[2]) and not evictor.evicted(nodes[1])
    with pytest.raises(CapacityError):
        evictor.reserve(budget * 10)


def test_device_pressure_and_telemetry():
    registry = DeviceTrimRegistry()
    freed = []

    class Cache:
        def trim(self, reason):
            freed.append(reason)
            return 100

    cache = Cache()
    registry.register("restorer:test", cache.trim)
    registry.register("decoder_pool", lambda reason: 1 / 0)
    result = registry.trim("oom", empty_cache=lambda: None)
    assert result["bytes"] == 100 and freed == ["oom"]
    assert result["trims"][0]["name"] == "decoder_pool" and "error" in result["trims"][0]
    del cache
    assert [r["name"] for r in registry.registered()] == ["decoder_pool"]
    collector = RuntimeTelemetry()
    with collector.capture():
        with span("store.read", nbytes=10):
            pass
    snap = collector.snapshot()
    assert snap["stages"]["store.read"]["completed_bytes"] == 10


def test_layer_prefetch_packed_prefetch_and_paired_decode(archived):
    from reelcache_b200.prefetch import LayerPrefetcher, PackedLayerPrefetcher, PairedDecoder
    runtime, nodes, sources = archived
    channels = MODEL.channels_for("K")
    prefetch = LayerPrefetcher(runtime, device="cpu", layers=MODEL.layers, channels=channels,
                               native_dtype=torch.float32, max_bytes=1 << 26)
    prefetch.begin(nodes[-1])
    for layer in range(MODEL.layers):
        tensors = prefetch.acquire(layer)
        expect = torch.cat([s[MatrixKey(layer, "V")] for s in sources])
        assert relative_error(tensors[("V", None)], expect) < 0.1
        prefetch.release(layer)
    assert prefetch.stats()["layers"] == MODEL.layers
    prefetch.close()
    pool = DecoderPool(2)
    restorer = PackedRestorer(runtime, pool, device="cpu")
    packed = PackedLayerPrefetcher(restorer, depth=1)
    packed.begin(nodes[-1], layers=MODEL.layers)
    heads, head_dim = 2, channels // 2
    caches = {(l, t): torch.zeros((1, 3 * TOKENS, heads, head_dim)) for l in range(MODEL.layers) for t in "KV"}
    table = rk.RopeTable.wan(head_dim, 32)
    for layer in range(packed.layers):
        packed.restore(layer, lambda l, w: caches[(l, w)],
                       lambda piece: (table, (2 * (piece.token_start // TOKENS), 0, 0))).synchronize()
    packed.end()
    got = caches[(0, "V")].reshape(3 * TOKENS, -1)
    assert relative_error(got, torch.cat([s[MatrixKey(0, "V")] for s in sources])) < 0.1
    prep = restorer.prepared(restorer.runtime.load_record(restorer.plan(nodes[-1])[0].entry.records[0][1]).packet_ref)
    paired = PairedDecoder(pool, max_output_bytes=1 << 26)
    k, v = paired.decode_pair((prep.stream, prep.stream_codec, prep.raw_shape), (prep.stream, prep.stream_codec,
                                                                                prep.raw_shape))
    assert k.tobytes() == v.tobytes() and paired.stats()["pairs"] == 1
    pool.close()


def test_raw_tier_machine_budgets_and_host_pool(tmp_path):
    """Host budgets come from the cgroup limit (v2 or v1) and MemAvailable, split over the node's workers; the
    pinned host pool hands back blocks by size class."""
    from reelcache_b200.raw_tier import HostPool, auto_host_budget, cgroup_memory_limit, meminfo_available
    root = tmp_path / "cg"
    (root).mkdir()
    (root / "memory.max").write_text("8589934592\n")
    meminfo = tmp_path / "meminfo"
    meminfo.write_text("MemTotal: 100000000 kB\nMemAvailable: 4194304 kB\n")
    assert cgroup_memory_limit(str(root)) == 8 << 30
    assert meminfo_available(str(meminfo)) == 4 << 30
    # the smaller of the two (4 GiB), half of it, over two workers
    assert auto_host_budget(fraction=0.5, workers=2, cgroup_root=str(root), meminfo=str(meminfo)) == 1 << 30
    (root / "memory.max").write_text("max\n")
    assert cgroup_memory_limit(str(root)) is None
    v1 = tmp_path / "v1"
    (v1 / "memory").mkdir(parents=True)
    (v1 / "memory" / "memory.limit_in_bytes").write_text(str(2 << 30))
    assert cgroup_memory_limit(str(v1)) == 2 << 30
    pool = HostPool(pinned=False, cached_bytes=8 << 20, min_block=1 << 20)
    a = pool.take(3 << 20)
    assert a.numel() == 4 << 20
    view = pool.view(a, (1024, 256), torch.float32)
    assert view.shape == (1024, 256)
    pool.give(a)
    b = pool.take((3 << 20) + 5)
    assert b.data_ptr() == a.data_ptr() and pool.stats["reused"] == 1


def test_layer_compute_model_lookup_and_route_record():
    from reelcache_b200.decoded_tier import LAYER_COMPUTE_MS, layer_compute_model, offer_decoded, open_tiers

    assert layer_compute_model("Wan-LongLive2-1.3B")[3] == "default:longlive2"      # longest contained name wins
    assert layer_compute_model("longlive1-x")[:3] == LAYER_COMPUTE_MS["longlive1"]
    assert layer_compute_model("unknown")[3].startswith("default:causvid")
    assert layer_compute_model("causvid", [1.0, 0.25]) == (1.0, 0.25, None, "configured")
    with pytest.raises(ConfigurationError):
        layer_compute_model(None, [1.0])
    tier = DecodedTier(1 << 20, route="deficit", layer_ms=[1.0, 0.0], decode_gbps=1.0, register=True)
    try:
        tiles = [np.full((100, 8), 3, dtype=np.uint8)]
        assert offer_decoded("digest-a", tiles) == 1 and tier in open_tiers()
        tier.bind("pack-a", "digest-a")
        # two packs of 2 MB over 1 layer at 1 GB/s: 4 ms predicted; the target is 0.85 x 1 ms
        chosen = tier.route([("pack-a", 2_000_000), ("pack-b", 2_000_000)], layers=1)
        assert chosen == ["pack-a"]
        record = tier.last_route
        assert record["hits"] == 1 and record["misses"] == 1 and record["c_model"] == "configured"
        assert record["predicted_decode_ms_per_layer"] == pytest.approx(4.0)
        assert record["predicted_decode_ms_per_layer_after"] == pytest.approx(2.0)
        tier.release(chosen)
    finally:
        tier.close()
    assert tier not in open_tiers()
