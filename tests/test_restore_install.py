"""Generation-first archival holds, the KV lease, RoPE table cache, dense installs and plan-slot placement of
lineage installs, on CPU."""

import threading
import time

import pytest
import torch

from reelcache_b200 import restore_kernels as rk
from reelcache_b200.archive_pipeline import ArchivePipeline
from reelcache_b200.archive_restore import SoftwareLineageRestorer
from reelcache_b200.errors import StateError
from reelcache_b200.integrations.sglang.generation_defer import GenerationDefer, decode_reason
from reelcache_b200.integrations.sglang.restore import (AttentionKVLease, DenseInstall, LineageInstall,
                                                        RopeTableCache, kernel_warmup_shapes)
from reelcache_b200.integrations.sglang.visibility import TokenSpan, VisibilityPlan
from reelcache_b200.lineage import LineageRuntime
from reelcache_b200.store import ObjectStore
from reelcache_b200.types import MatrixKey

from .lineage_support import FRAMES, HEIGHT, MODEL, TOKENS, WIDTH, chunk, method, relative_error
from .test_sglang_bridge import TINY, make_bridge

HEADS = 2


@pytest.fixture
def runtime(tmp_path):
    store = ObjectStore(tmp_path / "store")
    rt = LineageRuntime(store, MODEL)
    yield rt
    store.close()


def test_generation_hold_defers_fitting_until_closed(runtime):
    runtime.create_lineage("a")
    pipe = ArchivePipeline(runtime, method=method(), device="cpu", max_unpublished=4)
    try:
        record = pipe.open_generation("req-1")
        assert record["archival_defer_wait"] == 0.0
        m, c = chunk(0)
        ticket = pipe.submit("a", "c0", m, c)
        time.sleep(0.3)
        assert ticket.state == "queued" or not ticket.done()  # held: no planning inside the hold
        closed = pipe.close_generation("req-1")
        assert closed["held_seconds"] > 0.25
        ticket.result(60)
        stats = pipe.stats()["generation_defer"]
        assert stats["holds_opened"] == 1 and stats["open_holds"] == 0
        # a waiting drain overrides a hold (starvation guard)
        pipe.open_generation("req-2")
        m, c = chunk(1)
        pipe.submit("a", "c1", m, c)
        pipe.drain("a", timeout=60)
        assert pipe.stats()["generation_defer"]["starvation_overrides"] >= 1
        pipe.close_generation("req-2")
    finally:
        pipe.close()


def test_generation_hold_waits_for_inflight_node(runtime):
    runtime.create_lineage("a")
    pipe = ArchivePipeline(runtime, method=method(), device="cpu", max_unpublished=4)
    try:
        m, c = chunk(0)
        ticket = pipe.submit("a", "c0", m, c)
        deadline = time.monotonic() + 30
        while not pipe._planning and not ticket.done() and time.monotonic() < deadline:
            time.sleep(0.001)
        record = pipe.open_generation("r", inflight="wait")
        assert not pipe._planning  # the node on the GPU finished before the hold opened
        if record["archival_defer_wait"] > 0:
            assert pipe.stats()["generation_defer"]["inflight_waits"] == 1
        pipe.close_generation("r")
        ticket.result(60)
        with pipe.generation("o", inflight="overlap") as overlap:
            assert overlap["inflight_overlaps"] in (0, 1)
    finally:
        pipe.close()


def test_bridge_generation_defer_records(tmp_path):
    bridge = make_bridge(tmp_path, defer_archival_during_generation=True, archival_defer_inflight="overlap")
    try:
        assert bridge.defer is not None
        report = bridge.request("s", chunks=2, action="create", seed=1)
        assert report["archival_defer"]["closed_by"] == "finish"
        with bridge.memory_critical_section("vae_decode"):
            pass
        again = bridge.request("s", chunks=1, seed=1)
        assert again["archival_defer"] is not None
        bridge.pause("s")
    finally:
        bridge.shutdown()
    assert decode_reason("decode") and decode_reason("vae_decode") and not decode_reason("prefill")


def test_lease_and_rope_cache():
    released = []
    lease = AttentionKVLease(description={"x": 1})

    class Handle:
        def __init__(self):
            self.synced = False

        def synchronize(self):
            self.synced = True

    handle = Handle()
    lease.track(handle=handle, staging=torch.zeros(3), finalizer=lambda: released.append(1))
    lease.close()
    assert handle.synced and released == [1]
    with pytest.raises(StateError):
        lease.track(handle=Handle())
    cache = RopeTableCache(max_bytes=4096)
    calls = []
    bound = cache.bind(lambda start, frames: (calls.append(start) or torch.zeros(frames, 8),
                                              torch.ones(frames, 8)), grid=(4, 8), device="cpu")
    bound(0, 2)
    bound(0, 2)
    bound(3, 2)
    assert calls == [0, 3] and cache.stats()["hits"] == 1
    shapes = kernel_warmup_shapes(TINY)
    assert {s.source for s in shapes} == {"pictures", "dense"}


def _plan(nodes, spans):
    return VisibilityPlan(len(nodes), tuple(spans))


def test_dense_install_matches_reference_rope():
    head_dim = MODEL.channels_for("K") // HEADS
    table = rk.RopeTable.wan(head_dim, 64)
    caches = {(l, t): torch.zeros((1, 2 * TOKENS, HEADS, head_dim)) for l in range(MODEL.layers) for t in "KV"}
    m0, _ = chunk(0)
    m1, _ = chunk(1)
    rows = {"n0": m0, "n1": m1}
    # a window plan: chunk 1's second frame at slot 0, then chunk 0 whole at slot TOKENS // 2
    frame = HEIGHT * WIDTH
    spans = [TokenSpan("n1", 1, frame, frame, 0, TOKENS + frame, "window"),
             TokenSpan("n0", 0, 0, TOKENS, frame, 0, "sink")]
    plan = _plan(["n0", "n1"], spans)
    install = DenseInstall(plan=plan, destination=lambda l, t: caches[(l, t)],
                           rope=lambda span: (table, (FRAMES * span.chunk_index, 0, 0)),
                           rows_of=lambda span, key: rows[span.node_ref][key][span.node_offset:
                                                                               span.node_offset + span.length],
                           grid=(HEIGHT, WIDTH))
    for layer in range(MODEL.layers):
        install.layer(layer).release()
    k = caches[(0, "K")][0]
    expect = rk.apply_rope_reference(m1[MatrixKey(0, "K")][frame:2 * frame].reshape(frame, HEADS, head_dim),
                                     rk.RopePositions(table, (FRAMES * 1 + 1, 0, 0)), (1, HEIGHT, WIDTH))
    assert relative_error(k[:frame], expect) < 1e-6
    v = caches[(1, "V")][0].reshape(2 * TOKENS, -1)
    assert relative_error(v[frame:frame + TOKENS], m0[MatrixKey(1, "V")]) < 1e-7
    assert install.stats()["jobs"] == 2 * 2 * MODEL.layers


def test_lineage_install_places_pieces_at_plan_slots(runtime):
    runtime.create_lineage("main")
    node = None
    for index in range(3):
        m, c = chunk(index)
        node = runtime.commit_node("main", f"c{index}", m, c, method=method()).node_ref
    head_dim = MODEL.channels_for("K") // HEADS
    table = rk.RopeTable.wan(head_dim, 64)
    # attend to chunk 0 (sink) and chunk 2 (window), packed at slots 0 and TOKENS
    spans = [TokenSpan("n0", 0, 0, TOKENS, 0, 0, "sink"), TokenSpan("n2", 2, 0, TOKENS, TOKENS, 2 * TOKENS, "window")]
    plan = _plan(["n0", "n1", "n2"], spans)
    caches = {(l, t): torch.zeros((1, 2 * TOKENS, HEADS, head_dim)) for l in range(MODEL.layers) for t in "KV"}
    install = LineageInstall(plan=plan, destination=lambda l, t: caches[(l, t)],
                             rope_rows=lambda c: (FRAMES * c, 0, 0), table=table, tokens_per_frame=HEIGHT * WIDTH)
    result = install.restore(SoftwareLineageRestorer(runtime, "cpu"), node, overlapped=False)
    result.join()
    dense = runtime.acquire_node_history(node, MatrixKey(1, "V"))
    v = caches[(1, "V")][0].reshape(2 * TOKENS, -1)
    assert relative_error(v[:TOKENS], dense[:TOKENS]) < 5e-3
    assert relative_error(v[TOKENS:], dense[2 * TOKENS:]) < 5e-3


def test_overlapped_raw_install_marks_its_source():
    from reelcache_b200.errors import StateError
    from reelcache_b200.overlapped_restore import LayerReadiness, start_overlapped_install
    issued = []
    readiness = LayerReadiness(4, sources=("restore", "raw"))
    handle = start_overlapped_install(issued.append, 4, readiness=readiness, thread=True)
    for layer in range(4):
        readiness.mark(layer, None, source="restore")
    handle.join(30)
    for layer in range(4):
        readiness.wait(layer)
    assert issued == [0, 1, 2, 3]
    alone = start_overlapped_install(issued.append, 2, thread=False)
    alone.readiness.wait(1)
    with pytest.raises(StateError):
        start_overlapped_install(issued.append, 2, readiness=LayerReadiness(2), thread=False)
