"""Asynchronous archival (ordered publication, backpressure, failure propagation) and the raw tier's
invariants, on CPU."""

import threading

import pytest
import torch

from reelcache_b200.archive_pipeline import ArchivePipeline
from reelcache_b200.errors import CapacityError, StateError
from reelcache_b200.lineage import LineageRuntime
from reelcache_b200.predictor_registry import RankPredictorRegistry
from reelcache_b200.raw_tier import RawChunkTier
from reelcache_b200.store import ObjectStore
from reelcache_b200.types import MatrixKey

from .lineage_support import chunk, method, relative_error


@pytest.fixture
def runtime(tmp_path):
    store = ObjectStore(tmp_path / "store")
    rt = LineageRuntime(store, __import__("tests.lineage_support", fromlist=["MODEL"]).MODEL,
                        registry=RankPredictorRegistry("t"))
    yield rt
    store.close()


def test_pipeline_publishes_in_order_and_matches_sync(runtime, tmp_path):
    runtime.create_lineage("a")
    runtime.create_lineage("b")
    pipe = ArchivePipeline(runtime, method=method(), device="cpu", max_unpublished=3)
    tickets = []
    for index in range(3):
        m, c = chunk(index)
        tickets.append(pipe.submit("a", f"c{index}", m, c))
        m2, c2 = chunk(index, seed=5)
        pipe.submit("b", f"c{index}", m2, c2)
    pipe.drain(timeout=120)
    refs = [t.result(0) for t in tickets]
    assert runtime.lineage_head("a") == refs[-1]
    path = [ref for ref, _, _ in runtime.node_path(refs[-1])]
    assert path[-3:] == refs  # strict order: each node's parent is its predecessor
    assert pipe.frontiers("a")["generated"] == 3 and pipe.frontiers("a")["unpublished"] == 0
    # restored history equals what a synchronous commit chain would hold
    key = MatrixKey(1, "V")
    restored = runtime.acquire_node_history(refs[-1], key)
    source = torch.cat([chunk(i)[0][key] for i in range(3)])
    assert relative_error(restored, source) < 0.1
    pipe.close()


def test_failure_propagates_and_reset(runtime):
    runtime.create_lineage("a")
    pipe = ArchivePipeline(runtime, method=method(), device="cpu", max_unpublished=4)
    m, c = chunk(0)
    bad = {k: v[:-1] for k, v in m.items()}  # wrong token count: planning fails
    m1, c1 = chunk(1)
    with pipe.defer_gpu_work():  # both queued before the first one fails
        t0 = pipe.submit("a", "c0", bad, c)
        t1 = pipe.submit("a", "c1", m1, c1)
    with pytest.raises(StateError):
        pipe.drain("a", timeout=60)
    assert t0.state == "failed" and t1.state == "failed"
    with pytest.raises(StateError):
        pipe.submit("a", "c2", m1, c1)
    assert pipe.reset("a") is not None
    t = pipe.submit("a", "c0", m, c)
    assert t.result(60).startswith("manifest:")
    pipe.close()


def test_backpressure_capacity_error(runtime):
    runtime.create_lineage("a")
    pipe = ArchivePipeline(runtime, method=method(), device="cpu", max_unpublished=1, submit_timeout=0.0)
    with pipe.defer_gpu_work():  # nothing plans while deferred: the backlog stays full
        m, c = chunk(0)
        pipe.submit("a", "c0", m, c)
        m1, c1 = chunk(1)
        with pytest.raises(CapacityError):
            pipe.submit("a", "c1", m1, c1)
    pipe.drain(timeout=60)
    pipe.close()


def _tensors(n, value=1.0):
    return {MatrixKey(0, "K"): torch.full((n, 4), value), MatrixKey(0, "V"): torch.full((n, 4), value)}


def test_raw_tier_invariants():
    tier = RawChunkTier("cpu", gpu_budget_bytes=256, host_budget_bytes=512, retain="lru")
    a = tier.admit(_tensors(8, 1.0), "c0", holder="s")   # 256 B
    b = tier.admit(_tensors(8, 2.0), "c1", holder="s")   # device full: c0 demoted to host (copy first)
    s = tier.stats()
    assert s["gpu_bytes"] <= 256 and s["host_bytes"] == 256 and s["entries"] == 2
    assert torch.equal(tier.source(a)[MatrixKey(0, "K")], torch.full((8, 4), 1.0))  # re-staged from host
    tier.published(a, "manifest:a")
    tier.published(b, "manifest:b")
    with tier.lookup("manifest:a") as lease:
        assert torch.equal(lease.tensors[MatrixKey(0, "V")], torch.full((8, 4), 1.0))
    tier.release_holder("s")           # retain=lru: unheld entries stay as cache
    assert tier.stats()["entries"] == 2
    lease = tier.lookup("manifest:b")
    assert lease.retained
    lease.release()
    c = tier.admit(_tensors(16, 3.0), "c2")   # 512 B: unheld published entries are evicted first
    assert tier.stats()["unpublished"] == 1
    tier.failed(c)
    assert tier.lookup("manifest:missing") is None
    tier.close()


def test_raw_tier_backpressure_when_full_of_unpublished():
    tier = RawChunkTier("cpu", gpu_budget_bytes=256, host_budget_bytes=0, backpressure_timeout=0.2)
    tier.admit(_tensors(8), "c0")
    with pytest.raises(CapacityError):
        tier.admit(_tensors(8), "c1")
    done = threading.Event()

    def publish_later():
        tier.published(1, "manifest:x")
        done.set()

    threading.Timer(0.05, publish_later).start()
    tier.backpressure_timeout = 5.0
    tier.admit(_tensors(8), "c2")  # admitted once the first entry is published (and dropped: no holders)
    assert done.is_set()
    tier.close()


def test_pause_lands_at_a_planning_boundary(runtime):
    """A pause taken while a node plans is acknowledged at the planner's next lockstep round; the node waits
    there until the pause ends, then publishes."""
    import time
    runtime.create_lineage("a")
    pipe = ArchivePipeline(runtime, method=method(solver="topk_rr"), device="cpu", max_unpublished=2)
    entered, release = threading.Event(), threading.Event()
    original = pipe._step_boundary

    def gated():
        entered.set()
        release.wait(30)
        original()
    pipe._step_boundary = gated
    try:
        m, c = chunk(0)
        ticket = pipe.submit("a", "c0", m, c)
        assert entered.wait(30)
        records = []

        def pause():
            with pipe.pause_gpu_work(ack_timeout=20) as record:
                records.append(record)
                time.sleep(0.3)
                records.append(ticket.state)
        worker = threading.Thread(target=pause)
        worker.start()
        time.sleep(0.05)
        release.set()
        worker.join(60)
        assert records[0]["acked"] and records[0]["inflight"] and records[0]["landed"] == "boundary"
        assert records[1] == "planning"            # held at the boundary for the whole section
        assert ticket.result(60)
        stats = pipe.stats()["fitter_pause"]
        assert stats["requests"] == 1 and stats["acked"] == 1 and stats["paused_seconds"] > 0.2
        with pipe.pause_gpu_work() as record:      # nothing on the GPU: acknowledged at once
            assert record["landed"] == "idle"
    finally:
        release.set()
        pipe.close()


def test_detach_hands_unpublished_chunks_to_a_side_lineage(runtime):
    runtime.create_lineage("a")
    pipe = ArchivePipeline(runtime, method=method(), device="cpu", max_unpublished=4)
    try:
        m, c = chunk(0)
        pipe.submit("a", "c0", m, c).result(120)
        cut = runtime.lineage_head("a")
        with pipe.defer_gpu_work():                 # keep the next chunks queued
            tickets = [pipe.submit("a", f"c{i}", *chunk(i)) for i in (1, 2)]
            record = pipe.detach("a", "a-side")
        assert record == {"branch": "a-side", "moved": ["c1", "c2"], "cut": cut}
        pipe.drain("a-side", timeout=120)
        assert runtime.lineage_head("a") == cut    # the original head never moved
        side = runtime.lineage_head("a-side")
        assert tickets[1].result(0) == side and runtime.load_node(side).frontier == 3 * c[MatrixKey(0, "K")].token_count
        assert pipe.detach("a", "a-other")["moved"] == []
        report = pipe.prewarm(c)
        assert report["fresh_plan_seconds"] > 0 and report["decisions"] and pipe.stats()["prewarm"][0]["total_seconds"] > 0
    finally:
        pipe.close()
