"""The bridge's engine seam on CPU with a fake (synthetic) engine: an engine-driven request through
begin_request / restore / capture / end_chunk / finish, prompt-switch recaches (cache epochs that never touch the
sink), recompute restores from stored latents, in-flight controls, tree retention, the decode guard's records and
the plan cache."""

import pytest
import torch

from reelcache_b200.errors import IntegrityError, PendingError, StateError, UnsupportedError
from reelcache_b200.integrations.sglang import ReelCacheRuntimeConfig, SyntheticEngine, create_sglang_backend
from reelcache_b200.integrations.sglang.engine import model_identity_for
from reelcache_b200.integrations.sglang.profiles import ModelProfile
from reelcache_b200.integrations.sglang.seam import (CausalKVRequest, ChunkSlot, RestoreTarget, drive_request,
                                                     plan_recache)
from reelcache_b200.types import MatrixKey

SWITCH = ModelProfile("tiny-switch", backbone="tiny-wan", num_layers=2, num_heads=2, head_dim=32, chunk_frames=1,
                      grid=(4, 4), visibility="full_history", sink_frames=1, window_frames=None,
                      energy_profile="causvid", recache="kv_recache")
PLAIN = ModelProfile("tiny-plain", backbone="tiny-wan", num_layers=2, num_heads=2, head_dim=32, chunk_frames=1,
                     grid=(4, 4), visibility="full_history", sink_frames=0, window_frames=None,
                     energy_profile="causvid")


def make_bridge(tmp_path, profile=SWITCH, **overrides):
    fields = dict(store_root=str(tmp_path / "store"), fit_device="cpu", encode_workers=1, representation="raw")
    fields.update(overrides)
    engine = SyntheticEngine(profile, model_identity_for(profile, "synthetic"), "cpu", rank=4)
    return create_sglang_backend(ReelCacheRuntimeConfig(**fields), engine, cache_chunks=8)


def cache_rows(cache, tokens):
    return [(cache["k"][layer][:tokens].clone(), cache["v"][layer][:tokens].clone()) for layer in range(len(cache["k"]))]


def test_plan_recache_protects_the_sink_and_keeps_whole_chunks():
    assert plan_recache(generated_frames=0, window_frames=-1, sink_frames=1, frame_tokens=16, chunk_frames=1) is None
    plan = plan_recache(generated_frames=4, window_frames=-1, sink_frames=1, frame_tokens=16, chunk_frames=1)
    assert (plan.window_start_frame, plan.write_start_frame, plan.end_frame) == (0, 1, 4)
    assert plan.written_tokens == (16, 64) and plan.discarded_frames == (0, 1)
    # a window shorter than the history, a sink that ends mid-chunk: the partial chunk is re-run but not written
    plan = plan_recache(generated_frames=12, window_frames=9, sink_frames=4, frame_tokens=8, chunk_frames=3)
    assert (plan.window_start_frame, plan.write_start_frame) == (3, 6)
    plan = plan_recache(generated_frames=6, window_frames=-1, sink_frames=2, frame_tokens=8, chunk_frames=3,
                        global_sink=False)
    assert plan.write_start_frame == 0
    with pytest.raises(Exception):
        plan_recache(generated_frames=5, window_frames=-1, sink_frames=0, frame_tokens=8, chunk_frames=3)


def test_engine_driven_seam(tmp_path):
    """A stage that calls the seam itself; protocol violations are refused."""
    bridge = make_bridge(tmp_path, profile=PLAIN)
    engine = bridge.engine
    try:
        run = bridge.begin_request(CausalKVRequest("r1", "s", action="create", chunks=2, seed=3))
        with pytest.raises(PendingError):
            bridge.begin_request(CausalKVRequest("r2", "t", action="create"))
        target = RestoreTarget(engine)
        assert run.restore(target) == 0
        for index in range(2):
            slot = ChunkSlot.of(PLAIN, index)
            capture = run.begin_clean_forward(slot)
            latents = engine.generate_chunk(target.cache, index, capture, request_seed=3)
            run.end_clean_forward(capture)
            assert run.end_chunk(slot, latents) is False
        summary = run.finish(error=None)
        assert summary["chunks"] == 2 and summary["route"] == "none" and summary["error"] is None
        assert bridge.request_summary("r1")["generated"] == 2
        # an incomplete capture is an integrity error, and finish still releases the bridge
        run = bridge.begin_request(CausalKVRequest("r3", "s", chunks=1))
        target = RestoreTarget(engine)
        assert run.restore(target) == 2
        slot = ChunkSlot.of(PLAIN, 2)
        capture = run.begin_clean_forward(slot)
        run.capture_layer(capture, 0, torch.zeros(PLAIN.chunk_tokens, PLAIN.channels),
                          torch.zeros(PLAIN.chunk_tokens, PLAIN.channels))
        run.end_clean_forward(capture)
        with pytest.raises(IntegrityError):
            run.end_chunk(slot, torch.zeros(1))
        failed = run.finish(error=IntegrityError("incomplete"))
        assert failed["error"].startswith("IntegrityError") and bridge.sessions.get("s").resident is None
        assert not bridge.active_request
        # plain requests are not observed by default; with observe_plain_requests they are
        assert bridge.begin_request(CausalKVRequest("p", None, action="create")) is None
        assert [r["request"] for r in bridge.session_requests("s")] == ["r1", "r3"]
    finally:
        bridge.shutdown()
    observer = make_bridge(tmp_path / "o", profile=PLAIN, observe_plain_requests=True)
    try:
        summary = drive_request(observer, observer.engine, CausalKVRequest("p", None, action="create", chunks=2))
        assert summary["observed"] and summary["chunks"] == 2
        assert observer.sessions.sessions() == {}
    finally:
        observer.shutdown()


@pytest.mark.parametrize("representation", ["raw", "svd"])
def test_prompt_switch_recache(tmp_path, representation):
    bridge = make_bridge(tmp_path, representation=representation)
    engine = bridge.engine
    per_chunk = SWITCH.chunk_tokens
    try:
        bridge.request("s", action="create", chunks=3, seed=1, prompt="a cat")
        before = cache_rows(bridge.sessions.get("s").resident.cache, 3 * per_chunk)
        switched = bridge.request("s", chunks=1, seed=1, prompt="a dog")
        assert len(switched["recaches"]) == 1 and switched["recaches"][0]["ranges"] == ["chunk-1", "chunk-2"]
        assert engine.forwards["recache"] == 1
        after = cache_rows(bridge.sessions.get("s").resident.cache, 3 * per_chunk)
        for (k0, v0), (k1, v1) in zip(before, after):
            assert torch.equal(k0[:per_chunk], k1[:per_chunk])          # the sink keeps its KV
            assert not torch.allclose(k0[per_chunk:], k1[per_chunk:])  # the rest was recached
        bridge.pause("s")
        runtime = bridge.archive.runtime
        head = bridge.sessions.head("s")
        pieces = runtime.resolve_history(head, [(0, 4 * per_chunk)])
        assert [p.entry.source for p in pieces] == ["chunk", "epoch", "epoch", "chunk"]
        # the archive's newest KV of the recached range is the recache's (exact for RAW, close for SVD)
        restored = runtime.acquire_node_history(head, MatrixKey(0, "K"), ranges=[(per_chunk, 3 * per_chunk)])
        tol = 0 if representation == "raw" else 2e-2 * float(after[0][0].abs().max())
        assert float((restored - after[0][0][per_chunk:]).abs().max()) <= tol
        # an archive restore of the switched session reproduces the resident history
        resident = cache_rows(bridge.sessions.get("s").resident.cache, 4 * per_chunk)
        bridge.drop_resident("s")
        bridge.archive.raw_tier and bridge.archive.raw_tier.trim_device_cache("test")
        report = bridge.request("s", chunks=0, seed=1)
        assert report["route"] == "archive" and report["prompt"] == "a dog"
        for (k0, v0), (k1, v1) in zip(resident, cache_rows(bridge.sessions.get("s").resident.cache, 4 * per_chunk)):
            assert float((k0 - k1).abs().max()) <= tol and float((v0 - v1).abs().max()) <= max(tol, 0)
        # a profile without KV recache refuses a prompt change on a non-empty session
    finally:
        bridge.shutdown()
    plain = make_bridge(tmp_path / "p", profile=PLAIN)
    try:
        plain.request("s", action="create", chunks=1, prompt="a cat")
        with pytest.raises(UnsupportedError):
            plain.request("s", chunks=1, prompt="a dog")
    finally:
        plain.shutdown()


def test_recompute_restore_replays_the_path(tmp_path):
    """latents_only stores no KV: a restore replays each chunk from its stored latents and each recache under its
    prompt, bit for bit; a raw tier that holds every attended range is used instead of the replay."""
    bridge = make_bridge(tmp_path, representation="latents_only", restore_mode="recompute", raw_tier=False)
    engine = bridge.engine
    per_chunk = SWITCH.chunk_tokens
    try:
        bridge.request("s", action="create", chunks=3, seed=5, prompt="a cat")
        bridge.request("s", chunks=2, seed=5, prompt="a dog")
        resident = cache_rows(bridge.sessions.get("s").resident.cache, 5 * per_chunk)
        node = bridge.archive.runtime.load_node(bridge.sessions.head("s"))
        assert node.matrix_records == ()                           # no KV objects at all
        bridge.drop_resident("s")
        report = bridge.request("s", chunks=1, seed=5)
        assert report["route"] == "recompute" and report["restore"]["steps"] == 6   # 5 chunks + 1 recache
        assert engine.forwards["replay"] == 5
        replayed = cache_rows(bridge.sessions.get("s").resident.cache, 5 * per_chunk)
        for (k0, v0), (k1, v1) in zip(resident, replayed):
            assert torch.equal(k0, k1) and torch.equal(v0, v1)
    finally:
        bridge.shutdown()
    tiered = make_bridge(tmp_path / "t", representation="latents_only", restore_mode="recompute", raw_tier=True)
    try:
        tiered.request("s", action="create", chunks=2, seed=5)
        resident = cache_rows(tiered.sessions.get("s").resident.cache, 2 * per_chunk)
        tiered.drop_resident("s")
        report = tiered.request("s", chunks=0, seed=5)
        assert report["route"] == "raw_tier"
        for (k0, v0), (k1, v1) in zip(resident, cache_rows(tiered.sessions.get("s").resident.cache, 2 * per_chunk)):
            assert torch.equal(k0, k1) and torch.equal(v0, v1)
    finally:
        tiered.shutdown()


def test_inflight_pause_retention_sections_and_plan_cache(tmp_path):
    bridge = make_bridge(tmp_path, profile=PLAIN, tree_retention="full")
    try:
        # a pause queued while the request runs (here by the first boundary's hook) stops it at the next boundary
        bridge.set_boundary_hook(lambda run: bridge.inflight_control("pause", {"session": "s"}))
        report = bridge.request("s", action="create", chunks=4, seed=2)
        assert report["paused"] and report["chunks"] == 2 and report["requested_chunks"] == 4
        bridge.set_boundary_hook(None)
        assert bridge.request("s", chunks=3, seed=2, pause_after_chunks=2)["chunks"] == 2
        # decode sections are filed with the running request (CPU: no device guard)
        seen = []

        def decode(run):
            with bridge.memory_critical_section("vae_decode") as record:
                seen.append(record)
        bridge.set_boundary_hook(decode)
        report = bridge.request("s", chunks=1, seed=2)
        bridge.set_boundary_hook(None)
        assert report["sections"] and report["sections"][0]["reason"] == "vae_decode"
        with bridge.memory_critical_section("idle"):
            pass
        assert bridge.describe()["unattributed_sections"] == 1
        # full retention keeps the branch a rewind leaves
        bridge.pause("s")
        left = bridge.sessions.head("s")
        bridge.request("s", action="rewind", checkpoint=1, chunks=1, seed=9)
        assert bridge.sessions.retained("s") == [left]
        bridge.collect_garbage()
        assert bridge.archive.runtime.load_node(left).frontier == 5 * PLAIN.chunk_tokens
        # the plan cache serves a repeated restore of the same head
        bridge.pause("s")
        for _ in range(2):
            bridge.drop_resident("s")
            bridge.request("s", chunks=0)
        assert bridge.plans.hits >= 1
        with pytest.raises(StateError):
            bridge.begin_request(CausalKVRequest("x", "s")).begin_replay()
    finally:
        bridge._active = None
        bridge.shutdown()


def test_workload_record_of_a_restoring_request(tmp_path):
    bridge = make_bridge(tmp_path, profile=PLAIN, workload_telemetry=True)
    try:
        bridge.request("s", action="create", chunks=2, seed=1)
        bridge.pause("s")
        bridge.drop_resident("s")
        report = bridge.request("s", action="rewind", checkpoint=1, chunks=1, seed=1)
        record = report["workload"]
        names = [s["name"] for s in record["spans"]]
        assert {"request_begin", "drain", "restore_sync", "first_forward", "chunk_commit"} <= set(names)
        assert len(record["exposed_stalls"]) == PLAIN.num_layers and record["exposed_stall_ms"] >= 0
        assert record["bytes"]["restored_native_bytes"] == PLAIN.chunk_tokens * 2 * PLAIN.num_layers * PLAIN.channels * 2
        assert bridge.workload_record(report["request"]) is not None
    finally:
        bridge.shutdown()


def test_restore_records_tiers_gc_and_verification(tmp_path):
    import gc
    from reelcache_b200.integrations.sglang.restore import GC_PAUSES, check_restorable, gc_pause_record
    bridge = make_bridge(tmp_path, profile=PLAIN, verify_reads=True)
    try:
        bridge.request("s", action="create", chunks=2, seed=1)
        resident = bridge.request("s", chunks=1, seed=1)
        assert resident["restore"]["lease"]["tiers"]["chunks"] == {"resident": 2}
        bridge.pause("s")
        bridge.drop_resident("s")
        restored = bridge.request("s", chunks=0)
        lease = restored["restore"]["lease"]
        assert lease["verification"]["mode"] == "sync" and sum(lease["tiers"]["chunks"].values()) == 3
        assert set(lease["tiers"]["chunks"]) <= {"gpu_raw", "compressed"}
        assert restored["restore"]["gc"]["available"]
        before = GC_PAUSES.snapshot()
        gc.collect()
        assert gc_pause_record(before, GC_PAUSES.snapshot())["collections"][2] >= 1
        check_restorable(bridge.plans.get((bridge.sessions.head("s"), 3)) or type("P", (), {"spans": ()})())
    finally:
        bridge.shutdown()
