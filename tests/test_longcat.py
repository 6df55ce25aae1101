"""LongCat-shaped DiT on CPU (tiny geometry, plain-torch ops): context-parallel forward over Gloo equals
the single-rank forward, and the conditioning-cache seam archives a built cache as a segment node and
restores it (this rank's rows under CP)."""

import os
import socket
import traceback

import pytest
import torch
import torch.multiprocessing as mp

TINY = dict(layers=2, dim=128, heads=4, head_dim=32, ffn=256, text_dim=64, text_len=8, in_channels=4,
            latent_height=8, latent_width=12)


def _model():
    from reelcache_b200.models.longcat import LongCatConfig, LongCatDiT
    return LongCatDiT(LongCatConfig(**TINY), "cpu", seed=1, use_kernels=False, max_frames=16)


def _inputs(model, frames=2, seed=2):
    g = torch.Generator().manual_seed(seed)
    latents = torch.randn(model.cfg.in_channels, frames, model.cfg.latent_height, model.cfg.latent_width, generator=g)
    text = model.encode_text(torch.randn(model.cfg.text_len, model.cfg.text_dim, generator=g))
    return latents, text


def _cp_worker(rank, world, port, errors):
    import datetime
    import torch.distributed as dist
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    try:
        dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
        from reelcache_b200.models.longcat import ConditioningCacheEpoch
        model = _model()
        latents, text = _inputs(model)
        cond, _ = _inputs(model, frames=1, seed=5)
        epoch = ConditioningCacheEpoch("e0", 0, 0, 1)
        full_cache = model.build_conditioning_cache(cond, epoch)
        local_cache = model.build_conditioning_cache(cond, epoch, cp_group=dist.group.WORLD)
        ref = model.forward(latents, 0.5, text, first_frame=1, cache=full_cache)
        got = model.forward(latents, 0.5, text, first_frame=1, cache=local_cache, cp_group=dist.group.WORLD)
        assert torch.allclose(got, ref, atol=2e-2, rtol=2e-2), (got - ref).abs().max()
    except BaseException:  # noqa: BLE001
        errors.put((rank, traceback.format_exc()))
    finally:
        if torch.distributed.is_initialized():
            torch.distributed.destroy_process_group()


def test_context_parallel_matches_single_rank():
    ctx = mp.get_context("spawn")
    errors = ctx.Queue()
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    procs = [ctx.Process(target=_cp_worker, args=(r, 2, port, errors)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(180)
    failures = []
    while not errors.empty():
        failures.append(errors.get())
    assert not failures, "\n".join(tb for _, tb in failures)


def test_conditioning_cache_seam(tmp_path):
    from reelcache_b200.lineage import LineageRuntime
    from reelcache_b200.models.longcat import ConditioningCacheEpoch, ReelCacheConditioningCacheBackend
    from reelcache_b200.rank_method import RankMethodConfig
    from reelcache_b200.store import ObjectStore
    from reelcache_b200.types import CodecSpec, ModelIdentity, energy_targets
    model = _model()
    cfg = model.cfg
    store = ObjectStore(tmp_path / "store")
    identity = ModelIdentity("longcat-tiny", "seed1", cfg.layers, cfg.dim, "BTHD", "bfloat16")
    runtime = LineageRuntime(store, identity)
    runtime.create_lineage("session")
    method = RankMethodConfig(energy_targets("longcat_720p"), CodecSpec("svd_hevc", 32), solver="gram_eigh")
    backend = ReelCacheConditioningCacheBackend(runtime, "session", method, head_dim=cfg.head_dim, grid=cfg.grid)
    latents, text = _inputs(model)
    cond, _ = _inputs(model, frames=2, seed=9)
    epoch = ConditioningCacheEpoch("seg-0", 0, 0, 2)
    assert backend.restore(epoch) is None
    built = model.build_conditioning_cache(cond, epoch)
    backend.on_cache_built(built)
    restored = backend.restore(epoch)
    assert restored is not None and restored.tokens == built.tokens
    for a, b in zip(built.k, restored.k):
        rel = float((a.float() - b.float()).norm() / a.float().norm())
        assert rel < 0.2
    ref = model.forward(latents, 0.5, text, first_frame=2, cache=built)
    got = model.forward(latents, 0.5, text, first_frame=2, cache=restored)
    assert float((got - ref).norm() / ref.norm()) < 0.1
    store.close()


def test_epoch_tiers_planning_gate_and_session_provider(tmp_path):
    import threading
    import time

    from reelcache_b200.lineage import LineageRuntime
    from reelcache_b200.models.longcat import ConditioningCacheEpoch, ReelCacheConditioningCacheBackend
    from reelcache_b200.models.longcat_session import (EpochRawTiers, HostFull, LongCatSessionProvider, PlanningGate,
                                                       gated_plan_chunk)
    from reelcache_b200.rank_method import RankMethodConfig, plan_chunk
    from reelcache_b200.store import ObjectStore
    from reelcache_b200.types import CodecSpec, ModelIdentity, energy_targets
    model = _model()
    cfg = model.cfg
    store = ObjectStore(tmp_path / "store")
    identity = ModelIdentity("longcat-tiny", "seed1", cfg.layers, cfg.dim, "BTHD", "bfloat16")
    runtime = LineageRuntime(store, identity)
    runtime.create_lineage("s")
    method = RankMethodConfig(energy_targets("longcat_720p"), CodecSpec("svd_hevc", 32), solver="gram_eigh")
    backend = ReelCacheConditioningCacheBackend(runtime, "s", method, head_dim=cfg.head_dim, grid=cfg.grid)
    tiers = EpochRawTiers(host_raw_budget_bytes=1 << 30, pin_memory=False)
    provider = LongCatSessionProvider(model, backend, tiers)
    cond, text = _inputs(model, frames=2, seed=4)
    built, tier = provider.segment_cache("s", 0, cond, text, first_frame=0)
    assert tier == "built"
    again, tier = provider.segment_cache("s", 1, cond, text, first_frame=2)  # same content: the host tier serves it
    assert tier == "host_raw" and torch.equal(again.k[0], built.k[0])
    cond2, _ = _inputs(model, frames=2, seed=8)
    provider.segment_cache("s", 2, cond2, text, first_frame=4)
    assert [b["segment"] for b in provider.boundaries("s")] == [0, 1, 2]
    kept = provider.resume("s", 1, new_session="fork")
    assert [b["segment"] for b in provider.boundaries("fork")] == [0, 1] and len(kept) == 2
    # a fork whose epoch left every raw tier restores the archived node of the same content (its epoch id differs)
    provider.tiers = EpochRawTiers(host_raw_budget_bytes=0, pin_memory=False)
    forked, tier = provider.segment_cache("fork", 2, cond2, text, first_frame=4, base=kept)
    assert tier == "compressed_cold" and backend.stats["restored"] == 1
    assert forked.epoch.epoch_id.startswith("fork:2:") and forked.tokens == built.tokens
    fresh = LongCatSessionProvider(model, backend, EpochRawTiers(host_raw_budget_bytes=0, pin_memory=False))
    fresh.resume("s", 2, new_session="fork2")     # a new provider learns the nodes from the session record
    _, tier = fresh.segment_cache("fork2", 2, cond2, text, first_frame=4)
    assert tier == "compressed_cold"
    # the host tier evicts only published epochs; with no room for unpublished ones it refuses
    small = EpochRawTiers(host_raw_budget_bytes=1, host_slots=1, pin_memory=False)
    small.capture("a", built)
    with pytest.raises(HostFull):
        small.capture("b", built)
    small.published("a", "node-a")
    assert small.stats()["entries"] == 0 and small.stats()["evictions"] == 1
    # planning gate: a section waits for the unit in progress; a unit waits for an open section
    gate = PlanningGate()
    order = []

    def unit():
        with gate.unit():
            order.append("unit-start")
            time.sleep(0.2)
            order.append("unit-end")

    worker = threading.Thread(target=unit)
    worker.start()
    time.sleep(0.05)
    with gate.section(release_memory=False):
        order.append("section")
    worker.join()
    assert order == ["unit-start", "unit-end", "section"]
    # gated planning equals ungated planning
    from .lineage_support import chunk, method as lm
    matrices, contexts = chunk(0)
    a = plan_chunk(matrices, contexts, lm(), None, {}, {})
    b = gated_plan_chunk(gate, matrices, contexts, lm(), None, {}, {})
    assert all(torch.equal(a[k].rows, b[k].rows) for k in a)
    store.close()


def test_conditioning_cache_depends_only_on_latents():
    """Sessions share an archived segment through its content key (model, latents digest, grid), so the cache
    must not depend on the prompt or on where the segment sits in the video: two builds from the same latents
    with different epochs (first frames) are identical, and the content key ignores the text."""
    from reelcache_b200.models.longcat import ConditioningCacheEpoch
    from reelcache_b200.models.longcat_session import content_key
    model = _model()
    cond, _ = _inputs(model, frames=2, seed=9)
    a = model.build_conditioning_cache(cond, ConditioningCacheEpoch("a", 0, 0, 2))
    b = model.build_conditioning_cache(cond, ConditioningCacheEpoch("b", 3, 6, 2))
    for x, y in zip(a.k + a.v, b.k + b.v):
        assert torch.equal(x, y)
    other, _ = _inputs(model, frames=2, seed=10)
    assert content_key("m", cond, model.cfg.grid) == content_key("m", cond.clone(), model.cfg.grid)
    assert content_key("m", cond, model.cfg.grid) != content_key("m", other, model.cfg.grid)
