"""Serving bridge on CPU with the synthetic engine: create / resume / pause / checkpoint / rewind /
fork / close / delete through the typed controls; resident reuse, archive restores and the raw tier;
configuration round trips."""

import pytest
import torch

from reelcache_b200.integrations.sglang import (ReelCacheRuntimeConfig, SessionControlError, SyntheticEngine,
                                                create_sglang_backend, session_control)
from reelcache_b200.integrations.sglang.engine import model_identity_for
from reelcache_b200.integrations.sglang.profiles import ModelProfile
from reelcache_b200.errors import ConfigurationError

TINY = ModelProfile("tiny", backbone="tiny-wan", num_layers=2, num_heads=2, head_dim=64, chunk_frames=1,
                    grid=(4, 8), visibility="full_history", sink_frames=0, window_frames=None,
                    energy_profile="causvid")


def make_bridge(tmp_path, **overrides):
    config = ReelCacheRuntimeConfig(store_root=str(tmp_path / "store"), fit_device="cpu", encode_workers=1,
                                    **overrides)
    engine = SyntheticEngine(TINY, model_identity_for(TINY, "synthetic"), "cpu", rank=4)
    return create_sglang_backend(config, engine, cache_chunks=8)


def test_config_round_trip_and_validation(tmp_path):
    config = ReelCacheRuntimeConfig(store_root=str(tmp_path), durability="always", raw_tier_retain="lru")
    data = config.to_dict()
    assert data["schema"] == "reelcache.sglang.runtime_config.v1" and "tree_switch" not in data
    assert ReelCacheRuntimeConfig.from_dict(data) == config
    assert set(config.content_dict()) >= {"representation", "energy_key", "canvas"}
    with pytest.raises(ConfigurationError):
        ReelCacheRuntimeConfig(store_root=str(tmp_path), decoder="nope")
    with pytest.raises(ConfigurationError):
        ReelCacheRuntimeConfig.from_dict({"store_root": str(tmp_path), "unknown_field": 1})
    with pytest.raises(ConfigurationError):
        ReelCacheRuntimeConfig(store_root=str(tmp_path), tree_switch="merge")
    assert ReelCacheRuntimeConfig(store_root=str(tmp_path), tree_switch="detach").to_dict()["tree_switch"] == "detach"


def test_session_lifecycle(tmp_path):
    bridge = make_bridge(tmp_path)
    try:
        first = bridge.request("s", chunks=3, action="create", seed=1)
        assert first["route"] == "none" and first["generated"] == 3
        again = bridge.request("s", chunks=1, seed=1)          # resident cache: no restore
        assert again["route"] == "resident" and again["start_chunk"] == 3
        info = session_control(bridge, "checkpoint", {"session": "s", "name": "four"})
        assert info["chunks"] == 4
        # rewind onto a prefix of the resident path: still resident, the chunk regenerates identically
        session_control(bridge, "rewind", {"session": "s", "checkpoint": 2})
        redo = bridge.request("s", chunks=1, seed=1)
        assert redo["route"] == "resident" and redo["start_chunk"] == 2
        # fork from the named checkpoint: archive restore of 4 chunks, then continue
        fork = bridge.request("f", chunks=1, action="fork", source="s", checkpoint="four", seed=1)
        assert fork["route"] == "archive" and fork["start_chunk"] == 4
        assert fork["restore"]["attended_tokens"] == 4 * TINY.chunk_tokens
        # a resumed session without its resident cache restores from the raw tier / archive and
        # produces the same next chunk as the resident run did
        bridge.pause("s")
        bridge.drop_resident("s")
        resumed = bridge.request("s", chunks=1, seed=1)
        assert resumed["route"] == "archive" and resumed["start_chunk"] == 3
        listing = session_control(bridge, "list")["sessions"]
        assert set(listing) == {"s", "f"}
        described = session_control(bridge, "describe", {"session": "f"})
        assert described["generated"] == 5
        assert any(row.get("name") == "four" for row in session_control(bridge, "checkpoints", {"session": "s"})[
            "checkpoints"])
        session_control(bridge, "delete", {"session": "f"})
        with pytest.raises(SessionControlError) as err:
            session_control(bridge, "describe", {"session": "f"})
        assert err.value.status == 404
        gc = session_control(bridge, "gc")
        assert isinstance(gc, dict)
        assert session_control(bridge, "raw_tier")["enabled"]
    finally:
        bridge.shutdown()


def test_restore_matches_resident_history(tmp_path):
    """Chunks generated after an archive restore see (nearly) the same history as the resident run."""
    bridge = make_bridge(tmp_path, raw_tier=False)
    try:
        bridge.request("a", chunks=3, action="create", seed=7)
        resident = bridge.sessions.get("a").resident.cache
        bridge.pause("a")
        bridge.drop_resident("a")
        bridge.request("a", chunks=0, seed=7)  # restore only
        restored = bridge.sessions.get("a").resident.cache
        tokens = 3 * TINY.chunk_tokens
        for layer in range(TINY.num_layers):
            a, b = resident["k"][layer][:tokens], restored["k"][layer][:tokens]
            assert float((a - b).norm() / a.norm()) < 0.05
        assert bridge.archive.stats()["archive_installs"] > 0
    finally:
        bridge.shutdown()


def test_controls_errors(tmp_path):
    bridge = make_bridge(tmp_path)
    try:
        with pytest.raises(SessionControlError) as err:
            session_control(bridge, "nope")
        assert err.value.status == 404
        with pytest.raises(SessionControlError) as err:
            session_control(bridge, "rewind", {"session": "x"})
        assert err.value.status == 400
        caps = session_control(bridge, "capabilities")
        assert "fork" in caps["ops"]
    finally:
        bridge.shutdown()


@pytest.mark.parametrize("representation,raw_tier,bound", [("raw", False, 1e-7), ("raw_offload", True, 1e-7),
                                                           ("svd", False, 0.05)])
def test_other_representations_restore(tmp_path, representation, raw_tier, bound):
    """RAW (synchronous and write-behind) and SVD-only factor-pack archives restore the session history."""
    bridge = make_bridge(tmp_path, representation=representation, raw_tier=raw_tier, raw_restore="off"
                         if raw_tier else "prefer")
    try:
        bridge.request("a", chunks=3, action="create", seed=7)
        resident = bridge.sessions.get("a").resident.cache
        bridge.pause("a")
        bridge.drop_resident("a")
        report = bridge.request("a", chunks=0, seed=7)
        assert report["route"] == "archive"
        restored = bridge.sessions.get("a").resident.cache
        tokens = 3 * TINY.chunk_tokens
        for layer in range(TINY.num_layers):
            for which in ("k", "v"):
                a, b = resident[which][layer][:tokens], restored[which][layer][:tokens]
                assert float((a - b).norm() / a.norm()) < bound
        stats = bridge.archive.stats()["pipeline"]
        assert stats.get("representation", representation) == representation or representation == "svd"
    finally:
        bridge.shutdown()


def test_resident_caches_stay_under_the_budget(tmp_path):
    """``max_resident_bytes`` bounds the sessions' resident engine caches: creating more sessions than fit drops
    the least recently used residents, and a dropped session's next request restores its history instead."""
    bridge = make_bridge(tmp_path, max_resident_bytes=2 * 8 * 2 * TINY.num_layers * TINY.chunk_tokens
                         * TINY.num_heads * TINY.head_dim * 2)
    try:
        for name in ("a", "b", "c"):
            bridge.request(name, chunks=2, action="create", seed=1)
            bridge.pause(name)
        holders = [s.session_id for s in bridge.sessions.resident_states()]
        assert "c" in holders and len(holders) <= 2 and bridge.resident_evictions >= 1
        report = bridge.request("a", chunks=1, seed=1)
        assert report["route"] == "archive" and report["start_chunk"] == 2
    finally:
        bridge.shutdown()
