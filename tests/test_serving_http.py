"""The HTTP surface over a synthetic-engine bridge: generation requests with a ``causal_kv_session`` handle
(generate / resume / rewind / fork, durable), the session controls and their error statuses."""

import pytest

pytest.importorskip("fastapi")
pytest.importorskip("httpx")

from fastapi.testclient import TestClient  # noqa: E402

from reelcache_b200.integrations.sglang import ReelCacheRuntimeConfig, SyntheticEngine, create_sglang_backend  # noqa: E402
from reelcache_b200.integrations.sglang.engine import model_identity_for  # noqa: E402
from reelcache_b200.integrations.sglang.profiles import ModelProfile  # noqa: E402
from reelcache_b200.serving import create_app  # noqa: E402

TINY = ModelProfile("tiny-http", backbone="tiny-wan", num_layers=2, num_heads=2, head_dim=32, chunk_frames=1,
                    grid=(4, 4), visibility="full_history", sink_frames=0, window_frames=None, energy_profile="causvid")


@pytest.fixture
def client(tmp_path):
    engine = SyntheticEngine(TINY, model_identity_for(TINY, "synthetic"), "cpu", rank=4)
    bridge = create_sglang_backend(ReelCacheRuntimeConfig(store_root=str(tmp_path / "store"), fit_device="cpu",
                                                          encode_workers=1), engine, cache_chunks=8)
    with TestClient(create_app(bridge)) as test_client:
        yield test_client
    bridge.shutdown()


def test_generation_and_session_routes(client):
    first = client.post("/v1/videos", json={"prompt": "a cat", "num_chunks": 3, "request_id": "r1",
                                             "causal_kv_session": {"session_id": "s1", "durable": True}})
    assert first.status_code == 200, first.text
    body = first.json()
    assert body["generated"] == 3 and body["latents"]["shape"] and body["durable"]["chunks"] == 3
    again = client.post("/v1/videos", json={"num_chunks": 1, "causal_kv_session": {"session_id": "s1",
                                                                                   "action": "resume"}})
    assert again.json()["route"] == "resident"
    rewound = client.post("/v1/videos", json={"num_chunks": 1, "causal_kv_session": {
        "session_id": "s1", "action": "rewind", "checkpoint": 2}})
    assert rewound.json()["start_chunk"] == 2
    forked = client.post("/v1/videos", json={"num_chunks": 1, "causal_kv_session": {
        "session_id": "s2", "action": "fork", "from_session": "s1", "checkpoint": 2}})
    assert forked.status_code == 200 and forked.json()["route"] == "archive"
    assert set(client.get("/v1/sessions").json()["sessions"]) == {"s1", "s2"}
    assert client.get("/v1/sessions/s2").json()["generated"] == 3
    assert client.post("/v1/sessions/s1/pause").status_code == 200
    named = client.post("/v1/sessions/s1/checkpoints", json={"name": "keep"})
    assert named.status_code == 200 and named.json()["name"] == "keep"
    assert any(row.get("name") == "keep" for row in client.get("/v1/sessions/s1/checkpoints").json()["checkpoints"])
    assert client.get("/v1/session_requests/r1").json()["generated"] == 3
    assert client.get("/v1/session_capabilities").json()["profile"] == "tiny-http"
    assert client.delete("/v1/sessions/s2").status_code == 200
    assert client.get("/v1/sessions/s2").status_code == 404
    assert client.post("/v1/session_gc").status_code == 200


def test_errors_map_to_statuses(client):
    missing = client.post("/v1/videos", json={"causal_kv_session": {"action": "resume"}})
    assert missing.status_code == 400
    bad = client.post("/v1/videos", json={"causal_kv_session": {"session_id": "x", "path": "/tmp"}})
    assert bad.status_code == 400
    client.post("/v1/videos", json={"causal_kv_session": {"session_id": "x"}})
    duplicate = client.post("/v1/videos", json={"causal_kv_session": {"session_id": "x"}})
    assert duplicate.status_code == 409
    replaced = client.post("/v1/videos", json={"num_chunks": 2, "causal_kv_session": {"session_id": "x",
                                                                                     "replace": True}})
    assert replaced.status_code == 200 and replaced.json()["generated"] == 2
    assert client.get("/v1/session_requests/none").status_code == 404
    assert client.post("/v1/sessions/x/explode").status_code == 404
