"""LingBot integration on the CPU: the overlapped restore's per-layer waits (a layer is never read before the
restore marked it; the hooks go after the last layer; failures arrive typed), the archive's one node per chunk
with a fork on rewind, and restores into the stand-in world model's shared window cache that resume generation
exactly where an uninterrupted run continues (RAW bitwise, overlapped == synchronous bitwise, the compressed
representation within its energy target)."""

import threading
import time

import pytest
import torch

from reelcache_b200.integrations.lingbot import (ArchiveError, LINGBOT_WORLD_FAST, LingBotArchive, OverlapSession,
                                                 StallEvents, StandInWorldModel)
from reelcache_b200.overlapped_restore import LayerReadiness, RestoreFailure, start_overlapped_restore

# The stand-in's K / V have no low-rank structure, so the representation keeps exactly its energy targets
# (K 98 %, V 95 %): relative error sqrt(1 - target), plus 8-bit coefficient quantization.
K_BOUND = (1 - 0.98) ** 0.5 + 0.03
V_BOUND = (1 - 0.95) ** 0.5 + 0.03
GEOMETRY = LINGBOT_WORLD_FAST.scaled(layers=3, heads=2, head_dim=16, frames_per_chunk=1, latent_height=4,
                                     latent_width=4, window_latents=3, sink_latents=1)


def _inputs(count, seed=0):
    g = torch.Generator().manual_seed(seed)
    return [torch.randn(GEOMETRY.chunk_tokens, GEOMETRY.channels, generator=g) for _ in range(count)]


def _run(model, archive, session, xs, *, first=0, parent=None, prefix=""):
    outputs = []
    for offset, x in enumerate(xs):
        chunk = first + offset
        out, (k, v) = model.generate(chunk, x)
        key = f"{prefix}{session}/{chunk}"
        archive.commit(session, key, parent, chunk, k, v)
        parent = key
        outputs.append(out)
    return outputs, parent


def test_geometry_of_the_real_model():
    g = LINGBOT_WORLD_FAST
    assert (g.layers, g.heads, g.head_dim, g.channels) == (40, 40, 128, 5120)
    assert g.chunk_tokens == 3 * 30 * 52 and g.window_chunks == 7
    assert g.chunk_bytes() == 2 * 40 * 4680 * 5120 * 2
    with pytest.raises(ValueError):
        g.scaled(window_latents=20)


def test_overlap_session_waits_each_layer_then_detaches():
    layers = 4
    model = StandInWorldModel(GEOMETRY.scaled(layers=layers), dtype=torch.float32)
    order = []
    gate = threading.Event()

    def issue(layer):
        if layer == 2:
            gate.wait(5)
        order.append(("issued", layer))

    handle = start_overlapped_restore(issue, layers, thread=True, readiness=LayerReadiness(layers))

    class Result:
        readiness = handle.readiness

        def wait(self, layer, stream=None):
            handle.readiness.wait(layer, stream)
            order.append(("read", layer))

        def join(self):
            return handle.join() or {}

    session = OverlapSession(Result(), layers=layers, recorder=StallEvents("cpu"))
    model.attach_overlapped_restore(session)
    assert session.attached
    threading.Timer(0.05, gate.set).start()
    model.generate(0, _inputs(1)[0])
    for layer in range(layers):
        assert order.index(("issued", layer)) < order.index(("read", layer))
    assert not session.attached and session.state == "joined"
    assert session.record["layers_waited"] == layers
    assert session.gpu_summary()["layers_waited"] == layers
    model.generate(1, _inputs(2)[1])  # later forwards do not wait


def test_overlap_failure_reaches_the_forward_typed():
    layers = 3
    model = StandInWorldModel(GEOMETRY.scaled(layers=layers), dtype=torch.float32)

    def issue(layer):
        if layer == 1:
            raise RuntimeError("decoder lost")

    handle = start_overlapped_restore(issue, layers, thread=True, readiness=LayerReadiness(layers, timeout=5))

    class Result:
        readiness = handle.readiness

        def wait(self, layer, stream=None):
            handle.readiness.wait(layer, stream)

        def join(self):
            return handle.join()

    session = OverlapSession(Result(), layers=layers)
    model.attach_overlapped_restore(session)
    with pytest.raises(RestoreFailure):
        model.generate(0, _inputs(1)[0])
    assert not session.attached and session.state == "aborted"


def test_raw_resume_matches_the_uninterrupted_run(tmp_path):
    xs = _inputs(6)
    live = StandInWorldModel(GEOMETRY, dtype=torch.float32)
    archive = LingBotArchive(tmp_path / "store", GEOMETRY)
    archive.ensure_session("s")
    outputs, head = _run(live, archive, "s", xs[:5])
    assert archive.drain()["published"] == 5
    expected_next, _ = live.generate(5, xs[5])

    restarted = StandInWorldModel(GEOMETRY, dtype=torch.float32)
    record = archive.restore(head, restarted)
    assert record["chunks"] == [0, 3, 4]  # sink chunk 0, then the window before chunk 5
    for c in record["chunks"]:
        start, end = restarted.cache.place(c)
        for layer in range(GEOMETRY.layers):
            torch.testing.assert_close(restarted.cache.v[layer][0, start:end], live.cache.v[layer][0, start:end],
                                       rtol=0, atol=0)
            torch.testing.assert_close(restarted.cache.k[layer][0, start:end], live.cache.k[layer][0, start:end],
                                       rtol=1e-6, atol=1e-6)
    resumed, _ = restarted.generate(5, xs[5], capture=False)
    torch.testing.assert_close(resumed, expected_next, rtol=1e-5, atol=1e-5)
    archive.close()


def test_overlapped_restore_equals_synchronous(tmp_path):
    xs = _inputs(5, seed=3)
    archive = LingBotArchive(tmp_path / "store", GEOMETRY)
    archive.ensure_session("s")
    _, head = _run(StandInWorldModel(GEOMETRY, dtype=torch.float32), archive, "s", xs[:4])
    sync_model = StandInWorldModel(GEOMETRY, dtype=torch.float32)
    archive.restore(head, sync_model)
    sync_out, _ = sync_model.generate(4, xs[4], capture=False)
    over_model = StandInWorldModel(GEOMETRY, dtype=torch.float32)
    session = archive.restore(head, over_model, overlapped=True, thread=True)
    assert isinstance(session, OverlapSession) and session.attached
    over_out, _ = over_model.generate(4, xs[4], capture=False)
    assert session.state == "joined" and session.record["layers_waited"] == GEOMETRY.layers
    assert torch.equal(over_out, sync_out)
    for layer in range(GEOMETRY.layers):
        assert torch.equal(over_model.cache.k[layer], sync_model.cache.k[layer])
        assert torch.equal(over_model.cache.v[layer], sync_model.cache.v[layer])
    assert archive.stats()["overlapped_restores"] == 1
    archive.close()


def test_rewind_forks_a_branch_and_restores_the_new_history(tmp_path):
    xs = _inputs(7, seed=5)
    archive = LingBotArchive(tmp_path / "store", GEOMETRY)
    archive.ensure_session("s")
    live = StandInWorldModel(GEOMETRY, dtype=torch.float32)
    _run(live, archive, "s", xs[:5])  # chunks 0..4
    # rewind to chunk 2 and generate a different chunk 3 on the restored history
    rewound = StandInWorldModel(GEOMETRY, dtype=torch.float32)
    archive.restore("s/2", rewound)
    outputs, head = _run(rewound, archive, "s", [xs[6]], first=3, parent="s/2", prefix="alt-")
    report = archive.report(head)
    assert report["branch"] == "s~1" and report["forked_at"] == "s/2"
    assert archive.report("s/4")["branch"] == "s"
    fresh = StandInWorldModel(GEOMETRY, dtype=torch.float32)
    archive.restore(head, fresh)
    start, end = fresh.cache.place(3)
    for layer in range(GEOMETRY.layers):
        assert torch.equal(fresh.cache.v[layer][0, start:end], rewound.cache.v[layer][0, start:end])
    assert archive.stats()["forks"] == 1
    with pytest.raises(ArchiveError):  # a chunk must carry every layer
        archive.commit("s", "bad", "s/1", 2, [], [])
    assert archive.forget_session("s") == {"branches": 2, "chunks": 6}
    archive.close()


def test_commit_checks_parents_and_indices(tmp_path):
    archive = LingBotArchive(tmp_path / "store", GEOMETRY)
    k = [torch.zeros(GEOMETRY.chunk_tokens, GEOMETRY.channels)] * GEOMETRY.layers
    with pytest.raises(ArchiveError):
        archive.commit("nobody", "a", None, 0, k, k)
    archive.ensure_session("s")
    archive.commit("s", "a", None, 0, k, k)
    with pytest.raises(ArchiveError):
        archive.commit("s", "a", "a", 1, k, k)       # key reused
    with pytest.raises(ArchiveError):
        archive.commit("s", "b", "a", 2, k, k)       # index gap
    with pytest.raises(ArchiveError):
        archive.commit("s", "c", "missing", 1, k, k)
    with pytest.raises(ArchiveError):
        LingBotArchive(tmp_path / "other", GEOMETRY, representation="zip")
    archive.close()


def test_compressed_representation_within_its_energy_target(tmp_path):
    xs = _inputs(4, seed=9)
    live = StandInWorldModel(GEOMETRY, dtype=torch.float32)
    archive = LingBotArchive(tmp_path / "store", GEOMETRY, representation="svd_hevc")
    archive.ensure_session("s")
    _, head = _run(live, archive, "s", xs[:3])
    restored = StandInWorldModel(GEOMETRY, dtype=torch.float32)
    record = archive.restore(head, restored)
    for c in record["chunks"]:
        start, end = restored.cache.place(c)
        for layer in range(GEOMETRY.layers):
            for ours, theirs, bound in ((restored.cache.k[layer], live.cache.k[layer], K_BOUND),
                                        (restored.cache.v[layer], live.cache.v[layer], V_BOUND)):
                a, b = ours[0, start:end], theirs[0, start:end]
                assert float((a - b).norm() / b.norm()) < bound
    assert archive.stats()["restorer"] == "SoftwareLineageRestorer"
    archive.close()
