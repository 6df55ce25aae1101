"""KVRuntime: the CPU runtime demo flow (commit -> snapshot -> fork -> restart -> restore -> history),
streaming and asynchronous commits, validation, quarantine and garbage collection."""

import hashlib

import pytest
import torch

from reelcache_b200.errors import CapacityError, ConfigurationError, IntegrityError, PendingError, StateError
from reelcache_b200.execution import BoundedExecutor
from reelcache_b200.manager import KVRuntime
from reelcache_b200.types import CodecSpec, MatrixKey, ModelIdentity, TensorContext

MODEL = ModelIdentity("synthetic-demo", hashlib.sha256(b"seed7").hexdigest(), 2, 16, "canonical", "float32")
KEYS = [MatrixKey(layer, target) for layer in range(2) for target in ("K", "V")]


def matrices(seed, bases):
    generator = torch.Generator().manual_seed(seed)
    return {key: torch.randn(64, 4, generator=generator) @ bases[key] for key in KEYS}


def contexts(start, codec):
    return {key: TensorContext(MODEL, key, start, 2, 4, 8,
                               ("post_rope" if codec == "raw" else "pre_rope") if key.target == "K" else "none")
            for key in KEYS}


def metadata(chunk_id, end):
    return {"clean_boundary": {"chunk_id": chunk_id, "token_end": end, "clean": True},
            "conditioning": {"id": "synthetic"}, "execution": {"next_chunk": 1, "pending": False},
            "rng": {"tensor": "rng"}, "latent": {"native_latents": "n/a"}, "vae": {"native_decoder": "n/a"}}


@pytest.fixture
def bases():
    generator = torch.Generator().manual_seed(7)
    return {key: torch.randn(4, 16, generator=generator) for key in KEYS}


@pytest.mark.parametrize("codec", ["raw", "svd"])
def test_runtime_demo_flow(tmp_path, bases, codec):
    first, second = matrices(1, bases), matrices(2, bases)
    spec = CodecSpec() if codec == "raw" else CodecSpec(kind="svd", rank=4)
    runtime = KVRuntime(tmp_path / "state", MODEL, max_resident_bytes=1 << 20)
    runtime.create_branch("main")
    staged = sum(t.numel() * t.element_size() for t in first.values())
    with BoundedExecutor(max_staging_bytes=2 * staged) as executor:
        job = executor.submit(runtime.seal_chunk, "main", "chunk-0", first, contexts(0, codec), spec,
                              staging_bytes=staged)
        job.result()
    rng = torch.Generator().manual_seed(3).get_state()
    snapshot = runtime.snapshot("main", metadata=metadata("chunk-0", 64), tensors={"rng": rng})
    runtime.fork(snapshot, "child")
    with pytest.raises(StateError):
        runtime.fork(snapshot, "child")
    runtime.seal_chunk("child", "chunk-1", second, contexts(64, codec), spec,
                       reuse_threshold=0.01 if codec != "raw" else None)
    runtime.close()

    runtime = KVRuntime(tmp_path / "state", MODEL, max_resident_bytes=1 << 20)
    try:
        restored = runtime.restore(snapshot, "resumed")
        assert torch.equal(restored.tensors["rng"], rng)
        for key in KEYS:
            with runtime.acquire_history("resumed", key) as lease:
                error = float(torch.linalg.vector_norm(lease.tensor - first[key]) / torch.linalg.vector_norm(first[key]))
                if codec == "raw":
                    assert torch.equal(lease.tensor, first[key])
                else:
                    assert error < 0.03
                prefix = lease.tensor.clone()
            with runtime.acquire_history("main", key) as parent:
                assert torch.equal(parent.tensor, prefix)
            with runtime.acquire_history("child", key) as child:
                assert child.tensor.shape == (128, 16)
                assert torch.equal(child.tensor[:64], prefix)
                if codec == "raw":
                    assert torch.equal(child.tensor[64:], second[key])
        info = runtime.branch_info("child")
        assert info["chunk_ids"] == ["chunk-0", "chunk-1"] and info["token_end"] == 128
        assert runtime.resident_bytes == 0 and runtime.active_leases == 0
        if codec != "raw":
            # the child's second chunk reused the parent's basis: identical basis object
            ctx = runtime.history_specs("child", KEYS[0])
            assert len(ctx) == 2
    finally:
        runtime.close()


def test_validation_and_capacity(tmp_path, bases):
    runtime = KVRuntime(tmp_path / "s", MODEL, max_resident_bytes=64 * 16 * 4 - 1)
    runtime.create_branch("main")
    data = matrices(1, bases)
    with pytest.raises(ConfigurationError):
        runtime.seal_chunk("main", "c", data, contexts(64, "raw"))  # gap
    with pytest.raises(ConfigurationError):
        runtime.seal_chunk("main", "", data, contexts(0, "raw"))
    runtime.seal_chunk("main", "c", data, contexts(0, "raw"))
    with pytest.raises(ConfigurationError):
        runtime.seal_chunk("main", "c", data, contexts(64, "raw"))  # duplicate chunk id
    with pytest.raises(CapacityError):
        runtime.acquire_history("main", KEYS[0])
    lease = runtime.acquire_history("main", KEYS[0], columns=slice(0, 8))
    assert lease.tensor.shape == (64, 8)
    lease.release()
    with pytest.raises(StateError):
        _ = lease.tensor
    with pytest.raises(ConfigurationError):
        runtime.snapshot("main", metadata={**metadata("c", 64), "clean_boundary": {"chunk_id": "x", "token_end": 64}})
    with pytest.raises(PendingError):
        runtime.snapshot("main", metadata={**metadata("c", 64), "execution": {"pending": True}})
    runtime.close()


def test_streaming_and_async_commits(tmp_path, bases):
    runtime = KVRuntime(tmp_path / "s", MODEL, executor=BoundedExecutor(max_pending=4))
    runtime.create_branch("main")
    data = matrices(1, bases)
    stream = runtime.open_chunk("main", "c0", contexts(0, "raw"))
    with pytest.raises(PendingError):
        runtime.seal_chunk("main", "x", data, contexts(0, "raw"))
    for key in KEYS[:-1]:
        stream.add(key, data[key])
    with pytest.raises(StateError):
        stream.commit()
    stream.add(KEYS[-1], data[KEYS[-1]])
    chunk = stream.commit()
    assert stream.state == "committed" and chunk.startswith("manifest:")
    pending = runtime.submit_chunk("main", "c1", matrices(2, bases), contexts(64, "raw"))
    assert pending.result(timeout=30).startswith("manifest:")
    assert pending.status()["phase"] == "published"
    aborted = runtime.open_chunk("main", "c2", contexts(128, "raw"))
    aborted.add(KEYS[0], data[KEYS[0]])
    aborted.abort()
    assert runtime.branch_info("main")["chunk_ids"] == ["c0", "c1"]
    runtime.gc()
    with runtime.acquire_history("main", KEYS[1], token_start=32, token_end=96) as lease:
        assert torch.equal(lease.tensor[:32], data[KEYS[1]][32:])
    runtime.executor.close()
    runtime.close()


def test_quarantine_on_open(tmp_path, bases):
    runtime = KVRuntime(tmp_path / "s", MODEL)
    runtime.create_branch("good")
    runtime.create_branch("bad")
    runtime.seal_chunk("good", "c", matrices(1, bases), contexts(0, "raw"))
    runtime.seal_chunk("bad", "c", matrices(2, bases), contexts(0, "raw"))
    bad_head = runtime.branch_info("bad")["head_id"]
    chunk = runtime.branch_info("bad")["chunk_manifests"][0]
    tensor = runtime.store.get_manifest(chunk)["matrices"][0]["tensor"]
    payload = runtime.store.get_manifest(tensor)["encoded"]["payloads"]["tensor.bin"]
    runtime.close()
    path = runtime.store.path_for(payload)
    path.write_bytes(b"corrupt" + path.read_bytes()[7:])
    with pytest.raises(IntegrityError):
        KVRuntime(tmp_path / "s", MODEL, verify_reads=True)
    runtime = KVRuntime(tmp_path / "s", MODEL, verify_reads=True, on_open_error="quarantine")
    assert "branches/bad" in runtime.quarantined
    assert bad_head
    with runtime.acquire_history("good", KEYS[0]) as lease:
        assert lease.tensor.shape == (64, 16)
    with pytest.raises(IntegrityError):
        runtime.acquire_history("bad", KEYS[0])
    runtime.delete_branch("bad")
    assert "branches/bad" not in runtime.quarantined
    runtime.close()
