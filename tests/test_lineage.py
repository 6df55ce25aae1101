"""Lineage commits through the rank method: share/augment decisions, history, fork and rewind."""

import pytest
import torch

from reelcache_b200.errors import StateError
from reelcache_b200.lineage import LineageRuntime
from reelcache_b200.predictor_registry import RankPredictorRegistry
from reelcache_b200.store import ObjectStore
from reelcache_b200.types import MatrixKey

from .lineage_support import MODEL, TOKENS, chunk, method, relative_error


@pytest.fixture
def runtime(tmp_path):
    store = ObjectStore(tmp_path / "store")
    yield LineageRuntime(store, MODEL, registry=RankPredictorRegistry("test"))
    store.close()


def test_commit_history_and_decisions(runtime):
    runtime.create_lineage("main")
    cfg = method()
    decisions = []
    sources = []
    for index in range(4):
        matrices, contexts = chunk(index)
        sources.append(matrices)
        commit = runtime.commit_node("main", f"c{index}", matrices, contexts, method=cfg)
        decisions.append(commit.plan["decisions"])
    assert "fresh" in decisions[0]
    assert any("share" in d or "augment" in d for d in decisions[1:])
    head = runtime.lineage_head("main")
    key = MatrixKey(1, "K")
    history = runtime.acquire_node_history(head, key)
    assert history.shape == (4 * TOKENS, 128)
    for index in range(4):
        part = history[index * TOKENS:(index + 1) * TOKENS]
        # energy target K 98 % -> relative error about sqrt(0.02) plus 8-bit quantization
        assert relative_error(part, sources[index][key]) < 0.2
    pieces = runtime.resolve_history(head, [(TOKENS, 3 * TOKENS)])
    assert [p.entry.chunk_id for p in pieces] == ["c1", "c2"]
    assert runtime.registry.sequence >= 0


def test_fork_and_rewind(runtime):
    root = runtime.create_lineage("main")
    cfg = method()
    refs = []
    for index in range(3):
        matrices, contexts = chunk(index)
        refs.append(runtime.commit_node("main", f"c{index}", matrices, contexts, method=cfg).node_ref)
    runtime.fork_lineage(refs[0], "branch")
    matrices, contexts = chunk(1, seed=5)
    runtime.commit_node("branch", "b1", matrices, contexts, method=cfg)
    assert runtime.lineage_head("main") == refs[2]
    runtime.rewind_lineage("main", refs[1])
    assert runtime.lineage_head("main") == refs[1]
    with pytest.raises(StateError):
        runtime.rewind_lineage("main", runtime.lineage_head("branch"))
    assert set(runtime.list_lineages()) == {"main", "branch"}
    assert root != refs[0]


def test_raw_lineage_is_exact(runtime):
    runtime.create_lineage("raw")
    matrices, contexts = chunk(0)
    commit = runtime.commit_raw_node("raw", "c0", matrices, contexts, execution_state={"rng": torch.arange(3)})
    key = MatrixKey(0, "V")
    back = runtime.acquire_node_history(commit.node_ref, key)
    assert torch.equal(back, matrices[key])
    assert torch.equal(runtime.execution_state(commit.node_ref)["rng"], torch.arange(3))


def test_identical_content_identical_ids(tmp_path):
    refs = []
    for name in ("a", "b"):
        store = ObjectStore(tmp_path / name)
        rt = LineageRuntime(store, MODEL)
        rt.create_lineage("main")
        matrices, contexts = chunk(0)
        refs.append(rt.commit_node("main", "c0", matrices, contexts, method=method()).node_ref)
        store.close()
    assert refs[0] == refs[1]
