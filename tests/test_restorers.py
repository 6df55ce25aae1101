"""The RAW, software (host-decoded node packs) and factor-pack (SVD-only) lineage restorers on CPU: each restores
a node's attended history into native BTHD caches with RoPE on pre-RoPE keys, and matches the dense history of
``acquire_node_history`` (bitwise for RAW, within the representation's error otherwise)."""

import pytest
import torch

from reelcache_b200 import restore_kernels as rk
from reelcache_b200.archive_restore import RawLineageRestorer, SoftwareLineageRestorer
from reelcache_b200.errors import UnsupportedError
from reelcache_b200.factor_packs import FactorLineageRestorer, FactorRestorer
from reelcache_b200.lineage import LineageRuntime
from reelcache_b200.store import ObjectStore
from reelcache_b200.types import CodecSpec, MatrixKey

from .lineage_support import FRAMES, MODEL, TOKENS, chunk, method, relative_error

HEADS = 2


def _commit(tmp_path, kind, chunks=3):
    store = ObjectStore(tmp_path / kind)
    runtime = LineageRuntime(store, MODEL)
    runtime.create_lineage("main")
    node = None
    sources = []
    for index in range(chunks):
        m, c = chunk(index)
        sources.append(m)
        if kind == "raw":
            node = runtime.commit_raw_node("main", f"c{index}", m, c).node_ref
        else:
            node = runtime.commit_node("main", f"c{index}", m, c,
                                       method=method(codec=CodecSpec(kind, 32))).node_ref
    return runtime, node, sources


def _restore(restorer, runtime, node, chunks):
    head_dim = MODEL.channels_for("K") // HEADS
    caches = {(l, t): torch.zeros((1, chunks * TOKENS, HEADS, head_dim)) for l in range(MODEL.layers) for t in "KV"}
    table = rk.RopeTable.wan(head_dim, 64)
    rope_rows = lambda piece: (table, (FRAMES * (piece.token_start // TOKENS), 0, 0))  # noqa: E731
    result = restorer.restore(node, lambda l, t: caches[(l, t)], rope_rows, overlapped=False)
    for layer in range(MODEL.layers):
        result.wait(layer)
    result.join()
    return caches, table


def _expected_k(runtime, node, layer, table, chunks):
    head_dim = MODEL.channels_for("K") // HEADS
    dense = runtime.acquire_node_history(node, MatrixKey(layer, "K")).reshape(chunks * TOKENS, HEADS, head_dim)
    parts = []
    for index in range(chunks):
        positions = rk.RopePositions(table, (FRAMES * index, 0, 0))
        grid = (FRAMES, 8, 16)
        parts.append(rk.apply_rope_reference(dense[index * TOKENS:(index + 1) * TOKENS], positions, grid))
    return torch.cat(parts).float()


@pytest.mark.parametrize("kind", ["raw", "svd", "svd_hevc"])
def test_restorer_matches_history(tmp_path, kind):
    runtime, node, sources = _commit(tmp_path, kind)
    restorer = {"raw": RawLineageRestorer, "svd": FactorLineageRestorer, "svd_hevc": SoftwareLineageRestorer}[kind](
        runtime, "cpu")
    caches, table = _restore(restorer, runtime, node, 3)
    tolerance = 1e-6 if kind == "raw" else 5e-3
    for layer in range(MODEL.layers):
        v = caches[(layer, "V")].reshape(3 * TOKENS, -1)
        dense_v = runtime.acquire_node_history(node, MatrixKey(layer, "V"))
        assert relative_error(v, dense_v) < tolerance
        k = caches[(layer, "K")]
        assert relative_error(k, _expected_k(runtime, node, layer, table, 3)) < tolerance
        # and the representation tracks the source
        expect = torch.cat([s[MatrixKey(layer, "V")] for s in sources])
        assert relative_error(v, expect) < (1e-6 if kind == "raw" else 0.1)
    assert restorer.stats()["restores"] == 1


def test_factor_pack_storage_and_dense_history(tmp_path):
    runtime, node, sources = _commit(tmp_path, "svd", chunks=2)
    record_ref = runtime.resolve_history(node)[0].record(MatrixKey(0, "V"))
    record = runtime.load_record(record_ref)
    assert record.codec.kind == "svd" and record.decision["packet"]["stream_codec"] == "fp16"
    _, pack = runtime.factor_pack(record.packet_ref)
    assert pack.factors(record.decision["packet"]["tile"]).dtype.name == "float16"
    factors = FactorRestorer(runtime)
    dense = factors.history(node, MatrixKey(1, "K"))
    assert relative_error(dense, runtime.acquire_node_history(node, MatrixKey(1, "K"))) < 1e-6
    assert runtime.node_storage(node)["stream_bytes"] > 0
    # representation-specific restorers refuse other kinds
    with pytest.raises(UnsupportedError):
        _restore(RawLineageRestorer(runtime, "cpu"), runtime, node, 2)


def test_rank_report_of_a_lineage(tmp_path):
    """The rank-study report walks the head's path: one entry per node with per-layer K/V ranks, energy against
    the targets, bytes and a compression ratio above 1; comparing a report with itself shows equal columns."""
    from reelcache_b200.rank_report import compare, lineage_report, main
    runtime, node, _ = _commit(tmp_path, "svd_hevc")
    report = lineage_report(runtime, node)
    assert report["summary"]["nodes"] == 3 and report["summary"]["compression_ratio"] > 1
    first = report["nodes"][0]
    assert len(first["ranks"]["K"]) == MODEL.layers and first["energy"]["K"]["targets_met"] == MODEL.layers
    same = compare(report, report)
    assert all(row["bytes_a"] == row["bytes_b"] for row in same["nodes"])
    runtime.store.close()
    main(["--store", str(tmp_path / "svd_hevc"), "--node", node])
