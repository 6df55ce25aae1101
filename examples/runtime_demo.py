"""Durable clean chunks, restart and branching on synthetic KV, on the CPU.

Two scenarios (reference flow: examples/runtime_demo.py; the full run is the CPU runtime demo of the
benchmark table):

* ``--scenario lineage`` (default): 4 layers x 2 heads x head_dim 128 (256 channels), 1560 tokens per chunk
  (1 x 30 x 52 latent grid), FP32, 8 chunks. Every K / V of a chunk is ``U diag(sigma) W^T`` with random
  orthonormal ``U`` (per chunk, columns scaled by sqrt(1560)) and ``W`` (per matrix), ``sigma_i = 1 / i`` for ``i = 1..64``, plus
  N(0, 1e-3) noise, from fixed seeds. The chunks are committed through the rank method at the CausVid
  energy targets (pre-RoPE K 98 %, V 95 %) as 8-bit coefficient node packs (``svd_hevc`` records; the
  coefficient stream is HEVC when an FFmpeg with libx265 exists, else the same 8-bit planes uncompressed).
  Then the store is closed and reopened, the head's whole history is restored and compared with the
  sources, ``main`` is rewound to chunk 4 and continued, and chunk 6 is forked and extended; the fork and
  the rewound branch keep their parents' history bit for bit.
* ``--scenario kv_runtime``: the :class:`KVRuntime` flow on small matrices: commit a chunk on ``main``,
  snapshot it, fork ``child`` and extend it, close, reopen, restore the snapshot into ``resumed``.

    python examples/runtime_demo.py --output /tmp/demo
    python examples/runtime_demo.py --output /tmp/demo2 --scenario kv_runtime --codec svd
"""

from __future__ import annotations

import argparse
import hashlib
import json
import sys
import time
from pathlib import Path


def main(argv=None):
    ap = argparse.ArgumentParser(description=__doc__)
    ap.add_argument("--output", type=Path, required=True, help="new, empty output directory")
    ap.add_argument("--scenario", choices=("lineage", "kv_runtime"), default="lineage")
    ap.add_argument("--codec", choices=("raw", "svd", "svd_hevc"), default="raw",
                    help="representation of the kv_runtime scenario")
    ap.add_argument("--chunks", type=int, default=8, help="chunks of the lineage scenario (at least 6)")
    args = ap.parse_args(argv)
    if args.output.exists() and any(args.output.iterdir()):
        ap.error("--output must be new or empty")
    args.output.mkdir(parents=True, exist_ok=True)
    sys.path.insert(0, str(Path(__file__).resolve().parents[1]))
    if args.scenario == "lineage":
        if args.chunks < 6:
            ap.error("--chunks must be at least 6 (rewind to chunk 4, fork at chunk 6)")
        return lineage_scenario(args.output, args.chunks)
    import torch
    from reelcache_b200.execution import BoundedExecutor
    from reelcache_b200.manager import KVRuntime
    from reelcache_b200.types import CodecSpec, MatrixKey, ModelIdentity, TensorContext

    generator = torch.Generator().manual_seed(7)
    model = ModelIdentity("synthetic-demo", hashlib.sha256(b"reelcache-synthetic-v1-seed7-rank4").hexdigest(),
                          2, 16, "canonical", "float32")
    keys = [MatrixKey(layer, target) for layer in range(2) for target in ("K", "V")]
    bases = {key: torch.randn(4, 16, generator=generator) for key in keys}
    first = {key: torch.randn(64, 4, generator=generator) @ bases[key] for key in keys}
    second = {key: torch.randn(64, 4, generator=generator) @ bases[key] for key in keys}
    spec = CodecSpec() if args.codec == "raw" else CodecSpec(kind=args.codec, rank=4)

    def contexts(start):
        space = "post_rope" if args.codec == "raw" else "pre_rope"
        return {key: TensorContext(model, key, start, 2, 4, 8, space if key.target == "K" else "none") for key in keys}

    started = time.monotonic()
    runtime = KVRuntime(args.output / "state", model, max_resident_bytes=1 << 20)
    try:
        runtime.create_branch("main")
        staged = sum(t.numel() * t.element_size() for t in first.values())
        with BoundedExecutor(max_staging_bytes=2 * staged) as executor:
            job = executor.submit(runtime.seal_chunk, "main", "chunk-0", first, contexts(0), spec, staging_bytes=staged)
            job.result()
            timing = job.metrics()
        snapshot = runtime.snapshot("main", metadata={
            "clean_boundary": {"chunk_id": "chunk-0", "token_end": 64, "clean": True},
            "conditioning": {"id": "synthetic"}, "execution": {"next_chunk": 1, "pending": False},
            "rng": {"tensor": "rng"}, "latent": {"native_latents": "not applicable"},
            "vae": {"native_decoder": "not applicable"}}, tensors={"rng": generator.get_state()})
        runtime.fork(snapshot, "child")
        runtime.seal_chunk("child", "chunk-1", second, contexts(64), spec,
                           reuse_threshold=0.01 if args.codec != "raw" else None)
    finally:
        runtime.close()
    runtime = KVRuntime(args.output / "state", model, max_resident_bytes=1 << 20)
    errors = {}
    try:
        runtime.restore(snapshot, "resumed")
        for key in keys:
            with runtime.acquire_history("resumed", key) as lease:
                errors[f"{key.layer}:{key.target}"] = float(
                    torch.linalg.vector_norm(lease.tensor - first[key]) / torch.linalg.vector_norm(first[key]))
                prefix = lease.tensor.clone()
            with runtime.acquire_history("child", key) as child:
                assert child.tensor.shape == (128, 16) and torch.equal(child.tensor[:64], prefix)
    finally:
        runtime.close()
    report = {"schema": "reelcache_synthetic_demo_v1", "status": "passed", "codec": args.codec,
              "snapshot_id": snapshot, "restart_relative_KV_errors": errors, "parent_isolation": True,
              "state_store_bytes": sum(p.stat().st_size for p in (args.output / "state").rglob("*") if p.is_file()),
              "job_timing": timing, "wall_seconds": time.monotonic() - started}
    (args.output / "result.json").write_text(json.dumps(report, indent=2))
    print(json.dumps(report, indent=2))


LAYERS, HEADS, HEAD_DIM, RANK = 4, 2, 128, 64
FRAMES, HEIGHT, WIDTH = 1, 30, 52            # 1560 tokens per chunk


def synthetic_chunk(index, keys, bases, model):
    """One chunk's K and V: ``U diag(sigma) W^T + N(0, 1e-3)`` with a fresh orthonormal ``U`` per chunk, its
    columns scaled by ``sqrt(tokens)`` so that a token row carries O(1) signal next to the 1e-3 noise."""
    import torch
    from reelcache_b200.types import TensorContext

    tokens = FRAMES * HEIGHT * WIDTH
    sigma = 1.0 / torch.arange(1, RANK + 1, dtype=torch.float64)
    matrices, contexts = {}, {}
    for key in keys:
        gen = torch.Generator().manual_seed(10_000 + 100 * index + 2 * key.layer + (key.target == "V"))
        u = torch.linalg.qr(torch.randn(tokens, RANK, dtype=torch.float64, generator=gen))[0] * tokens ** 0.5
        x = (u * sigma) @ bases[key].t() + 1e-3 * torch.randn(tokens, HEADS * HEAD_DIM, dtype=torch.float64,
                                                               generator=gen)
        matrices[key] = x.float()
        contexts[key] = TensorContext(model, key, index * tokens, FRAMES, HEIGHT, WIDTH,
                                      "pre_rope" if key.target == "K" else "none")
    return matrices, contexts


def lineage_scenario(output: Path, chunks: int):
    import torch
    from reelcache_b200.lineage import LineageRuntime
    from reelcache_b200.predictor_registry import RankPredictorRegistry
    from reelcache_b200.rank_method import RankMethodConfig
    from reelcache_b200.store import ObjectStore
    from reelcache_b200.types import CodecSpec, MatrixKey, ModelIdentity, energy_targets

    started = time.monotonic()
    model = ModelIdentity("synthetic-demo", hashlib.sha256(b"reelcache-synthetic-4x2x128-seed7").hexdigest(),
                          LAYERS, HEADS * HEAD_DIM, "BTHD", "float32")
    keys = [MatrixKey(layer, target) for layer in range(LAYERS) for target in ("K", "V")]
    gen = torch.Generator().manual_seed(7)
    bases = {key: torch.linalg.qr(torch.randn(HEADS * HEAD_DIM, RANK, dtype=torch.float64, generator=gen))[0]
             for key in keys}
    method = RankMethodConfig(targets=energy_targets("causvid"), codec=CodecSpec("svd_hevc", RANK),
                              solver="gram_eigh")
    tokens = FRAMES * HEIGHT * WIDTH
    sources = [synthetic_chunk(index, keys, bases, model) for index in range(chunks)]
    state = output / "state"

    # ---- commit every chunk on main ----
    store = ObjectStore(state)
    runtime = LineageRuntime(store, model, registry=RankPredictorRegistry("demo"))
    runtime.create_lineage("main")
    refs, decisions, commit_seconds = [], [], []
    for index, (matrices, contexts) in enumerate(sources):
        t0 = time.monotonic()
        commit = runtime.commit_node("main", f"chunk-{index + 1}", matrices, contexts, method=method)
        commit_seconds.append(time.monotonic() - t0)
        refs.append(commit.node_ref)
        decisions.append(commit.plan["decisions"])
    head = runtime.lineage_head("main")
    store.close()

    # ---- restart: reopen the store, restore the head's whole history ----
    store = ObjectStore(state)
    runtime = LineageRuntime(store, model, registry=RankPredictorRegistry("demo"))
    errors, ranks = {}, {}
    t0 = time.monotonic()
    restored = {}
    packs = {}
    for key in keys:
        history = runtime.acquire_node_history(runtime.lineage_head("main"), key, packs=packs)
        if history.shape != (chunks * tokens, HEADS * HEAD_DIM):
            raise SystemExit(f"restored history of {key} has shape {tuple(history.shape)}")
        restored[key] = history
        errors[f"{key.layer}:{key.target}"] = max(
            float(torch.linalg.vector_norm(history[i * tokens:(i + 1) * tokens] - sources[i][0][key])
                  / torch.linalg.vector_norm(sources[i][0][key])) for i in range(chunks))
    restore_seconds = time.monotonic() - t0
    for key in keys:
        ranks[f"{key.layer}:{key.target}"] = [
            runtime.load_record(piece.record(key, None)).rank_view for piece in runtime.resolve_history(head)]

    # ---- rewind main to chunk 4 and continue it with a new chunk 5 ----
    runtime.rewind_lineage("main", refs[3])
    replacement, contexts = synthetic_chunk(chunks + 1, keys, bases, model)
    contexts = {key: type(ctx)(model, key, 4 * tokens, FRAMES, HEIGHT, WIDTH, ctx.key_space)
                for key, ctx in contexts.items()}
    runtime.commit_node("main", "chunk-5-rewound", replacement, contexts, method=method)
    # ---- fork at chunk 6 and extend the fork with a new chunk 7 ----
    runtime.fork_lineage(refs[5], "fork")
    extension, contexts = synthetic_chunk(chunks + 2, keys, bases, model)
    contexts = {key: type(ctx)(model, key, 6 * tokens, FRAMES, HEIGHT, WIDTH, ctx.key_space)
                for key, ctx in contexts.items()}
    runtime.commit_node("fork", "chunk-7-fork", extension, contexts, method=method)
    isolation = True
    for key in keys:
        rewound = runtime.acquire_node_history(runtime.lineage_head("main"), key, packs=packs)
        forked = runtime.acquire_node_history(runtime.lineage_head("fork"), key, packs=packs)
        original = runtime.acquire_node_history(head, key, packs=packs)
        isolation &= bool(torch.equal(rewound[:4 * tokens], restored[key][:4 * tokens]))
        isolation &= bool(torch.equal(forked[:6 * tokens], restored[key][:6 * tokens]))
        isolation &= bool(torch.equal(original, restored[key]))
        isolation &= rewound.shape[0] == 5 * tokens and forked.shape[0] == 7 * tokens
    store_bytes = sum(p.stat().st_size for p in state.rglob("*") if p.is_file())
    store.close()
    source_bytes = chunks * len(keys) * tokens * HEADS * HEAD_DIM * 4
    report = {"schema": "reelcache_synthetic_demo_v1", "scenario": "lineage",
              "status": "passed" if isolation else "failed",
              "geometry": {"layers": LAYERS, "heads": HEADS, "head_dim": HEAD_DIM, "tokens_per_chunk": tokens,
                           "chunks": chunks, "dtype": "float32", "synthetic_rank": RANK},
              "energy_targets": {"K": method.targets.key, "V": method.targets.value},
              "decisions": decisions, "ranks": ranks,
              "restart_relative_KV_errors": errors, "parent_isolation": isolation,
              "state_store_bytes": store_bytes, "source_bytes": source_bytes,
              "compression": round(source_bytes / max(1, store_bytes), 2),
              "commit_seconds": [round(x, 3) for x in commit_seconds],
              "restore_seconds": round(restore_seconds, 3), "wall_seconds": time.monotonic() - started}
    (output / "result.json").write_text(json.dumps(report, indent=2))
    print(json.dumps({k: v for k, v in report.items() if k not in ("decisions", "ranks")}, indent=2))
    return report


if __name__ == "__main__":
    main()
