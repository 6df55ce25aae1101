"""Durable clean chunks, restart and branching on small synthetic KV with the KVRuntime (BASELINE
config 1 flow): commit a chunk on ``main``, snapshot it, fork ``child`` and extend it, close, reopen the
store, restore the snapshot into ``resumed`` and compare every history against its source.

    python examples/runtime_demo.py --output /tmp/demo --codec svd
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
    ap.add_argument("--codec", choices=("raw", "svd", "svd_hevc"), default="raw")
    args = ap.parse_args(argv)
    if args.output.exists() and any(args.output.iterdir()):
        ap.error("--output must be new or empty")
    args.output.mkdir(parents=True, exist_ok=True)
    sys.path.insert(0, str(Path(__file__).resolve().parents[1]))
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


if __name__ == "__main__":
    main()
