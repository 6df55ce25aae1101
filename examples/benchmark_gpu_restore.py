"""Restore paths on one GPU (the counterpart of reference examples/benchmark_gpu_restore.py): the same CausVid-shaped
history (30 layers x K/V of [4680, 1536] per chunk, synthetic low-rank data) archived as ``svd_hevc`` node packs,
``svd`` FP16 factor packs and RAW, restored into native bf16 BTHD caches with RoPE by

* ``fused``    -- LineageRestorer (prepared packs, per-layer H2D on a copy stream, fused tcgen05 restore),
* ``software`` -- SoftwareLineageRestorer (host decode of every pack per restore, then the fused kernel),
* ``factor``   -- FactorLineageRestorer (FP16 factors, hi/lo-split fused restore),
* ``raw``      -- RawLineageRestorer (dense rows, the RoPE-and-store kernel).

    python examples/benchmark_gpu_restore.py --chunks 4 [--out result.json]

Times are CUDA-event means per full restore (all layers), after warm-up; GB/s counts the bf16 bytes written.
"""

from __future__ import annotations

import argparse
import json
import sys
import tempfile
from pathlib import Path


def main(argv=None):
    ap = argparse.ArgumentParser(description=__doc__)
    ap.add_argument("--chunks", type=int, default=4)
    ap.add_argument("--layers", type=int, default=30)
    ap.add_argument("--reps", type=int, default=5)
    ap.add_argument("--out", type=Path)
    args = ap.parse_args(argv)
    sys.path.insert(0, str(Path(__file__).resolve().parents[1]))
    import torch
    from reelcache_b200 import restore_kernels as rk
    from reelcache_b200.archive_restore import LineageRestorer, RawLineageRestorer, SoftwareLineageRestorer
    from reelcache_b200.factor_packs import FactorLineageRestorer
    from reelcache_b200.lineage import LineageRuntime
    from reelcache_b200.rank_method import RankMethodConfig
    from reelcache_b200.store import ObjectStore
    from reelcache_b200.types import CodecSpec, MatrixKey, ModelIdentity, TensorContext, energy_targets

    device = torch.device("cuda", 0)
    frames, height, width, heads, head_dim = 3, 30, 52, 12, 128
    tokens, channels = frames * height * width, heads * head_dim
    model = ModelIdentity("causvid-shaped", "bench", args.layers, channels, "BTHD", "bfloat16")
    g = torch.Generator(device=device).manual_seed(0)
    chunks = []
    for index in range(args.chunks):
        matrices, contexts = {}, {}
        for layer in range(args.layers):
            for target in ("K", "V"):
                key = MatrixKey(layer, target)
                base = torch.randn(tokens, 48, device=device, generator=g) @ torch.randn(48, channels, device=device,
                                                                                         generator=g)
                matrices[key] = (base + 0.05 * torch.randn(tokens, channels, device=device, generator=g)).bfloat16()
                contexts[key] = TensorContext(model, key, index * tokens, frames, height, width,
                                              "pre_rope" if target == "K" else "none")
        chunks.append((matrices, contexts))
    table = rk.RopeTable.wan(head_dim, 1024, device=device)
    caches = {(l, t): torch.zeros((1, args.chunks * tokens, heads, head_dim), dtype=torch.bfloat16, device=device)
              for l in range(args.layers) for t in "KV"}
    written = 2 * args.layers * args.chunks * tokens * channels * 2
    out = {"device": torch.cuda.get_device_name(0), "chunks": args.chunks, "layers": args.layers,
           "bytes_written_per_restore": written}
    with tempfile.TemporaryDirectory() as root:
        for name, kind, cls in (("fused", "svd_hevc", LineageRestorer), ("software", "svd_hevc", SoftwareLineageRestorer),
                                ("factor", "svd", FactorLineageRestorer), ("raw", "raw", RawLineageRestorer)):
            store = ObjectStore(f"{root}/{name}")
            runtime = LineageRuntime(store, model)
            runtime.create_lineage("s")
            method = RankMethodConfig(energy_targets("causvid"), CodecSpec("svd_hevc" if kind == "raw" else kind, 32))
            node = None
            for index, (matrices, contexts) in enumerate(chunks):
                if kind == "raw":
                    node = runtime.commit_raw_node("s", f"c{index}", matrices, contexts).node_ref
                else:
                    node = runtime.commit_node("s", f"c{index}", matrices, contexts, method=method,
                                               device=device).node_ref
            restorer = cls(runtime, device)
            stream = torch.cuda.Stream(device)

            def restore():
                result = restorer.restore(node, lambda l, t: caches[(l, t)],
                                          lambda piece: (table, (frames * (piece.token_start // tokens), 0, 0)),
                                          stream=stream, overlapped=False)
                result.join()
                torch.cuda.current_stream(device).wait_stream(stream)

            for _ in range(2):
                restore()
            torch.cuda.synchronize()
            start, stop = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            start.record()
            for _ in range(args.reps):
                restore()
            stop.record()
            torch.cuda.synchronize()
            ms = start.elapsed_time(stop) / args.reps
            dense = runtime.acquire_node_history(node, MatrixKey(0, "V"), device=device)
            error = float((caches[(0, "V")][0].reshape(-1, channels).float() - dense).norm() / dense.norm())
            out[name] = {"ms_per_restore": round(ms, 3), "GB_per_s": round(written / (ms * 1e-3) / 1e9, 1),
                         "v_error_vs_history": error, "archive_bytes": runtime.node_storage(node)["total_bytes"]}
            store.close()
    text = json.dumps(out, indent=1)
    print(text)
    if args.out:
        args.out.write_text(text)


if __name__ == "__main__":
    main()
