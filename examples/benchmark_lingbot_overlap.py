"""LingBot-World-Fast resume on one GPU: time to the first chunk after a restart, with the history restored
synchronously or layer-overlapped with the chunk's forward (pre-hooks on every block's self-attention).

The stand-in world model has LingBot's per-layer geometry (40 heads x 128 = 5,120 channels, 3-frame chunks of 30 x
52 latent tokens, a 7-chunk window) with ``--layers`` blocks and random weights; a session of ``--chunks`` chunks is
generated and archived (``svd_hevc``, the fused restore kernels), then a fresh model instance (an empty cache)
resumes after the last chunk ``--trials`` times per mode. Time = CUDA events from before the restore call to the
end of the next chunk's forward, synchronized on both sides; the overlapped mode also reports the per-layer stall
of the generation stream (StallEvents).

    python examples/benchmark_lingbot_overlap.py [--layers 8] [--chunks 8] [--trials 3] [--out result.json]

Progress and the time of each phase go to stderr.
"""

import argparse
import json
import sys
import tempfile
import time
from pathlib import Path

import torch

sys.path.insert(0, str(Path(__file__).resolve().parents[1]))


def main(argv=None):
    ap = argparse.ArgumentParser(description=__doc__)
    ap.add_argument("--layers", type=int, default=8)
    ap.add_argument("--chunks", type=int, default=8)
    ap.add_argument("--trials", type=int, default=3)
    ap.add_argument("--out", type=Path)
    args = ap.parse_args(argv)
    from reelcache_b200.integrations.lingbot import LINGBOT_WORLD_FAST, LingBotArchive, StallEvents, StandInWorldModel

    dev = torch.device("cuda", 0)
    geometry = LINGBOT_WORLD_FAST.scaled(layers=args.layers)
    g = torch.Generator().manual_seed(0)
    xs = [torch.randn(geometry.chunk_tokens, geometry.channels, generator=g) for _ in range(args.chunks + 1)]
    rows = {"synchronous": [], "overlapped": []}
    stalls = []
    with tempfile.TemporaryDirectory() as tmp:
        archive = LingBotArchive(Path(tmp) / "store", geometry, representation="svd_hevc", device=dev)
        archive.ensure_session("s")
        live = StandInWorldModel(geometry, device=dev)
        parent = None
        started = time.perf_counter()
        for chunk in range(args.chunks):
            _, (k, v) = live.generate(chunk, xs[chunk])
            archive.commit("s", f"s/{chunk}", parent, chunk, k, v)
            parent = f"s/{chunk}"
            print(f"chunk {chunk} generated and queued: {time.perf_counter() - started:.1f} s", file=sys.stderr,
                  flush=True)
        archive.drain()
        print(f"archive drained: {time.perf_counter() - started:.1f} s", file=sys.stderr, flush=True)
        del live
        model = StandInWorldModel(geometry, device=dev)
        model.generate(args.chunks, xs[args.chunks], capture=False)  # warm-up (kernels, allocator)
        torch.cuda.synchronize()
        for trial in range(args.trials + 1):
            for mode in ("synchronous", "overlapped"):
                torch.cuda.synchronize()
                start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                start.record()
                recorder = StallEvents(dev, start) if mode == "overlapped" else None
                session = archive.restore(parent, model, overlapped=mode == "overlapped", recorder=recorder)
                model.generate(args.chunks, xs[args.chunks], capture=False)
                end.record()
                torch.cuda.synchronize()
                if trial == 0:
                    continue  # the first restore builds and caches its plan
                rows[mode].append(start.elapsed_time(end))
                print(f"trial {trial} {mode}: {rows[mode][-1]:.1f} ms", file=sys.stderr, flush=True)
                if recorder is not None:
                    stalls.append(session.gpu_summary()["stall_ms_total"])
        archive.close()
    result = {
        "geometry": {"layers": geometry.layers, "heads": geometry.heads, "head_dim": geometry.head_dim,
                     "chunk_tokens": geometry.chunk_tokens, "window_chunks": geometry.window_chunks},
        "history_chunks_restored": min(args.chunks, geometry.window_chunks - 1),
        "restored_bytes": 2 * geometry.layers * min(args.chunks, geometry.window_chunks - 1) * geometry.chunk_tokens
        * geometry.channels * 2,
        "ttfc_ms": {mode: sorted(values)[len(values) // 2] for mode, values in rows.items()},
        "ttfc_ms_all": {mode: [round(v, 2) for v in values] for mode, values in rows.items()},
        "overlapped_stall_ms_total": [round(v, 2) for v in stalls],
    }
    print(json.dumps(result))
    if args.out:
        args.out.write_text(json.dumps(result, indent=1))


if __name__ == "__main__":
    main()
