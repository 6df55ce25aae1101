"""Fork time-to-first-chunk on a LongCat-Video-shaped DiT (one GPU, context parallelism 1).

A main session of ``--depth`` segments is built: each segment's conditioning cache (48 layers of pre-RoPE K and V
over one 4-frame 720p chunk, 14,400 tokens x 4096 channels each) is built by the model, captured into the raw
tiers and archived as a segment node (rank method on the GPU). Then the session forks at each of ``--forks``:
``resume(main, b, new_session)`` cuts the record after boundary ``b``, the fork's conditioning cache is fetched from
the best tier (with ``--host-gb`` 0 the raw tiers hold nothing and every fork restores the archived node) and the
first denoising forward of the fork's next chunk runs on it. Fork TTFC = record cut + cache fetch + that forward,
timed with CUDA events around the whole request on the compute stream (host work included, synchronised on both
sides). The reference quotes this workload on 8 GPUs with CP 8; this run keeps the full model and chunk shape on
one GPU, so each rank-equivalent restores and multiplies 8x the rows.

    python examples/benchmark_longcat_fork.py [--depth 16] [--forks 4,8,12] [--trials 3] [--out result.json]
"""

from __future__ import annotations

import argparse
import json
import statistics
import sys
import tempfile
import time
from pathlib import Path

import torch

sys.path.insert(0, str(Path(__file__).resolve().parent.parent))

from reelcache_b200.lineage import LineageRuntime  # noqa: E402
from reelcache_b200.models.longcat import LONGCAT_720P, LongCatDiT, ReelCacheConditioningCacheBackend  # noqa: E402
from reelcache_b200.models.longcat_session import EpochRawTiers, LongCatSessionProvider  # noqa: E402
from reelcache_b200.rank_method import RankMethodConfig  # noqa: E402
from reelcache_b200.store import ObjectStore  # noqa: E402
from reelcache_b200.types import CodecSpec, ModelIdentity, energy_targets  # noqa: E402


def main(argv=None) -> dict:
    ap = argparse.ArgumentParser(description=__doc__)
    ap.add_argument("--depth", type=int, default=16)
    ap.add_argument("--forks", default="4,8,12")
    ap.add_argument("--trials", type=int, default=3)
    ap.add_argument("--layers", type=int, default=LONGCAT_720P.layers)
    ap.add_argument("--host-gb", type=float, default=0.0, help="host raw tier budget (0: forks restore the archive)")
    ap.add_argument("--tiny", action="store_true", help="a small config for a CPU check of the procedure")
    ap.add_argument("--out", type=Path)
    args = ap.parse_args(argv)

    device = torch.device("cuda" if torch.cuda.is_available() else "cpu")
    cfg = LONGCAT_720P.scaled(layers=args.layers)
    if args.tiny:
        cfg = cfg.scaled(layers=2, dim=256, heads=2, ffn=512, text_dim=64, text_len=8, latent_height=8,
                         latent_width=16, frames_per_chunk=2)
    frames = cfg.frames_per_chunk
    model = LongCatDiT(cfg, device, seed=0, max_frames=(args.depth + 1) * frames)
    gen = torch.Generator(device=device).manual_seed(0)

    def latents(seed):
        g = torch.Generator(device=device).manual_seed(seed)
        return torch.randn((cfg.in_channels, frames, cfg.latent_height, cfg.latent_width), generator=g,
                           device=device)

    text = model.encode_text(torch.randn((cfg.text_len, cfg.text_dim), generator=gen, device=device))
    with tempfile.TemporaryDirectory() as tmp:
        store = ObjectStore(Path(tmp) / "store")
        identity = ModelIdentity("longcat-720p-shaped", "seed0", cfg.layers, cfg.dim, "BTHD", "bfloat16")
        runtime = LineageRuntime(store, identity)
        runtime.create_lineage("main")
        method = RankMethodConfig(energy_targets("longcat_720p"), CodecSpec("svd_hevc", 32), solver="topk_rr")
        # on CUDA the backend restores segments on the fused kernels (restorer="auto")
        backend = ReelCacheConditioningCacheBackend(runtime, "main", method, head_dim=cfg.head_dim, grid=cfg.grid,
                                                    device=device)
        tiers = EpochRawTiers(gpu_raw_budget_bytes=0, host_raw_budget_bytes=int(args.host_gb * (1 << 30)),
                              pin_memory=device.type == "cuda")
        provider = LongCatSessionProvider(model, backend, tiers)

        build_s = []
        for s in range(args.depth):
            started = time.perf_counter()
            _, tier = provider.segment_cache("main", s, latents(100 + s), text, first_frame=s * frames)
            if device.type == "cuda":
                torch.cuda.synchronize()
            build_s.append(time.perf_counter() - started)
            print(f"segment {s}: {tier} {build_s[-1]:.2f} s", file=sys.stderr, flush=True)

        noise = latents(7)
        # warm-up: one forward with a built cache (kernels loaded, allocator primed)
        warm, _ = provider.segment_cache("main", args.depth - 1, latents(100 + args.depth - 1), text,
                                         first_frame=(args.depth - 1) * frames)
        model.forward(noise, 0.9, text, first_frame=args.depth * frames, cache=warm)
        del warm
        if device.type == "cuda":
            torch.cuda.synchronize()

        forks = [int(b) for b in args.forks.split(",") if b]
        rows = []
        for trial in range(args.trials):
            for b in forks:
                session = f"fork{b}-{trial}"
                if device.type == "cuda":
                    torch.cuda.synchronize()
                    start, fetched, end = (torch.cuda.Event(enable_timing=True) for _ in range(3))
                    start.record()
                wall = time.perf_counter()
                provider.resume("main", b, new_session=session)
                cache, tier = provider.segment_cache(session, b, latents(100 + b), text, first_frame=b * frames,
                                                     base=provider.boundaries(session)[:-1])
                if device.type == "cuda":
                    fetched.record()
                out = model.forward(noise, 0.9, text, first_frame=(b + 1) * frames, cache=cache)
                if device.type == "cuda":
                    end.record()
                    torch.cuda.synchronize()
                    ttfc, fetch = start.elapsed_time(end), start.elapsed_time(fetched)
                else:
                    ttfc = fetch = (time.perf_counter() - wall) * 1e3
                rows.append({"fork": b, "trial": trial, "tier": tier, "ttfc_ms": round(ttfc, 2),
                             "fetch_ms": round(fetch, 2), "finite": bool(torch.isfinite(out).all())})
                print(f"fork at {b} trial {trial}: {tier} fetch {fetch:.1f} ms ttfc {ttfc:.1f} ms",
                      file=sys.stderr, flush=True)
                del cache, out
        stored = runtime.node_storage(provider.nodes[next(iter(provider.nodes))])
        store.close()

    ttfc = [r["ttfc_ms"] for r in rows]
    result = {
        "workload": f"LongCat-Video-shaped DiT ({cfg.layers} x {cfg.dim}, {cfg.heads} x {cfg.head_dim}, "
                    f"{cfg.latent_height * 8}p, {frames} latent frames per chunk), fork tree of depth {args.depth} "
                    f"with forks at {args.forks}, 1 GPU",
        "tokens_per_chunk": frames * cfg.tokens_per_frame,
        "segment_cache_bytes": 2 * cfg.layers * frames * cfg.tokens_per_frame * cfg.dim * 2,
        "segment_node_bytes": stored.get("total_bytes"),
        "p50_fork_ttfc_ms": round(statistics.median(ttfc), 2),
        "p90_fork_ttfc_ms": round(sorted(ttfc)[int(0.9 * (len(ttfc) - 1))], 2),
        "p50_fetch_ms": round(statistics.median(r["fetch_ms"] for r in rows), 2),
        "mean_segment_build_and_archive_s": round(statistics.mean(build_s), 2),
        "tiers": sorted({r["tier"] for r in rows}),
        "rows": rows,
        "data": "synthetic latents and text, random-init weights",
    }
    print(json.dumps(result))
    if args.out:
        args.out.write_text(json.dumps(result, indent=1))
    return result


if __name__ == "__main__":
    main()
