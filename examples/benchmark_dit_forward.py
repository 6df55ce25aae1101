"""One denoising forward of the CausVid-shaped DiT (chunk 4 attending to a 4-chunk history, 30 layers), timed with
CUDA events; ``--profile-window`` wraps one more forward in cudaProfilerStart/Stop for an ncu launch list.

    python examples/benchmark_dit_forward.py --backend auto --iters 10
    ncu --metrics gpu__time_duration.sum --clock-control none --profile-from-start off --csv \\
        python examples/benchmark_dit_forward.py --iters 5 --profile-window
"""

from __future__ import annotations

import argparse
import json
import sys
import time
from pathlib import Path


def main(argv=None):
    ap = argparse.ArgumentParser(description=__doc__)
    ap.add_argument("--backend", default="auto", choices=("auto", "sdpa", "fused"), help="attention backend")
    ap.add_argument("--iters", type=int, default=10)
    ap.add_argument("--history", type=int, default=4)
    ap.add_argument("--profile-window", action="store_true")
    args = ap.parse_args(argv)
    sys.path.insert(0, str(Path(__file__).resolve().parents[1]))
    import torch
    from reelcache_b200.models.causal_wan import CAUSVID, CausalWanDiT, KVCache

    cfg = CAUSVID
    torch.manual_seed(0)
    model = CausalWanDiT(cfg, "cuda")
    cache = KVCache(cfg, args.history + 1, "cuda")
    for layer in range(cfg.layers):
        cache.k[layer].normal_()
        cache.v[layer].normal_()
    text_kv = model.encode_text(torch.randn(cfg.text_len, cfg.text_dim, device="cuda"))
    latents = torch.randn(cfg.in_dim, cfg.frames_per_chunk, cfg.latent_height, cfg.latent_width, device="cuda")

    def forward():
        return model.forward_chunk(latents, 757.0, args.history, cache, text_kv, attention_backend=args.backend)

    for _ in range(3):
        forward()
    torch.cuda.synchronize()
    times = []
    for _ in range(args.iters):
        start, stop = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        start.record()
        forward()
        stop.record()
        torch.cuda.synchronize()
        times.append(start.elapsed_time(stop))
    wall = time.perf_counter()
    forward()
    enqueue_ms = (time.perf_counter() - wall) * 1e3
    torch.cuda.synchronize()
    median = sorted(times)[len(times) // 2]
    flops = model.flops_per_forward(args.history * cfg.chunk_tokens)
    print(json.dumps({"backend": args.backend, "forward_ms": round(median, 3), "min_ms": round(min(times), 3),
                      "host_enqueue_ms": round(enqueue_ms, 2), "tflops": round(flops / (median * 1e9), 1)}))
    if args.profile_window:
        torch.cuda.profiler.start()
        forward()
        torch.cuda.synchronize()
        torch.cuda.profiler.stop()


if __name__ == "__main__":
    main()
