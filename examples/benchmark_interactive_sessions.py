"""Interactive session mix on one GPU (the 64-session resume / rewind / fork mix scaled to one device; the counterpart of reference
examples/benchmark_interactive_sessions.py): sessions of the CausVid-shaped DiT (random-init bf16, full-history
visibility) created with histories of ``--min-history..--max-history`` chunks, then a Poisson trace of resume /
rewind-to-an-earlier-chunk / fork requests (50 / 30 / 20 %) served through the bridge
(``create_sglang_backend`` -> ``CausalWanKVBridge.request``), each generating one chunk. Reports p50 / p90 / p99
time to first chunk per action and the restore routes taken (resident cursor, archive restore).

    python examples/benchmark_interactive_sessions.py --sessions 8 --requests 40 [--out result.json]

TTFC is the bridge's own host clock from the request to the first generated chunk's latents on the host (it
includes the archive restore, overlapped layer by layer with the first denoising step).
"""

from __future__ import annotations

import argparse
import json
import sys
import tempfile
from pathlib import Path


def main(argv=None):
    ap = argparse.ArgumentParser(description=__doc__)
    ap.add_argument("--sessions", type=int, default=8)
    ap.add_argument("--requests", type=int, default=40)
    ap.add_argument("--min-history", type=int, default=4)
    ap.add_argument("--max-history", type=int, default=8)
    ap.add_argument("--rate", type=float, default=2.0)
    ap.add_argument("--layers", type=int, default=30)
    ap.add_argument("--realtime", action="store_true", help="honour the Poisson arrival times")
    ap.add_argument("--resident-gb", type=float, default=40.0, help="budget of the sessions' resident caches")
    ap.add_argument("--out", type=Path)
    args = ap.parse_args(argv)
    sys.path.insert(0, str(Path(__file__).resolve().parents[1]))
    import torch
    from reelcache_b200.integrations.sglang import ReelCacheRuntimeConfig, create_sglang_backend
    from reelcache_b200.models.causal_wan import CAUSVID, CausalWanDiT
    from reelcache_b200.workloads import WorkloadSpec, run

    device = torch.device("cuda", 0)
    cfg = CAUSVID if args.layers == 30 else CAUSVID.scaled(layers=args.layers)
    model = CausalWanDiT(cfg, device, seed=0)
    gen = torch.Generator(device=device).manual_seed(1)
    text_kv = model.encode_text(torch.randn((cfg.text_len, cfg.text_dim), generator=gen, device=device))
    spec = WorkloadSpec(sessions=args.sessions, rate_per_s=args.rate, requests=args.requests,
                        min_history=args.min_history, max_history=args.max_history)
    with tempfile.TemporaryDirectory(prefix="reelcache-sessions-") as root:
        config = ReelCacheRuntimeConfig(store_root=root, fit_device="cuda", encode_workers=2,
                                        max_resident_bytes=int(args.resident_gb * (1 << 30)))
        bridge = create_sglang_backend(config, (model, text_kv), cache_chunks=args.max_history + 4)
        try:
            result = run(bridge, spec, realtime=args.realtime)
        finally:
            bridge.shutdown()
    summary = result.summary()
    summary.update(device=torch.cuda.get_device_name(0), layers=cfg.layers, spec=vars(args) | {"out": None},
                   resident_evictions=bridge.resident_evictions)
    text = json.dumps(summary, indent=1, default=str)
    print(text)
    if args.out:
        args.out.write_text(text)


if __name__ == "__main__":
    main()
