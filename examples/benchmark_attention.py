"""Attention forward on one B200: the sm_100a tcgen05 kernel (``backend="fused"``) against cuDNN's fused SDPA
(``backend="sdpa"``) on the DiT shapes, bf16, head_dim 128, non-causal.

Times are CUDA-event means of ``--reps`` back-to-back calls after 3 warm-up calls on the launching stream;
TFLOP/s counts 4 * Tq * Tk * 128 * heads. Every call reads K and V of at least 18 MB per head group; the
self-attention shapes read 110-230 MB of K / V per call (above the 126 MB L2 for the larger ones).

    python examples/benchmark_attention.py [--shapes causvid|longcat|all] [--out result.json]
    python examples/benchmark_attention.py --small      # one fused call on 4680 x 4680 x 12 (an ncu case)
"""

import argparse
import json
import math
import sys
from pathlib import Path

import torch

sys.path.insert(0, str(Path(__file__).resolve().parents[1]))

SHAPES = {
    "causvid": [(4680, 23400, 12), (4680, 18720, 12), (4680, 4680, 12), (4680, 512, 12)],
    "longcat": [(14432, 14432, 32)],
}


def timed(fn, reps):
    for _ in range(3):
        fn()
    torch.cuda.synchronize()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    start.record()
    for _ in range(reps):
        fn()
    end.record()
    torch.cuda.synchronize()
    return start.elapsed_time(end) / reps


def main():
    ap = argparse.ArgumentParser(description=__doc__)
    ap.add_argument("--shapes", choices=("causvid", "longcat", "all"), default="all")
    ap.add_argument("--reps", type=int, default=20)
    ap.add_argument("--small", action="store_true")
    ap.add_argument("--trace", action="store_true", help="clock64 timeline of one CTA (cycles per phase)")
    ap.add_argument("--out", type=Path)
    args = ap.parse_args()
    from reelcache_b200.ops import _ext
    from reelcache_b200.ops.attention import OPT_NO_TURNS, OPT_POLY_EXP, attention

    dev = torch.device("cuda", 0)
    g = torch.Generator(device=dev).manual_seed(0)
    if args.small:
        q = torch.randn(4680, 12, 128, device=dev, generator=g).bfloat16()
        k = torch.randn(4680, 12, 128, device=dev, generator=g).bfloat16()
        v = torch.randn(4680, 12, 128, device=dev, generator=g).bfloat16()
        for _ in range(3):
            attention(q, k, v, backend="fused")
        torch.cuda.synchronize()
        _ext.check_status(dev)
        print(json.dumps({"small": "ok"}))
        return
    if args.trace:
        for tq, tk, heads in [(4680, 18720, 12), (14432, 14432, 32)]:
            q = torch.randn(tq, heads, 128, device=dev, generator=g).bfloat16()
            k = torch.randn(tk, heads, 128, device=dev, generator=g).bfloat16()
            v = torch.randn(tk, heads, 128, device=dev, generator=g).bfloat16()
            for options in (1, 1 | OPT_POLY_EXP, 1 | OPT_NO_TURNS):
                trace = torch.zeros(512, dtype=torch.int64, device=dev)
                out = torch.empty_like(q)
                for _ in range(2):
                    _ext.ext().attention_fwd(q, k, v, out, 1.0 / math.sqrt(128), _ext.status_word(dev), options | 32, trace)
                torch.cuda.synchronize()
                t = trace.view(32, 16).cpu().tolist()
                phases = {"ld0": [], "sm0": [], "st0": [], "next0": [], "ld1": [], "sm1": [], "st1": [], "next1": [],
                          "mma_wait_p0": [], "mma_wait_p1": [], "period": []}
                for i in range(4, 30):
                    a, b = t[i], t[i + 1]
                    for gi in (0, 1):
                        e = 4 * gi
                        phases[f"ld{gi}"].append(a[e + 1] - a[e])
                        phases[f"sm{gi}"].append(a[e + 2] - a[e + 1])
                        phases[f"st{gi}"].append(a[e + 3] - a[e + 2])
                        phases[f"next{gi}"].append(b[e] - a[e + 3])
                    phases["mma_wait_p0"].append(b[9] - b[8])
                    phases["mma_wait_p1"].append(b[11] - b[10])
                    phases["period"].append(b[0] - a[0])
                med = {k2: sorted(v2)[len(v2) // 2] for k2, v2 in phases.items()}
                print(json.dumps({"trace_shape": [tq, tk, heads], "options": options, "median_cycles": med}), flush=True)
        return
    shapes = SHAPES["causvid"] + SHAPES["longcat"] if args.shapes == "all" else SHAPES[args.shapes]
    rows = []
    for tq, tk, heads in shapes:
        q = torch.randn(tq, heads, 128, device=dev, generator=g).bfloat16()
        k = torch.randn(tk, heads, 128, device=dev, generator=g).bfloat16()
        v = torch.randn(tk, heads, 128, device=dev, generator=g).bfloat16()
        scale = 1.0 / math.sqrt(128)
        flops = 4.0 * tq * tk * 128 * heads
        row = {"shape": [tq, tk, heads]}
        variants = {"fused": 0, "fused_one_range": 1, "fused_poly8": OPT_POLY_EXP, "fused_no_turns": OPT_NO_TURNS}
        for name, options in variants.items():
            ms = timed(lambda: attention(q, k, v, backend="fused", scale=scale, options=options), args.reps)
            row[name] = {"ms": round(ms, 4), "tflops": round(flops / ms / 1e9, 1)}
        ms = timed(lambda: attention(q, k, v, backend="sdpa", scale=scale), args.reps)
        row["cudnn_sdpa"] = {"ms": round(ms, 4), "tflops": round(flops / ms / 1e9, 1)}
        ref = attention(q, k, v, backend="sdpa", scale=scale).float()
        got = attention(q, k, v, backend="fused", scale=scale).float()
        row["rel_diff_vs_cudnn"] = float((got - ref).norm() / ref.norm())
        _ext.check_status(dev)
        rows.append(row)
        print(json.dumps(row), flush=True)
        del q, k, v
    if args.out:
        args.out.write_text(json.dumps(rows, indent=1))


if __name__ == "__main__":
    main()
