"""Ulysses projections of one LongCat-shaped attention block on N GPUs: the fused kernels (QKV GEMM with the
head scatter in its epilogue over NVLink peer stores; output projection whose TMA producer gathers the
attention outputs from the owners' memory) against the library path (the same tcgen05 GEMM followed or
preceded by NCCL ``all_to_all_single``).

    python -m torch.distributed.run --nproc-per-node 8 --master-addr 127.0.0.1 examples/benchmark_ulysses_fused.py

Per op: device time (CUDA events around ``--reps`` repetitions after warm-up, max over ranks), the fused
result checked against the library result, and the roofline of the fused op: the slower of its GEMM FLOPs
at the measured bf16 peak and its NVLink bytes at 770 GB/s per direction. Rank 0 prints one JSON line.
"""

from __future__ import annotations

import argparse
import datetime
import json
import os
import sys
from pathlib import Path


def main(argv=None):
    ap = argparse.ArgumentParser(description=__doc__)
    ap.add_argument("--tokens", type=int, default=14400, help="tokens of the chunk (all ranks together)")
    ap.add_argument("--dim", type=int, default=4096)
    ap.add_argument("--heads", type=int, default=32)
    ap.add_argument("--reps", type=int, default=20)
    args = ap.parse_args(argv)
    sys.path.insert(0, str(Path(__file__).resolve().parents[1]))
    import torch
    import torch.distributed as dist
    from reelcache_b200.ops import gemm
    from reelcache_b200.parallel.context_parallel import ulysses_in, ulysses_out
    from reelcache_b200.parallel.ulysses_fused import FusedUlysses

    local = int(os.environ.get("LOCAL_RANK", 0))
    torch.cuda.set_device(local)
    device = torch.device("cuda", local)
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=device)
    rank, world = dist.get_rank(), dist.get_world_size()
    d = args.dim // args.heads
    hp = args.heads // world
    n_loc = args.tokens // world
    rows = world * n_loc
    g = torch.Generator(device=device).manual_seed(0)
    y = torch.randn(n_loc, args.dim, device=device, generator=g).bfloat16()
    w_qkv = (torch.randn(3 * args.dim, args.dim, device=device, generator=torch.Generator(device=device).manual_seed(1))
             / args.dim ** 0.5).bfloat16()
    b_qkv = torch.randn(3 * args.dim, device=device, generator=torch.Generator(device=device).manual_seed(2)).bfloat16()
    w_o = (torch.randn(args.dim, args.dim, device=device, generator=torch.Generator(device=device).manual_seed(3))
           / args.dim ** 0.5).bfloat16()
    b_o = torch.randn(args.dim, device=device, generator=torch.Generator(device=device).manual_seed(4)).bfloat16()
    gate = torch.rand(args.dim, device=device, generator=torch.Generator(device=device).manual_seed(5))
    o_local = torch.randn(rows, hp, d, device=device, generator=g).bfloat16()
    x0 = torch.randn(n_loc, args.dim, device=device, generator=g)
    fused = FusedUlysses(None, device, heads=args.heads, head_dim=d, rows=rows)
    fused.local["o"][:rows].copy_(o_local.reshape(rows, hp * d))
    torch.cuda.synchronize()
    dist.barrier()

    def library_qkv():
        qkv = gemm.linear(y, w_qkv, b_qkv).reshape(n_loc, 3, args.heads, d)
        return [ulysses_in(qkv[:, s].contiguous()) for s in range(3)]

    def fused_qkv():
        return fused.qkv(y, w_qkv, b_qkv)

    def library_out(x):
        o = ulysses_out(o_local)  # [n_loc, heads, d]
        x.add_(gate * gemm.linear(o.reshape(n_loc, args.dim), w_o, b_o).float())
        return x

    def fused_out(x):
        return fused.out(x, w_o, b_o, gate)

    # correctness: fused against library
    ref = library_qkv()
    got = fused_qkv()
    torch.cuda.synchronize()
    qkv_err = max(float((a.float() - b.float()).abs().max()) for a, b in zip(got, ref))
    xr, xf = x0.clone(), x0.clone()
    library_out(xr)
    fused_out(xf)
    torch.cuda.synchronize()
    out_err = float((xr - xf).abs().max())
    fused.check()

    def timed(fn, reps=args.reps):
        for _ in range(3):
            fn()
        torch.cuda.synchronize()
        dist.barrier()
        start, stop = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        start.record()
        for _ in range(reps):
            fn()
        stop.record()
        torch.cuda.synchronize()
        t = torch.tensor([start.elapsed_time(stop) / reps], device=device)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t)

    xb = x0.clone()
    res = {"world": world, "tokens": rows, "n_loc": n_loc, "dim": args.dim, "heads": args.heads,
           "qkv_library_ms": timed(library_qkv), "qkv_fused_ms": timed(fused_qkv),
           "out_library_ms": timed(lambda: library_out(xb)), "out_fused_ms": timed(lambda: fused_out(xb)),
           "qkv_max_abs_diff": qkv_err, "out_max_abs_diff": out_err}
    fused.check()
    peaks_path = Path(__file__).resolve().parents[1] / "MEASURED_PEAKS.json"
    peak = json.loads(peaks_path.read_text())["bf16_tflops"] * 1e12 if peaks_path.exists() else 1.59e15
    link = 770e9
    for name, n, k in (("qkv", 3 * args.dim, args.dim), ("out", args.dim, args.dim)):
        flops = 2.0 * n_loc * n * k
        nv = (n_loc * (n if name == "qkv" else k) * 2) * (world - 1) / world
        bound_ms = max(flops / peak, nv / link) * 1e3
        res[f"{name}_roofline_ms"] = round(bound_ms, 4)
        res[f"{name}_fused_frac_of_roofline"] = round(bound_ms / res[f"{name}_fused_ms"], 3)
        res[f"{name}_nvlink_bytes_per_rank"] = int(nv)
    if rank == 0:
        print(json.dumps(res))
    fused.close()
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
