"""Sequence-parallel Gram fit on N GPUs: the fused kernel (upper-triangular partial Gram tiles of every rank's
token shard stored straight into the fit owners' buffers over NVLink, owner-side rank-order sum) against the
library path (the same FP32-accurate tcgen05 Gram per matrix, then an NCCL reduce of the full FP32 Gram to the
owner). Shapes: one chunk of the CausVid-shaped DiT under SP N -- ``--matrices`` captured K/V matrices of
[4680, 1536] with 4680 / N tokens per rank, owners round-robin.

    python -m torch.distributed.run --nproc-per-node 8 --master-addr 127.0.0.1 examples/benchmark_gram_rs.py

Device time per batch (CUDA events around ``--reps`` repetitions after warm-up, max over ranks), the fused
Gram checked against the library Gram on every owner, and the fused path's roofline: the slower of its GEMM
FLOPs at the measured bf16 peak and the NVLink bytes the busiest rank sends at 770 GB/s. Rank 0 prints one
JSON line.
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
    ap.add_argument("--tokens", type=int, default=4680)
    ap.add_argument("--channels", type=int, default=1536)
    ap.add_argument("--matrices", type=int, default=16)
    ap.add_argument("--reps", type=int, default=10)
    args = ap.parse_args(argv)
    sys.path.insert(0, str(Path(__file__).resolve().parents[1]))
    import torch
    import torch.distributed as dist
    from reelcache_b200.ops.fitter import matmul_promoted
    from reelcache_b200.parallel.gram_rs import GramReduceScatter

    local = int(os.environ.get("LOCAL_RANK", 0))
    torch.cuda.set_device(local)
    device = torch.device("cuda", local)
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=device)
    rank, world = dist.get_rank(), dist.get_world_size()
    n_r = (args.tokens // world + 7) // 8 * 8
    owners = [b % world for b in range(args.matrices)]
    g = torch.Generator(device=device).manual_seed(rank)
    shards = [torch.randn(n_r, args.channels, device=device, generator=g).bfloat16() for _ in range(args.matrices)]
    xt = torch.cat([x.t() for x in shards]).contiguous()
    slots = GramReduceScatter.slots_for(owners)
    fused = GramReduceScatter(None, device, channels=args.channels, max_slots=max(slots) + 1)
    in_switch = GramReduceScatter(None, device, channels=args.channels, max_slots=max(slots) + 1, nvls="auto")

    def library():
        out = {}
        for b, owner in enumerate(owners):
            gram = matmul_promoted(xt[b * args.channels:(b + 1) * args.channels],
                                   xt[b * args.channels:(b + 1) * args.channels])
            dist.reduce(gram, dst=owner)
            if owner == rank:
                out[b] = gram
        return out

    def run_fused():
        return fused.run(xt, owners)

    ref = library()
    got = run_fused()
    torch.cuda.synchronize()
    fused.check()
    err = max((float((got[b] - ref[b]).norm() / ref[b].norm()) for b in got), default=0.0)
    errt = torch.tensor([err], device=device)
    dist.all_reduce(errt, op=dist.ReduceOp.MAX)

    def timed(fn):
        for _ in range(3):
            fn()
        torch.cuda.synchronize()
        dist.barrier()
        start, stop = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        start.record()
        for _ in range(args.reps):
            fn()
        stop.record()
        torch.cuda.synchronize()
        t = torch.tensor([start.elapsed_time(stop) / args.reps], device=device)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t)

    res = {"world": world, "matrices": args.matrices, "tokens_per_rank": n_r, "channels": args.channels,
           "library_ms": timed(library), "fused_ms": timed(run_fused), "max_rel_diff": float(errt)}
    if in_switch.nvls:
        got_nvls = in_switch.run(xt, owners)
        torch.cuda.synchronize()
        in_switch.check()
        err_n = max((float((got_nvls[b] - ref[b]).norm() / ref[b].norm()) for b in got_nvls), default=0.0)
        errn = torch.tensor([err_n], device=device)
        dist.all_reduce(errn, op=dist.ReduceOp.MAX)
        res.update(nvls_ms=timed(lambda: in_switch.run(xt, owners)), nvls_max_rel_diff=float(errn))
    else:
        res.update(nvls_ms=None, nvls_note="no NVLink multicast object on these GPUs")
    fused.check()
    nt = args.channels // 128
    tiles = nt * (nt + 1) // 2
    flops = 2.0 * n_r * tiles * 128 * 128 * args.matrices
    remote = sum(1 for o in owners if o != rank)
    nv_bytes = remote * tiles * 128 * 128 * 4
    peaks = Path(__file__).resolve().parents[1] / "MEASURED_PEAKS.json"
    peak = json.loads(peaks.read_text())["bf16_tflops"] * 1e12 if peaks.exists() else 1.59e15
    bound = max(flops / peak, nv_bytes / 770e9) * 1e3
    res.update(roofline_ms=round(bound, 4), fused_frac_of_roofline=round(bound / res["fused_ms"], 3),
               nvlink_bytes_per_rank=nv_bytes)
    if rank == 0:
        print(json.dumps(res))
    fused.close()
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
