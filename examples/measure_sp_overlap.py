"""Overlap of the sequence-parallel history exchange with compute on 2+ GPUs (the counterpart of reference
examples/measure_sp_overlap.py): the NCCL all-gather of one layer's head slices (the tiered SP history's
distribution step) timed alone, a GEMM timed alone, and both issued on separate streams;
``hidden = (T_sync - T_overlap) / (T_sync - T_compute)`` is the fraction of the exchange hidden behind compute.

    python -m torch.distributed.run --nproc-per-node 2 --master-addr 127.0.0.1 examples/measure_sp_overlap.py

Device times (CUDA events), max over ranks; rank 0 prints one JSON line.
"""

from __future__ import annotations

import datetime
import json
import os
import sys
from pathlib import Path


def main():
    sys.path.insert(0, str(Path(__file__).resolve().parents[1]))
    import torch
    import torch.distributed as dist
    local = int(os.environ.get("LOCAL_RANK", 0))
    torch.cuda.set_device(local)
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120))
    rank, world = dist.get_rank(), dist.get_world_size()
    tokens, channels = 4680 * 8, 1536
    local_cols = channels // world
    piece = torch.randn(tokens, local_cols, device="cuda", dtype=torch.bfloat16)
    gathered = [torch.empty_like(piece) for _ in range(world)]
    a = torch.randn(8192, 8192, device="cuda", dtype=torch.bfloat16)
    comm, compute = torch.cuda.Stream(), torch.cuda.Stream()

    def timed(fn, reps=10):
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
        value = torch.tensor([start.elapsed_time(stop) / reps], device="cuda")
        dist.all_reduce(value, op=dist.ReduceOp.MAX)
        return float(value)

    def exchange():
        with torch.cuda.stream(comm):
            dist.all_gather(gathered, piece)
        torch.cuda.current_stream().wait_stream(comm)

    def gemm():
        with torch.cuda.stream(compute):
            a @ a
        torch.cuda.current_stream().wait_stream(compute)

    def both():
        with torch.cuda.stream(comm):
            dist.all_gather(gathered, piece)
        with torch.cuda.stream(compute):
            a @ a
        torch.cuda.current_stream().wait_stream(comm)
        torch.cuda.current_stream().wait_stream(compute)

    t_comm, t_compute, t_overlap = timed(exchange), timed(gemm), timed(both)
    t_sync = t_comm + t_compute
    hidden = (t_sync - t_overlap) / max(t_sync - t_compute, 1e-9)
    if rank == 0:
        print(json.dumps({"world": world, "exchange_ms": t_comm, "compute_ms": t_compute, "overlap_ms": t_overlap,
                          "hidden_fraction": hidden, "bytes_per_rank": piece.numel() * 2 * (world - 1)}))
    dist.barrier()
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
