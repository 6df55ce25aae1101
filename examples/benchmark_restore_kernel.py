"""One fused restore launch on one GPU: ``--jobs`` jobs of the CausVid geometry (4680 tokens x 1536 channels,
u8 coefficients of rank ``--rank``; even jobs K with Wan 3-axis RoPE, odd jobs V) restored into bf16 BTHD caches
by ``RestoreProgram`` (one ``restore_run`` per 48 jobs). Optional measurement variants (``--modes``, the kernel's
``ablate`` word): 1 drops the stores, 2 also the arithmetic, 4 the TMEM reads, 5 also the MMAs, 7 also the
tcgen05 commits, 8 also the TMA loads.

    python examples/benchmark_restore_kernel.py --jobs 48 --rank 64 --modes 0,1,2,4,8

Device time per launch: CUDA events around 20 back-to-back launches after 3 warm-up launches, with the GPU
held busy while the host enqueues them (the events time the device only). GB/s counts the bf16 bytes written.
"""

from __future__ import annotations

import argparse
import json
import sys
from pathlib import Path


def main(argv=None):
    ap = argparse.ArgumentParser(description=__doc__)
    ap.add_argument("--jobs", type=int, default=8)
    ap.add_argument("--rank", type=int, default=64)
    ap.add_argument("--modes", default="0")
    ap.add_argument("--iters", type=int, default=20)
    args = ap.parse_args(argv)
    sys.path.insert(0, str(Path(__file__).resolve().parents[1]))
    import numpy as np
    import torch
    from reelcache_b200 import restore_kernels as rk
    from reelcache_b200.ops import _ext
    from reelcache_b200.ops.restore import RestoreProgram

    device = torch.device("cuda", 0)
    frames, height, width, heads, head_dim = 3, 30, 52, 12, 128
    tokens, channels = frames * height * width, heads * head_dim
    pairs = max(1, args.jobs // 2)
    caches = {t: torch.zeros((1, pairs * tokens, heads, head_dim), dtype=torch.bfloat16, device=device) for t in "KV"}
    table = rk.RopeTable.wan(head_dim, 1024, device=device)
    rng = np.random.default_rng(0)
    stream = torch.cuda.current_stream(device)
    program = RestoreProgram(device, stream, precision="fp16")
    for index in range(args.jobs):
        chunk, target = index // 2, "KV"[index % 2]
        values = torch.from_numpy(rng.integers(0, 256, (tokens, args.rank), dtype=np.uint8)).to(device)
        basis = (torch.randn(args.rank, channels, device=device) / channels ** 0.5).half()
        rows = caches[target][0, chunk * tokens:(chunk + 1) * tokens]
        job = {"kind": "u8", "values": values, "tokens": tokens, "rank": args.rank, "grid": (frames, height, width),
               "basis": basis, "qmax": float(basis.abs().amax()),
               "scale": rng.uniform(0.001, 0.01, args.rank).astype(np.float32),
               "offset": rng.uniform(-1.0, 1.0, args.rank).astype(np.float32),
               "dest": (rows.data_ptr(), rows.stride(), rows.dtype, channels, head_dim), "rope": None}
        if target == "K":
            job["rope"] = rk.restore_rope_item(rk.RopePositions(table, (frames * chunk, 0, 0)), (frames, height, width),
                                               device, stream, program.keepalive)
        program.add(job)
    program.prepare()
    torch.cuda.synchronize()
    status = _ext.status_word(device)
    blobs = [blob for group in program.blobs.values() for blob in group]
    written = args.jobs * tokens * channels * 2
    out = {"device": torch.cuda.get_device_name(0), "jobs": args.jobs, "rank": args.rank, "launches": len(blobs),
           "bytes_written": written}
    for mode in (int(m, 0) for m in args.modes.split(",")):
        def launch():
            for blob in blobs:
                _ext.ext().restore_run(blob, device.index, status, mode)

        for _ in range(3):
            launch()
        torch.cuda.synchronize()
        start, stop = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        torch.cuda._sleep(20_000_000)
        start.record()
        for _ in range(args.iters):
            launch()
        stop.record()
        torch.cuda.synchronize()
        us = start.elapsed_time(stop) / args.iters * 1e3
        out[f"mode_{mode:#x}"] = {"us": round(us, 1), "GB_per_s": round(written / us / 1e3, 1)}
    _ext.check_status(device)
    print(json.dumps(out))


if __name__ == "__main__":
    main()
