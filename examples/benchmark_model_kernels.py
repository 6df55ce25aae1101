"""The DiT's and the raw tier's hot ops on one GPU at CausVid geometry (4680 tokens per chunk, dim 1536, 12 heads x
128): AdaLN LayerNorm + modulation, fused q/k RMSNorm + RoPE writing the KV-cache slots, RMSNorm, the dense RoPE
store of a raw-tier matrix into the native cache (``restore_kernels.reconstruct`` with a ``DenseSource``), the
block's GEMMs on the tcgen05 kernel against cuBLAS (``torch.matmul``), and the raw tier's device<->host staging
copies of one chunk's 60 K/V matrices on a side stream (copy engines, pinned host memory).

    python examples/benchmark_model_kernels.py [--out result.json]

Every kernel time is a CUDA-event mean over back-to-back calls after 3 warm-up calls; each call reads a
different copy of its inputs from a ring larger than the 126 MB L2, so DRAM figures are not L2 hits.
``GB/s`` counts the bytes each op must read and write once; ``frac`` divides by the measured copy bandwidth
(MEASURED_PEAKS.json ``hbm_gbs``) or, for GEMMs, the measured cuBLAS bf16 burst peak.
"""

from __future__ import annotations

import argparse
import json
import sys
from pathlib import Path


def main(argv=None):
    ap = argparse.ArgumentParser(description=__doc__)
    ap.add_argument("--tokens", type=int, default=4680)
    ap.add_argument("--reps", type=int, default=20)
    ap.add_argument("--only", choices=("all", "norms"), default="all",
                    help="norms: only the memory-bound ops (a short run for profiling)")
    ap.add_argument("--gemm", help="M,N,K: only run gemm.linear on this shape three times (a small case for ncu)")
    ap.add_argument("--out", type=Path)
    args = ap.parse_args(argv)
    root = Path(__file__).resolve().parents[1]
    sys.path.insert(0, str(root))
    import torch
    from reelcache_b200 import restore_kernels as rk
    from reelcache_b200.ops import _ext, gemm, norms

    device = torch.device("cuda", 0)
    if args.gemm:
        m, n, k = (int(v) for v in args.gemm.split(","))
        a = torch.randn(m, k, device=device).bfloat16()
        w = (torch.randn(n, k, device=device) / k ** 0.5).bfloat16()
        for _ in range(3):
            gemm.linear(a, w)
        torch.cuda.synchronize()
        _ext.check_status(device)
        return
    peaks_path = root / "MEASURED_PEAKS.json"
    peaks = json.loads(peaks_path.read_text()) if peaks_path.exists() else {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0}
    hbm, tflops = peaks["hbm_gbs"], peaks["bf16_tflops"]
    T, C, H, D, F = args.tokens, 1536, 12, 128, 8960
    ring_bytes = 512 << 20

    def ring(make, nbytes):
        return [make() for _ in range(max(2, -(-ring_bytes // max(nbytes, 1))))]

    def timed(fn, n):
        for i in range(3):
            fn(i % n)
        torch.cuda.synchronize()
        start, stop = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        start.record()
        for i in range(args.reps):
            fn(i % n)
        stop.record()
        torch.cuda.synchronize()
        return start.elapsed_time(stop) / args.reps

    out = {"device": torch.cuda.get_device_name(0), "tokens": T, "dim": C, "hbm_gbs_measured": hbm,
           "bf16_tflops_measured": tflops}

    def record(name, ms, nbytes=None, flops=None):
        row = {"ms": round(ms, 4)}
        if nbytes is not None:
            row.update(GB_per_s=round(nbytes / ms / 1e6, 1), frac_of_measured_hbm=round(nbytes / ms / 1e6 / hbm, 3))
        if flops is not None:
            row.update(TFLOPs=round(flops / ms / 1e9, 1), frac_of_measured_bf16=round(flops / ms / 1e9 / tflops, 3))
        out[name] = row

    # AdaLN LayerNorm + modulation: x bf16 [T, C] -> y bf16
    xs = ring(lambda: torch.randn(T, C, device=device).bfloat16(), T * C * 2)
    ys = [torch.empty_like(xs[0]) for _ in range(2)]
    shift, scale = torch.randn(C, device=device), torch.randn(C, device=device)
    record("ln_modulate", timed(lambda i: norms.ln_modulate(xs[i], shift=shift, scale=scale, out=ys[i % 2]), len(xs)),
           nbytes=2 * T * C * 2)
    # RMSNorm over the channel dim
    w = torch.rand(C, device=device) + 0.5
    record("rms_norm", timed(lambda i: norms.rms_norm(xs[i], w, out=ys[i % 2]), len(xs)), nbytes=2 * T * C * 2)
    # fused q/k RMSNorm + RoPE from qkv into q, the pre-RoPE K capture and the K/V cache slots
    qkvs = ring(lambda: torch.randn(T, 3 * C, device=device).bfloat16(), T * 3 * C * 2)
    table = rk.RopeTable.wan(D, 1024, device=device)
    cos, sin = table.token_tables((0, 0, 0), (3, 30, 52), device)
    wq, wk = torch.rand(C, device=device) + 0.5, torch.rand(C, device=device) + 0.5
    q_out = torch.empty(T, C, device=device, dtype=torch.bfloat16)
    k_pre, k_cache, v_cache = torch.empty_like(q_out), torch.empty_like(q_out), torch.empty_like(q_out)
    record("qkv_norm_rope", timed(lambda i: norms.qkv_norm_rope(qkvs[i], wq, wk, cos, sin, q_out, k_cache, v_cache,
                                                               head_dim=D, k_pre=k_pre), len(qkvs)),
           nbytes=T * 3 * C * 2 + 4 * T * C * 2)
    # dense RoPE store of one raw-tier K matrix into a native BTHD slot
    dests = ring(lambda: torch.empty((1, T, H, D), device=device, dtype=torch.bfloat16), T * C * 2)
    jobs = [rk.ReconstructionJob(rk.DenseSource(xs[i]), rk.NativeView(dests[i % len(dests)]), (3, 30, 52),
                                 rope=rk.RopePositions(table, (0, 0, 0))) for i in range(len(xs))]
    record("dense_rope_store", timed(lambda i: rk.reconstruct([jobs[i]], backend="fused"), len(jobs)),
           nbytes=2 * T * C * 2)
    # the block's GEMMs: tcgen05 kernel vs cuBLAS (bf16 in, bf16 out)
    gemms = () if args.only == "norms" else ((("qkv", 3 * C, C), ("out_proj", C, C), ("ffn_up", F, C),
                                               ("ffn_down", C, F)))
    for name, n, k in gemms:
        a_ring = ring(lambda: torch.randn(T, k, device=device).bfloat16(), T * k * 2)
        wt = (torch.randn(n, k, device=device) / k ** 0.5).bfloat16()
        outs = [torch.empty(T, n, device=device, dtype=torch.bfloat16) for _ in range(2)]
        flops = 2.0 * T * n * k
        record(f"gemm_{name}_tcgen05", timed(lambda i: gemm.linear(a_ring[i], wt, out=outs[i % 2]), len(a_ring)),
               flops=flops)
        record(f"gemm_{name}_cublas", timed(lambda i: torch.matmul(a_ring[i], wt.t(), out=outs[i % 2]), len(a_ring)),
               flops=flops)
    # the block's GEMMs with the epilogues the DiT uses: bias + tanh-GELU (FFN up), bias + gate * (.) + residual
    # (out-projection, FFN down); the library rows are cuBLAS followed by the same elementwise math in torch
    fused = () if args.only == "norms" else (("ffn_up_gelu", F, C, "gelu"), ("out_proj_gated", C, C, "gated"),
                                             ("ffn_down_gated", C, F, "gated"))
    for name, n, k, kind in fused:
        a_ring = ring(lambda: torch.randn(T, k, device=device).bfloat16(), T * k * 2)
        wt = (torch.randn(n, k, device=device) / k ** 0.5).bfloat16()
        bias = (0.02 * torch.randn(n, device=device)).bfloat16()
        gate = 1.0 + 0.05 * torch.randn(n, device=device)
        resid = [torch.randn(T, n, device=device).bfloat16() for _ in range(2)]
        flops = 2.0 * T * n * k
        if kind == "gelu":
            outs = [torch.empty(T, n, device=device, dtype=torch.bfloat16) for _ in range(2)]
            ours = lambda i: gemm.linear_gelu(a_ring[i], wt, bias, out=outs[i % 2])
            library = lambda i: torch.nn.functional.gelu(torch.addmm(bias, a_ring[i], wt.t()), approximate="tanh")
        else:
            ours = lambda i: gemm.linear_gated_residual(a_ring[i], wt, bias, gate, resid[i % 2])
            library = lambda i: resid[i % 2].add_((torch.addmm(bias, a_ring[i], wt.t()).float() * gate).bfloat16())
        record(f"gemm_{name}_tcgen05", timed(ours, len(a_ring)), flops=flops)
        record(f"gemm_{name}_cublas_torch", timed(library, len(a_ring)), flops=flops)
    # raw-tier staging: one chunk's 60 K/V matrices device -> pinned host -> device on a side stream
    mats = [torch.randn(T, C, device=device).bfloat16() for _ in range(60 if args.only == "all" else 0)]
    hosts = [torch.empty(T, C, dtype=torch.bfloat16, pin_memory=True) for _ in range(len(mats))]
    side = torch.cuda.Stream(device)
    nbytes = 60 * T * C * 2
    for direction in ("d2h", "h2d") if mats else ():
        def copy_all(_):
            with torch.cuda.stream(side):
                for m, h in zip(mats, hosts):
                    (h.copy_(m, non_blocking=True) if direction == "d2h" else m.copy_(h, non_blocking=True))
            torch.cuda.current_stream(device).wait_stream(side)
        ms = timed(copy_all, 1)
        out[f"raw_tier_{direction}"] = {"ms": round(ms, 3), "GB_per_s": round(nbytes / ms / 1e6, 1),
                                        "bytes": nbytes, "engine": "copy engine (cudaMemcpyAsync), side stream"}
    _ext.check_status(device)
    text = json.dumps(out, indent=1)
    print(text)
    if args.out:
        args.out.write_text(text)


if __name__ == "__main__":
    main()
