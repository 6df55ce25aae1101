"""The chunk planner of CausVid geometry on one GPU: 60 matrices [4680, 1536] (bf16, decaying spectra), a fresh
chunk and a second chunk against the first one's rows (share / augment), planned matrix by matrix, in lockstep,
and in lockstep over CUDA stream lanes; plus the thin FP32-accurate products the planner issues (split-K promoted
GEMM) against cuBLAS SGEMM.

    python examples/benchmark_planner.py [--out result.json] [--gemm-only] [--shape "G B"]

Times are host wall clock around each plan (synchronized on both sides) and CUDA-event means for the GEMMs; the
plans of every mode are checked bitwise equal.
"""

from __future__ import annotations

import argparse
import json
import sys
import time
from pathlib import Path


def gemm_shapes(device, only: str | None = None) -> list[dict]:
    import torch
    from reelcache_b200.ops.fitter import SPLIT_A, SPLIT_A_BF16, SPLIT_B, SPLIT_B_BF16, matmul_promoted, split_operand

    def timed(fn, reps=20):
        for _ in range(3):
            fn()
        torch.cuda.synchronize()
        start, stop = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        start.record()
        for _ in range(reps):
            fn()
        stop.record()
        torch.cuda.synchronize()
        return start.elapsed_time(stop) / reps * 1e3

    rows = []
    for m, n, k, a_dtype, label in ((1536, 1536, 4680, torch.float32, "residual Gram (FP32)"),
                                    (1536, 1536, 4680, torch.bfloat16, "source Gram (bf16)"),
                                    (4680, 112, 1536, torch.bfloat16, "projection X Q^T"),
                                    (4680, 1536, 112, torch.float32, "reconstruction P Q"),
                                    (1536, 176, 1536, torch.float32, "subspace step G B"),
                                    (1536, 32, 1536, torch.float32, "sketch G Omega")):
        if only is not None and only not in label:
            continue
        a = torch.randn(m, k, device=device).to(a_dtype)
        b = torch.randn(k, n, device=device)
        parts_a, parts_b = (SPLIT_A_BF16, SPLIT_B_BF16) if a_dtype == torch.bfloat16 else (SPLIT_A, SPLIT_B)
        a_split, _ = split_operand(a, parts_a)
        b_split, _ = split_operand(b.t(), parts_b)
        gemm_us = timed(lambda: matmul_promoted(a_split, b_split))
        ref = a.double() @ b.double()
        err = float((matmul_promoted(a_split, b_split).double() - ref).abs().max() / ref.abs().max())
        old = torch.backends.cuda.matmul.allow_tf32
        torch.backends.cuda.matmul.allow_tf32 = False
        sgemm_us = timed(lambda: a.float() @ b)
        torch.backends.cuda.matmul.allow_tf32 = old
        rows.append({"product": label, "m": m, "n": n, "k": k, "promoted_gemm_us": round(gemm_us, 1),
                     "cublas_sgemm_us": round(sgemm_us, 1), "rel_err_vs_fp64": err})
    return rows


def chunk(model, index, bases, device, gen):
    import torch
    from reelcache_b200.types import MatrixKey, TensorContext
    matrices, contexts = {}, {}
    for layer in range(30):
        for target in "KV":
            key = MatrixKey(layer, target)
            if key not in bases:
                bases[key] = torch.linalg.qr(torch.randn(1536, 1536, device=device, generator=gen))[0]
            spectrum = torch.exp(-torch.arange(1536, device=device) / (40.0 if target == "K" else 80.0))
            x = (torch.randn(4680, 1536, device=device, generator=gen) * spectrum) @ bases[key].t()
            x = x + 0.02 * index * torch.randn(4680, 1536, device=device, generator=gen) * spectrum[200]
            matrices[key] = x.to(torch.bfloat16)
            contexts[key] = TensorContext(model, key, index * 4680, 3, 30, 52, "pre_rope" if target == "K" else "none")
    return matrices, contexts


def plans(device) -> dict:
    import torch
    import reelcache_b200.rank_method as rank_method
    from reelcache_b200 import deferred_reads
    from reelcache_b200.rank_method import RankMethodConfig, plan_chunk
    from reelcache_b200.types import ActiveBasisBinding, CodecSpec, ModelIdentity, energy_targets
    model = ModelIdentity("causvid-planner-bench", "synthetic", 30, 1536, "BTHD", "bfloat16")
    gen = torch.Generator(device=device).manual_seed(0)
    bases = {}
    first, first_ctx = chunk(model, 0, bases, device, gen)
    second, second_ctx = chunk(model, 1, bases, device, gen)
    results, out = {}, {}
    for label, batch, lanes in (("warm-up", 60, 8), ("sequential", 1, 1), ("lockstep", 60, 1),
                                ("lockstep + 8 lanes", 60, 8)):
        rank_method.PLANNER_STREAMS = lanes
        cfg = RankMethodConfig(energy_targets("causvid"), CodecSpec("svd_hevc", 32), solver="topk_rr",
                               batch_size=batch)
        torch.cuda.synchronize()
        rounds, clock = deferred_reads.STATS["rounds"], time.perf_counter()
        p0 = plan_chunk(first, first_ctx, cfg, None, {}, {})
        torch.cuda.synchronize()
        fresh = time.perf_counter() - clock
        fresh_rounds = deferred_reads.STATS["rounds"] - rounds
        bindings = {k: ActiveBasisBinding("manifest:" + "0" * 64, p.rows.shape[0], "1" * 64, p.rows.shape[0], "c0")
                    for k, p in p0.items()}
        rounds, clock = deferred_reads.STATS["rounds"], time.perf_counter()
        p1 = plan_chunk(second, second_ctx, cfg, None, bindings, {k: p.rows for k, p in p0.items()})
        torch.cuda.synchronize()
        reuse = time.perf_counter() - clock
        results[label] = (p0, p1)
        if label != "warm-up":
            decisions = {}
            for p in p1.values():
                decisions[p.decision] = decisions.get(p.decision, 0) + 1
            out[label] = {"fresh_chunk_ms": round(fresh * 1e3, 1), "fresh_rounds": fresh_rounds,
                          "second_chunk_ms": round(reuse * 1e3, 1),
                          "second_rounds": deferred_reads.STATS["rounds"] - rounds, "second_decisions": decisions}
    rank_method.PLANNER_STREAMS = 8
    same = all(torch.equal(results["sequential"][j][k].rows, results[label][j][k].rows)
               and torch.equal(results["sequential"][j][k].coefficients, results[label][j][k].coefficients)
               for label in ("lockstep", "lockstep + 8 lanes") for j in (0, 1) for k in results["sequential"][0])
    out["plans_bitwise_equal"] = same
    return out


def main(argv=None) -> None:
    sys.path.insert(0, str(Path(__file__).resolve().parents[1]))
    import torch
    parser = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    parser.add_argument("--out", default=None)
    parser.add_argument("--gemm-only", action="store_true")
    parser.add_argument("--shape", default=None, help="only the GEMM shapes whose label contains this text")
    args = parser.parse_args(argv)
    device = torch.device("cuda")
    result = {"gemms": gemm_shapes(device, args.shape)}
    if not args.gemm_only:
        result["plans"] = plans(device)
    text = json.dumps(result, indent=2)
    print(text)
    if args.out:
        Path(args.out).write_text(text)


if __name__ == "__main__":
    main()
