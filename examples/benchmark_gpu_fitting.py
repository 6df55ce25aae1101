"""Fitter kernels against their library baselines on one GPU (the counterpart of reference
examples/benchmark_gpu_fitting.py): the batched Jacobi eigensolver vs cuSOLVER's batched eigh, the FP32-accurate
split-bf16 tcgen05 GEMM (promoted accumulation) vs cuBLAS SGEMM -- time and relative error against FP64 --, the
promoted bf16 Gram of bf16 sources, the fused square sums, exact fingerprints and the compensated Dot2 GEMM, and
one chunk plan of CausVid geometry (60 matrices [4680, 1536]).

    python examples/benchmark_gpu_fitting.py [--out result.json]

Every time is a CUDA-event mean over repetitions after warm-up.
"""

from __future__ import annotations

import argparse
import json
import sys
from pathlib import Path


def timed(fn, reps=10, warmup=3):
    import torch
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    start, stop = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    start.record()
    for _ in range(reps):
        fn()
    stop.record()
    torch.cuda.synchronize()
    return start.elapsed_time(stop) / reps


def rel_err(got, ref):
    return float((got.double() - ref).norm() / ref.norm())


def main(argv=None):
    ap = argparse.ArgumentParser(description=__doc__)
    ap.add_argument("--out", type=Path)
    ap.add_argument("--plan", action="store_true", help="also time one CausVid-shaped chunk plan")
    args = ap.parse_args(argv)
    sys.path.insert(0, str(Path(__file__).resolve().parents[1]))
    import torch
    from reelcache_b200 import exact_blas
    from reelcache_b200.ops.fitter import dot2_gemm, fingerprint_partials, jacobi_eigh, matmul_promoted, sq_partials
    from reelcache_b200.ops.gemm import matmul_tn

    torch.backends.cuda.matmul.allow_tf32 = False
    out = {"device": torch.cuda.get_device_name(0)}
    for n in (64, 128, 160):
        x = torch.randn(60, 2 * n, n, device="cuda")
        mats = x.transpose(1, 2) @ x
        _, _, info, sweeps = jacobi_eigh(mats)
        out[f"eigh_b60_n{n}"] = {"jacobi_ms": timed(lambda: jacobi_eigh(mats), 5),
                                 "cusolver_ms": timed(lambda: torch.linalg.eigh(mats), 5),
                                 "jacobi_max_sweeps": int(sweeps.max()), "converged": bool((info == 0).all())}
    for m, k, n in ((1536, 4680, 1536), (4680, 1536, 256), (4096, 14432, 4096), (160, 1536, 160)):
        a, b = torch.randn(m, k, device="cuda"), torch.randn(k, n, device="cuda")
        ref = a.double() @ b.double()
        out[f"mm_{m}x{k}x{n}"] = {"split_ms": timed(lambda: exact_blas.mm(a, b)), "sgemm_ms": timed(lambda: a @ b),
                                  "split_rel_err": rel_err(exact_blas.mm(a, b), ref),
                                  "sgemm_rel_err": rel_err(a @ b, ref)}
    x = torch.randn(4680, 1536, device="cuda").bfloat16()
    xt = x.t().contiguous()
    ref = xt.double() @ xt.double().t()
    out["gram_bf16_4680x1536"] = {"promoted_ms": timed(lambda: matmul_promoted(xt, xt)),
                                  "plain_ms": timed(lambda: matmul_tn(xt, xt)),
                                  "sgemm_ms": timed(lambda: xt.float() @ xt.float().t()),
                                  "promoted_rel_err": rel_err(matmul_promoted(xt, xt), ref),
                                  "plain_rel_err": rel_err(matmul_tn(xt, xt), ref),
                                  "sgemm_rel_err": rel_err(xt.float() @ xt.float().t(), ref)}
    out["sq_partials_4680x1536_bf16_us"] = 1000 * timed(lambda: sq_partials(x))
    out["fingerprint_4680x1536_bf16_us"] = 1000 * timed(lambda: fingerprint_partials(x, 0, 2147483629))
    xf, rows = torch.randn(4680, 1536, device="cuda"), torch.randn(256, 1536, device="cuda")
    out["dot2_4680x1536x256_ms"] = timed(lambda: dot2_gemm(xf, rows), 3)
    if args.plan:
        from reelcache_b200.rank_method import RankMethodConfig, plan_chunk
        from reelcache_b200.types import CodecSpec, MatrixKey, ModelIdentity, TensorContext, energy_targets
        model = ModelIdentity("causvid-shaped", "bench", 30, 1536, "BTHD", "bfloat16")
        matrices, contexts = {}, {}
        for layer in range(30):
            for target in ("K", "V"):
                key = MatrixKey(layer, target)
                base = torch.randn(4680, 48, device="cuda") @ torch.randn(48, 1536, device="cuda")
                matrices[key] = (base + 0.05 * torch.randn(4680, 1536, device="cuda")).bfloat16()
                contexts[key] = TensorContext(model, key, 0, 3, 30, 52, "pre_rope" if target == "K" else "none")
        cfg = RankMethodConfig(energy_targets("causvid"), CodecSpec("svd_hevc", 32))
        out["plan_chunk_causvid_ms"] = timed(lambda: plan_chunk(matrices, contexts, cfg, None, {}, {}), 2, 1)
    text = json.dumps(out, indent=1)
    print(text)
    if args.out:
        args.out.write_text(text)


if __name__ == "__main__":
    main()
