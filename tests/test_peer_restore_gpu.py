"""Sequence-parallel restore with the all-gather fused into the restore GEMM (peer-memory A operands),
on 2 GPUs: every rank restores its head columns of the whole history from tiles staged on both ranks,
and matches a single-GPU restore of the full matrices (sliced). Skipped with fewer than 2 GPUs."""

import os
import socket
import traceback

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu


def _port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, errors):
    import datetime
    import torch.distributed as dist
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    try:
        torch.cuda.set_device(rank)
        device = torch.device("cuda", rank)
        dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=120),
                                device_id=device)
        from reelcache_b200 import restore_kernels as rk
        from reelcache_b200.ops.peer_restore import PeerRestoreDomain, column_basis, plan_tiles
        from reelcache_b200.restore_kernels import restore_rope_item

        chunks, frames, h, w, heads, head_dim, rank_k = 4, 3, 30, 52, 12, 128, 64
        tokens, channels = frames * h * w, heads * head_dim
        local_heads = heads // world
        cols = slice(rank * local_heads * head_dim, (rank + 1) * local_heads * head_dim)
        rng = np.random.default_rng(0)  # identical data on every rank
        table = rk.RopeTable.wan(head_dim, 64, device=device)
        tiles_data = []
        for c in range(chunks):
            for target in ("K", "V"):
                pixels = rng.integers(0, 256, (tokens, rank_k), dtype=np.uint8)
                scale = rng.uniform(0.001, 0.05, rank_k).astype(np.float32)
                offset = rng.uniform(-3, 3, rank_k).astype(np.float32)
                basis = (rng.standard_normal((rank_k, channels)) / 40).astype(np.float16)
                tiles_data.append((c, target, pixels, scale, offset, basis))
        shapes = [(i % world, tokens, rank_k) for i in range(len(tiles_data))]
        tiles = plan_tiles(shapes)
        domain = PeerRestoreDomain(None, device, 2 * sum(t.nbytes for t in tiles) // world + (1 << 20))
        sources = {i: torch.from_numpy(d[2]).to(device) for i, d in enumerate(tiles_data) if tiles[i].owner == rank}
        domain.stage(tiles, sources)

        cache_k = torch.zeros((1, chunks * tokens, local_heads, head_dim), dtype=torch.bfloat16, device=device)
        cache_v = torch.zeros_like(cache_k)
        keep, jobs = [], []
        for i, (c, target, pixels, scale, offset, basis) in enumerate(tiles_data):
            dest = (cache_k if target == "K" else cache_v)[0, c * tokens:(c + 1) * tokens]
            b = column_basis(torch.from_numpy(basis).to(device), rank_k, cols)
            rope = restore_rope_item(rk.RopePositions(table, (3 * c, 0, 0)), (frames, h, w), device, None, keep) \
                if target == "K" else None
            jobs.append({"grid": (frames, h, w), "basis": b, "scale": scale, "offset": offset, "rope": rope,
                         "dest": (dest.data_ptr(), (dest.stride(0), dest.stride(1), dest.stride(2)), dest.dtype,
                                  local_heads * head_dim, head_dim)})
        domain.restore(tiles, jobs)
        torch.cuda.synchronize()
        assert domain.stats["remote_a_bytes"] > 0 and domain.stats["local_a_bytes"] > 0

        # single-GPU reference: the full matrices restored locally, this rank's columns compared
        full_k = torch.zeros((1, chunks * tokens, heads, head_dim), dtype=torch.bfloat16, device=device)
        full_v = torch.zeros_like(full_k)
        ref_jobs = []
        for c, target, pixels, scale, offset, basis in tiles_data:
            view = rk.NativeView(full_k if target == "K" else full_v, "BTHD", c * tokens)
            ref_jobs.append(rk.ReconstructionJob(
                rk.CoefficientSource(torch.from_numpy(pixels).to(device), scale, offset), view, (frames, h, w),
                torch.from_numpy(basis).to(device), rope=rk.RopePositions(table, (3 * c, 0, 0)) if target == "K" else None))
        rk.reconstruct(ref_jobs, backend="fused", precision="fp16").synchronize()
        for got, full in ((cache_k, full_k), (cache_v, full_v)):
            expect = full[:, :, rank * local_heads:(rank + 1) * local_heads].float()
            err = (got.float() - expect).abs().max().item()
            scale_ref = expect.abs().max().item()
            assert err <= 2e-2 * scale_ref, (err, scale_ref)
        dist.barrier()
        del domain
    except BaseException:  # noqa: BLE001
        errors.put((rank, traceback.format_exc()))
    finally:
        if torch.distributed.is_initialized():
            torch.distributed.destroy_process_group()


def test_peer_memory_restore_two_gpus():
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    ctx = mp.get_context("spawn")
    errors = ctx.Queue()
    port = _port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, errors)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(300)
        if p.is_alive():
            p.kill()
            raise AssertionError("a rank did not finish")
    failures = []
    while not errors.empty():
        failures.append(errors.get())
    assert not failures, "\n".join(f"rank {r}:\n{tb}" for r, tb in failures)
