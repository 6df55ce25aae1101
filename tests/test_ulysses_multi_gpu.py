"""Fused Ulysses on 2+ GPUs (NVLink peer memory): the LongCat-shaped DiT's context-parallel forward with the
all-to-alls fused into the projection GEMMs equals the same forward with NCCL all-to-alls, with and without a
conditioning cache. Skipped unless the box has at least two GPUs."""

import os
import socket

import pytest
import torch

pytestmark = pytest.mark.gpu


def _free_port() -> int:
    with socket.socket() as sock:
        sock.bind(("127.0.0.1", 0))
        return sock.getsockname()[1]


def _worker(rank, world, port, result_path):
    import datetime
    import torch.distributed as dist
    from reelcache_b200.models.longcat import ConditioningCacheEpoch, LongCatConfig, LongCatDiT
    from reelcache_b200.parallel.ulysses_fused import FusedUlysses

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    torch.cuda.set_device(rank)
    device = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60),
                            device_id=device)
    try:
        heads = 2 * world
        cfg = LongCatConfig(layers=2, dim=heads * 128, heads=heads, head_dim=128, ffn=1024, text_dim=256, text_len=16,
                            latent_height=16, latent_width=32, frames_per_chunk=2)
        model = LongCatDiT(cfg, device, seed=3)
        gen = torch.Generator(device=device).manual_seed(0)
        latents = torch.randn((cfg.in_channels, 2, cfg.latent_height, cfg.latent_width), generator=gen, device=device)
        cond = torch.randn((cfg.in_channels, 2, cfg.latent_height, cfg.latent_width), generator=gen, device=device)
        text = model.encode_text(torch.randn((cfg.text_len, cfg.text_dim), generator=gen, device=device))
        epoch = ConditioningCacheEpoch("e0", 0, 0, 2)
        cache = model.build_conditioning_cache(cond, epoch, cp_group=dist.group.WORLD)
        tokens = 2 * cfg.tokens_per_frame
        errors = []
        for use_cache in (False, True):
            c = cache if use_cache else None
            ref = model.forward(latents, 0.5, text, first_frame=2, cache=c, cp_group=dist.group.WORLD)
            fused = FusedUlysses(None, device, heads=cfg.heads, head_dim=cfg.head_dim, rows=tokens,
                                 cache_rows=tokens if use_cache else 0)
            got = model.forward(latents, 0.5, text, first_frame=2, cache=c, cp_group=dist.group.WORLD, ulysses=fused)
            torch.cuda.synchronize()
            fused.check()
            errors.append(float((got - ref).norm() / ref.norm()))
            fused.close()
        # fused Gram reduce-scatter: every owner's Gram equals the FP64 Gram of all ranks' shards
        from reelcache_b200.parallel.gram_rs import GramReduceScatter
        channels, matrices = 256, 3
        owners = [b % world for b in range(matrices)]
        grs = GramReduceScatter(None, device, channels=channels, max_slots=matrices)
        gram_err = 0.0
        # several calls back to back with different inputs: a call must not overwrite partials an owner is
        # still summing from the previous call
        for call in range(4):
            gen_r = torch.Generator(device=device).manual_seed(10 + 97 * call + rank)
            shards = [torch.randn(96 + 32 * call, channels, device=device, generator=gen_r).bfloat16()
                      for _ in range(matrices)]
            grams = grs.run(torch.cat([x.t() for x in shards]).contiguous(), owners)
            gathered = [[torch.empty_like(x) for _ in range(world)] for x in shards]
            for b in range(matrices):
                dist.all_gather(gathered[b], shards[b])
            for b, gram in grams.items():
                full = torch.cat(gathered[b]).double()
                ref = full.t() @ full
                gram_err = max(gram_err, float((gram.double() - ref).norm() / ref.norm()))
        torch.cuda.synchronize()
        grs.check()
        errors.append(gram_err)
        grs.close()
        # the in-switch (NVLS multimem.ld_reduce) variant, where the GPUs share an NVLink multicast object
        nvls = GramReduceScatter(None, device, channels=channels, max_slots=matrices, nvls="auto")
        nvls_err = -1.0
        if nvls.nvls:
            nvls_err = 0.0
            for call in range(4):
                gen_r = torch.Generator(device=device).manual_seed(20 + 89 * call + rank)
                shards = [torch.randn(64 + 32 * call, channels, device=device, generator=gen_r).bfloat16()
                          for _ in range(matrices)]
                grams = nvls.run(torch.cat([x.t() for x in shards]).contiguous(), owners)
                gathered = [[torch.empty_like(x) for _ in range(world)] for x in shards]
                for b in range(matrices):
                    dist.all_gather(gathered[b], shards[b])
                for b, gram in grams.items():
                    full = torch.cat(gathered[b]).double()
                    ref = full.t() @ full
                    nvls_err = max(nvls_err, float((gram.double() - ref).norm() / ref.norm()))
            torch.cuda.synchronize()
            nvls.check()
        errors.append(nvls_err)
        nvls.close()
        if rank == 0:
            with open(result_path, "w") as handle:
                handle.write(",".join(str(e) for e in errors))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2])
def test_fused_ulysses_forward_matches_nccl(tmp_path, world):
    if not torch.cuda.is_available() or torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    import torch.multiprocessing as mp
    result = tmp_path / "errors.txt"
    mp.spawn(_worker, args=(world, _free_port(), str(result)), nprocs=world, join=True)
    errors = [float(v) for v in result.read_text().split(",")]
    assert all(e < 2e-2 for e in errors[:2]), errors
    assert errors[2] < 1e-6, errors
    assert errors[3] < 1e-6, errors  # -1: no NVLink multicast object on these GPUs (the NVLS variant did not run)
    try:
        import torch.distributed._symmetric_memory as symm
        multicast = bool(symm._SymmetricMemory.has_multicast_support(symm.DeviceType.CUDA, 0))
    except Exception:  # noqa: BLE001 - a torch without the query leaves the NVLS run optional
        multicast = False
    if multicast:
        assert errors[3] >= 0, "the GPUs support multicast but the in-switch (NVLS) variant did not run"
