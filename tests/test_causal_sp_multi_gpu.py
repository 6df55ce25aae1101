"""The CausVid-shaped DiT under Ulysses sequence parallelism on 2 GPUs: a chunk generated with the SP forward (each
rank its token rows, all-to-alls around attention) equals the single-GPU forward -- the flow prediction, and
every rank's cache holds exactly its heads of the single-GPU cache -- and a second chunk attends to that history.
Skipped unless the box has at least two GPUs."""

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
    from reelcache_b200.models.causal_wan import CAUSVID, CausalWanDiT, KVCache, SPKVCache
    from reelcache_b200.models.sampler import ChunkGenerator

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    torch.cuda.set_device(rank)
    device = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60),
                            device_id=device)
    try:
        cfg = CAUSVID.scaled(layers=2)
        model = CausalWanDiT(cfg, device, seed=3)
        gen = torch.Generator(device=device).manual_seed(0)
        text_kv = model.encode_text(torch.randn((cfg.text_len, cfg.text_dim), generator=gen, device=device))
        full = KVCache(cfg, 3, device)
        shard = SPKVCache(cfg, 3, device, world=world, rank=rank)
        single = ChunkGenerator(model, full, text_kv, seed=5)
        sp = ChunkGenerator(model, shard, text_kv, seed=5, group=dist.group.WORLD)
        errors = []
        captured = {}
        for index in range(2):
            a = single.denoise(index)
            b = sp.denoise(index)
            errors.append(float((a - b).norm() / a.norm()))
            single.commit_clean(index, a)
            sp.commit_clean(index, a, capture=lambda layer, k, v: captured.setdefault(layer, k.clone()))
        hp = cfg.heads // world
        end = 2 * cfg.chunk_tokens
        cache_err = 0.0
        for layer in range(cfg.layers):
            for mine, ref in ((shard.k[layer], full.k[layer]), (shard.v[layer], full.v[layer])):
                want = ref[0, :end, rank * hp:(rank + 1) * hp].float()
                cache_err = max(cache_err, float((mine[0, :end].float() - want).norm() / want.norm()))
        errors.append(cache_err)
        errors.append(float(captured[0].shape[0]))  # this rank's rows only
        torch.cuda.synchronize()
        if rank == 0:
            with open(result_path, "w") as handle:
                handle.write(",".join(str(e) for e in errors))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2])
def test_ulysses_causal_forward_matches_single_gpu(tmp_path, world):
    if not torch.cuda.is_available() or torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    import torch.multiprocessing as mp
    from reelcache_b200.models.causal_wan import CAUSVID
    result = tmp_path / "errors.txt"
    mp.spawn(_worker, args=(world, _free_port(), str(result)), nprocs=world, join=True)
    errors = [float(v) for v in result.read_text().split(",")]
    assert errors[0] < 2e-2 and errors[1] < 2e-2, errors      # flow of chunk 0 and of chunk 1 (with history)
    assert errors[2] < 2e-2, errors                           # cache shards = the single-GPU cache's heads
    assert errors[3] == CAUSVID.chunk_tokens // world, errors
