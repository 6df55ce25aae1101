"""LongCat conditioning-cache restore on the fused sm_100a kernels: each context-parallel rank gathers only its
rows of the segment's coefficient tiles (row runs in the unpack kernel) and gets the values the host decode of
the same node gives for those rows."""

import pytest
import torch

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("cp", [1, 2, 4])
def test_fused_segment_restore_matches_host_decode(tmp_path, cp):
    from reelcache_b200.archive_restore import LineageRestorer
    from reelcache_b200.lineage import LineageRuntime
    from reelcache_b200.models.longcat import (ConditioningCacheEpoch, LongCatConfig, LongCatDiT,
                                               ReelCacheConditioningCacheBackend)
    from reelcache_b200.parallel.context_parallel import RowShard
    from reelcache_b200.rank_method import RankMethodConfig
    from reelcache_b200.store import ObjectStore
    from reelcache_b200.types import CodecSpec, ModelIdentity, energy_targets
    cfg = LongCatConfig(layers=2, dim=256, heads=2, head_dim=128, ffn=512, text_dim=64, text_len=8, in_channels=4,
                        latent_height=8, latent_width=12)
    model = LongCatDiT(cfg, "cuda", seed=1, use_kernels=False, max_frames=8)
    g = torch.Generator(device="cuda").manual_seed(3)
    cond = torch.randn(cfg.in_channels, 3, cfg.latent_height, cfg.latent_width, generator=g, device="cuda")
    store = ObjectStore(tmp_path / "store")
    runtime = LineageRuntime(store, ModelIdentity("longcat-small", "seed1", cfg.layers, cfg.dim, "BTHD", "bfloat16"))
    runtime.create_lineage("s")
    method = RankMethodConfig(energy_targets("longcat_720p"), CodecSpec("svd_hevc", 32))
    writer = ReelCacheConditioningCacheBackend(runtime, "s", method, head_dim=cfg.head_dim, grid=cfg.grid,
                                               device="cuda")
    epoch = ConditioningCacheEpoch("seg-0", 0, 0, 3)
    node = writer.on_cache_built(model.build_conditioning_cache(cond, epoch))
    restorer = LineageRestorer(runtime, torch.device("cuda"))
    for rank in range(cp):
        shard = None if cp == 1 else RowShard(rank, cp, 3, *cfg.grid)
        host = ReelCacheConditioningCacheBackend(runtime, "s", method, head_dim=cfg.head_dim, grid=cfg.grid,
                                                 device="cuda", cp_shard=shard, restorer=None)
        fused = ReelCacheConditioningCacheBackend(runtime, "s", method, head_dim=cfg.head_dim, grid=cfg.grid,
                                                  device="cuda", cp_shard=shard, restorer=restorer)
        want = host.restore(epoch, node)
        got = fused.restore(epoch, node)
        torch.cuda.synchronize()
        assert fused.stats.get("fused") == 1 and got.tokens == want.tokens
        for a, b in zip(want.k + want.v, got.k + got.v):
            assert a.shape == b.shape
            err = float((a.float() - b.float()).abs().max())
            assert err <= 2e-2 * float(a.float().abs().max()) + 1e-3, err
    store.close()


@pytest.mark.parametrize("head_dim", [64, 128])
def test_head_norm_rope_matches_fp32_reference(head_dim):
    from reelcache_b200.ops.norms import head_norm_rope
    g = torch.Generator(device="cuda").manual_seed(1)
    tokens, heads = 300, 6
    base = torch.randn(tokens, 3, heads, head_dim, generator=g, device="cuda").to(torch.bfloat16)
    x = base[:, 1]                                   # a strided view, as a fused qkv's K
    w = torch.rand(head_dim, generator=g, device="cuda") + 0.5
    angle = torch.rand(tokens, head_dim // 2, generator=g, device="cuda") * 6.28
    cos, sin = angle.cos(), angle.sin()
    xf = x.float()
    normed = xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + 1e-6) * w
    e, o = normed[..., 0::2], normed[..., 1::2]
    ref = torch.stack((e * cos[:, None] - o * sin[:, None], e * sin[:, None] + o * cos[:, None]), -1).flatten(-2)
    got = head_norm_rope(x, w, cos, sin, eps=1e-6).float()
    assert float((got - ref).abs().max()) <= 1e-2 * float(ref.abs().max())
    only_norm = head_norm_rope(x, w, eps=1e-6).float()
    assert float((only_norm - normed).abs().max()) <= 1e-2 * float(normed.abs().max())
    inplace = x.clone()
    head_norm_rope(inplace, None, cos, sin, out=inplace)
    xe, xo = xf[..., 0::2], xf[..., 1::2]
    rot = torch.stack((xe * cos[:, None] - xo * sin[:, None], xe * sin[:, None] + xo * cos[:, None]), -1).flatten(-2)
    assert float((inplace.float() - rot).abs().max()) <= 1e-2 * float(rot.abs().max())
