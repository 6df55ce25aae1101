"""The fused-kernel causal DiT matches its FP32 PyTorch reference on a small geometry."""

import pytest
import torch

pytestmark = pytest.mark.gpu


def _small():
    from reelcache_b200.models.causal_wan import CAUSVID
    return CAUSVID.scaled(layers=2, dim=256, heads=2, ffn=512, text_dim=128, text_len=16, latent_height=8,
                          latent_width=16)


def test_forward_matches_reference(cuda_device):
    from reelcache_b200.models.causal_wan import CausalWanDiT, KVCache
    from reelcache_b200.models.reference import reference_forward
    from reelcache_b200.ops import _ext

    cfg = _small()
    model = CausalWanDiT(cfg, cuda_device, seed=3)
    cache = KVCache(cfg, 4, cuda_device)
    context = torch.randn(cfg.text_len, cfg.text_dim, device=cuda_device)
    text_kv = model.encode_text(context)
    torch.manual_seed(0)
    hist_k, hist_v = None, None
    for chunk in range(2):
        latents = torch.randn(cfg.in_dim, cfg.frames_per_chunk, cfg.latent_height, cfg.latent_width,
                              device=cuda_device)
        captured = {}

        def capture(layer, k_pre, v):
            captured[layer] = (k_pre.clone(), v.clone())

        out = model.forward_chunk(latents, 500.0, chunk, cache, text_kv, capture=capture)
        torch.cuda.synchronize()
        _ext.check_status(cuda_device)
        ref, k_pres, vs, k_posts = reference_forward(model, latents, 500.0, chunk, hist_k, hist_v, context)
        err = (out - ref).norm() / ref.norm()
        assert err < 5e-2, float(err)
        for layer in range(cfg.layers):
            kp, v = captured[layer]
            assert (kp.float() - k_pres[layer]).norm() / k_pres[layer].norm() < 3e-2
            assert (v.float() - vs[layer]).norm() / vs[layer].norm() < 3e-2
        t = cfg.chunk_tokens
        hist_k = [torch.cat([hist_k[l], k_posts[l]]) if hist_k else k_posts[l] for l in range(cfg.layers)]
        hist_v = [torch.cat([hist_v[l], vs[l].reshape(t, cfg.heads, cfg.head_dim)]) if hist_v
                  else vs[l].reshape(t, cfg.heads, cfg.head_dim) for l in range(cfg.layers)]


def test_norm_kernels(cuda_device):
    from reelcache_b200.ops import norms

    x = torch.randn(100, 1536, device=cuda_device, dtype=torch.bfloat16)
    shift = torch.randn(1536, device=cuda_device)
    scale = torch.randn(1536, device=cuda_device) * 0.1
    y = norms.ln_modulate(x, shift=shift, scale=scale)
    ref = torch.nn.functional.layer_norm(x.float(), (1536,), eps=1e-6) * (1 + scale) + shift
    assert torch.allclose(y.float(), ref, atol=3e-2, rtol=2e-2)
    w = torch.rand(1536, device=cuda_device) + 0.5
    z = norms.rms_norm(x, w)
    ref = x.float() * torch.rsqrt(x.float().square().mean(-1, keepdim=True) + 1e-6) * w
    assert torch.allclose(z.float(), ref, atol=3e-2, rtol=2e-2)


def test_longcat_kernels_match_torch_path(cuda_device):
    """The LongCat-shaped DiT on the sm_100a ops agrees with the same weights on plain torch ops."""
    from reelcache_b200.models.longcat import ConditioningCacheEpoch, LongCatConfig, LongCatDiT
    cfg = LongCatConfig(layers=2, dim=512, heads=4, head_dim=128, ffn=1024, text_dim=256, text_len=16,
                        in_channels=16, latent_height=16, latent_width=24)
    fast = LongCatDiT(cfg, cuda_device, seed=3, use_kernels=True)
    slow = LongCatDiT(cfg, cuda_device, seed=3, use_kernels=False)
    g = torch.Generator(device="cpu").manual_seed(4)
    latents = torch.randn(16, 2, 16, 24, generator=g).to(cuda_device)
    context = torch.randn(16, 256, generator=g).to(cuda_device)
    cond = torch.randn(16, 1, 16, 24, generator=g).to(cuda_device)
    epoch = ConditioningCacheEpoch("e", 0, 0, 1)
    outs = []
    for model in (fast, slow):
        text = model.encode_text(context)
        cache = model.build_conditioning_cache(cond, epoch)
        outs.append(model.forward(latents, 0.7, text, first_frame=1, cache=cache))
    rel = float((outs[0] - outs[1]).norm() / outs[1].norm())
    assert rel < 0.05, rel


def test_bridge_with_the_dit_restores_a_fork_from_the_archive(cuda_device, tmp_path):
    """The serving bridge around the fused-kernel DiT: a session is created, paused (durable archive) and forked
    from an earlier checkpoint -- a restore overlapped with the first denoising step, the DiT waiting per layer
    (with its stream) on the restore -- and the fork's first chunk is generated."""
    import dataclasses
    from reelcache_b200.integrations.sglang import ReelCacheRuntimeConfig, create_sglang_backend, get_profile
    from reelcache_b200.models.causal_wan import CausalWanDiT
    cfg = _small()
    profile = dataclasses.replace(get_profile("causvid"), name="causvid-small", num_layers=cfg.layers,
                                  num_heads=cfg.heads, head_dim=cfg.head_dim, chunk_frames=cfg.frames_per_chunk,
                                  grid=(cfg.grid_h, cfg.grid_w))
    model = CausalWanDiT(cfg, cuda_device, seed=3)
    text_kv = model.encode_text(torch.randn(cfg.text_len, cfg.text_dim, device=cuda_device,
                                            generator=torch.Generator(device=cuda_device).manual_seed(1)))
    config = ReelCacheRuntimeConfig(store_root=str(tmp_path / "store"), fit_device="cuda", encode_workers=1,
                                    profile_fields=profile.to_dict())
    bridge = create_sglang_backend(config, (model, text_kv), cache_chunks=6)
    try:
        first = bridge.request("s", chunks=3, action="create", seed=1)
        assert first["generated"] == 3
        bridge.pause("s")
        fork = bridge.request("f", chunks=1, action="fork", source="s", checkpoint=2, seed=1)
        assert fork["route"] in ("archive", "raw_tier") and fork["start_chunk"] == 2
        assert fork["ttfc_ms"] is not None and fork["ttfc_ms"] > 0
    finally:
        bridge.shutdown()
