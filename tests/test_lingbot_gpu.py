"""LingBot archive on a B200: the compressed representation restored by the fused sm_100a restore kernels into
the stand-in world model's shared window cache (LingBot's real frame size, 30 x 52 latent tokens, 3 frames per
chunk), layer-overlapped with the next chunk's forward and bitwise equal to the synchronous restore."""

import pytest
import torch

from reelcache_b200.integrations.lingbot import LINGBOT_WORLD_FAST, LingBotArchive, StallEvents, StandInWorldModel

pytestmark = pytest.mark.gpu

# The stand-in's K / V have no low-rank structure, so the representation keeps exactly its energy targets
# (K 98 %, V 95 %): relative error sqrt(1 - target), plus 8-bit coefficient quantization.
K_BOUND = (1 - 0.98) ** 0.5 + 0.03
V_BOUND = (1 - 0.95) ** 0.5 + 0.03
GEOMETRY = LINGBOT_WORLD_FAST.scaled(layers=2, heads=2, window_latents=9)


@pytest.fixture(autouse=True)
def _cuda():
    if not torch.cuda.is_available():
        pytest.skip("needs a GPU")


def test_fused_restore_overlapped_equals_synchronous(tmp_path):
    dev = torch.device("cuda", 0)
    g = torch.Generator().manual_seed(0)
    xs = [torch.randn(GEOMETRY.chunk_tokens, GEOMETRY.channels, generator=g) for _ in range(4)]
    live = StandInWorldModel(GEOMETRY, device=dev)
    archive = LingBotArchive(tmp_path / "store", GEOMETRY, representation="svd_hevc", device=dev)
    archive.ensure_session("s")
    parent = None
    for chunk in range(3):
        _, (k, v) = live.generate(chunk, xs[chunk])
        archive.commit("s", f"s/{chunk}", parent, chunk, k, v)
        parent = f"s/{chunk}"
    assert archive.stats()["restorer"] == "LineageRestorer"
    sync_model = StandInWorldModel(GEOMETRY, device=dev)
    record = archive.restore(parent, sync_model)
    assert record["chunks"] == [1, 2]  # the window before chunk 3 (3 chunks of 3 latent frames)
    for c in record["chunks"]:
        start, end = sync_model.cache.place(c)
        for layer in range(GEOMETRY.layers):
            for ours, theirs, bound in ((sync_model.cache.k[layer], live.cache.k[layer], K_BOUND),
                                        (sync_model.cache.v[layer], live.cache.v[layer], V_BOUND)):
                a, b = ours[0, start:end].float(), theirs[0, start:end].float()
                assert float((a - b).norm() / b.norm()) < bound
    sync_out, _ = sync_model.generate(3, xs[3], capture=False)
    over_model = StandInWorldModel(GEOMETRY, device=dev)
    anchor = torch.cuda.Event(enable_timing=True)
    anchor.record()
    recorder = StallEvents(dev, anchor)
    session = archive.restore(parent, over_model, overlapped=True, recorder=recorder)
    over_out, _ = over_model.generate(3, xs[3], capture=False)
    torch.cuda.synchronize()
    assert session.state == "joined"
    assert torch.equal(over_out, sync_out)
    summary = session.gpu_summary()
    assert summary["layers_waited"] == GEOMETRY.layers and len(summary["stall_ms"]) == GEOMETRY.layers
    assert "restore_window_ms" in summary
    archive.close()
