"""The RAW, software and factor-pack lineage restorers on a B200 (fused restore kernels) against the same
restorers on the host."""

import pytest
import torch

from reelcache_b200 import restore_kernels as rk
from reelcache_b200.archive_restore import RawLineageRestorer, SoftwareLineageRestorer
from reelcache_b200.factor_packs import FactorLineageRestorer

from .lineage_support import FRAMES, MODEL, TOKENS, relative_error
from .test_restorers import HEADS, _commit

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("kind", ["raw", "svd", "svd_hevc"])
def test_restorers_on_gpu_match_host(tmp_path, kind):
    if not torch.cuda.is_available():
        pytest.skip("needs a GPU")
    from reelcache_b200.ops import _ext
    _ext.ext()
    runtime, node, _ = _commit(tmp_path, kind)
    cls = {"raw": RawLineageRestorer, "svd": FactorLineageRestorer, "svd_hevc": SoftwareLineageRestorer}[kind]
    head_dim = MODEL.channels_for("K") // HEADS
    out = {}
    for device in ("cpu", "cuda"):
        caches = {(l, t): torch.zeros((1, 3 * TOKENS, HEADS, head_dim), device=device, dtype=torch.float32)
                  for l in range(MODEL.layers) for t in "KV"}
        table = rk.RopeTable.wan(head_dim, 64, device=device)
        result = cls(runtime, device).restore(node, lambda l, t: caches[(l, t)],
                                              lambda piece: (table, (FRAMES * (piece.token_start // TOKENS), 0, 0)))
        for layer in range(MODEL.layers):
            result.wait(layer)
        result.join()
        torch.cuda.synchronize()
        out[device] = {k: v.cpu() for k, v in caches.items()}
    for key in out["cpu"]:
        assert relative_error(out["cuda"][key], out["cpu"][key]) < 1e-5, key


def test_fused_restore_batched_matches_per_layer(tmp_path):
    """A non-overlapped restore packs consecutive layers into shared launches; the caches it writes are
    bit-identical to the per-layer (overlapped) launches and it issues fewer restore launches."""
    if not torch.cuda.is_available():
        pytest.skip("needs a GPU")
    from reelcache_b200.archive_restore import LineageRestorer
    runtime, node, _ = _commit(tmp_path, "svd_hevc")
    head_dim = MODEL.channels_for("K") // HEADS
    table = rk.RopeTable.wan(head_dim, 64, device="cuda")
    out, launches = {}, {}
    for overlapped in (True, False):
        caches = {(l, t): torch.zeros((1, 3 * TOKENS, HEADS, head_dim), device="cuda", dtype=torch.bfloat16)
                  for l in range(MODEL.layers) for t in "KV"}
        restorer = LineageRestorer(runtime, "cuda")
        result = restorer.restore(node, lambda l, t: caches[(l, t)],
                                  lambda piece: (table, (FRAMES * (piece.token_start // TOKENS), 0, 0)),
                                  overlapped=overlapped)
        for layer in range(MODEL.layers):
            result.wait(layer)
        result.join()
        torch.cuda.synchronize()
        out[overlapped] = {k: v.cpu() for k, v in caches.items()}
        program = result.program
        launches[overlapped] = program.batch_launch_count(aux=False) if not overlapped else \
            sum(len(b) for b in program.blobs.values())
    for key in out[True]:
        assert torch.equal(out[True][key], out[False][key]), key
        assert out[True][key].abs().amax() > 0
    assert launches[False] < launches[True]
