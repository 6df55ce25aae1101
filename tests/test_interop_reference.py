"""On-disk interoperability with the reference implementation (installed under ``baseline/_ref``): each side
reads the other's store -- lineage heads, nodes, cache epochs, matrix records, packets and basis versions --
and continues it. RAW history is bit for bit; SVD history (FP32 coefficients on an FP16 basis prefix) decodes to
the same values as the writer's own read. Node packs of HEVC streams need an HEVC codec neither machine has, so
they are not exercised here."""

import os
import sys
import tempfile

import pytest
import torch

REF = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "baseline", "_ref")


@pytest.fixture(scope="module")
def ref():
    if not os.path.isdir(os.path.join(REF, "reelcache")):
        pytest.skip("the reference is not installed under baseline/_ref")
    sys.path.insert(0, REF)
    try:
        import reelcache.manager
        import reelcache.predictor_registry
        import reelcache.rank_method
        import reelcache.types
    except Exception as error:  # noqa: BLE001 - an unusable install skips the interop checks
        pytest.skip(f"the reference does not import: {error}")
    finally:
        sys.path.remove(REF)
    return reelcache


class Side:
    """One implementation's runtime, types and method classes."""

    def __init__(self, package):
        import importlib
        self.types = importlib.import_module(f"{package}.types")
        self.KVRuntime = importlib.import_module(f"{package}.manager").KVRuntime
        self.rank_method = importlib.import_module(f"{package}.rank_method")
        self.registry = importlib.import_module(f"{package}.predictor_registry").RankPredictorRegistry
        self.ours = package == "reelcache_b200"

    def runtime(self, root):
        return self.KVRuntime(root, self.types.ModelIdentity("tiny", "fp", 2, 128, "BTHD", "bfloat16"))

    def chunk(self, runtime, index, seed=0):
        t = self.types
        g = torch.Generator().manual_seed(seed * 100 + index)
        basis = torch.linalg.qr(torch.randn(128, 8, generator=torch.Generator().manual_seed(seed)))[0].t()
        matrices, contexts = {}, {}
        for layer in range(2):
            for target in "KV":
                key = t.MatrixKey(layer, target)
                x = torch.randn(32, 8, generator=g) @ basis + 1e-3 * torch.randn(32, 128, generator=g)
                matrices[key] = x.to(torch.bfloat16)
                contexts[key] = t.TensorContext(runtime.model, key, 32 * index, 2, 4, 4,
                                                "pre_rope" if target == "K" else "none")
        return matrices, contexts

    def commit(self, runtime, index, representation, branch="a"):
        matrices, contexts = self.chunk(runtime, index)
        if representation == "raw":
            runtime.commit_raw_node(branch, f"c{index}", matrices, contexts)
        else:
            t = self.types
            method = self.rank_method.RankMethodConfig(t.energy_targets("causvid"), t.CodecSpec("svd", 32))
            extra = {}
            if self.ours:
                from reelcache_b200.lineage_commit import ArchiveOptions
                extra["options"] = ArchiveOptions(packed=False)  # per-matrix packets, the layout both read
            runtime.commit_node(branch, f"c{index}", matrices, contexts, method=method,
                                registry=self.registry("interop"), **extra)
        return matrices

    def history(self, runtime, head):
        out = {}
        for layer in range(2):
            for target in "KV":
                value = runtime.acquire_node_history(head, self.types.MatrixKey(layer, target))
                if hasattr(value, "release"):
                    tensor = value.tensor.clone()
                    value.release()
                    value = tensor
                out[(layer, target)] = value.to(torch.bfloat16)
        return out


def _sides(ref):
    return Side("reelcache"), Side("reelcache_b200")


@pytest.mark.parametrize("representation", ["raw", "svd"])
@pytest.mark.parametrize("writer_first", ["reference", "ours"])
def test_each_side_reads_and_continues_the_other(ref, representation, writer_first):
    theirs, ours = _sides(ref)
    first, second = (theirs, ours) if writer_first == "reference" else (ours, theirs)
    root = tempfile.mkdtemp(prefix="reelcache-interop-")
    a = first.runtime(root)
    a.create_lineage("a")
    sources = [first.commit(a, 0, representation), first.commit(a, 1, representation)]
    head = a.lineage_head("a")
    expected = first.history(a, head)
    b = second.runtime(root)
    assert b.lineage_head("a") == head
    got = second.history(b, head)
    for key in expected:
        assert torch.equal(got[key], expected[key])
    if representation == "raw":
        for key in expected:
            source = torch.cat([sources[0][first.types.MatrixKey(*key)], sources[1][first.types.MatrixKey(*key)]])
            assert torch.equal(got[key], source)
    # the second implementation continues the lineage, and forks it; the first reads both heads
    second.commit(b, 2, representation)
    b.fork_lineage(head, "f")
    second.commit(b, 2, representation, branch="f")
    a2 = first.runtime(root)
    for branch in ("a", "f"):
        tip = b.lineage_head(branch)
        assert a2.lineage_head(branch) == tip
        left, right = first.history(a2, tip), second.history(b, tip)
        for key in left:
            assert torch.equal(left[key], right[key])
            assert left[key].shape[0] == 96


@pytest.mark.parametrize("kind", ["raw", "svd"])
@pytest.mark.parametrize("writer_first", ["reference", "ours"])
def test_manager_snapshots_cross_over(ref, kind, writer_first):
    """The manager API's branches and snapshots: a snapshot one side takes is restored into a branch by the other,
    whose history reads back the writer's values."""
    theirs, ours = _sides(ref)
    first, second = (theirs, ours) if writer_first == "reference" else (ours, theirs)
    root = tempfile.mkdtemp(prefix="reelcache-interop-manager-")
    a = first.runtime(root)
    a.create_branch("main")
    for index in range(2):
        matrices, contexts = first.chunk(a, index)
        spec = first.types.CodecSpec("raw") if kind == "raw" else first.types.CodecSpec("svd", 8)
        a.seal_chunk("main", index, matrices, contexts, spec)
    metadata = {"origin": writer_first, "clean_boundary": {"chunk_id": 1, "token_end": 64},
                "conditioning": "prompt", "execution": {},
                "rng": {"seed": 1}, "latent": {"frames": 4}, "vae": "wan"}
    snapshot = a.snapshot("main", metadata=metadata, tensors={"latents": torch.arange(6.0)})
    key = first.types.MatrixKey(1, "V")

    def read(runtime, side, branch):
        lease = runtime.acquire_history(branch, side.types.MatrixKey(1, "V"))
        value = lease.tensor.clone() if hasattr(lease, "tensor") else lease
        if hasattr(lease, "release"):
            lease.release()
        return value.float()

    expected = read(a, first, "main")
    b = second.runtime(root)
    restored = b.restore(snapshot, "copy")
    assert dict(restored.metadata)["origin"] == writer_first
    assert torch.equal(restored.tensors["latents"].cpu(), torch.arange(6.0))
    got = read(b, second, "copy")
    assert got.shape == expected.shape == (64, 128)
    assert torch.equal(got.to(torch.bfloat16), expected.to(torch.bfloat16))
    assert key.layer == 1
