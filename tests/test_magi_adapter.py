"""MAGI Ulysses clean-history adapter on CPU with Gloo ranks (world size 2): each rank captures the normalized
pre-RoPE K and the V of its token rows through the attention's get_k / get_v, seal_chunk gathers them into one
lineage node on the owner and broadcasts the head, and restore_history hands every rank exactly its KV-head
columns of the whole history, rotated at global positions (RAW exact, svd_hevc within its energy target). A rank
whose capture is incomplete makes the seal fail on every rank, typed, before anything is committed."""

import os
import socket
import traceback

import pytest
import torch
import torch.multiprocessing as mp

from reelcache_b200.adapters import MagiGeometry
from reelcache_b200.errors import ConfigurationError

GEOMETRY = MagiGeometry(layers=2, kv_heads=4, head_dim=16, frames=2, height=4, width=4, world_size=2)
HIDDEN = 48


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _entry(rank, world, port, fn_name, args, errors):
    import datetime
    import torch.distributed as dist
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    try:
        dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
        globals()[fn_name](rank, world, *args)
    except BaseException:  # noqa: BLE001
        errors.put((rank, traceback.format_exc()))
    finally:
        if dist.is_initialized():
            dist.destroy_process_group()


def _run(fn_name, *args, world=2):
    ctx = mp.get_context("spawn")
    errors = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_entry, args=(r, world, port, fn_name, args, errors)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(180)
        if p.is_alive():
            p.kill()
            raise AssertionError("a rank hung")
    failures = []
    while not errors.empty():
        failures.append(errors.get())
    assert not failures, "\n".join(f"rank {r}:\n{tb}" for r, tb in failures)


def _rotary(values, first):
    """1-D rotary embedding of interleaved channel pairs at global token positions first, first + 1, ..."""
    tokens, _, dim = values.shape
    pos = torch.arange(first, first + tokens, dtype=torch.float64)
    inv = 1.0 / 10000.0 ** (torch.arange(0, dim, 2, dtype=torch.float64) / dim)
    angle = torch.outer(pos, inv)[:, None, :]
    x = values.double().reshape(tokens, values.shape[1], dim // 2, 2)
    even, odd = x[..., 0], x[..., 1]
    out = torch.stack((even * angle.cos() - odd * angle.sin(), even * angle.sin() + odd * angle.cos()), -1)
    return out.reshape(values.shape).to(values.dtype)


class _Norm(torch.nn.Module):
    def forward(self, x):
        return x * torch.rsqrt(x.pow(2).mean(-1, keepdim=True) + 1e-6)


class _Attention(torch.nn.Module):
    def __init__(self):
        super().__init__()
        channels = GEOMETRY.channels
        self.k_proj = torch.nn.Linear(HIDDEN, channels)
        self.v_proj = torch.nn.Linear(HIDDEN, channels)
        self.k_norm = _Norm()

    def get_k(self, mixed, first):
        k = self.k_norm(self.k_proj(mixed))
        return _rotary(k.reshape(-1, GEOMETRY.kv_heads, GEOMETRY.head_dim), first)

    def get_v(self, mixed):
        return self.v_proj(mixed)


class _Block(torch.nn.Module):
    def __init__(self):
        super().__init__()
        self.attention = _Attention()


class _Model(torch.nn.Module):
    def __init__(self):
        super().__init__()
        torch.manual_seed(0)
        self.layers = torch.nn.ModuleList(_Block() for _ in range(GEOMETRY.layers))


def _chunk_input(chunk):
    return torch.randn(GEOMETRY.tokens, HIDDEN, generator=torch.Generator().manual_seed(100 + chunk))


def _adapter(rank, store_dir, representation):
    from reelcache_b200.adapters import MagiAdapter
    from reelcache_b200.lineage import LineageRuntime
    from reelcache_b200.parallel.distributed import DistributedOwner
    from reelcache_b200.store import ObjectStore
    transport = DistributedOwner(device="cpu")
    runtime = None
    if transport.is_owner:
        runtime = LineageRuntime(ObjectStore(store_dir), GEOMETRY.identity())
        runtime.create_lineage("main")
    model = _Model()
    adapter = MagiAdapter(model, geometry=GEOMETRY, transport=transport, branch_id="main", rotary=_rotary,
                          runtime=runtime, representation=representation).attach()
    return model, adapter, runtime


def _forward(model, adapter, chunk, rank, *, skip_v_layer=None):
    rows = GEOMETRY.layout.rows(rank)
    x = _chunk_input(chunk)[rows]
    with adapter.execution(chunk_index=chunk, clean=True):
        for layer, block in enumerate(model.layers):
            block.attention.get_k(x, chunk * GEOMETRY.tokens + rows.start)
            if layer != skip_v_layer:
                block.attention.get_v(x)


def w_roundtrip(rank, world, store_dir, representation):
    model, adapter, _ = _adapter(rank, store_dir, representation)
    heads = []
    for chunk in range(3):
        _forward(model, adapter, chunk, rank)
        heads.append(adapter.seal_chunk())
    assert adapter.chunks == 3 and len(set(heads)) == 3
    restored = adapter.restore_history(dtype=torch.float32)
    local = slice(rank * GEOMETRY.kv_heads // world, (rank + 1) * GEOMETRY.kv_heads // world)
    x = torch.cat([_chunk_input(c) for c in range(3)])
    with torch.no_grad():
        for layer, block in enumerate(model.layers):
            attn = block.attention
            k_full = _rotary(attn.k_norm(attn.k_proj(x)).reshape(-1, GEOMETRY.kv_heads, GEOMETRY.head_dim), 0)
            v_full = attn.v_proj(x).reshape(-1, GEOMETRY.kv_heads, GEOMETRY.head_dim)
            k, v = restored[layer]
            assert k.shape == (3 * GEOMETRY.tokens, GEOMETRY.kv_heads // world, GEOMETRY.head_dim)
            for got, want in ((k, k_full[:, local]), (v, v_full[:, local])):
                if representation == "raw":
                    torch.testing.assert_close(got, want, rtol=1e-5, atol=1e-5)
                else:
                    assert float((got - want).norm() / want.norm()) < 0.2
    # a denoising execution captures nothing
    with adapter.execution(chunk_index=3, clean=False):
        model.layers[0].attention.get_v(_chunk_input(3)[GEOMETRY.layout.rows(rank)])
    assert adapter._captured == {}
    adapter.detach()
    assert "get_k" not in model.layers[0].attention.__dict__


def w_capture_failure(rank, world, store_dir):
    from reelcache_b200.parallel.distributed import PeerFailure
    model, adapter, runtime = _adapter(rank, store_dir, "raw")
    _forward(model, adapter, 0, rank)
    head = adapter.seal_chunk()
    _forward(model, adapter, 1, rank, skip_v_layer=1 if rank == 1 else None)
    with pytest.raises(PeerFailure, match="rank 1"):
        adapter.seal_chunk()
    assert adapter.head_ref == head and adapter.chunks == 1
    if runtime is not None:
        assert runtime.lineage_head("main") == head


@pytest.mark.parametrize("representation", ["raw", "svd_hevc"])
def test_magi_roundtrip_two_ranks(tmp_path, representation):
    _run("w_roundtrip", str(tmp_path / "store"), representation)


def test_magi_capture_failure_agreed(tmp_path):
    _run("w_capture_failure", str(tmp_path / "store"))


def test_magi_geometry():
    g = MagiGeometry()
    assert (g.layers, g.kv_heads, g.head_dim, g.tokens, g.channels) == (48, 8, 128, 6 * 68 * 120, 1024)
    assert g.layout.columns(1) == slice(512, 1024)
    with pytest.raises(ConfigurationError):
        MagiGeometry(kv_heads=8, world_size=3)
