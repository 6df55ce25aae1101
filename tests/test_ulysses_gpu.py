"""Fused Ulysses projections (QKV GEMM + head scatter, gather + output-projection GEMM) against FP32 PyTorch
references. One GPU emulates ``world`` ranks: every "owner" buffer is a separate allocation on the device and
the kernel runs once per rank (separate launches that do not wait on one another), which exercises every
index of the scatter and gather; the NVLink path is the same code with peer-mapped addresses."""

import pytest
import torch

pytestmark = pytest.mark.gpu


def _ext():
    if not torch.cuda.is_available():
        pytest.skip("needs a GPU")
    from reelcache_b200.ops import _ext
    return _ext


@pytest.mark.parametrize("world,n_loc", [(1, 256), (2, 200), (4, 136)])
def test_qkv_scatter_matches_reference(world, n_loc):
    E = _ext()
    torch.manual_seed(0)
    heads, d, k_in = 8, 128, 1024
    hp = heads // world
    xs = [torch.randn(n_loc, k_in, device="cuda").bfloat16() for _ in range(world)]
    w = (torch.randn(3 * heads * d, k_in, device="cuda") / k_in ** 0.5).bfloat16()
    b = torch.randn(3 * heads * d, device="cuda").bfloat16()
    rows = world * n_loc
    q = [torch.zeros(rows, hp, d, device="cuda", dtype=torch.bfloat16) for _ in range(world)]
    k = [torch.zeros_like(q[0]) for _ in range(world)]
    v = [torch.zeros_like(q[0]) for _ in range(world)]
    status = E.status_word("cuda")
    for r in range(world):
        E.ext().ulysses_qkv(xs[r], w, b, q, k, v, r, d, status)
    torch.cuda.synchronize()
    E.check_status("cuda")
    full = (torch.cat(xs).float() @ w.float().t() + b.float()).reshape(rows, 3, heads, d)
    for p in range(world):
        for s, got in enumerate((q[p], k[p], v[p])):
            ref = full[:, s, p * hp:(p + 1) * hp]
            err = (got.float() - ref).abs().max().item()
            assert err <= 0.02 * ref.abs().max().item() + 1e-3, (p, s, err)


@pytest.mark.parametrize("world,n_loc", [(1, 256), (2, 200), (4, 136)])
def test_out_gather_matches_reference(world, n_loc):
    E = _ext()
    torch.manual_seed(1)
    heads, d, n_out = 8, 128, 1024
    hp = heads // world
    rows = world * n_loc
    owners = [torch.randn(rows, hp * d, device="cuda").bfloat16() for _ in range(world)]
    w = (torch.randn(n_out, heads * d, device="cuda") / (heads * d) ** 0.5).bfloat16()
    b = torch.randn(n_out, device="cuda").bfloat16()
    gate = torch.rand(n_out, device="cuda")
    status = E.status_word("cuda")
    gathered = torch.cat(owners, dim=1).float()  # [rows, heads * d], owner-major columns
    m_tiles = (n_loc + 127) // 128
    stage = torch.empty(m_tiles * 128, heads * d, device="cuda", dtype=torch.bfloat16)
    flags = torch.zeros(m_tiles + 2, dtype=torch.int32, device="cuda")  # spare counters are signalled too
    call = 0
    for r in range(world):
        out = torch.empty(n_loc, n_out, device="cuda", dtype=torch.bfloat16)
        call += 1
        E.ext().ulysses_out(owners, w, b, None, out, r, n_loc, 0, stage, flags, call, status)
        resid = torch.randn(n_loc, n_out, device="cuda")
        x = resid.clone()
        call += 1
        E.ext().ulysses_out(owners, w, b, gate, x, r, n_loc, 1, stage, flags, call, status)
        torch.cuda.synchronize()
        ref = gathered[r * n_loc:(r + 1) * n_loc] @ w.float().t() + b.float()
        err = (out.float() - ref).abs().max().item()
        assert err <= 0.02 * ref.abs().max().item() + 1e-3, (r, err)
        ref_x = resid + gate * ref
        err = (x - ref_x).abs().max().item()
        assert err <= 2e-3 * ref_x.abs().max().item() + 1e-3, (r, err)
    E.check_status("cuda")
    assert int(flags.min()) == call * (world - 1)


def test_peer_barrier_single_rank_and_timeout():
    """The barrier returns at once when every flag holds the epoch; a flag that nothing sets makes it give up
    after its bounded wait and report the peer timeout in the status word (the context stays usable)."""
    E = _ext()
    flags = torch.zeros(2, dtype=torch.int32, device="cuda")
    table = torch.tensor([flags.data_ptr()], dtype=torch.int64, device="cuda")
    status = E.status_word("cuda")
    E.ext().peer_barrier(table, 0, 1, status)
    torch.cuda.synchronize()
    assert int(flags[0]) == 1 and int(status[0]) == 0
    # two "ranks" whose second flag slot nothing writes: rank 0 waits for slot 1 and times out
    table2 = torch.tensor([flags.data_ptr(), flags.data_ptr()], dtype=torch.int64, device="cuda")
    E.ext().peer_barrier(table2, 0, 5, status)
    torch.cuda.synchronize()
    assert int(status[0]) == 0x201
    status.zero_()
    torch.zeros(1, device="cuda").add_(1)  # the context still runs work
    torch.cuda.synchronize()


@pytest.mark.parametrize("world", [1, 3])
def test_gram_reduce_scatter_matches_fp64(world):
    """Partial Grams of every emulated rank's token shard land in the owners' buffers; the owner's rank-order
    sum (mirrored upper triangle) equals the FP64 Gram of all shards to FP32 accuracy."""
    E = _ext()
    from reelcache_b200.parallel.gram_rs import GramReduceScatter, symmetric_from_upper
    torch.manual_seed(2)
    channels, matrices = 256, 4
    owners = [b % world for b in range(matrices)][::-1]
    slots = GramReduceScatter.slots_for(owners)
    shards = [[torch.randn(100 + 24 * r, channels, device="cuda").bfloat16() for _ in range(matrices)]
              for r in range(world)]
    partials = [torch.zeros(world, max(slots) + 1, channels, channels, device="cuda") for _ in range(world)]
    status = E.status_word("cuda")
    from reelcache_b200.parallel.gram_rs import stacked_transpose
    for r in range(world):
        xt = stacked_transpose(shards[r])  # token count padded with zero columns to a multiple of 8
        assert xt.shape[1] % 8 == 0
        E.ext().gram_reduce_scatter(xt, matrices, partials, torch.tensor(owners), torch.tensor(slots), r, status)
    torch.cuda.synchronize()
    E.check_status("cuda")
    for b in range(matrices):
        full = torch.cat([shards[r][b] for r in range(world)]).double()
        ref = full.t() @ full
        got = symmetric_from_upper(partials[owners[b]][:, slots[b]].double().sum(0))
        err = float((got - ref).norm() / ref.norm())
        assert err < 1e-6, (b, err)
