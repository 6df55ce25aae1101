"""The chunk planner in lockstep: a group of matrices planned together gives, matrix by matrix, the plan of
planning each alone (decision, rank, rows, coefficients and energies bit for bit) in far fewer host rounds; on
CUDA the round's Rayleigh-Ritz problems share Jacobi launches."""

import pytest
import torch

from .lineage_support import chunk, method
from reelcache_b200 import deferred_reads
from reelcache_b200.rank_method import plan_chunk
from reelcache_b200.types import ActiveBasisBinding


def _same(a, b):
    assert a.decision == b.decision and a.rank_view == b.rank_view
    assert torch.equal(a.rows, b.rows) and torch.equal(a.coefficients, b.coefficients)
    assert a.energy == b.energy
    assert (a.new_rows is None) == (b.new_rows is None)
    if a.new_rows is not None:
        assert torch.equal(a.new_rows, b.new_rows)


def _plan_pair(matrices, contexts, bindings, inherited, device=None, **overrides):
    rounds = []
    plans = []
    for batch in (1, 60):
        cfg = method(batch_size=batch, **overrides)
        before = deferred_reads.STATS["rounds"]
        plans.append(plan_chunk(matrices, contexts, cfg, None, bindings, inherited, chunk_id="c", device=device))
        rounds.append(deferred_reads.STATS["rounds"] - before)
    return plans, rounds


@pytest.mark.parametrize("solver", ["topk_rr", "gram_eigh"])
def test_lockstep_plans_equal_sequential(solver):
    matrices, contexts = chunk(0, rank=12)
    (alone, together), rounds = _plan_pair(matrices, contexts, {}, {}, solver=solver, anchor_rank=16, bucket=16,
                                           topk_margin=8)
    for entry in alone:
        _same(alone[entry], together[entry])
    assert rounds[1] * 2 <= rounds[0]
    # a second chunk against the first chunk's rows: share / augment decisions in lockstep as well
    later, later_contexts = chunk(1, rank=12)
    bindings = {e: ActiveBasisBinding("manifest:" + "0" * 64, p.rows.shape[0], "1" * 64, p.rows.shape[0], "c")
                for e, p in alone.items()}
    inherited = {e: p.rows for e, p in alone.items()}
    (alone2, together2), rounds2 = _plan_pair(later, later_contexts, bindings, inherited, solver=solver,
                                              anchor_rank=16, bucket=16, topk_margin=8)
    assert {p.decision for p in alone2.values()} & {"share", "augment", "refit"}
    for entry in alone2:
        _same(alone2[entry], together2[entry])
    assert rounds2[1] < rounds2[0]


@pytest.mark.gpu
def test_lockstep_plans_equal_sequential_on_cuda():
    from reelcache_b200 import gpu_fitting
    matrices, contexts = chunk(0, rank=12, dtype=torch.bfloat16)
    before = gpu_fitting.STATS.get("jacobi_calls", 0)
    (alone, together), rounds = _plan_pair(matrices, contexts, {}, {}, device="cuda", solver="topk_rr",
                                           anchor_rank=16, bucket=16, topk_margin=8)
    assert gpu_fitting.STATS["jacobi_calls"] > before
    for entry in alone:
        _same(alone[entry], together[entry])
    assert rounds[1] * 2 <= rounds[0]


def test_condition_transfers_and_step_points():
    import math
    q = torch.linalg.qr(torch.randn(64, 16, generator=torch.Generator().manual_seed(0)))[0].t()
    assert abs(deferred_reads.run_one(deferred_reads.condition_routine(q)) - 1.0) < 1e-5
    assert math.isinf(deferred_reads.run_one(deferred_reads.condition_routine(torch.ones(2, 8))))
    tensors = [torch.randn(3, 4), torch.arange(5, dtype=torch.int32), torch.randn(2, dtype=torch.float64)]
    for a, b in zip(deferred_reads.download(tensors), tensors):
        assert torch.equal(a, b) and a.dtype == b.dtype
    seen = []
    deferred_reads.set_step_hook(lambda: seen.append(deferred_reads.current_phase()))
    try:
        deferred_reads.step_phase("plan")
        with deferred_reads.blocked_wait("staging"):
            pass
        deferred_reads.run_lockstep([deferred_reads.source_energy_routine(torch.ones(4, 4))])
    finally:
        deferred_reads.set_step_hook(None)
    assert seen[0] == "plan" and len(seen) >= 2
