"""The session-mix workload generator: reproducible traces and a short replay on the synthetic engine."""

import pytest

from reelcache_b200.workloads import WorkloadSpec, generate, main


def test_trace_is_reproducible_and_mixed():
    spec = WorkloadSpec(sessions=8, requests=200, seed=3)
    a, b = generate(spec), generate(spec)
    assert [(r.session, r.action, r.checkpoint) for r in a] == [(r.session, r.action, r.checkpoint) for r in b]
    actions = {r.action for r in a}
    assert actions == {"create", "resume", "rewind", "fork"}
    assert all(x.at < y.at for x, y in zip(a, a[1:]))


def test_replay_on_synthetic_engine(tmp_path, capsys):
    main(["--store", str(tmp_path / "store"), "--sessions", "2", "--requests", "6", "--min-history", "2",
          "--max-history", "3"])
    out = capsys.readouterr().out
    assert '"requests": 6' in out


def test_session_tree_workloads_are_reproducible_and_rate_independent():
    from reelcache_b200.session_workloads import (InfeasibleError, SessionTree, WorkloadSetting, gap_distribution,
                                                  schedule_requests)
    base = WorkloadSetting(seed=11, n_sessions=3, requests_per_session=6, p_historical=0.7, gap_profile="recent")
    a = schedule_requests(base)
    b = schedule_requests(WorkloadSetting(**{**base.to_dict(), "rho": 3.0, "arrival_cv": 0.2}))
    c = schedule_requests(WorkloadSetting(**{**base.to_dict(), "arrival_mode": "closed"}))
    key = lambda w: sorted((r["session"], r["ordinal"], r["age"], r["node"]) for r in w["schedule"])  # noqa: E731
    assert key(a) == key(b) == key(c)
    assert a == schedule_requests(base)
    times = [r["at"] for r in a["schedule"]]
    assert times == sorted(times) and all(r["think_s"] > 0 for r in c["schedule"])
    tree = SessionTree("x", 3)
    assert tree.legal_ages(min_switch_depth=2, max_depth=None) == [1]
    with pytest.raises(InfeasibleError):
        gap_distribution("fixed", [1, 2], gap_k=5)
    support, probabilities = gap_distribution("far", [1, 2, 3, 4])
    assert support == [1, 2, 3, 4] and probabilities[:2] == [0.0, 0.0]


def test_verify_receipt_binds_the_tree(tmp_path):
    import json
    from reelcache_b200 import verify
    digest, files = verify.source_identity()
    assert len(digest) == 64 and "reelcache_b200/verify.py" in files
    receipt = tmp_path / "r.json"
    receipt.write_text(json.dumps({"tree_sha256": digest, "exit_code": 0, "counts": {"passed": 1}}))
    assert verify.check(receipt) == 0
    receipt.write_text(json.dumps({"tree_sha256": "0" * 64, "exit_code": 0, "counts": {"passed": 1}}))
    assert verify.check(receipt) == 2
