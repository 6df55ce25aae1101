"""The session-mix workload generator: reproducible traces and a short replay on the synthetic engine."""

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
