"""Clean-boundary workload traces: a synthetic prompt session compiles into a fork DAG that validates, replays on
the CPU KVRuntime (bitwise histories, parent isolation, durable pause), and equals the reference's compilation."""

import copy
import importlib
import os
import sys

import pytest

from reelcache_b200.errors import ConfigurationError
from reelcache_b200.workload_traces import (HISTORY_LENGTHS, bundle_summary, compile_session, replay_cpu_control,
                                            validate_session, validate_workload)


def _prompt(tag, i, words=20):
    return " ".join(f"{tag}{i}w{j}" for j in range(words))


def session(index=100, prompts=20):
    sid = f"s{index:04d}"
    return {"session_id": sid, "title": f"title {sid}", "category": "nature",
            "prompts": [_prompt(f"{sid}m", i) for i in range(prompts)],
            "forks": [{"history_prompt_count": h, "change_type": "camera",
                       "prompts": [_prompt(f"{sid}f{h}x", i) for i in range(2)]} for h in HISTORY_LENGTHS]}


def test_compile_validate_and_replay(tmp_path):
    workload = compile_session(session(), chunks_per_prompt=1, seed=3)
    ops = workload["summary"]["operations"]
    assert ops == {"generate": 20 + 2 * len(HISTORY_LENGTHS), "fork": 5, "resume": 5}
    report = replay_cpu_control(workload, tmp_path / "store")
    assert report["status"] == "passed" and len(report["events"]) == len(workload["events"])


def test_pause_reopens_the_store(tmp_path):
    workload = compile_session(session(), seed=1)
    events = workload["events"]
    last = max(i for i, e in enumerate(events) if e["operation"] == "generate" and e["branch_id"] == "main"
               and i < 6)
    pause = {**events[last], "operation": "pause", "target_checkpoint": events[last]["output_checkpoint"]}
    pause.pop("output_checkpoint")
    events = events[:last + 1] + [pause] + events[last + 1:]
    for i, e in enumerate(events):
        e["event_id"] = e["source_event_index"] = i
    workload["events"] = events
    validate_workload(workload)
    assert replay_cpu_control(workload, tmp_path / "store")["operations"]["pause"] == 1


def test_invalid_sessions_and_workloads():
    bad = session()
    bad["forks"][0]["prompts"][0] = bad["prompts"][3]               # a fork copies a main prompt
    with pytest.raises(ConfigurationError):
        validate_session(bad)
    with pytest.raises(ConfigurationError):
        validate_session({**session(), "session_id": "x1"})
    workload = compile_session(session())
    forward = copy.deepcopy(workload)
    gen = next(e for e in forward["events"] if e["operation"] == "generate" and e["target_clean_chunk"] == 0)
    forward["events"].append({**gen, "event_id": len(forward["events"]), "operation": "rewind",
                              "source_event_index": len(forward["events"]),
                              "target_checkpoint": forward["events"][-2]["output_checkpoint"]})
    with pytest.raises(ConfigurationError):
        validate_workload(forward)
    assert bundle_summary([session(0), session(1)])["sessions"] == 2
    with pytest.raises(ConfigurationError):
        bundle_summary([session(1)])


def test_compilation_matches_the_reference():
    ref = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "baseline", "_ref")
    if not os.path.isdir(ref):
        pytest.skip("the reference is not installed under baseline/_ref")
    sys.path.insert(0, ref)
    try:
        theirs = importlib.import_module("reelcache.synthetic_workloads")
    except Exception as error:  # noqa: BLE001
        pytest.skip(f"reference module not importable: {error}")
    finally:
        sys.path.remove(ref)
    s = session()
    for chunks, seed in ((1, 0), (2, 5)):
        assert compile_session(s, chunks_per_prompt=chunks, seed=seed) == \
            theirs.compile_session(s, chunks_per_prompt=chunks, seed=seed)
