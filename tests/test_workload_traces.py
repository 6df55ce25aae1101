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


def _browser_replay():
    """An authored browser replay: two tabs, a pause, a revisit of an earlier document, a closed tab."""
    def row(t, intent, tab, **props):
        return {"timestamp": t, "type": "browser",
                "action": {"intent": intent, "arguments": {"properties": {"tabId": tab, **props}, "metadata": {}}}}
    return {"data": [
        {"timestamp": -1.0, "type": "chat", "action": {"intent": "say", "arguments": {}}},
        row(0.0, "load", 1, documentId="doc-a"),
        row(2.0, "click", 1),
        row(4.0, "scroll", 1),
        row(5.0, "tabcreate", 2, openerTabId=1),
        row(6.0, "tabswitch", 2),
        row(7.0, "load", 2, documentId="doc-b"),
        row(8.0, "tabswitch", 1),
        row(60.0, "click", 1),
        row(61.0, "load", 1, documentId="doc-a"),
        row(62.0, "tabremove", 2),
        row(63.0, "click", 2),
    ]}


def test_browser_trace_compiles_into_a_valid_workload(tmp_path):
    from reelcache_b200.workload_traces import (WorkloadPolicy, browser_observations, compile_browser_workload,
                                                read_narratives, replay_cpu_control, validate_workload)
    narrative = read_narratives('{"prompts": ["a quiet street", "rain starts", "night falls"]}\n')[0]
    observations = browser_observations(_browser_replay())
    workload = compile_browser_workload(observations, narrative, WorkloadPolicy(chunk_seconds=5.0),
                                        source_id="fixture", episode_id="e1", source_provenance="authored_fixture")
    validate_workload(workload)
    ops = [e["operation"] for e in workload["events"]]
    assert ops.count("fork") == 1 and ops.count("retire") == 1 and ops.count("rewind") == 1
    assert ("pause", "resume") in list(zip(ops, ops[1:]))
    fork = next(e for e in workload["events"] if e["operation"] == "fork")
    assert fork["parent_branch_id"] == "main" and fork["mapping_rule"] == "tabcreate_from_opener"
    statuses = {r["source_event_index"]: r["mapping_status"] for r in workload["source_audit"]}
    assert statuses[0] == "pre_recording"
    assert statuses[11] == "audit_only"  # tab 2 was closed before this click: nothing is invented for it
    assert statuses[10] == "mapped"  # closing the inactive tab 2 retired its branch
    assert workload["claims"]["native_model_executed"] is False
    report = replay_cpu_control(workload, tmp_path / "store")
    assert report["schema"] == "reelcache.workload_cpu_control.v1"


def test_browser_policy_and_narratives_are_checked():
    from reelcache_b200.errors import ConfigurationError
    from reelcache_b200.workload_traces import WorkloadPolicy, read_narratives
    with pytest.raises(ConfigurationError):
        WorkloadPolicy(chunk_seconds=0)
    with pytest.raises(ConfigurationError):
        WorkloadPolicy(chunk_seconds=1.0, branch_content="remix")
    with pytest.raises(ConfigurationError):
        read_narratives('{"prompts": ["x"]}\n{"prompts": ["x"]}\n')
    with pytest.raises(ConfigurationError):
        read_narratives("")
