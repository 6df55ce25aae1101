"""Clean-boundary workload traces: prompt sessions compiled into fork DAGs of generate / fork / resume / rewind /
pause / retire events, their validation, and a model-free CPU replay on the KVRuntime (reference counterparts:
reelcache/synthetic_workloads.py and reelcache/workloads.py:273-426).

A **session** (one JSON object per line of a sessions file) is a main path of prompts plus one fork at each of the
declared history lengths (:data:`HISTORY_LENGTHS` prompts), each fork a short list of new continuation prompts of
one change type. :func:`compile_session` turns it into a ``reelcache.trace_mapped_video_workload.v1`` workload:
one ``generate`` event per prompt segment and chunk (``chunks_per_prompt``), a ``fork`` from the main path's
checkpoint after each forked prefix (a new seed derived from the session, history and seed), the fork's
generations, then a ``resume`` of the main path. :func:`validate_workload` replays the event DAG without a model
and rejects dangling checkpoints, cursor jumps and forward rewinds. :func:`replay_cpu_control` runs the events on a
real :class:`~reelcache_b200.manager.KVRuntime` with tiny RAW matrices and checks restored histories bit for bit,
parent isolation across forks and durable reopen at pauses. No video, token or timing claim is derived from these
traces: the workload records that no native model ran.
"""

from __future__ import annotations

import hashlib
import json
import re
from collections import Counter
from typing import Any, Mapping, Sequence

from .errors import ConfigurationError

TRACE_SCHEMA = "reelcache.trace_mapped_video_workload.v1"
CONTROL_SCHEMA = "reelcache.workload_cpu_control.v1"
HISTORY_LENGTHS = (4, 8, 12, 16, 20)
CHANGE_TYPES = frozenset(("action", "camera", "object", "environment", "goal"))
OPERATIONS = ("generate", "fork", "resume", "rewind", "pause", "retire")
_SESSION_ID = re.compile(r"s\d{4}")


def normalized_prompt(text: str) -> str:
    """Lower-case alphanumeric words joined by single spaces (duplicate detection ignores punctuation)."""
    return " ".join(re.findall(r"[a-z0-9]+", text.lower()))


def _words(prompt: Any) -> int:
    return len(prompt.split()) if isinstance(prompt, str) else -1


def validate_session(session: Mapping[str, Any]) -> None:
    """A session: ``s0000``-style id, title, category, >= 20 main prompts of 18-35 words (sessions below s0100
    may keep a six-prompt inherited prefix of >= 12 words each), and one fork per history length in order."""
    if not isinstance(session, Mapping):
        raise ConfigurationError(f"a session is a JSON object, not {type(session).__name__}")
    missing = {"session_id", "title", "category", "prompts", "forks"} - set(session)
    if missing:
        raise ConfigurationError(f"session lacks {sorted(missing)}")
    sid = session["session_id"]
    if not (isinstance(sid, str) and _SESSION_ID.fullmatch(sid)):
        raise ConfigurationError(f"session_id {sid!r} is not of the form s0000")
    for name in ("title", "category"):
        if not (isinstance(session[name], str) and session[name].strip()):
            raise ConfigurationError(f"{sid}: {name} must be a non-blank string")
    prompts = session["prompts"]
    if not (isinstance(prompts, list) and len(prompts) >= 20):
        raise ConfigurationError(f"{sid}: needs at least 20 main-path prompts")
    inherited_prefix = 6 if int(sid[1:]) < 100 else 0
    for index, prompt in enumerate(prompts):
        words = _words(prompt)
        ok = words >= 12 if index < inherited_prefix else 18 <= words <= 35
        if not ok:
            raise ConfigurationError(f"{sid}: main prompt {index} has {words} words "
                                     f"({'>= 12' if index < inherited_prefix else '18-35'} required)")
    forks = session["forks"]
    if not (isinstance(forks, list) and len(forks) == len(HISTORY_LENGTHS)):
        raise ConfigurationError(f"{sid}: needs one fork per history length {HISTORY_LENGTHS}")
    main = {normalized_prompt(p) for p in prompts}
    for fork, history in zip(forks, HISTORY_LENGTHS):
        if not (isinstance(fork, Mapping) and set(fork) == {"history_prompt_count", "change_type", "prompts"}):
            raise ConfigurationError(f"{sid}: a fork has exactly history_prompt_count, change_type and prompts")
        if fork["history_prompt_count"] != history:
            raise ConfigurationError(f"{sid}: forks must branch after {HISTORY_LENGTHS} prompts, in that order")
        if fork["change_type"] not in CHANGE_TYPES:
            raise ConfigurationError(f"{sid}: change_type {fork['change_type']!r} is not one of {sorted(CHANGE_TYPES)}")
        branch = fork["prompts"]
        if not (isinstance(branch, list) and len(branch) >= 2 and all(18 <= _words(p) <= 35 for p in branch)):
            raise ConfigurationError(f"{sid}: fork at {history} needs >= 2 new prompts of 18-35 words")
        seen = [normalized_prompt(p) for p in branch]
        if len(set(seen)) != len(seen) or set(seen) & main:
            raise ConfigurationError(f"{sid}: fork at {history} repeats a prompt of itself or of the main path")


def read_sessions(path) -> list[dict[str, Any]]:
    """Validated sessions of a JSON-lines file (blank lines skipped)."""
    sessions = []
    with open(path) as source:
        for number, line in enumerate(source, 1):
            if line.strip():
                try:
                    session = json.loads(line)
                except ValueError as error:
                    raise ConfigurationError(f"{path}:{number} is not JSON") from error
                validate_session(session)
                sessions.append(session)
    return sessions


def _fork_seed(session_id: str, history: int, seed: int) -> int:
    digest = hashlib.sha256(f"{session_id}:{history}:{seed}".encode()).digest()
    return int.from_bytes(digest[:8], "little") % (1 << 63)


def compile_session(session: Mapping[str, Any], *, chunks_per_prompt: int = 1, seed: int = 0) -> dict[str, Any]:
    """The fork-DAG workload of one session (see the module docstring)."""
    validate_session(session)
    if not (type(chunks_per_prompt) is int and chunks_per_prompt > 0):
        raise ConfigurationError(f"chunks_per_prompt={chunks_per_prompt!r}: expected an int >= 1")
    if not (type(seed) is int and 0 <= seed < (1 << 63)):
        raise ConfigurationError(f"seed={seed!r}: expected an int in [0, 2**63)")
    sid = session["session_id"]
    source = f"llm-authored:{sid}"
    prompts = list(session["prompts"])
    fork_prompts = {}
    for fork in session["forks"]:
        first = len(prompts)
        prompts.extend(fork["prompts"])
        fork_prompts[fork["history_prompt_count"]] = (fork, range(first, len(prompts)))
    events: list[dict[str, Any]] = []
    cursor, head = {"main": 0}, {"main": "main:0"}

    def event(operation, branch, prompt_index, **extra):
        record = {"event_id": len(events), "operation": operation, "branch_id": branch, "source_id": source,
                  "source_event_index": len(events), "source_timestamp": None, "source_action": operation,
                  "source_state_id": None, "mapping_rule": "declared_synthetic_fork_schedule",
                  "provenance_class": "controlled_synthetic", "target_clean_chunk": cursor[branch],
                  "checkpoint_id": head[branch], "prompt_index": prompt_index, "seed": seed}
        record.update(extra)
        events.append(record)

    def generate(branch, prompt_index, branch_seed):
        for _ in range(chunks_per_prompt):
            checkpoint = f"{branch}:generated-{len(events)}"
            event("generate", branch, prompt_index, seed=branch_seed, output_checkpoint=checkpoint)
            cursor[branch] += 1
            head[branch] = checkpoint

    main_length = len(session["prompts"])
    for index in range(main_length):
        generate("main", index, seed)
        if index + 1 not in fork_prompts:
            continue
        history = index + 1
        fork, indices = fork_prompts[history]
        branch, parent = f"fork-h{history:02d}", head["main"]
        cursor[branch], head[branch] = cursor["main"], f"fork-h{history:02d}:fork"
        branch_seed = _fork_seed(sid, history, seed)
        event("fork", branch, indices[0], parent_branch_id="main", target_checkpoint=parent,
              history_prompt_count=history, seed=branch_seed, seed_policy="new_seed",
              content_policy="authored_alternative", change_type=fork["change_type"])
        for prompt_index in indices:
            generate(branch, prompt_index, branch_seed)
        event("resume", "main", min(history, main_length - 1), target_checkpoint=parent)
    workload = {"schema": TRACE_SCHEMA, "episode_id": sid, "source_id": source,
                "source_provenance": "llm_authored_synthetic", "narrative_id": sid, "prompts": prompts,
                "policy": {"seed": seed},
                "history_mapping": {"unit": "completed_prompt_segments", "chunks_per_prompt": chunks_per_prompt,
                                    "native_geometry_qualified": False},
                "events": events, "source_audit": [],
                "claims": {"recorded_video_user_trace": False, "recorded_agent_trace": False,
                           "native_model_executed": False, "video_quality_measured": False},
                "summary": {"operations": dict(Counter(e["operation"] for e in events)),
                            "branches": 1 + len(session["forks"]), "source_events": 0}}
    validate_workload(workload)
    return workload


def validate_workload(workload: Mapping[str, Any]) -> None:
    """Replay the event DAG: every checkpoint a restore or fork names was saved before on the right branch,
    generations advance their branch's cursor by one and publish a new checkpoint, rewinds go backwards."""
    if workload.get("schema") != TRACE_SCHEMA:
        raise ConfigurationError(f"workload schema {workload.get('schema')!r} is not {TRACE_SCHEMA}")
    position = {"main": 0}                       # branch -> clean chunks generated so far
    checkpoints = {"main:0": ("main", 0)}        # checkpoint -> (branch, position)
    retired: set[str] = set()
    previous_source = -1
    for index, ev in enumerate(workload.get("events", [])):
        where = f"event {index}"
        if ev.get("event_id") != index or ev.get("source_event_index", -1) < previous_source:
            raise ConfigurationError(f"{where}: event ids or source order are not monotone")
        previous_source = ev["source_event_index"]
        branch, operation = ev.get("branch_id"), ev.get("operation")
        if operation not in OPERATIONS:
            raise ConfigurationError(f"{where}: operation {operation!r} is not one of {OPERATIONS}")
        if operation == "fork":
            saved = checkpoints.get(ev.get("target_checkpoint"))
            if branch in position or saved is None or saved[0] != ev.get("parent_branch_id"):
                raise ConfigurationError(f"{where}: a fork opens a new branch from a saved checkpoint of its parent")
            if ev.get("checkpoint_id") in checkpoints:
                raise ConfigurationError(f"{where}: the fork's checkpoint {ev.get('checkpoint_id')!r} exists already")
            position[branch] = saved[1]
            checkpoints[ev["checkpoint_id"]] = (branch, saved[1])
            continue
        if branch not in position or branch in retired:
            raise ConfigurationError(f"{where}: branch {branch!r} does not exist or was retired")
        if operation in ("resume", "rewind"):
            saved = checkpoints.get(ev.get("target_checkpoint"))
            if saved is None or saved[0] != branch:
                raise ConfigurationError(f"{where}: {operation} target is not a checkpoint of {branch!r}")
            if operation == "rewind" and saved[1] >= position[branch]:
                raise ConfigurationError(f"{where}: a rewind must go to an earlier clean boundary")
            position[branch] = saved[1]
        elif operation == "generate":
            if ev.get("target_clean_chunk") != position[branch]:
                raise ConfigurationError(f"{where}: generates chunk {ev.get('target_clean_chunk')} of {branch!r}, "
                                         f"which is at {position[branch]}")
            if not 0 <= ev.get("prompt_index", -1) < len(workload["prompts"]):
                raise ConfigurationError(f"{where}: prompt index {ev.get('prompt_index')} is out of range")
            output = ev.get("output_checkpoint")
            if not (isinstance(output, str) and output) or output in checkpoints:
                raise ConfigurationError(f"{where}: a generation must publish a new checkpoint")
            position[branch] += 1
            checkpoints[output] = (branch, position[branch])
        elif operation == "pause":
            if checkpoints.get(ev.get("target_checkpoint")) != (branch, position[branch]):
                raise ConfigurationError(f"{where}: a pause names the branch's current clean boundary")
        else:  # retire
            retired.add(branch)


def replay_cpu_control(workload: Mapping[str, Any], store_root) -> dict[str, Any]:
    """Run a workload's events on a KVRuntime with one layer of 4-channel RAW K / V matrices (6 tokens per
    chunk): histories after every restore equal the recorded ones bit for bit, forks leave their parent's head
    untouched, the RNG continues across snapshots, and a pause closes and reopens the store."""
    import torch

    from .manager import KVRuntime
    from .types import CodecSpec, MatrixKey, ModelIdentity, TensorContext

    validate_workload(workload)
    if not any(ev["operation"] == "generate" for ev in workload["events"]):
        raise ConfigurationError("the CPU replay needs at least one generate event")
    model = ModelIdentity("workload-control", "synthetic-clean-kv-v1", 1, 4, "tokens_channels", "float32")
    keys = (MatrixKey(0, "K"), MatrixKey(0, "V"))

    def open_runtime():
        return KVRuntime(store_root, model, max_resident_bytes=1 << 20, verify_reads=True)

    runtime = open_runtime()
    live: dict[str, tuple[torch.Generator, dict]] = {}
    saved: dict[str, dict] = {}

    def check(branch, history):
        for key in keys:
            with runtime.acquire_history(branch, key) as lease:
                if not torch.equal(lease.tensor, history[key]):
                    raise ConfigurationError(f"restored {key} of {branch!r} differs from its recorded history")

    def save(branch, checkpoint):
        generator, history = live[branch]
        info = runtime.branch_info(branch)
        metadata = {"clean_boundary": {"chunk_id": info["chunk_id"], "token_end": info["token_end"], "clean": True},
                    "conditioning": {"id": workload["narrative_id"]},
                    "execution": {"pending": False, "workload_control": True}, "rng": {"tensor": "rng"},
                    "latent": {"native_latents": "not applicable to synthetic matrices"},
                    "vae": {"native_decoder": "not applicable to synthetic matrices"}}
        saved[checkpoint] = {"snapshot": runtime.snapshot(branch, metadata=metadata,
                                                          tensors={"rng": generator.get_state()}),
                             "history": {k: v.clone() for k, v in history.items()}}

    def restore(ev, fork):
        branch, record = ev["branch_id"], saved[ev["target_checkpoint"]]
        point = runtime.fork if fork else runtime.restore
        state = point(record["snapshot"], branch)
        generator = torch.Generator().set_state(state.tensors["rng"])
        if fork:
            generator.manual_seed(ev["seed"])
        live[branch] = (generator, {k: v.clone() for k, v in record["history"].items()})
        check(branch, live[branch][1])
        if fork:
            save(branch, ev["checkpoint_id"])

    results = []
    try:
        runtime.create_branch("main")
        live["main"] = (torch.Generator().manual_seed(workload["policy"]["seed"]),
                        {key: torch.empty(0, 4) for key in keys})
        save("main", "main:0")
        for ev in workload["events"]:
            branch, operation = ev["branch_id"], ev["operation"]
            if operation == "generate":
                generator, history = live[branch]
                start = runtime.branch_info(branch)["token_end"]
                prompt = workload["prompts"][ev["prompt_index"]]
                shift = int(hashlib.sha256(prompt.encode()).hexdigest()[:4], 16) / 65536
                chunk = {key: torch.randn(6, 4, generator=generator) + shift for key in keys}
                contexts = {key: TensorContext(model, key, start, 1, 2, 3, "pre_rope" if key.target == "K" else "none")
                            for key in keys}
                runtime.seal_chunk(branch, f"event-{ev['event_id']}", chunk, contexts, CodecSpec())
                for key in keys:
                    history[key] = torch.cat((history[key], chunk[key]))
                check(branch, history)
                save(branch, ev["output_checkpoint"])
            elif operation == "fork":
                parent_head = runtime.branch_info(ev["parent_branch_id"])["head_id"]
                restore(ev, fork=True)
                if runtime.branch_info(ev["parent_branch_id"])["head_id"] != parent_head:
                    raise ConfigurationError("a fork moved its parent's head")
            elif operation in ("resume", "rewind"):
                restore(ev, fork=False)
            elif operation == "pause":
                runtime.close()
                runtime = open_runtime()
            else:
                runtime.delete_branch(branch)
                del live[branch]
            results.append({"event_id": ev["event_id"], "operation": operation, "status": "passed"})
        return {"schema": CONTROL_SCHEMA, "status": "passed",
                "scope": "synthetic CPU matrices and the durable KVRuntime lifecycle only",
                "native_model_executed": False, "video_quality_measured": False,
                "source_provenance": workload["source_provenance"], "events": results,
                "operations": dict(Counter(r["operation"] for r in results)), "store": runtime.store.stats()}
    finally:
        runtime.close()


def bundle_summary(sessions: Sequence[Mapping[str, Any]]) -> dict[str, Any]:
    """Counts of a session bundle after validating each session and rejecting prompts repeated across it."""
    owners: dict[str, str] = {}
    categories, changes = Counter(), Counter()
    main_prompts = fork_prompts = 0
    for index, session in enumerate(sessions):
        validate_session(session)
        if session["session_id"] != f"s{index:04d}":
            raise ConfigurationError(f"session {index} is {session['session_id']}, expected s{index:04d}")
        categories[session["category"]] += 1
        texts = list(session["prompts"])
        main_prompts += len(session["prompts"])
        for fork in session["forks"]:
            changes[fork["change_type"]] += 1
            fork_prompts += len(fork["prompts"])
            texts += fork["prompts"]
        for text in texts:
            token = normalized_prompt(text)
            if owners.setdefault(token, session["session_id"]) != session["session_id"]:
                raise ConfigurationError(f"{session['session_id']} repeats a prompt of {owners[token]}")
    return {"sessions": len(sessions), "main_prompts": main_prompts, "fork_prompts": fork_prompts,
            "forks": len(sessions) * len(HISTORY_LENGTHS), "categories": dict(categories),
            "change_types": dict(changes), "history_prompt_counts": list(HISTORY_LENGTHS),
            "native_model_executed": False}


__all__ = ["CHANGE_TYPES", "CONTROL_SCHEMA", "HISTORY_LENGTHS", "OPERATIONS", "TRACE_SCHEMA", "bundle_summary",
           "compile_session", "normalized_prompt", "read_sessions", "replay_cpu_control", "validate_session",
           "validate_workload"]
