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


# -- recorded browser traces ------------------------------------------------------------------------------------------
# A browser session recorded as events (WebLINX-style replays) mapped onto clean-boundary video operations under an
# explicit policy (reference reelcache/workloads.py:21-272): every content-producing action of the active tab
# generates ``chunks_per_action`` clean chunks; a new tab forks a branch from its opener's (or the active tab's)
# newest checkpoint; switching tabs resumes that tab's branch; closing an inactive tab retires its branch; loading a
# document the branch produced before rewinds (or resumes) to the checkpoint it was seen at; an idle gap of at least
# ``pause_gap_seconds`` pauses and resumes the branch. Events the policy cannot map stay in the source audit with
# the reason, never as invented operations. The output is the same trace-mapped workload schema as above.

from dataclasses import asdict, dataclass  # noqa: E402
import math  # noqa: E402


@dataclass(frozen=True)
class WorkloadPolicy:
    chunk_seconds: float
    prompt_seconds: float = 10.0
    chunks_per_action: int = 1
    pause_gap_seconds: float = 30.0
    seed: int = 0
    branch_content: str = "new_seed"
    generation_intents: tuple[str, ...] = ("load", "click", "scroll", "paste")
    infer_url_rewind: bool = False

    def __post_init__(self):
        def seconds(value, name, *, positive):
            ok = not isinstance(value, bool) and isinstance(value, (int, float)) and math.isfinite(value)
            if not ok or (value <= 0 if positive else value < 0):
                raise ConfigurationError(f"workload policy: {name} must be {'positive' if positive else 'nonnegative'}"
                                         f" finite seconds, got {value!r}")
        seconds(self.chunk_seconds, "chunk_seconds", positive=True)
        seconds(self.prompt_seconds, "prompt_seconds", positive=True)
        seconds(self.pause_gap_seconds, "pause_gap_seconds", positive=False)
        if type(self.chunks_per_action) is not int or self.chunks_per_action < 1:
            raise ConfigurationError(f"workload policy: chunks_per_action must be >= 1, got {self.chunks_per_action!r}")
        if type(self.seed) is not int or not 0 <= self.seed < 2 ** 63:
            raise ConfigurationError(f"workload policy: seed must be in [0, 2**63), got {self.seed!r}")
        if self.branch_content not in ("new_seed", "next_prompt"):
            raise ConfigurationError(f"workload policy: branch_content {self.branch_content!r} is neither new_seed "
                                     "nor next_prompt")
        if type(self.infer_url_rewind) is not bool:
            raise ConfigurationError("workload policy: infer_url_rewind is a boolean")
        if not self.generation_intents or not all(isinstance(i, str) and i for i in self.generation_intents):
            raise ConfigurationError("workload policy: generation_intents are nonempty strings")


def read_narratives(text: str) -> list[dict[str, Any]]:
    """Narratives (JSONL of ``{"prompts": [...]}``), each identified by the SHA-256 of its canonical prompt list;
    a repeated narrative is refused (split datasets at whole narratives)."""
    out, ids = [], set()
    for number, line in enumerate(text.splitlines(), 1):
        if not line.strip():
            continue
        try:
            row = json.loads(line)
        except ValueError as error:
            raise ConfigurationError(f"narrative line {number} is not JSON") from error
        prompts = row.get("prompts") if isinstance(row, dict) else None
        if not isinstance(prompts, list) or not prompts or not all(isinstance(p, str) and p.strip() for p in prompts):
            raise ConfigurationError(f"narrative line {number} needs a nonempty list of nonempty prompts")
        prompts = json.loads(json.dumps(prompts))
        identity = hashlib.sha256(json.dumps(prompts, ensure_ascii=True).encode()).hexdigest()
        if identity in ids:
            raise ConfigurationError(f"narrative line {number} repeats an earlier narrative")
        ids.add(identity)
        out.append({"narrative_id": identity, "prompts": prompts})
    if not out:
        raise ConfigurationError("there are no narratives")
    return out


def _tab_id(value) -> str | None:
    if isinstance(value, bool) or not isinstance(value, (str, int)):
        return None
    text = str(value)
    return None if text in ("", "-1") else text


def _opaque(value) -> str | None:
    """A short digest standing for a document or URL (the trace keeps no page content)."""
    return hashlib.sha256(str(value).encode()).hexdigest()[:24] if value else None


def browser_observations(replay: Mapping[str, Any]) -> list[dict[str, Any]]:
    """Timing and navigation metadata of a browser replay (``{"data": [rows]}``), without dialogue or page content."""
    rows = replay.get("data") if isinstance(replay, Mapping) else None
    if not isinstance(rows, list):
        raise ConfigurationError("a browser replay is a mapping with a 'data' list of events")
    out = []
    for index, row in enumerate(rows):
        if not isinstance(row, Mapping):
            raise ConfigurationError(f"replay row {index} is not a mapping")
        stamp = row.get("timestamp")
        if stamp is not None and (isinstance(stamp, bool) or not isinstance(stamp, (int, float))
                                  or not math.isfinite(stamp)):
            raise ConfigurationError(f"replay row {index} has a non-finite timestamp")
        action = row.get("action", {})
        arguments = action.get("arguments", {}) if isinstance(action, Mapping) else None
        properties = arguments.get("properties", {}) if isinstance(arguments, Mapping) else None
        metadata = arguments.get("metadata", {}) if isinstance(arguments, Mapping) else None
        if not isinstance(properties, Mapping) or not isinstance(metadata, Mapping):
            raise ConfigurationError(f"replay row {index} has malformed action arguments")
        qualifiers = properties.get("transitionQualifiers", [])
        if not isinstance(qualifiers, list):
            raise ConfigurationError(f"replay row {index} has malformed navigation qualifiers")
        out.append({
            "source_event_index": index, "source_timestamp": stamp, "source_type": row.get("type"),
            "source_action": action.get("intent", row.get("type")),
            "tab_id": _tab_id(properties.get("tabId")) or _tab_id(metadata.get("tabId")),
            "origin_tab_id": _tab_id(properties.get("openerTabId")) or _tab_id(properties.get("tabIdOrigin")),
            "source_state_id": _opaque(properties.get("documentId")),
            "source_url_id": _opaque(metadata.get("url") or properties.get("url")),
            "back_forward": "forward_back" in qualifiers,
        })
    return out


class _BrowserMapper:
    """The mapping state of one browser trace: branches (cursor, seed, prompt offset, newest checkpoint), the
    live tabs, the checkpoints documents and URLs were seen at, the emitted events and the audit rows."""

    def __init__(self, prompts, policy: WorkloadPolicy, source_id: str, episode_id: str):
        self.prompts, self.policy = prompts, policy
        self.source_id, self.episode_id = source_id, episode_id
        self.branches = {"main": {"cursor": 0, "seed": policy.seed, "prompt_offset": 0, "checkpoint": "main:0"}}
        self.tabs: dict[str, str] = {}
        self.seen_state: dict[tuple, tuple] = {}
        self.seen_url: dict[tuple, tuple] = {}
        self.events: list[dict[str, Any]] = []
        self.audit: list[dict[str, Any]] = []
        self.active = "main"

    def prompt_index(self, branch: str) -> int:
        state = self.branches[branch]
        seconds = state["cursor"] * self.policy.chunk_seconds
        return min(len(self.prompts) - 1, int(seconds / self.policy.prompt_seconds) + state["prompt_offset"])

    def emit(self, operation: str, obs, rule: str, branch: str | None = None, **extra) -> None:
        branch = self.active if branch is None else branch
        state = self.branches[branch]
        self.events.append({
            "event_id": len(self.events), "operation": operation, "branch_id": branch, "source_id": self.source_id,
            "source_event_index": obs["source_event_index"], "source_timestamp": obs.get("source_timestamp"),
            "source_action": obs.get("source_action"), "source_state_id": obs.get("source_state_id"),
            "mapping_rule": rule, "provenance_class": "trace_mapped", "target_clean_chunk": state["cursor"],
            "checkpoint_id": state["checkpoint"], "prompt_index": self.prompt_index(branch), "seed": state["seed"],
            **extra})

    # each handler returns the audit reason when the event cannot be mapped (None when it was)
    def tab_create(self, obs):
        tab = obs.get("tab_id")
        if tab is None:
            return "missing_new_tab_id"
        if tab in self.tabs:
            raise ConfigurationError(f"source event {obs['source_event_index']} creates tab {tab}, which is open")
        if self.branches[self.active]["cursor"] == 0:
            return "no_clean_video_checkpoint_yet"
        opener = obs.get("origin_tab_id")
        inferred = opener not in self.tabs
        parent = self.active if inferred else self.tabs[opener]
        child = f"branch-{len(self.branches)}"
        index = obs["source_event_index"]
        digest = hashlib.sha256(f"{self.episode_id}:{index}:{self.policy.seed}".encode()).digest()
        offset = self.branches[parent]["prompt_offset"] + (1 if self.policy.branch_content == "next_prompt" else 0)
        self.branches[child] = {"cursor": self.branches[parent]["cursor"],
                                "seed": int.from_bytes(digest[:8], "little") % (2 ** 63),
                                "prompt_offset": offset, "checkpoint": f"{child}:fork-{index}"}
        self.emit("fork", obs, "tabcreate_from_active_tab" if inferred else "tabcreate_from_opener", branch=child,
                  parent_branch_id=parent, target_checkpoint=self.branches[parent]["checkpoint"],
                  provenance_class="inferred_relationship" if inferred else "trace_mapped", seed_policy="new_seed",
                  content_policy=self.policy.branch_content)
        self.tabs[tab] = child
        return None

    def tab_switch(self, obs):
        branch = self.tabs.get(obs.get("tab_id"))
        if branch is None:
            return "target_tab_has_no_mapped_branch"
        if branch != self.active:
            self.active = branch
            if self.branches[branch]["cursor"] > 0:
                self.emit("resume", obs, "reactivate_recorded_tab", target_checkpoint=self.branches[branch]["checkpoint"])
        return None

    def tab_remove(self, obs):
        branch = self.tabs.get(obs.get("tab_id"))
        if branch is None or branch == self.active:
            return "cannot_retire_active_or_unknown_tab_without_a_recorded_switch"
        self.emit("retire", obs, "close_recorded_inactive_tab", branch=branch)
        del self.tabs[obs["tab_id"]]
        return None

    def revisit(self, obs):
        state_id, url_id = obs.get("source_state_id"), obs.get("source_url_id")
        target = self.seen_state.get((self.active, state_id)) if state_id else None
        inferred = False
        if target is None and self.policy.infer_url_rewind and obs.get("back_forward"):
            target = self.seen_url.get((self.active, url_id))
            inferred = target is not None
        current = self.branches[self.active]
        if target is not None and target[2] != current["checkpoint"]:
            operation = "rewind" if target[1] < current["cursor"] else "resume"
            self.emit(operation, obs, "back_to_visited_url" if inferred else "revisit_recorded_document",
                      target_checkpoint=target[2], target_clean_chunk=target[1],
                      provenance_class="inferred_relationship" if inferred else "trace_mapped")
            current["cursor"], current["checkpoint"] = target[1], target[2]
            return None
        return "back_forward_has_no_identifiable_checkpoint_target" if obs.get("back_forward") else None

    def generate(self, obs):
        if self.tabs.get(obs.get("tab_id")) != self.active:
            return "generation_event_belongs_to_inactive_tab"
        state = self.branches[self.active]
        for _ in range(self.policy.chunks_per_action):
            produced = f"{self.active}:generated-{len(self.events)}"
            self.emit("generate", obs, "native_clean_chunks_per_selected_action", output_checkpoint=produced)
            state["cursor"] += 1
            state["checkpoint"] = produced
        seen = (self.active, state["cursor"], state["checkpoint"])
        if obs.get("source_state_id"):
            self.seen_state.setdefault((self.active, obs["source_state_id"]), seen)
        if obs.get("source_url_id"):
            self.seen_url.setdefault((self.active, obs["source_url_id"]), seen)
        return None


def compile_browser_workload(observations: Sequence[Mapping[str, Any]], narrative: Mapping[str, Any],
                             policy: WorkloadPolicy, *, source_id: str, episode_id: str,
                             source_provenance: str = "recorded_trace") -> dict[str, Any]:
    """A recorded browser trace (:func:`browser_observations`) as a trace-mapped video workload over the
    narrative's prompts (see the section comment); validated before it is returned."""
    if not source_id or not episode_id:
        raise ConfigurationError("a browser workload needs a source id and an episode id")
    if not isinstance(policy, WorkloadPolicy):
        raise ConfigurationError("the mapping policy must be a WorkloadPolicy")
    if source_provenance not in ("recorded_trace", "authored_fixture"):
        raise ConfigurationError(f"source_provenance {source_provenance!r} is neither recorded_trace nor "
                                 "authored_fixture")
    prompts = narrative.get("prompts")
    if not isinstance(prompts, list) or not prompts or not all(isinstance(p, str) and p.strip() for p in prompts):
        raise ConfigurationError("the narrative needs a nonempty list of nonempty prompts")
    mapper = _BrowserMapper(prompts, policy, source_id, episode_id)
    last_index, last_stamp = -1, None
    for raw in observations:
        obs = json.loads(json.dumps(raw))
        index, stamp = obs.get("source_event_index"), obs.get("source_timestamp")
        if type(index) is not int or index <= last_index:
            raise ConfigurationError("source event indices must increase strictly (the trace keeps its order)")
        last_index = index
        if stamp is not None and (isinstance(stamp, bool) or not isinstance(stamp, (int, float))
                                  or not math.isfinite(stamp)):
            raise ConfigurationError(f"source event {index} has a non-finite timestamp")
        if stamp is not None and stamp < 0:
            mapper.audit.append({**obs, "mapping_status": "pre_recording", "event_ids": []})
            continue
        first = len(mapper.events)
        if stamp is not None and last_stamp is not None:
            gap = stamp - last_stamp
            if gap < 0:
                raise ConfigurationError(f"source event {index}: timestamps go backwards (audit the clock first)")
            active = mapper.branches[mapper.active]
            if gap > 0 and gap >= policy.pause_gap_seconds and active["cursor"] > 0:
                mapper.emit("pause", obs, "interaction_gap_threshold", idle_seconds=gap,
                            target_checkpoint=active["checkpoint"])
                mapper.emit("resume", obs, "same_branch_after_measured_gap", target_checkpoint=active["checkpoint"])
        if stamp is not None:
            last_stamp = stamp
        intent, tab = obs.get("source_action"), obs.get("tab_id")
        if obs.get("source_type") == "browser" and tab is not None and not mapper.tabs and intent != "tabcreate":
            mapper.tabs[tab] = mapper.active  # the first browser tab seen carries the main branch
        reason = None
        if intent == "tabcreate":
            reason = mapper.tab_create(obs)
        elif intent == "tabswitch":
            reason = mapper.tab_switch(obs)
        elif intent == "tabremove":
            reason = mapper.tab_remove(obs)
        if intent == "load":
            reason = mapper.revisit(obs) or reason
        if obs.get("source_type") == "browser" and intent in policy.generation_intents and tab in mapper.tabs:
            reason = mapper.generate(obs) or reason
        mapped = len(mapper.events) > first
        mapper.audit.append({**obs, "mapping_status": reason or ("mapped" if mapped else "audit_only"),
                             "event_ids": list(range(first, len(mapper.events)))})
    skipped = Counter(r["mapping_status"] for r in mapper.audit
                      if r["mapping_status"] not in ("mapped", "audit_only", "pre_recording"))
    workload = {
        "schema": TRACE_SCHEMA, "episode_id": episode_id, "source_id": source_id,
        "source_provenance": source_provenance, "narrative_id": narrative.get("narrative_id"),
        "prompts": list(prompts), "policy": asdict(policy), "events": mapper.events, "source_audit": mapper.audit,
        "claims": {"recorded_video_user_trace": False, "source_interaction_order_preserved": True,
                   "native_model_executed": False, "video_quality_measured": False},
        "summary": {"source_events": len(observations),
                    "operations": dict(Counter(e["operation"] for e in mapper.events)),
                    "branches": len(mapper.branches), "unmapped_reasons": dict(skipped)},
    }
    validate_workload(workload)
    return workload
