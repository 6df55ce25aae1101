"""Serving sessions: per-session state and the controller of the session tree (the counterpart of
reference reelcache/integrations/sglang/session.py:79-1337).

A session is one lineage in the archive. Its **published head** is the newest checkpoint in the store;
its **generated frontier** counts submitted chunks (ahead of the head while archival runs). Operations:
create / open / fork / rewind / pause / checkpoint (named, refs ``sglang/checkpoints/<session>/<name>``)
/ close / delete / gc. Failures of a session's archival are surfaced once and must be acknowledged
(``acknowledge``) before the session accepts new work.
"""

from __future__ import annotations

import threading
import time
from dataclasses import dataclass, field
from typing import Any

import torch

from ...errors import ConfigurationError, StateError
from .nodes import chunk_nodes, path_nodes

CHECKPOINT_PREFIX = "sglang/checkpoints/"
STATUSES = ("idle", "running", "paused", "failed", "closed")


def checkpoint_ref(session_id: str, name: str) -> str:
    for part in (session_id, name):
        if not isinstance(part, str) or not part or "/" in part or "\x00" in part:
            raise ConfigurationError("session ids and checkpoint names are nonempty single-component strings")
    return f"{CHECKPOINT_PREFIX}{session_id}/{name}"


@dataclass
class SGLangSessionState:
    session_id: str
    created: float = field(default_factory=time.time)
    status: str = "idle"
    generated: int = 0                 # chunks submitted (generated frontier)
    resident: Any = None               # engine cache currently holding this session's history
    resident_chunks: int = 0           # chunks of history the resident cache holds (of the generated path)
    resident_used: int = 0             # request counter of the last use of the resident cache (LRU order)
    pending: list = field(default_factory=list)   # archive tickets not yet published
    prompt: str | None = None          # conditioning of the newest chunk / recache (None: the default)
    recaches: list = field(default_factory=list)  # chunk counts at which the resident cache was recached
    failure: BaseException | None = None
    pause_requested: bool = False
    events: list = field(default_factory=list)

    def log(self, event: str, **details: Any) -> None:
        self.events.append({"t": time.time(), "event": event, **details})
        if len(self.events) > 256:
            del self.events[:64]

    def describe(self) -> dict:
        return {"session": self.session_id, "status": self.status, "generated": self.generated,
                "resident_chunks": self.resident_chunks, "pending": len([t for t in self.pending if not t.done()]),
                "failure": None if self.failure is None else str(self.failure)}


RETAINED_PREFIX = "sglang/retained/"
#: Infix of the side lineages a detaching rewind hands a session's unpublished chunks to.
DETACHED = ".detached."


def node_prompt(runtime, node_ref: str) -> str | None:
    """The prompt a node was generated (or recached) under, from its execution state (None: the default)."""
    state = runtime.execution_state(node_ref)
    prompt = state.get("prompt")
    return None if prompt is None else bytes(prompt.to(torch.uint8).tolist()).decode()


def prompt_tensor(prompt: str | None) -> dict:
    """The execution-state entry recording a prompt (none for the default conditioning)."""
    return {} if prompt is None else {"prompt": torch.tensor(list(prompt.encode()), dtype=torch.uint8)}


class SGLangSessionController:
    """``retention="full"`` keeps every abandoned branch reachable: a rewind first pins the head it leaves under
    ``sglang/retained/<session>/<n>`` (garbage collection keeps what refs reach); ``"head"`` keeps the current
    head (and named checkpoints) only."""

    def __init__(self, archive, *, retention: str = "head", tree_switch: str = "drain"):
        if retention not in ("head", "full"):
            raise ConfigurationError("retention is 'head' or 'full'")
        if tree_switch not in ("drain", "detach"):
            raise ConfigurationError("tree_switch is 'drain' or 'detach'")
        self.archive = archive
        self.store = archive.store
        self.runtime = archive.runtime
        self.retention = retention
        self.tree_switch = tree_switch
        self.detached: dict[str, list[dict]] = {}
        self._lock = threading.RLock()
        self._states: dict[str, SGLangSessionState] = {}

    # -- lookup ---------------------------------------------------------------------------------------------------

    def resident_states(self) -> list[SGLangSessionState]:
        """Sessions holding a resident engine cache."""
        with self._lock:
            return [state for state in self._states.values() if state.resident is not None]

    def get(self, session_id: str, *, required: bool = True) -> SGLangSessionState | None:
        with self._lock:
            state = self._states.get(session_id)
            if state is None and self.archive.exists(session_id):
                state = self._reopen(session_id)
            if state is None and required:
                raise StateError(f"unknown session {session_id!r}")
            return state

    def _reopen(self, session_id: str) -> SGLangSessionState:
        from .workload_telemetry import active_telemetry
        record = active_telemetry()
        if record is not None:
            with record.span("session_open", gpu=False):
                return self._reopen_state(session_id)
        return self._reopen_state(session_id)

    def _reopen_state(self, session_id: str) -> SGLangSessionState:
        head = self.archive.head(session_id)
        state = SGLangSessionState(session_id, generated=len(chunk_nodes(self.runtime, head)),
                                   prompt=node_prompt(self.runtime, head))
        state.log("reopened", head=head)
        self._states[session_id] = state
        return state

    def sessions(self) -> dict[str, dict]:
        with self._lock:
            names = {name.split("/", 1)[1] for name in self.store.list_refs("lineages/")}
            names = {name for name in names if DETACHED not in name}
            return {name: self.get(name).describe() for name in sorted(names)}

    def head(self, session_id: str) -> str:
        return self.archive.head(session_id)

    def chunks(self, session_id: str) -> list[str]:
        return chunk_nodes(self.runtime, self.head(session_id))

    # -- lifecycle ------------------------------------------------------------------------------------------------

    def create(self, session_id: str) -> SGLangSessionState:
        with self._lock:
            if self.archive.exists(session_id):
                raise StateError(f"session {session_id!r} already exists")
            head = self.archive.create(session_id)
            state = SGLangSessionState(session_id)
            state.log("created", head=head)
            self._states[session_id] = state
            return state

    def open(self, session_id: str) -> dict:
        return self.get(session_id).describe()

    def reconcile(self, state: SGLangSessionState) -> None:
        """Drop finished tickets; record the first failure (surfaced until acknowledged)."""
        still = []
        for ticket in state.pending:
            if not ticket.done():
                still.append(ticket)
            elif ticket.state != "published" and state.failure is None:
                state.failure = ticket.error or StateError(ticket.state)
                state.status = "failed"
                state.log("archival_failed", chunk=ticket.chunk_id, error=str(state.failure))
        state.pending = still

    def check_ready(self, state: SGLangSessionState) -> None:
        self.reconcile(state)
        if state.failure is not None:
            raise StateError(f"session {state.session_id} has an unacknowledged archival failure: {state.failure}")
        if state.status == "closed":
            raise StateError(f"session {state.session_id} is closed")

    def acknowledge(self, session_id: str) -> dict:
        """Accept a failure: the session falls back to its published head; the archive lineage is reset."""
        with self._lock:
            state = self.get(session_id)
            error = state.failure
            self.archive.pipeline.reset(session_id)
            state.failure = None
            state.status = "idle"
            state.generated = len(self.chunks(session_id))
            state.resident = None
            state.resident_chunks = 0
            state.log("acknowledged", error=None if error is None else str(error))
            return {"session": session_id, "acknowledged": None if error is None else str(error),
                    "head": self.head(session_id)}

    def pause(self, session_id: str, *, timeout: float | None = None) -> dict:
        """Wait until every generated chunk is published (durable), then mark the session paused."""
        state = self.get(session_id)
        waited = self.archive.drain(session_id, timeout)
        self.reconcile(state)
        if state.failure is None:
            state.status = "paused"
        state.log("paused", waited=waited)
        return {"session": session_id, "head": self.head(session_id), "waited_seconds": waited,
                "chunks": len(self.chunks(session_id))}

    def checkpoint(self, session_id: str, name: str | None = None, *, timeout: float | None = None,
                   replace: bool = False) -> dict:
        """Pause, then (optionally) pin the published head under a name."""
        info = self.pause(session_id, timeout=timeout)
        if name is not None:
            ref = checkpoint_ref(session_id, name)
            current = self.store.get_ref(ref)
            if current is not None and not replace:
                raise StateError(f"checkpoint {name!r} of {session_id} exists")
            self.store.set_ref(ref, info["head"])
            info["name"] = name
        return info

    def retained(self, session_id: str) -> list[str]:
        """Heads a rewind left behind (``retention="full"``), oldest first."""
        refs = self.store.list_refs(f"{RETAINED_PREFIX}{session_id}/")
        return [refs[name] for name in sorted(refs, key=lambda name: int(name.rsplit("/", 1)[1]))]

    def checkpoints(self, session_id: str) -> list[dict]:
        """Every chunk checkpoint of the session's published path, plus its named checkpoints."""
        named = {ref.rsplit("/", 1)[1]: node for ref, node in
                 self.store.list_refs(f"{CHECKPOINT_PREFIX}{session_id}/").items()}
        rows = [n.to_dict() for n in path_nodes(self.runtime, self.head(session_id)) if n.kind == "chunk"]
        for name, node in sorted(named.items()):
            rows.append({"name": name, "node": node})
        return rows

    def resolve(self, session_id: str, checkpoint: Any) -> str:
        """A checkpoint (chunk count int, name, or node ref) of the session -> node ref."""
        if isinstance(checkpoint, int) and not isinstance(checkpoint, bool):
            path = [n for n in path_nodes(self.runtime, self.head(session_id))]
            chunks = [n for n in path if n.kind == "chunk"]
            if checkpoint == 0:
                return path[0].node_ref
            if not 1 <= checkpoint <= len(chunks):
                raise ConfigurationError(f"checkpoint {checkpoint} is outside 0..{len(chunks)} published chunks")
            return chunks[checkpoint - 1].node_ref
        if isinstance(checkpoint, str) and checkpoint.startswith("manifest:"):
            return checkpoint
        if isinstance(checkpoint, str):
            node = self.store.get_ref(checkpoint_ref(session_id, checkpoint))
            if node is None:
                raise StateError(f"no checkpoint {checkpoint!r} in session {session_id}")
            return node
        raise ConfigurationError("a checkpoint is a chunk count, a name or a node reference")

    def fork(self, source_id: str, session_id: str, *, checkpoint: Any = None) -> SGLangSessionState:
        with self._lock:
            source = self.get(source_id)
            self.check_ready(source)
            if checkpoint is None:
                self.archive.drain(source_id)
                node = self.head(source_id)
            else:
                node = self.resolve(source_id, checkpoint)
            if self.archive.exists(session_id):
                raise StateError(f"session {session_id!r} already exists")
            self.archive.fork(node, session_id)
            state = SGLangSessionState(session_id, generated=len(chunk_nodes(self.runtime, node)),
                                       prompt=node_prompt(self.runtime, node))
            state.log("forked", source=source_id, node=node)
            self._states[session_id] = state
            return state

    def rewind(self, session_id: str, checkpoint: Any) -> SGLangSessionState:
        with self._lock:
            state = self.get(session_id)
            self.check_ready(state)
            node = self._switch_point(session_id, checkpoint)
            left = self.head(session_id)
            if self.retention == "full" and left != node:
                taken = self.store.list_refs(f"{RETAINED_PREFIX}{session_id}/")
                self.store.set_ref(f"{RETAINED_PREFIX}{session_id}/{len(taken)}", left)
            self.archive.rewind(session_id, node)
            state.generated = len(chunk_nodes(self.runtime, node))
            state.prompt = node_prompt(self.runtime, node)
            if any(at >= state.generated for at in state.recaches):
                state.resident = None  # the resident cache holds KV recached after the rewind point
                state.resident_chunks = 0
                state.recaches = []
            elif state.resident_chunks > state.generated:
                state.resident_chunks = state.generated  # the resident prefix stays valid (same path)
            state.status = "idle"
            state.log("rewound", node=node)
            return state

    def _switch_point(self, session_id: str, checkpoint: Any) -> str:
        """The node a rewind moves to. ``tree_switch="drain"`` first waits until every submitted chunk is
        published; ``"detach"`` resolves against the published head when it can and hands the unpublished chunks
        to a side lineage (``<session>.detached.<n>``) that keeps publishing them, so the rewind does not wait."""
        pipeline = getattr(self.archive, "pipeline", None)
        if self.tree_switch == "detach" and hasattr(pipeline, "detach"):
            try:
                node = self.resolve(session_id, checkpoint)
            except (ConfigurationError, StateError):
                node = None  # the checkpoint is not published yet: drain for it
            if node is not None:
                history = self.detached.setdefault(session_id, [])
                record = pipeline.detach(session_id, f"{session_id}{DETACHED}{len(history)}")
                if record["moved"]:
                    history.append(record)
                return node
        self.archive.drain(session_id)
        return self.resolve(session_id, checkpoint)

    def close(self, session_id: str, *, delete: bool = False, drain: bool = True) -> dict:
        with self._lock:
            state = self.get(session_id)
            if drain and not delete:
                try:
                    self.archive.drain(session_id)
                except StateError:
                    pass
            state.resident = None
            state.resident_chunks = 0
            state.status = "closed"
            result = {"session": session_id, "deleted": delete}
            if delete:
                for prefix in (CHECKPOINT_PREFIX, RETAINED_PREFIX):
                    for ref in self.store.list_refs(f"{prefix}{session_id}/"):
                        self.store.delete_ref(ref)
                self.archive.delete(session_id)
                self._states.pop(session_id, None)
            else:
                result["head"] = self.head(session_id)
            state.log("closed", delete=delete)
            return result

    def gc(self) -> dict:
        with self._lock:
            return self.archive.gc()
