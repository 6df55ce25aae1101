"""The engine seam of the serving bridge: what a chunked causal video engine hands the bridge, and in which
order (the counterpart of the ``CausalKVBackend`` protocol that reference
reelcache/integrations/sglang/bridge.py:997-3173 implements for SGLang).

A request runs as::

    run = bridge.begin_request(CausalKVRequest(...))   # None: a plain request the bridge does not observe
    done = run.restore(target)                         # chunks already generated; the cache is ready (or
                                                       # becoming ready layer by layer: target.layer_wait)
    for each chunk to generate:
        [run.begin_recache(prompt) -> recache; engine rewrites the window; run.end_recache(recache)]
        capture = run.begin_clean_forward(chunk)       # the clean forward hands every layer's pre-RoPE K / V
        run.capture_layer(capture, layer, k, v, stream)
        run.end_clean_forward(capture)
        stop = run.end_chunk(chunk, latents)           # True: the session was paused at this boundary
    summary = run.finish(error=None)                   # always called, with the error when the stage failed

A replay (``restore_mode="recompute"``) is driven the same way between ``begin_replay`` and ``end_replay``: the
engine re-runs each recorded step (a chunk's clean forward from its stored latents, or a recache under its
recorded prompt) and the bridge captures nothing.

:func:`drive_request` is that loop over one of this package's engines (:mod:`.engine`); the bridge's own
``request`` call uses it. :func:`plan_recache` is the index arithmetic of a prompt-switch KV recache (LongLive's
``_recache_after_switch``): which frames a recache forward re-runs and which of them are written back (the
sink's are kept when the sink is global).
"""

from __future__ import annotations

from dataclasses import dataclass, field
from typing import Any, Callable

import torch

from ...errors import ConfigurationError, IntegrityError, StateError
from .capture import CleanChunkBuilder

ACTIONS = ("create", "resume", "rewind", "fork")
CLEAN_COMMIT = "clean_commit"
KV_RECACHE = "kv_recache"


@dataclass(frozen=True)
class CausalKVRequest:
    """One engine request on a session (``session_id=None``: a plain generation the bridge may only observe)."""

    request_id: Any
    session_id: str | None
    action: str = "resume"
    chunks: int = 1
    checkpoint: Any = None
    source: str | None = None
    seed: int = 0
    prompt: str | None = None              # conditioning of the new chunks; None keeps the session's
    overlap_restore: bool | None = None    # per-request override of the runtime configuration
    pause_after_chunks: int | None = None

    def __post_init__(self) -> None:
        if self.action not in ACTIONS:
            raise ConfigurationError(f"action must be one of {ACTIONS}")
        if type(self.chunks) is not int or self.chunks < 0:
            raise ConfigurationError("chunks must be a nonnegative integer")
        if self.action == "fork" and self.source is None:
            raise ConfigurationError("fork needs a source session")
        if self.pause_after_chunks is not None and (type(self.pause_after_chunks) is not int
                                                    or self.pause_after_chunks < 1):
            raise ConfigurationError("pause_after_chunks must be a positive integer")
        if self.prompt is not None and (not isinstance(self.prompt, str) or not self.prompt):
            raise ConfigurationError("a prompt is a nonempty string")


@dataclass(frozen=True)
class ChunkSlot:
    """Where chunk ``index`` sits: its first latent frame and its token range."""

    index: int
    start_frame: int
    num_frames: int
    token_start: int
    num_tokens: int

    @classmethod
    def of(cls, profile, index: int) -> "ChunkSlot":
        frames = profile.chunk_frames
        return cls(index, index * frames, frames, index * profile.chunk_tokens, profile.chunk_tokens)


@dataclass
class CaptureScope:
    """The capture of one clean forward: a chunk's (``clean_commit``) or a recache window's (``kv_recache``)."""

    kind: str
    slot: ChunkSlot
    builder: CleanChunkBuilder | None
    forwards: int = 0
    ended: bool = False

    def capture_layer(self, layer: int, k_pre: torch.Tensor, v: torch.Tensor, stream: str = "cond") -> None:
        """Engines call this from the clean forward; the bridge keeps the tensors (the engine must not reuse them)."""
        if self.ended:
            raise StateError("capture after the clean forward ended")
        if self.builder is not None:
            self.builder.capture_layer(layer, k_pre, v, stream)

    @property
    def complete(self) -> bool:
        return self.builder is None or self.builder.complete()


@dataclass(frozen=True)
class RecachePlan:
    """One prompt-switch recache before chunk ``before_chunk`` (frame indices are global latent frames)."""

    before_chunk: int
    window_start_frame: int      # first frame the recache forward re-runs
    end_frame: int               # frames generated so far (the recache ends there)
    write_start_frame: int       # first frame written back (the sink's frames are kept when the sink is global)
    frame_tokens: int
    sink_frames: int

    @property
    def window_tokens(self) -> tuple[int, int]:
        return self.window_start_frame * self.frame_tokens, self.end_frame * self.frame_tokens

    @property
    def written_tokens(self) -> tuple[int, int]:
        return self.write_start_frame * self.frame_tokens, self.end_frame * self.frame_tokens

    @property
    def discarded_frames(self) -> tuple[int, int]:
        """Frames the forward re-runs but does not write back."""
        return self.window_start_frame, self.write_start_frame

    def to_dict(self) -> dict[str, Any]:
        return {"before_chunk": self.before_chunk, "window_frames": [self.window_start_frame, self.end_frame],
                "written_frames": [self.write_start_frame, self.end_frame],
                "discarded_frames": list(self.discarded_frames), "window_tokens": list(self.window_tokens),
                "written_tokens": list(self.written_tokens), "sink_frames": self.sink_frames}


def plan_recache(*, generated_frames: int, window_frames: int, sink_frames: int, frame_tokens: int,
                 chunk_frames: int, global_sink: bool = True) -> RecachePlan | None:
    """The recache of a prompt switch before the next chunk (None before the first chunk: nothing to re-run).

    The forward re-runs the last ``window_frames`` generated frames (``-1``: all of them). With a global sink the
    sink frames keep their KV; the write-back then starts at the first whole chunk after the sink, so every
    written range is a union of whole archived chunks (a partly-sink chunk is re-run and discarded)."""
    for name, value in (("generated_frames", generated_frames), ("sink_frames", sink_frames),
                        ("frame_tokens", frame_tokens), ("chunk_frames", chunk_frames)):
        if type(value) is not int or value < 0:
            raise ConfigurationError(f"{name} must be a nonnegative integer")
    if frame_tokens == 0 or chunk_frames == 0 or generated_frames % chunk_frames:
        raise ConfigurationError("a recache runs at a chunk boundary of whole frames")
    if generated_frames == 0:
        return None
    span = generated_frames if window_frames == -1 else min(window_frames, generated_frames)
    if type(span) is not int or span <= 0:
        raise ConfigurationError("window_frames is -1 (all history) or a positive frame count")
    start = generated_frames - span
    write = start
    if global_sink and sink_frames:
        write = max(write, -(-sink_frames // chunk_frames) * chunk_frames)
    write = -(-write // chunk_frames) * chunk_frames          # whole chunks only
    write = min(write, generated_frames)
    return RecachePlan(generated_frames // chunk_frames, start, generated_frames, write, frame_tokens, sink_frames)


@dataclass
class KVRecache:
    """A recache in flight: its plan, epoch id, the prompt it runs under and its capture scope."""

    plan: RecachePlan
    epoch_id: str
    prompt: str
    capture: CaptureScope
    cause: str = "prompt_switch"
    details: dict = field(default_factory=dict)

    @property
    def written(self) -> list[tuple[int, int]]:
        start, end = self.plan.written_tokens
        return [(start, end - start)] if end > start else []


@dataclass
class ReplayStep:
    """One step of a recompute replay: a chunk's clean forward or a recache under its recorded prompt."""

    kind: str                       # "chunk" | "recache"
    slot: ChunkSlot | None
    prompt: str | None
    latents: torch.Tensor | None = None
    plan: RecachePlan | None = None


@dataclass
class RestoreTarget:
    """What the engine hands ``run.restore``: its engine object; the run fills in the cache to generate into and
    the per-layer wait of the first forward (None when the history is already in place)."""

    engine: Any
    cache: Any = None
    layer_wait: Callable[..., None] | None = None
    replay: list[ReplayStep] = field(default_factory=list)
    latents: dict[int, torch.Tensor] = field(default_factory=dict)


def drive_request(bridge, engine, request: CausalKVRequest) -> dict[str, Any]:
    """The stage loop over the seam for one of this package's engines; returns ``run.finish``'s summary.

    The engine provides ``new_cache``, ``generate_chunk``, ``replay_chunk``, ``recache`` and ``install``
    (:mod:`.engine`)."""
    run = bridge.begin_request(request)
    if run is None:
        raise StateError("a plain request is not observed (observe_plain_requests is off)")
    error = None
    try:
        target = RestoreTarget(engine)
        done = run.restore(target)
        if target.replay:
            run.begin_replay()
            for step in target.replay:
                if step.kind == "chunk":
                    engine.replay_chunk(target.cache, step.slot.index, step.latents, prompt=step.prompt)
                else:
                    engine.recache(target.cache, step.plan, None, prompt=step.prompt, latents=target.latents)
            run.end_replay()
        for i in range(request.chunks):
            index = done + i
            if run.needs_recache(index):
                recache = run.begin_recache(index)
                engine.recache(target.cache, recache.plan, recache.capture, prompt=recache.prompt,
                               latents=target.latents)
                run.end_recache(recache)
            slot = ChunkSlot.of(bridge.profile, index)
            capture = run.begin_clean_forward(slot)
            wait = target.layer_wait if i == 0 else None
            latents = engine.generate_chunk(target.cache, index, capture, request_seed=request.seed, layer_wait=wait,
                                            prompt=run.prompt)
            run.end_clean_forward(capture)
            target.latents[index] = latents
            if run.end_chunk(slot, latents):
                break
    except BaseException as exc:
        error = exc
        raise
    finally:
        summary = run.finish(error=error)
    return summary


def check_capture(scope: CaptureScope, kind: str, slot: ChunkSlot) -> None:
    if scope.kind != kind or scope.slot != slot or not scope.ended or not scope.complete:
        raise IntegrityError(f"{kind} {slot.index} ended without a complete clean capture")
