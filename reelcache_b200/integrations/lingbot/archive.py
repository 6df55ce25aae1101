"""LingBot session archive: one lineage node per generated chunk, a fork when a session rewinds, asynchronous
publication and synchronous or layer-overlapped restores into the model's shared cache (reference:
integrations/lingbot/reelcache_lingbot/lb_archive.py:150-540).

Every session starts a lineage branch. ``commit(session, key, parent_key, chunk, k_pre, v)`` appends the chunk
under ``parent_key``: when the parent is the session's newest chunk the branch just grows; when it is an older
chunk (the user rewound) the session continues on a new branch forked at the parent's node, and the old branch
keeps its chunks for other forks. Commits copy the captured K / V (they stay on the capturing device) and are
published in submission order by one worker thread, so a fork always finds its parent published; at most
``max_inflight`` chunks wait at a time (``commit`` blocks beyond that).

``restore(head_key, model)`` resolves the history the model attends when it generates the chunk after
``head_key`` (its sink chunks and the window before it) and writes it into the model's cache slots, RoPE
applied at each chunk's absolute frame position. ``overlapped=True`` returns at once with an
:class:`~.overlap.OverlapSession` attached to the model's self-attention modules; the model joins it at the
end of its first forward.

Representations: ``raw`` (exact pre-RoPE rows; restores are bitwise the captured K / V) and ``svd_hevc`` (the
lineage runtime's low-rank node packs at the energy targets; HEVC where an encoder exists, else the same 8-bit
coefficient planes uncompressed). CUDA archives restore ``svd_hevc`` with the fused restore kernels.
"""

from __future__ import annotations

import threading
from concurrent.futures import Future, ThreadPoolExecutor
from typing import Any, Hashable

import torch

from ...archive_restore import LineageRestorer, RawLineageRestorer, SoftwareLineageRestorer
from ...errors import ReelCacheError
from ...lineage import LineageRuntime
from ...rank_method import RankMethodConfig
from ...store import ObjectStore
from ...types import CodecSpec, MatrixKey, TensorContext, energy_targets
from .geometry import LingBotGeometry
from .overlap import OverlapSession, StallEvents

REPRESENTATIONS = ("raw", "svd_hevc")


class ArchiveError(ReelCacheError):
    """A LingBot archive operation failed (the message names the session, key or node)."""


class LingBotArchive:
    def __init__(self, root, geometry: LingBotGeometry, *, representation: str = "raw", device: Any = "cpu",
                 targets: str = "causvid", max_inflight: int = 2, precision: str = "auto"):
        if representation not in REPRESENTATIONS:
            raise ArchiveError(f"representation must be one of {REPRESENTATIONS}, got {representation!r}")
        if type(max_inflight) is not int or max_inflight < 1:
            raise ArchiveError(f"max_inflight must be a positive integer, got {max_inflight!r}")
        self.geometry = geometry
        self.representation = representation
        self.device = torch.device(device)
        self.store = ObjectStore(root)
        self.runtime = LineageRuntime(self.store, geometry.identity())
        self.method = (None if representation == "raw" else
                       RankMethodConfig(targets=energy_targets(targets), codec=CodecSpec("svd_hevc", 32),
                                        solver="gram_eigh"))
        if representation == "raw":
            self.restorer = RawLineageRestorer(self.runtime, self.device)
        elif self.device.type == "cuda":
            self.restorer = LineageRestorer(self.runtime, self.device, precision=precision)
        else:
            self.restorer = SoftwareLineageRestorer(self.runtime, self.device)
        self._lock = threading.Lock()
        self._worker = ThreadPoolExecutor(max_workers=1, thread_name_prefix="lingbot-archive")
        self._slots = threading.Semaphore(max_inflight)
        self._branch: dict[str, str] = {}       # session -> the branch it grows
        self._branches: dict[str, list[str]] = {}  # session -> every branch it made
        self._head: dict[str, Hashable] = {}    # session -> key of its newest chunk
        self._keys: dict[Hashable, dict] = {}   # key -> session, branch, chunk, node, state, error
        self._futures: dict[Hashable, Future] = {}
        self.counters = {"commits": 0, "forks": 0, "restores": 0, "overlapped_restores": 0, "failed": 0}

    # -- sessions and commits --------------------------------------------------------------------------------------

    def ensure_session(self, session: str) -> None:
        with self._lock:
            if session in self._branch:
                return
            branch = str(session)
            self.runtime.create_lineage(branch)
            self._branch[session] = branch
            self._branches[session] = [branch]

    def commit(self, session: str, key: Hashable, parent_key: Hashable | None, chunk: int, k_pre, v) -> None:
        """Queue chunk ``chunk`` (per-layer pre-RoPE K and V ``[chunk_tokens, channels]``) under ``parent_key``."""
        g = self.geometry
        if len(k_pre) != g.layers or len(v) != g.layers:
            raise ArchiveError(f"chunk {key!r}: {len(k_pre)} K and {len(v)} V layers for a {g.layers}-layer model")
        with self._lock:
            if session not in self._branch:
                raise ArchiveError(f"session {session!r} is not open (ensure_session first)")
            if key in self._keys:
                raise ArchiveError(f"chunk key {key!r} was already committed")
            head = self._head.get(session)
            fork_at = None
            if parent_key is None:
                if head is not None:
                    raise ArchiveError(f"session {session!r} already has chunks; its next chunk needs a parent")
            elif parent_key != head:
                parent = self._keys.get(parent_key)
                if parent is None:
                    raise ArchiveError(f"chunk {key!r}: parent {parent_key!r} was never committed")
                if chunk != parent["chunk"] + 1:
                    raise ArchiveError(f"chunk {key!r}: index {chunk} does not follow its parent's {parent['chunk']}")
                fork_at = parent_key
                branch = f"{session}~{len(self._branches[session])}"
                self._branches[session].append(branch)
                self._branch[session] = branch
            elif chunk != self._keys[head]["chunk"] + 1:
                raise ArchiveError(f"chunk {key!r}: index {chunk} does not follow the head's {self._keys[head]['chunk']}")
            branch = self._branch[session]
            self._head[session] = key
            self._keys[key] = {"session": session, "branch": branch, "chunk": chunk, "node": None,
                               "state": "pending", "error": None, "fork_at": fork_at}
        self._slots.acquire()
        try:
            k_copy = [t.detach().reshape(g.chunk_tokens, g.channels).clone() for t in k_pre]
            v_copy = [t.detach().reshape(g.chunk_tokens, g.channels).clone() for t in v]
            copied = None
            if k_copy[0].is_cuda:  # the worker's stream must not read the copies before the caller's stream made them
                copied = torch.cuda.Event()
                copied.record(torch.cuda.current_stream(k_copy[0].device))
            self._futures[key] = self._worker.submit(self._publish, key, k_copy, v_copy, copied)
        except BaseException:
            self._slots.release()
            raise

    def _publish(self, key: Hashable, k_pre: list, v: list, copied=None) -> str:
        info = self._keys[key]
        g = self.geometry
        try:
            if copied is not None:
                torch.cuda.current_stream(k_pre[0].device).wait_event(copied)
            if info["fork_at"] is not None:
                parent = self._keys[info["fork_at"]]
                if parent["node"] is None:
                    raise ArchiveError(f"cannot fork at {info['fork_at']!r}: {parent['error'] or 'not published'}")
                self.runtime.fork_lineage(parent["node"], info["branch"])
                self.counters["forks"] += 1
            model = self.runtime.model
            start = info["chunk"] * g.chunk_tokens
            matrices, contexts = {}, {}
            for layer in range(g.layers):
                for target, rows in (("K", k_pre[layer]), ("V", v[layer])):
                    mk = MatrixKey(layer, target)
                    matrices[mk] = rows
                    contexts[mk] = TensorContext(model, mk, start, g.frames_per_chunk, g.latent_height,
                                                 g.latent_width, "pre_rope" if target == "K" else "none")
            chunk_id = f"chunk{info['chunk']}"
            if self.method is None:
                commit = self.runtime.commit_raw_node(info["branch"], chunk_id, matrices, contexts)
            else:
                commit = self.runtime.commit_node(info["branch"], chunk_id, matrices, contexts, method=self.method,
                                                  device=self.device)
            info["node"] = commit.node_ref
            info["state"] = "published"
            self.counters["commits"] += 1
            return commit.node_ref
        except BaseException as error:
            info["state"], info["error"] = "failed", error
            self.counters["failed"] += 1
            raise
        finally:
            self._slots.release()

    def published(self, key: Hashable) -> bool:
        info = self._keys.get(key)
        return info is not None and info["state"] == "published"

    def wait_published(self, key: Hashable, timeout: float | None = None) -> str:
        """The node of ``key`` once published (raises :class:`ArchiveError` with the cause if it failed)."""
        future = self._futures.get(key)
        if future is None:
            raise ArchiveError(f"chunk key {key!r} was never committed")
        try:
            return future.result(timeout)
        except ArchiveError:
            raise
        except BaseException as error:  # noqa: BLE001 - re-raised typed with the key
            raise ArchiveError(f"chunk {key!r} failed to publish: {error}") from error

    def drain(self, timeout: float | None = None) -> dict[str, Any]:
        """Wait for every queued chunk; returns the published and failed counts."""
        for key in list(self._futures):
            try:
                self.wait_published(key, timeout)
            except ArchiveError:
                pass
        states = [info["state"] for info in self._keys.values()]
        return {"published": states.count("published"), "failed": states.count("failed"),
                "pending": states.count("pending")}

    def inflight(self) -> int:
        return sum(1 for info in self._keys.values() if info["state"] == "pending")

    def report(self, key: Hashable) -> dict[str, Any]:
        node = self.wait_published(key)
        info = self._keys[key]
        return {"key": key, "session": info["session"], "branch": info["branch"], "chunk": info["chunk"],
                "node": node, "forked_at": info["fork_at"], "commit": dict(self.runtime.node_commit_report(node))}

    # -- restores ---------------------------------------------------------------------------------------------------

    def restore(self, head_key: Hashable, model, *, overlapped: bool = False, thread: bool = True, stream=None,
                recorder: StallEvents | None = None):
        """Restore the history the model attends after ``head_key`` into ``model.cache``.

        Synchronous: returns the record once every layer is written. Overlapped: returns the attached
        :class:`OverlapSession` (the model's next forward waits per layer and joins it)."""
        node = self.wait_published(head_key)
        g = self.geometry
        head_chunk = self._keys[head_key]["chunk"]
        chunks = [c for c in model.cache.attended(head_chunk + 1) if c <= head_chunk]
        ranges = _merge([(c * g.chunk_tokens, (c + 1) * g.chunk_tokens) for c in chunks])
        tokens = g.chunk_tokens
        table = model.rope_table

        def rope(piece):
            return table, (g.frames_per_chunk * (piece.token_start // tokens), 0, 0)

        def slot_of(piece):
            return model.cache.place(piece.token_start // tokens)[0] + piece.token_start % tokens

        cuda = self.device.type == "cuda"
        if cuda and stream is None:
            stream = torch.cuda.Stream(self.device)
        window = recorder.window_begin("restore", stream) if recorder is not None else None
        result = self.restorer.restore(node, model.cache.destination, rope, stream=stream, overlapped=overlapped,
                                       ranges=ranges, thread=thread and overlapped, slot_of=slot_of)
        record = {"node": node, "head_chunk": head_chunk, "chunks": chunks, "overlapped": overlapped}
        for c in chunks:
            model.cache.resident[model.cache.slot(c)] = c

        def finish(_info):
            if window is not None:
                recorder.window_end(window)
            return {}

        self.counters["restores"] += 1
        if not overlapped:
            for layer in range(g.layers):
                result.wait(layer)
            record["restore"] = dict(result.join() or {})
            finish(None)
            if cuda:
                torch.cuda.current_stream(self.device).synchronize()
            return record
        self.counters["overlapped_restores"] += 1
        session = OverlapSession(result, layers=g.layers, record=record, recorder=recorder,
                                 stream=torch.cuda.current_stream(self.device) if cuda else None, finish=finish)
        model.attach_overlapped_restore(session)
        return session

    # -- lifetime ---------------------------------------------------------------------------------------------------

    def forget_session(self, session: str) -> dict[str, Any]:
        """Delete every branch the session made (after its queued chunks finished)."""
        with self._lock:
            branches = self._branches.pop(session, [])
            self._branch.pop(session, None)
            self._head.pop(session, None)
            keys = [k for k, info in self._keys.items() if info["session"] == session]
        for key in keys:
            try:
                self.wait_published(key)
            except ArchiveError:
                pass
        for branch in branches:
            self.runtime.delete_lineage(branch)
        for key in keys:
            self._keys.pop(key, None)
            self._futures.pop(key, None)
        return {"branches": len(branches), "chunks": len(keys)}

    def archive_bytes(self) -> int:
        return int(self.store.stats().get("bytes", 0)) if hasattr(self.store, "stats") else 0

    def stats(self) -> dict[str, Any]:
        return {**self.counters, "sessions": len(self._branch), "inflight": self.inflight(),
                "representation": self.representation, "restorer": type(self.restorer).__name__}

    def close(self) -> None:
        self.drain()
        self._worker.shutdown(wait=True)


def _merge(ranges: list[tuple[int, int]]) -> list[tuple[int, int]]:
    merged: list[list[int]] = []
    for start, end in sorted(ranges):
        if merged and merged[-1][1] == start:
            merged[-1][1] = end
        else:
            merged.append([start, end])
    return [(a, b) for a, b in merged]
