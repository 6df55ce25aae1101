"""Interactive session-mix workload generator (64 sessions, Poisson arrivals, resume / rewind / fork mix; the counterpart of reference
reelcache/workloads.py): concurrent sessions with Poisson arrivals, an action mix of resume / rewind
to a uniform earlier chunk / fork, histories of ``min_history..max_history`` chunks, driven through
a serving bridge (:class:`CausalWanKVBridge`). Records per-action time to first chunk and summarizes
p50 / p90 / p99.

``python -m reelcache_b200.workloads --store DIR`` runs a small mix on the synthetic engine (CPU, or
the current GPU with ``--device cuda``).
"""

from __future__ import annotations

import argparse
import json
import random
import time
from dataclasses import dataclass, field
from typing import Any

import numpy as np

ACTIONS = ("resume", "rewind", "fork")


@dataclass(frozen=True)
class WorkloadSpec:
    sessions: int = 64
    rate_per_s: float = 2.0
    mix: tuple[float, float, float] = (0.5, 0.3, 0.2)   # resume, rewind, fork
    min_history: int = 8
    max_history: int = 32
    chunks_per_request: int = 1
    requests: int = 200
    seed: int = 0


@dataclass
class Request:
    at: float
    session: str
    action: str
    checkpoint: Any = None
    source: str | None = None


@dataclass
class WorkloadResult:
    records: list = field(default_factory=list)

    def summary(self) -> dict:
        out: dict[str, Any] = {"requests": len(self.records)}
        for action in ACTIONS + ("create",):
            values = [r["ttfc_ms"] for r in self.records if r["action"] == action and r.get("ttfc_ms") is not None]
            if values:
                out[action] = {"count": len(values), "p50_ttfc_ms": float(np.percentile(values, 50)),
                               "p90_ttfc_ms": float(np.percentile(values, 90)),
                               "p99_ttfc_ms": float(np.percentile(values, 99))}
        routes: dict[str, int] = {}
        for r in self.records:
            routes[r.get("route", "?")] = routes.get(r.get("route", "?"), 0) + 1
        out["routes"] = routes
        return out


def generate(spec: WorkloadSpec) -> list[Request]:
    """A reproducible request trace: Poisson arrivals over randomly chosen sessions."""
    rng = random.Random(spec.seed)
    t = 0.0
    histories: dict[str, int] = {}
    trace = []
    forks = 0
    for _ in range(spec.requests):
        t += rng.expovariate(spec.rate_per_s)
        session = f"s{rng.randrange(spec.sessions)}"
        if session not in histories:
            histories[session] = rng.randint(spec.min_history, spec.max_history)
            trace.append(Request(t, session, "create", checkpoint=histories[session]))
            continue
        action = rng.choices(ACTIONS, weights=spec.mix)[0]
        if action == "rewind":
            trace.append(Request(t, session, "rewind", checkpoint=rng.randint(1, max(1, histories[session] - 1))))
        elif action == "fork":
            forks += 1
            child = f"{session}-f{forks}"
            trace.append(Request(t, child, "fork", checkpoint=rng.randint(1, histories[session]), source=session))
            histories[child] = histories[session]
        else:
            trace.append(Request(t, session, "resume"))
    return trace


def run(bridge, spec: WorkloadSpec, *, realtime: bool = False) -> WorkloadResult:
    """Replay a trace through ``bridge`` (sequentially; ``realtime`` honours the arrival times)."""
    result = WorkloadResult()
    start = time.perf_counter()
    for request in generate(spec):
        if realtime:
            delay = request.at - (time.perf_counter() - start)
            if delay > 0:
                time.sleep(delay)
        if request.action == "create":
            report = bridge.request(request.session, chunks=request.checkpoint, action="create", seed=spec.seed)
            bridge.pause(request.session)  # durable history before it is rewound or forked
        elif request.action == "rewind":
            report = bridge.request(request.session, chunks=spec.chunks_per_request, action="rewind",
                                    checkpoint=request.checkpoint, seed=spec.seed)
        elif request.action == "fork":
            bridge.pause(request.source)
            report = bridge.request(request.session, chunks=spec.chunks_per_request, action="fork",
                                    source=request.source, checkpoint=request.checkpoint, seed=spec.seed)
        else:
            report = bridge.request(request.session, chunks=spec.chunks_per_request, seed=spec.seed)
        result.records.append({"session": request.session, "action": request.action, "ttfc_ms": report["ttfc_ms"],
                               "route": report["route"], "start_chunk": report["start_chunk"]})
    return result


def main(argv=None):
    ap = argparse.ArgumentParser(description=__doc__)
    ap.add_argument("--store", required=True)
    ap.add_argument("--device", default="cpu")
    ap.add_argument("--sessions", type=int, default=4)
    ap.add_argument("--requests", type=int, default=24)
    ap.add_argument("--min-history", type=int, default=2)
    ap.add_argument("--max-history", type=int, default=4)
    args = ap.parse_args(argv)
    from .integrations.sglang import ReelCacheRuntimeConfig, SyntheticEngine, create_sglang_backend
    from .integrations.sglang.engine import model_identity_for
    from .integrations.sglang.profiles import ModelProfile
    profile = ModelProfile("workload-tiny", backbone="tiny-wan", num_layers=2, num_heads=2, head_dim=64, chunk_frames=1,
                           grid=(4, 8), visibility="full_history", sink_frames=0, window_frames=None,
                           energy_profile="causvid")
    engine = SyntheticEngine(profile, model_identity_for(profile, "synthetic"), args.device, rank=4)
    config = ReelCacheRuntimeConfig(store_root=args.store, fit_device="cuda" if args.device != "cpu" else "cpu",
                                    encode_workers=1)
    bridge = create_sglang_backend(config, engine, cache_chunks=args.max_history + 8)
    spec = WorkloadSpec(sessions=args.sessions, requests=args.requests, min_history=args.min_history,
                        max_history=args.max_history)
    try:
        print(json.dumps(run(bridge, spec).summary(), indent=2))
    finally:
        bridge.shutdown()


if __name__ == "__main__":
    main()
