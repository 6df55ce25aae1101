"""Session-tree rewind-and-generate workloads (the counterpart of reference reelcache/session_workloads.py:1-40 for
the design; ``SessionTree`` :708, ``gap_distribution`` :786, ``choose_age`` :822, ``rewind_and_generate`` :836,
``plan_session`` :854, ``open_loop_arrivals`` :912, ``schedule_requests`` :950).

One request selects a session, picks a source node and generates exactly one new chunk as its child.

* **Node age.** Every node gets a monotonically increasing *generation index* (setup nodes 1..d0, then one per
  request). ``k = 0`` targets the latest node; ``k > 0`` the node generated ``k`` generations ago, wherever it is
  in the tree. ``p_historical`` is the probability of ``k > 0``; the positive gap follows a profile over the
  request's **legal** ages: ``uniform``, ``recent`` (geometric with mean ``recent_mean``, truncated), ``far``
  (uniform over the upper half) or ``fixed`` (``gap_k``). An empty support or an illegal fixed gap raises
  :class:`InfeasibleError` -- ages are never snapped or replaced.
* **Legal targets.** ``depth >= min_switch_depth`` and ``depth + 1 <= max_depth``.
* **Arrivals.** Open loop: gamma inter-arrivals with mean ``S / rho`` and coefficient of variation ``arrival_cv``
  (0 constant, 1 Poisson), each arrival to a uniformly chosen eligible session. Closed loop: each session's next
  request ``think`` seconds after its previous chunk returned (lognormal, mean ``think_time_mult * S``, CV
  ``think_cv``).
* **Independent streams.** Every random choice draws uniform doubles from its own PCG64 stream
  (``SeedSequence(seed, spawn_key=(stream word, ...))``): cohort, arrivals, session choice, think times and
  targeting are independent, so trees and targets are identical across rates, burstiness and arrival modes.
  Normal, gamma and lognormal variates are derived here from those uniforms (Box-Muller; Marsaglia-Tsang), so a
  frozen plan does not depend on numpy's distribution code.

Standard library and numpy only.
"""

from __future__ import annotations

import hashlib
import json
import math
from dataclasses import dataclass, field
from typing import Any, Iterable, Mapping, Sequence

import numpy as np

from .errors import ConfigurationError

GAP_PROFILES = ("uniform", "recent", "far", "fixed")


class InfeasibleError(ConfigurationError):
    """The requested workload cannot be realized without changing its distribution."""


def canonical_json(value: Any) -> str:
    return json.dumps(value, sort_keys=True, separators=(",", ":"), allow_nan=False)


def stream_word(name: str) -> int:
    """A stable 32-bit word naming an RNG stream."""
    return int(hashlib.sha256(name.encode()).hexdigest()[:8], 16)


class Uniforms:
    """Uniform doubles in (0, 1) from one PCG64 stream keyed by (seed, name, *keys)."""

    def __init__(self, seed: int, name: str, *keys: int):
        sequence = np.random.SeedSequence(int(seed), spawn_key=(stream_word(name), *[int(k) for k in keys]))
        self._gen = np.random.Generator(np.random.PCG64(sequence))

    def next(self) -> float:
        u = float(self._gen.random())
        while u <= 0.0:
            u = float(self._gen.random())
        return u

    def normal(self) -> float:
        """Standard normal by Box-Muller (one variate per two uniforms)."""
        u1, u2 = self.next(), self.next()
        return math.sqrt(-2.0 * math.log(u1)) * math.cos(2.0 * math.pi * u2)

    def gamma(self, shape: float) -> float:
        """Gamma(shape, 1) by Marsaglia-Tsang (with the u^(1/shape) boost below shape 1)."""
        if shape <= 0:
            raise ConfigurationError("gamma shape must be positive")
        if shape < 1.0:
            return self.gamma(shape + 1.0) * self.next() ** (1.0 / shape)
        d = shape - 1.0 / 3.0
        c = 1.0 / math.sqrt(9.0 * d)
        while True:
            x = self.normal()
            v = (1.0 + c * x) ** 3
            if v <= 0:
                continue
            u = self.next()
            if math.log(u) < 0.5 * x * x + d - d * v + d * math.log(v):
                return d * v


def session_number(session_id: str) -> int:
    return int(hashlib.sha256(session_id.encode()).hexdigest()[:8], 16)


def think_seconds(seed: int, session_id: str, ordinal: int, mean: float, cv: float) -> float:
    """Lognormal think time with the given mean and coefficient of variation (0: constant)."""
    if cv <= 0:
        return float(mean)
    sigma2 = math.log(1.0 + cv * cv)
    mu = math.log(mean) - 0.5 * sigma2
    z = Uniforms(seed, "think", session_number(session_id), ordinal).normal()
    return math.exp(mu + math.sqrt(sigma2) * z)


@dataclass
class WorkloadSetting:
    seed: int = 0
    n_sessions: int = 8
    requests_per_session: int = 4
    setup_depth: int = 3                       # d0
    p_historical: float = 0.5
    gap_profile: str = "uniform"
    recent_mean: float = 2.0
    gap_k: int | None = None
    min_switch_depth: int = 1
    max_depth: int | None = None
    service_time_s: float = 1.0
    rho: float = 0.5
    arrival_cv: float = 1.0
    arrival_mode: str = "open"                 # "open" | "closed"
    think_time_mult: float = 1.0
    think_cv: float = 0.5
    cooldown_s: float = 0.0

    def __post_init__(self):
        if not 0.0 <= self.p_historical <= 1.0:
            raise ConfigurationError("p_historical must lie in [0, 1]")
        if self.gap_profile not in GAP_PROFILES:
            raise ConfigurationError(f"gap_profile must be one of {GAP_PROFILES}")
        if self.gap_profile == "fixed" and (self.gap_k is None or self.gap_k < 1):
            raise ConfigurationError("the fixed gap profile needs gap_k >= 1")
        if self.arrival_mode not in ("open", "closed"):
            raise ConfigurationError("arrival_mode is open or closed")
        if self.setup_depth < 1 or self.n_sessions < 1 or self.requests_per_session < 0:
            raise ConfigurationError("setup_depth and n_sessions must be positive")
        if self.rho <= 0 or self.service_time_s <= 0 or self.arrival_cv < 0:
            raise ConfigurationError("rho and service time must be positive, arrival_cv nonnegative")

    def to_dict(self) -> dict:
        return {name: getattr(self, name) for name in self.__dataclass_fields__}


def setting_id_hash(setting: WorkloadSetting) -> str:
    return hashlib.sha256(canonical_json(setting.to_dict()).encode()).hexdigest()


@dataclass
class TreeNode:
    node_id: str
    parent: str | None
    depth: int                 # chunks on the path including this node
    generation: int            # monotonically increasing per session
    children: list = field(default_factory=list)


class SessionTree:
    """A session's node tree with generation indices."""

    def __init__(self, session_id: str, setup_depth: int):
        self.session_id = session_id
        self.nodes: dict[str, TreeNode] = {}
        self.by_generation: list[str] = []
        parent = None
        for depth in range(1, setup_depth + 1):
            parent = self._add(parent, depth)

    def _add(self, parent: str | None, depth: int) -> str:
        generation = len(self.by_generation) + 1
        node_id = f"{self.session_id}/g{generation}"
        self.nodes[node_id] = TreeNode(node_id, parent, depth, generation)
        if parent is not None:
            self.nodes[parent].children.append(node_id)
        self.by_generation.append(node_id)
        return node_id

    @property
    def latest(self) -> TreeNode:
        return self.nodes[self.by_generation[-1]]

    def node_at_age(self, k: int) -> TreeNode:
        return self.nodes[self.by_generation[len(self.by_generation) - 1 - k]]

    def legal_ages(self, *, min_switch_depth: int, max_depth: int | None) -> list[int]:
        ages = []
        for k in range(1, len(self.by_generation)):
            node = self.node_at_age(k)
            if node.depth >= min_switch_depth and (max_depth is None or node.depth + 1 <= max_depth):
                ages.append(k)
        return ages

    def path(self, node_id: str) -> list[str]:
        out = []
        while node_id is not None:
            out.append(node_id)
            node_id = self.nodes[node_id].parent
        return out[::-1]


def gap_distribution(profile: str, legal_ages: Iterable[int], *, gap_k: int | None = None,
                     recent_mean: float = 2.0) -> tuple[list[int], list[float]]:
    """(support, probabilities) of the positive gap over the request's legal ages."""
    ages = sorted(set(int(a) for a in legal_ages))
    if not ages:
        raise InfeasibleError("no legal historical target")
    if profile == "uniform":
        return ages, [1.0 / len(ages)] * len(ages)
    if profile == "fixed":
        if gap_k not in ages:
            raise InfeasibleError(f"the fixed gap {gap_k} is not a legal age here")
        return [gap_k], [1.0]
    if profile == "recent":
        p = 1.0 / max(recent_mean, 1.0)
        weights = [p * (1.0 - p) ** (a - 1) for a in ages]
    elif profile == "far":
        half = ages[len(ages) // 2:] if len(ages) > 1 else ages
        weights = [1.0 if a in half else 0.0 for a in ages]
    else:
        raise ConfigurationError(f"unknown gap profile {profile!r}")
    total = sum(weights)
    return ages, [w / total for w in weights]


def choose_age(support: Sequence[int], probabilities: Sequence[float], u: float) -> int:
    """Inverse-CDF choice from one uniform."""
    cumulative = 0.0
    for age, p in zip(support, probabilities):
        cumulative += p
        if u <= cumulative:
            return age
    return support[-1]


def rewind_and_generate(tree: SessionTree, k: int, *, min_switch_depth: int, max_depth: int | None) -> str:
    """Generate one child of the node ``k`` generations back (``k = 0``: the latest)."""
    if k < 0 or k >= len(tree.by_generation):
        raise InfeasibleError(f"age {k} does not exist")
    target = tree.node_at_age(k)
    if k > 0 and target.depth < min_switch_depth:
        raise InfeasibleError("the target is shallower than the minimum switch depth")
    if max_depth is not None and target.depth + 1 > max_depth:
        raise InfeasibleError("the child would exceed the maximum depth")
    return tree._add(target.node_id, target.depth + 1)


def plan_session(session_id: str, setting: WorkloadSetting) -> dict[str, Any]:
    """Every request of one session: (target node, age, new node, depth), from the targeting stream."""
    tree = SessionTree(session_id, setting.setup_depth)
    requests = []
    for ordinal in range(setting.requests_per_session):
        stream = Uniforms(setting.seed, "targeting", session_number(session_id), ordinal)
        k = 0
        support: list[int] = []
        if stream.next() < setting.p_historical:
            ages = tree.legal_ages(min_switch_depth=setting.min_switch_depth, max_depth=setting.max_depth)
            support, probabilities = gap_distribution(setting.gap_profile, ages, gap_k=setting.gap_k,
                                                      recent_mean=setting.recent_mean)
            k = choose_age(support, probabilities, stream.next())
        target = tree.node_at_age(k)
        child = rewind_and_generate(tree, k, min_switch_depth=setting.min_switch_depth, max_depth=setting.max_depth)
        requests.append({"ordinal": ordinal, "age": k, "target": target.node_id, "target_depth": target.depth,
                         "target_generation": target.generation, "node": child, "legal_ages": support})
    return {"session": session_id, "tree": tree, "requests": requests}


def open_loop_arrivals(setting: WorkloadSetting, count: int) -> list[float]:
    """Gamma inter-arrivals with mean S / rho and CV ``arrival_cv`` (0: constant spacing)."""
    mean = setting.service_time_s / setting.rho
    stream = Uniforms(setting.seed, "arrivals")
    t, times = 0.0, []
    for _ in range(count):
        if setting.arrival_cv == 0:
            gap = mean
        else:
            shape = 1.0 / (setting.arrival_cv ** 2)
            gap = stream.gamma(shape) * mean / shape
        t += gap
        times.append(t)
    return times


def schedule_requests(setting: WorkloadSetting, session_ids: Sequence[str] | None = None) -> dict[str, Any]:
    """A frozen workload: per-session plans and, for open loop, every request's arrival time and session."""
    session_ids = list(session_ids or [f"s{i:03d}" for i in range(setting.n_sessions)])
    plans = {sid: plan_session(sid, setting) for sid in session_ids}
    schedule = []
    if setting.arrival_mode == "open":
        budget = {sid: setting.requests_per_session for sid in session_ids}
        last = {sid: -math.inf for sid in session_ids}
        choice = Uniforms(setting.seed, "session_choice")
        total = setting.requests_per_session * len(session_ids)
        for at in open_loop_arrivals(setting, total):
            eligible = [sid for sid in session_ids if budget[sid] > 0 and at - last[sid] >= setting.cooldown_s]
            if not eligible:
                raise InfeasibleError(f"no eligible session at t={at:.3f}s (cooldown or budget)")
            sid = eligible[min(len(eligible) - 1, int(choice.next() * len(eligible)))]
            ordinal = setting.requests_per_session - budget[sid]
            budget[sid] -= 1
            last[sid] = at
            schedule.append({"at": at, "session": sid, **{k: v for k, v in plans[sid]["requests"][ordinal].items()
                                                         if k != "legal_ages"}})
    else:
        mean = setting.think_time_mult * setting.service_time_s
        for sid in session_ids:
            for request in plans[sid]["requests"]:
                schedule.append({"session": sid, "think_s": think_seconds(setting.seed, sid, request["ordinal"],
                                                                          mean, setting.think_cv),
                                 **{k: v for k, v in request.items() if k != "legal_ages"}})
    ages = [r["age"] for r in schedule]
    return {"setting": setting.to_dict(), "setting_id": setting_id_hash(setting), "schedule": schedule,
            "summary": {"requests": len(schedule), "historical_fraction": float(np.mean([a > 0 for a in ages]))
                        if ages else 0.0, "mean_age": float(np.mean(ages)) if ages else 0.0}}


__all__ = ["GAP_PROFILES", "InfeasibleError", "SessionTree", "TreeNode", "Uniforms", "WorkloadSetting",
           "choose_age", "gap_distribution", "open_loop_arrivals", "plan_session", "rewind_and_generate",
           "schedule_requests", "setting_id_hash", "think_seconds"]
