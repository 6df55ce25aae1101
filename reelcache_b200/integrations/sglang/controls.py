"""Typed plain-JSON session controls (the counterpart of reference
reelcache/integrations/sglang/controls.py:120-698): ``capabilities, list, describe, checkpoints,
request, open, pause, checkpoint, fork, rewind, close, delete, gc, raw_tier, acknowledge``. Errors are
:class:`SessionControlError` with an HTTP-like status."""

from __future__ import annotations

from typing import Any, Mapping

from ...errors import CapacityError, ConfigurationError, PendingError, ReelCacheError, StateError

OPS = ("capabilities", "list", "describe", "checkpoints", "request", "open", "pause", "checkpoint", "fork", "rewind",
       "close", "delete", "gc", "raw_tier", "acknowledge")


class SessionControlError(ReelCacheError):
    def __init__(self, code: str, status: int, message: str):
        super().__init__(message)
        self.code = code
        self.status = status

    def to_dict(self) -> dict:
        return {"error": {"code": self.code, "status": self.status, "message": str(self)}}


def _str(payload, name, required=True):
    value = payload.get(name)
    if value is None and not required:
        return None
    if not isinstance(value, str) or not value:
        raise SessionControlError("bad_request", 400, f"{name} must be a nonempty string")
    return value


def session_control(bridge, op: str, payload: Mapping[str, Any] | None = None) -> dict:
    """Run one control operation; returns a JSON-able dict or raises :class:`SessionControlError`."""
    payload = dict(payload or {})
    if op not in OPS:
        raise SessionControlError("unknown_op", 404, f"unknown control {op!r}; supported: {OPS}")
    sessions = bridge.sessions
    try:
        if op == "capabilities":
            return {"ops": list(OPS), "profile": bridge.profile.name, "representation": bridge.config.representation,
                    "durability": bridge.config.durability, "raw_tier": bridge.archive.raw_tier is not None,
                    "device": str(bridge.device)}
        if op == "list":
            return {"sessions": sessions.sessions()}
        if op in ("describe", "open"):
            sid = _str(payload, "session")
            state = sessions.get(sid)
            sessions.reconcile(state)
            return {**state.describe(), "head": sessions.head(sid),
                    "published_chunks": len(sessions.chunks(sid))}
        if op == "checkpoints":
            return {"checkpoints": sessions.checkpoints(_str(payload, "session"))}
        if op == "request":
            report = bridge.request(_str(payload, "session"), chunks=int(payload.get("chunks", 1)),
                                    action=payload.get("action", "resume"), checkpoint=payload.get("checkpoint"),
                                    source=payload.get("source"), seed=int(payload.get("seed", 0)),
                                    prompt=payload.get("prompt"), request_id=payload.get("request_id"))
            report.pop("latents", None)
            return report
        if op == "pause":
            return sessions.pause(_str(payload, "session"), timeout=payload.get("timeout"))
        if op == "checkpoint":
            return sessions.checkpoint(_str(payload, "session"), payload.get("name"), timeout=payload.get("timeout"),
                                       replace=bool(payload.get("replace", False)))
        if op == "fork":
            state = sessions.fork(_str(payload, "source"), _str(payload, "session"),
                                  checkpoint=payload.get("checkpoint"))
            return state.describe()
        if op == "rewind":
            if "checkpoint" not in payload:
                raise SessionControlError("bad_request", 400, "rewind needs a checkpoint")
            return sessions.rewind(_str(payload, "session"), payload["checkpoint"]).describe()
        if op == "close":
            return sessions.close(_str(payload, "session"))
        if op == "delete":
            return sessions.close(_str(payload, "session"), delete=True)
        if op == "gc":
            return sessions.gc()
        if op == "acknowledge":
            return sessions.acknowledge(_str(payload, "session"))
        if op == "raw_tier":
            tier = bridge.archive.raw_tier
            return {"enabled": tier is not None, **({} if tier is None else tier.stats())}
    except SessionControlError:
        raise
    except ConfigurationError as error:
        raise SessionControlError("bad_request", 400, str(error)) from error
    except PendingError as error:
        raise SessionControlError("busy", 409, str(error)) from error
    except CapacityError as error:
        raise SessionControlError("capacity", 503, str(error)) from error
    except StateError as error:
        code, status = ("not_found", 404) if "unknown session" in str(error) else ("conflict", 409)
        raise SessionControlError(code, status, str(error)) from error
    raise SessionControlError("unknown_op", 404, op)  # pragma: no cover
