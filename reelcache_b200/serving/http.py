"""The HTTP surface of a serving bridge (the counterpart of the reference's ``/v1/videos`` and ``/v1/sessions/*``
routes, docs/usage.md:49-79): generation requests carry a ``causal_kv_session`` handle, and session controls need
no generation. Requests run one at a time per bridge (a concurrent one answers 409); no endpoint takes a
filesystem path.

``create_app(bridge)`` returns a FastAPI application; ``python -m reelcache_b200.serving.http --help`` serves one
over a synthetic-engine bridge for local use.
"""

from __future__ import annotations

import uuid
from typing import Any

from ..errors import ConfigurationError, PendingError, ReelCacheError, StateError, UnsupportedError

#: Handle keys a generation request may carry.
HANDLE_KEYS = ("session_id", "action", "from_session", "checkpoint", "pause_after_chunks", "durable", "output",
               "overlap_restore", "replace")
_ACTIONS = {"generate": "create", "resume": "resume", "fork": "fork", "rewind": "rewind"}


def _status(error: BaseException) -> int:
    from ..integrations.sglang.controls import SessionControlError
    if isinstance(error, SessionControlError):
        return error.status
    if isinstance(error, PendingError):
        return 409
    if isinstance(error, (ConfigurationError, UnsupportedError)):
        return 400
    if isinstance(error, StateError):
        return 404 if "unknown session" in str(error) else 409
    return 500


def _plain(summary: dict) -> dict:
    """A JSON-able summary: tensors become their shapes."""
    out = {}
    for key, value in summary.items():
        if hasattr(value, "shape") and hasattr(value, "dtype"):
            out[key] = {"shape": list(value.shape), "dtype": str(value.dtype).removeprefix("torch.")}
        else:
            out[key] = value
    return out


def generation_request(bridge, body: dict) -> dict:
    """Run one ``POST /v1/videos`` body through the bridge; returns the request summary."""
    handle = dict(body.get("causal_kv_session") or {})
    unknown = set(handle) - set(HANDLE_KEYS)
    if unknown:
        raise ConfigurationError(f"unknown causal_kv_session keys {sorted(unknown)}")
    if "session_id" not in handle:
        raise ConfigurationError("causal_kv_session needs a session_id")
    action = _ACTIONS.get(handle.get("action", "generate"))
    if action is None:
        raise ConfigurationError(f"action must be one of {sorted(_ACTIONS)}")
    if action == "create" and handle.get("replace"):
        state = bridge.sessions.get(handle["session_id"], required=False)
        if state is not None:
            bridge.close(handle["session_id"], delete=True)
    request_id = body.get("request_id") or f"video-{uuid.uuid4().hex[:12]}"
    summary = bridge.request(handle["session_id"], chunks=int(body.get("num_chunks", 1)), action=action,
                             checkpoint=handle.get("checkpoint"), source=handle.get("from_session"),
                             seed=int(body.get("seed", 0)), prompt=body.get("prompt"), request_id=request_id,
                             overlap_restore=handle.get("overlap_restore"),
                             pause_after_chunks=handle.get("pause_after_chunks"))
    if handle.get("durable"):
        summary["durable"] = bridge.pause(handle["session_id"])
    summary["output"] = handle.get("output", "new")
    return _plain(summary)


def create_app(bridge):
    """The FastAPI application serving ``bridge``."""
    from fastapi import Body, FastAPI
    from fastapi.responses import JSONResponse

    from ..integrations.sglang.controls import session_control

    app = FastAPI(title="reelcache-b200")

    def answer(call):
        try:
            return call()
        except ReelCacheError as error:
            return JSONResponse({"error": type(error).__name__, "message": str(error)}, status_code=_status(error))

    def control(op: str, payload: dict | None = None):
        return answer(lambda: session_control(bridge, op, payload or {}))

    @app.post("/v1/videos")
    def videos(body: dict = Body(...)):
        return answer(lambda: generation_request(bridge, body))

    @app.get("/v1/sessions")
    def sessions():
        return control("list")

    @app.get("/v1/sessions/{session_id}")
    def describe(session_id: str):
        return control("describe", {"session": session_id})

    @app.delete("/v1/sessions/{session_id}")
    def delete(session_id: str):
        return control("delete", {"session": session_id})

    @app.get("/v1/sessions/{session_id}/checkpoints")
    def checkpoints(session_id: str):
        return control("checkpoints", {"session": session_id})

    @app.post("/v1/sessions/{session_id}/checkpoints")
    def checkpoint(session_id: str, body: dict | None = Body(None)):
        return control("checkpoint", {"session": session_id, **(body or {})})

    @app.get("/v1/sessions/{session_id}/raw_tier")
    def raw_tier(session_id: str):
        return control("raw_tier", {"session": session_id})

    @app.post("/v1/sessions/{session_id}/{op}")
    def session_op(session_id: str, op: str, body: dict | None = Body(None)):
        payload = dict(body or {})
        if op not in ("open", "pause", "fork", "rewind", "close", "acknowledge"):
            return JSONResponse({"error": "unknown_op", "message": op}, status_code=404)
        if op == "fork":
            payload.setdefault("source", session_id)
            return control("fork", payload)
        payload["session"] = session_id
        return control(op, payload)

    @app.get("/v1/session_capabilities")
    def capabilities():
        return control("capabilities")

    @app.get("/v1/session_requests/{request_id}")
    def request_summary(request_id: str):
        summary = bridge.request_summary(request_id)
        if summary is None:
            return JSONResponse({"error": "not_found", "message": request_id}, status_code=404)
        return _plain(summary)

    @app.post("/v1/session_gc")
    def gc():
        return control("gc")

    return app


def main(argv=None) -> None:
    import argparse

    import uvicorn

    from ..integrations.sglang import ReelCacheRuntimeConfig, SyntheticEngine, create_sglang_backend, get_profile
    from ..integrations.sglang.engine import model_identity_for
    parser = argparse.ArgumentParser(description="serve a synthetic-engine bridge over HTTP")
    parser.add_argument("--store", required=True)
    parser.add_argument("--profile", default="causvid")
    parser.add_argument("--host", default="127.0.0.1")
    parser.add_argument("--port", type=int, default=8000)
    args = parser.parse_args(argv)
    profile = get_profile(args.profile)
    engine = SyntheticEngine(profile, model_identity_for(profile, "synthetic"), "cpu")
    bridge = create_sglang_backend(ReelCacheRuntimeConfig(store_root=args.store, fit_device="cpu"), engine)
    try:
        uvicorn.run(create_app(bridge), host=args.host, port=args.port)
    finally:
        bridge.shutdown()


if __name__ == "__main__":
    main()
