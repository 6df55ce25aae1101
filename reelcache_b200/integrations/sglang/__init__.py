"""Serving bridge (the engine-side counterpart of reference reelcache/integrations/sglang/):
configuration, model profiles, sessions and their controls, archival and restore of session KV.

``create_sglang_backend(config=, pipeline=, server_args=)`` validates the configuration, picks the
model profile and returns a :class:`CausalWanKVBridge` around an engine: ``pipeline`` is a chunk
engine (:class:`CausalWanEngine`, :class:`SyntheticEngine`) or a :class:`CausalWanDiT` with its
encoded text context (``(model, text_kv)``). An engine drives each request through the bridge's seam
(:mod:`.seam`: ``begin_request`` / ``restore`` / capture / ``end_chunk`` / ``finish``); ``bridge.request`` is that
loop over the bridge's own engine.
"""

from __future__ import annotations

from typing import Any, Mapping

from ...errors import ConfigurationError
from .bridge import CausalWanKVBridge, PlanCache, ResidentKV
from .config import ReelCacheRuntimeConfig
from .controls import SessionControlError, session_control
from .engine import CausalWanEngine, SyntheticEngine, model_identity_for
from .profiles import ModelProfile, get_profile, register_profile
from .seam import (CausalKVRequest, CaptureScope, ChunkSlot, KVRecache, RecachePlan, RestoreTarget, drive_request,
                   plan_recache)
from .session import SGLangSessionController, SGLangSessionState, checkpoint_ref


def create_sglang_backend(config: ReelCacheRuntimeConfig | Mapping[str, Any], pipeline: Any = None,
                          server_args: Any = None, **kwargs) -> CausalWanKVBridge:
    if not isinstance(config, ReelCacheRuntimeConfig):
        config = ReelCacheRuntimeConfig.from_dict(config)
    if pipeline is None:
        raise ConfigurationError("create_sglang_backend needs a pipeline (engine or (model, text_kv))")
    if config.profile_fields is not None:
        profile = ModelProfile.from_dict(config.profile_fields)
    elif config.profile is None and getattr(pipeline, "profile", None) is not None:
        profile = pipeline.profile  # an engine carries its own profile
    else:
        profile = get_profile(config.profile or getattr(server_args, "reelcache_profile", None) or "causvid")
    if isinstance(pipeline, tuple):
        model, text_kv = pipeline
        identity = model_identity_for(profile, f"random-init-seed{getattr(model, 'seed', 0)}")
        engine = CausalWanEngine(model, text_kv, profile, identity)
    else:
        engine = pipeline
    return CausalWanKVBridge(config, engine, profile, **kwargs)


__all__ = ["CaptureScope", "CausalKVRequest", "CausalWanKVBridge", "CausalWanEngine", "ChunkSlot", "KVRecache",
           "ModelProfile", "PlanCache", "RecachePlan", "ReelCacheRuntimeConfig", "ResidentKV", "RestoreTarget",
           "SGLangSessionController", "SGLangSessionState", "SessionControlError", "SyntheticEngine", "checkpoint_ref",
           "create_sglang_backend", "drive_request", "get_profile", "plan_recache", "register_profile",
           "session_control"]
