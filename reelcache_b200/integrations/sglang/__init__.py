"""Serving bridge (the engine-side counterpart of reference reelcache/integrations/sglang/):
configuration, model profiles, sessions and their controls, archival and restore of session KV.

``create_sglang_backend(config=, pipeline=, server_args=)`` validates the configuration, picks the
model profile and returns a :class:`CausalWanKVBridge` around an engine: ``pipeline`` is a chunk
engine (:class:`CausalWanEngine`, :class:`SyntheticEngine`) or a :class:`CausalWanDiT` with its
encoded text context (``(model, text_kv)``).
"""

from __future__ import annotations

from typing import Any, Mapping

from ...errors import ConfigurationError
from .bridge import CausalWanKVBridge
from .config import ReelCacheRuntimeConfig
from .controls import SessionControlError, session_control
from .engine import CausalWanEngine, SyntheticEngine, model_identity_for
from .profiles import ModelProfile, get_profile, register_profile
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


__all__ = ["CausalWanKVBridge", "CausalWanEngine", "ModelProfile", "ReelCacheRuntimeConfig", "SGLangSessionController",
           "SGLangSessionState", "SessionControlError", "SyntheticEngine", "checkpoint_ref", "create_sglang_backend",
           "get_profile", "register_profile", "session_control"]
