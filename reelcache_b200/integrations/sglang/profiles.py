"""Model profiles of the serving bridge: per-model geometry, attention-visibility policy, capture
dtypes and energy targets as plain data (the counterpart of reference
reelcache/integrations/sglang/profiles.py:51-334 and causal_wan/profiles.py).

Built in: the three Wan2.1-1.3B causal profiles (CausVid, LongLive 1.0, RAVEN: 30 layers, 12 x 128
heads, 3-latent-frame chunks, 480p -> 30 x 52 tokens per frame) and LongLive 2.0. ``register_profile``
adds more (e.g. a LongCat-Video profile).
"""

from __future__ import annotations

import threading
from dataclasses import asdict, dataclass, field
from typing import Any, Mapping

from ...errors import ConfigurationError

VISIBILITIES = ("full_history", "sink_window")


@dataclass(frozen=True)
class ModelProfile:
    name: str
    backbone: str
    num_layers: int
    num_heads: int
    head_dim: int
    chunk_frames: int
    grid: tuple[int, int]                 # tokens per latent frame: (rows, columns)
    visibility: str                       # full_history | sink_window
    sink_frames: int
    window_frames: int | None             # KV buffer length in latent frames (sink included); None: full
    energy_profile: str
    native_dtype: str = "bfloat16"
    rope: str = "wan_3d"
    cfg_streams: tuple[str, ...] = ("cond",)
    recache: str = "none"
    capture_dtypes: Mapping[str, str] | None = None
    timesteps: tuple[float, ...] = (1000.0, 757.0, 522.0)
    defaults: Mapping[str, Any] = field(default_factory=dict)

    def __post_init__(self) -> None:
        if not self.name or self.visibility not in VISIBILITIES:
            raise ConfigurationError(f"profile needs a name and a visibility in {VISIBILITIES}")
        for value in (self.num_layers, self.num_heads, self.head_dim, self.chunk_frames, *self.grid):
            if type(value) is not int or value < 1:
                raise ConfigurationError("profile geometry must be positive integers")
        if self.visibility == "sink_window" and (self.window_frames is None or self.window_frames <= self.sink_frames):
            raise ConfigurationError("sink_window profiles need window_frames > sink_frames")
        object.__setattr__(self, "grid", tuple(self.grid))
        object.__setattr__(self, "cfg_streams", tuple(self.cfg_streams))
        object.__setattr__(self, "timesteps", tuple(self.timesteps))

    @property
    def channels(self) -> int:
        return self.num_heads * self.head_dim

    @property
    def tokens_per_frame(self) -> int:
        return self.grid[0] * self.grid[1]

    @property
    def chunk_tokens(self) -> int:
        return self.chunk_frames * self.tokens_per_frame

    def capture_dtype(self, target: str) -> str:
        return (self.capture_dtypes or {}).get(target, self.native_dtype)

    def to_dict(self) -> dict:
        data = asdict(self)
        data["grid"] = list(self.grid)
        data["cfg_streams"] = list(self.cfg_streams)
        data["timesteps"] = list(self.timesteps)
        return data

    @classmethod
    def from_dict(cls, data: Mapping[str, Any]) -> "ModelProfile":
        values = dict(data)
        values["grid"] = tuple(values.get("grid", ()))
        values["cfg_streams"] = tuple(values.get("cfg_streams", ("cond",)))
        values["timesteps"] = tuple(values.get("timesteps", (1000.0, 757.0, 522.0)))
        return cls(**values)


_WAN = dict(backbone="wan2.1-t2v-1.3b", num_layers=30, num_heads=12, head_dim=128, chunk_frames=3, grid=(30, 52))
_REGISTRY: dict[str, ModelProfile] = {}
_LOCK = threading.Lock()


def register_profile(profile: ModelProfile | Mapping[str, Any], *, replace: bool = False) -> ModelProfile:
    if not isinstance(profile, ModelProfile):
        profile = ModelProfile.from_dict(profile)
    with _LOCK:
        if profile.name in _REGISTRY and not replace:
            raise ConfigurationError(f"profile {profile.name!r} is already registered")
        _REGISTRY[profile.name] = profile
    return profile


def get_profile(name: str) -> ModelProfile:
    try:
        return _REGISTRY[name]
    except KeyError:
        raise ConfigurationError(f"unknown model profile {name!r}; registered: {sorted(_REGISTRY)}") from None


def profiles() -> dict[str, ModelProfile]:
    return dict(_REGISTRY)


register_profile(ModelProfile("causvid", visibility="full_history", sink_frames=0, window_frames=None,
                              energy_profile="causvid", **_WAN))
register_profile(ModelProfile("longlive", visibility="sink_window", sink_frames=3, window_frames=21,
                              energy_profile="longlive1", recache="kv_recache", **_WAN))
register_profile(ModelProfile("raven", visibility="full_history", sink_frames=0, window_frames=None,
                              energy_profile="raven", capture_dtypes={"K": "float32", "V": "bfloat16"}, **_WAN))
register_profile(ModelProfile("longlive2", backbone="wan2.1-t2v-1.3b", num_layers=30, num_heads=12, head_dim=128,
                              chunk_frames=3, grid=(30, 52), visibility="sink_window", sink_frames=3, window_frames=21,
                              energy_profile="longlive2", recache="kv_recache"))
