"""ReelCache-B200: immutable, compressed clean-chunk KV state for autoregressive video diffusion,
rebuilt for NVIDIA B200 (sm_100a).

Every generated chunk's clean (t = 0) self-attention K/V is archived as a low-rank, 8-bit-quantized,
content-addressed node in a per-session tree; any committed node can be resumed, rewound to or
forked from by restoring its history straight into the engine's KV cache. The hot paths are
hand-written CUDA kernels for sm_100a (``reelcache_b200.ops``); the runtime around them (store,
lineages, pipelines, sessions) keeps the reference's public API and on-disk format.
"""

__version__ = "0.1.0"

__all__ = [
    "__version__", "RankPolicy", "RankDecision", "RankState",
    "RankPreparation", "PreparedRankMatrix", "RankAbstention",
]


def __getattr__(name):
    if name in __all__ and name != "__version__":
        from . import online_rank
        return getattr(online_rank, name)
    raise AttributeError(f"module {__name__!r} has no attribute {name!r}")
