"""LingBot-World-Fast integration: the world model's KV history archived and restored through this package's
lineage runtime, with the restore layer-overlapped with the next chunk's first forward.

LingBot-World-Fast (an image-to-video world model with camera control on the Wan2.2 A14B geometry) keeps one
persistent self-attention cache: each chunk of 3 latent frames is written once by a clean pass and never
recomputed. This package wraps any pipeline with that shape (reference: integrations/lingbot/README.md:1-41):

* :mod:`.geometry` -- the model geometry and its store identity;
* :mod:`.model` -- :class:`ChunkKV` hooks capturing a chunk's pre-RoPE K and V from its clean pass and
  installing restored rows, the shared window cache, and :class:`StandInWorldModel`, a small model of the same
  interface that runs on CPU or GPU without the official weights;
* :mod:`.archive` -- :class:`LingBotArchive`: one lineage node per chunk, a fork when a session rewinds,
  asynchronous publication, synchronous or layer-overlapped restores;
* :mod:`.overlap` -- :class:`OverlapSession` (forward pre-hooks on ``blocks[l].self_attn`` wait for layer
  ``l``) and :class:`StallEvents` (per-layer stall and restore-window events).
"""

from .archive import ArchiveError, LingBotArchive, REPRESENTATIONS
from .geometry import LINGBOT_WORLD_FAST, LingBotGeometry
from .model import ChunkKV, SharedWindowCache, StandInWorldModel
from .overlap import OverlapSession, StallEvents

__all__ = ["ArchiveError", "ChunkKV", "LINGBOT_WORLD_FAST", "LingBotArchive", "LingBotGeometry", "OverlapSession",
           "REPRESENTATIONS", "SharedWindowCache", "StallEvents", "StandInWorldModel"]
