"""Clean-chunk capture: per-layer pre-RoPE K and V of each CFG stream gathered into the canonical
``[tokens, channels]`` matrices of one commit, with their contexts (the counterpart of reference
reelcache/integrations/sglang/capture.py:25 and commit.py:20-53)."""

from __future__ import annotations

from typing import Any

import torch

from ...errors import ConfigurationError, StateError
from ...types import MatrixKey, ModelIdentity, TensorContext


class CleanChunkBuilder:
    def __init__(self, model: ModelIdentity, chunk_index: int, token_start: int, frames: int, height: int, width: int,
                 streams: tuple[str, ...] = ("cond",), key_space: str = "pre_rope"):
        self.model = model
        self.chunk_index = chunk_index
        self.token_start = token_start
        self.geometry = (frames, height, width)
        self.streams = tuple(streams)
        self.key_space = key_space
        self.matrices: dict[Any, torch.Tensor] = {}
        self._sealed = False

    def entry(self, layer: int, target: str, stream: str):
        key = MatrixKey(layer, target)
        return key if len(self.streams) == 1 else (key, stream)

    def capture_layer(self, layer: int, k_pre: torch.Tensor, v: torch.Tensor, stream: str = "cond") -> None:
        if self._sealed:
            raise StateError("chunk already sealed")
        if stream not in self.streams:
            raise ConfigurationError(f"unknown CFG stream {stream!r}")
        tokens = self.geometry[0] * self.geometry[1] * self.geometry[2]
        for target, tensor in (("K", k_pre), ("V", v)):
            matrix = tensor.reshape(tokens, -1)
            if matrix.shape[1] != self.model.channels_for(target):
                raise ConfigurationError("captured matrix width differs from the model's KV channels")
            self.matrices[self.entry(layer, target, stream)] = matrix

    def complete(self) -> bool:
        return len(self.matrices) == 2 * self.model.layers * len(self.streams)

    def seal(self) -> tuple[dict, dict]:
        if not self.complete():
            raise StateError("chunk capture is missing layers")
        self._sealed = True
        frames, height, width = self.geometry
        contexts = {}
        for entry in self.matrices:
            key = entry if isinstance(entry, MatrixKey) else entry[0]
            contexts[entry] = TensorContext(self.model, key, self.token_start, frames, height, width,
                                            self.key_space if key.target == "K" else "none")
        return dict(self.matrices), contexts
