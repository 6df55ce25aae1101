"""LongCat-Video LoRA branches (reference counterpart: reelcache_sglang_models/longcat_video/lora.py).

A LoRA adds ``multiplier * alpha * up(down(x))`` to the output of one linear layer without touching its weights
(merging into the bf16 weights would change their rounding). ``up`` may be split into ``n`` blocks applied to
``n`` equal slices of ``down(x)`` and concatenated (the fused QKV projection uses 3, the cross-attention KV
projection 2). Branches are stored per block of :class:`~reelcache_b200.models.longcat.LongCatDiT` under the
weight names of that block (``qkv``, ``proj``, ``cq``, ``ckv``, ``cproj``, ``w1``, ``w2``, ``w3``); every
projection of the forward passes through :func:`apply_branches`.

The state-dict format is the native checkpoint's (interface): ``<name>.lora_down.weight`` ``[r, in]``, either
``<name>.lora_up.weight`` ``[out, r]`` or ``<name>.lora_up.blocks.<i>.weight`` ``[out_i, r / n]``, and
``<name>.alpha_scale``; ``<name>`` is the module path with ``.`` spelled ``___lorahyphen___`` behind the prefix
``lora___lorahyphen___``.
"""

from __future__ import annotations

import re
from collections import OrderedDict
from dataclasses import dataclass, field
from typing import Mapping

import torch

LORA_PREFIX = "lora___lorahyphen___"
LORA_HYPHEN = "___lorahyphen___"

#: native module path inside a transformer block -> the weight name of a LongCatDiT block
NATIVE_TARGETS = {"attn.qkv": "qkv", "attn.proj": "proj", "cross_attn.q_linear": "cq",
                  "cross_attn.kv_linear": "ckv", "cross_attn.proj": "cproj", "ffn.w1": "w1", "ffn.w2": "w2",
                  "ffn.w3": "w3"}
_BLOCK_PATH = re.compile(r"^blocks\.(\d+)\.(.+)$")


@dataclass
class LoRABranch:
    """One additive branch: ``down`` ``[r, in]``, ``ups`` (``[out_i, r / n]`` each), FP32 ``alpha``."""

    name: str
    down: torch.Tensor
    ups: tuple
    alpha: float
    multiplier: float = 1.0
    enabled: bool = True
    _up_cat: torch.Tensor | None = field(default=None, repr=False)

    @property
    def in_features(self) -> int:
        return int(self.down.shape[1])

    @property
    def out_features(self) -> int:
        return int(sum(u.shape[0] for u in self.ups))

    def delta(self, x: torch.Tensor, linear) -> torch.Tensor:
        """``multiplier * alpha * up(down(x))`` in FP32 (``linear(x, w)`` is the model's GEMM)."""
        low = linear(x.to(self.down.dtype), self.down)
        if len(self.ups) == 1:
            high = linear(low, self.ups[0], out_dtype=torch.float32)
        else:
            parts = low.chunk(len(self.ups), dim=-1)
            high = torch.cat([linear(p.contiguous(), u, out_dtype=torch.float32) for p, u in zip(parts, self.ups)],
                             dim=-1)
        return high * (self.multiplier * self.alpha)


def module_name(lora_name: str) -> str:
    """Native module path of a LoRA key stem (``lora___lorahyphen___blocks___lorahyphen___0...`` -> ``blocks.0...``)."""
    return lora_name.replace(LORA_PREFIX, "", 1).replace(LORA_HYPHEN, ".")


def parse_state_dict(state_dict: Mapping[str, torch.Tensor]) -> "OrderedDict[str, tuple]":
    """``{module path: (down, ups, alpha)}`` of a native LoRA state dict; every key must belong to a branch."""
    stems = sorted(key[:-len(".lora_down.weight")] for key in state_dict if key.endswith(".lora_down.weight"))
    used: set[str] = set()
    parsed: "OrderedDict[str, tuple]" = OrderedDict()
    for stem in stems:
        down_key, alpha_key = f"{stem}.lora_down.weight", f"{stem}.alpha_scale"
        block_keys = [key for key in state_dict if key.startswith(f"{stem}.lora_up.blocks.")]
        if block_keys:
            count = len(block_keys)
            wanted = [f"{stem}.lora_up.blocks.{i}.weight" for i in range(count)]
            if sorted(block_keys) != sorted(wanted):
                raise ValueError(f"LoRA {stem}: up blocks {sorted(block_keys)} are not 0..{count - 1}")
            up_keys = wanted
        else:
            up_keys = [f"{stem}.lora_up.weight"]
            if up_keys[0] not in state_dict:
                raise ValueError(f"LoRA {stem} has no {up_keys[0]}")
        if alpha_key not in state_dict:
            raise ValueError(f"LoRA {stem} has no {alpha_key}")
        down, ups = state_dict[down_key], tuple(state_dict[key] for key in up_keys)
        consistent = down.ndim == 2 and all(u.ndim == 2 and u.shape[1] * len(ups) == down.shape[0] for u in ups)
        if not consistent:
            raise ValueError(f"LoRA {stem}: down {tuple(down.shape)} does not feed ups {[tuple(u.shape) for u in ups]}")
        path = module_name(stem)
        if path in parsed:
            raise ValueError(f"two LoRA stems target {path}")
        parsed[path] = (down, ups, float(torch.as_tensor(state_dict[alpha_key]).float().reshape(())))
        used.update((down_key, alpha_key, *up_keys))
    unused = sorted(set(state_dict) - used)
    if unused:
        raise ValueError(f"{len(unused)} keys belong to no LoRA branch, e.g. {unused[:4]}")
    return parsed


def attach(blocks, state_dict: Mapping[str, torch.Tensor], *, multiplier: float = 1.0, dtype=torch.bfloat16,
           device=None) -> list[str]:
    """Attach the branches of ``state_dict`` to the matching LongCatDiT ``blocks`` (each target once); returns
    the module paths attached."""
    attached = []
    for path, (down, ups, alpha) in parse_state_dict(state_dict).items():
        found = _BLOCK_PATH.match(path)
        target = NATIVE_TARGETS.get(found.group(2)) if found else None
        if target is None or int(found.group(1)) >= len(blocks):
            raise ValueError(f"LoRA target {path} is not a projection of this model")
        blk = blocks[int(found.group(1))]
        weight = blk[f"{target}_w" if f"{target}_w" in blk else target]
        out_features, in_features = weight.shape
        if down.shape[1] != in_features or sum(u.shape[0] for u in ups) != out_features:
            raise ValueError(f"LoRA {path}: {down.shape[1]} -> {sum(u.shape[0] for u in ups)} does not match the "
                             f"projection's {in_features} -> {out_features}")
        branches = blk.setdefault("lora", {})
        if target in branches:
            raise ValueError(f"LoRA target {path} already has a branch")
        device = device or weight.device
        branches[target] = [LoRABranch(path, down.to(device=device, dtype=dtype).contiguous(),
                                       tuple(u.to(device=device, dtype=dtype).contiguous() for u in ups),
                                       alpha, float(multiplier))]
        attached.append(path)
    return attached


def apply_branches(blk: dict, target: str, x: torch.Tensor, out: torch.Tensor, linear) -> torch.Tensor:
    """``out`` plus the enabled branches of ``blk[target]`` evaluated on ``x`` (``out`` unchanged without any)."""
    branches = [b for b in blk.get("lora", {}).get(target, ()) if b.enabled]
    if not branches:
        return out
    total = out.float()
    for branch in branches:
        total = total + branch.delta(x, linear)
    return total.to(out.dtype)


def detach(blocks) -> int:
    """Remove every branch; returns how many were attached."""
    count = 0
    for blk in blocks:
        count += sum(len(v) for v in blk.pop("lora", {}).values())
    return count


def set_enabled(blocks, enabled: bool) -> None:
    for blk in blocks:
        for branches in blk.get("lora", {}).values():
            for branch in branches:
                branch.enabled = bool(enabled)


__all__ = ["LORA_HYPHEN", "LORA_PREFIX", "LoRABranch", "NATIVE_TARGETS", "apply_branches", "attach", "detach",
           "module_name", "parse_state_dict", "set_enabled"]
