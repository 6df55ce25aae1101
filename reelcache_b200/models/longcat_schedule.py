"""Distilled LongCat-Video continuation schedule (reference counterpart:
reelcache_sglang_models/longcat_video/schedule.py).

The distilled checkpoint samples ``n`` of the ``S = 50`` distillation steps of ``T = 1000`` training timesteps:
distillation step ``k`` (1..S) sits at timestep ``k * (T // S)``; taken from the noisiest down, the inference
steps use every ``S / n``-th of them (``floor`` of ``n`` evenly spaced positions in ``[0, S)``). Each sigma
``t / T`` is then shifted for the flow-matching Euler scheduler, ``s' = shift s / (1 + (shift - 1) s)`` with the
checkpoint's ``shift = 12``; the timesteps fed to the DiT are ``s' T`` and a terminal sigma 0 closes the list.
The values must be those of the native pipeline bit for bit (its scheduler state is what a resumed session
continues), so the spacing uses the same ``numpy.linspace`` evaluation and FP32 arithmetic.
"""

from __future__ import annotations

import numpy as np
import torch


def distill_sigmas(num_inference_steps: int = 16, num_train_timesteps: int = 1000,
                   num_distill_sample_steps: int = 50) -> torch.Tensor:
    """FP32 sigmas of the sampled distillation steps, noisiest first, before the shift."""
    steps, train, distill = num_inference_steps, num_train_timesteps, num_distill_sample_steps
    if not (isinstance(steps, int) and 0 < steps <= distill):
        raise ValueError(f"num_inference_steps {steps!r} must be an int in [1, {distill}]")
    stride = train // distill
    positions = np.floor(np.linspace(0, distill, num=steps, endpoint=False)).astype(np.int64)
    timesteps = (distill - positions) * stride          # distillation step distill - p, noisiest first
    return torch.from_numpy(timesteps.astype(np.float32) / np.float32(train))


def shift_sigmas(sigmas, shift: float = 12.0) -> np.ndarray:
    """The static flow shift ``shift s / (1 + (shift - 1) s)`` in FP32."""
    s = np.asarray(sigmas, dtype=np.float32)
    return shift * s / (1 + (shift - 1) * s)


def continuation_schedule(num_inference_steps: int = 16, shift: float = 12.0, num_train_timesteps: int = 1000,
                          num_distill_sample_steps: int = 50, device=None) -> tuple[torch.Tensor, torch.Tensor]:
    """``(timesteps [n], sigmas [n + 1])`` FP32 on ``device``, the terminal sigma 0 appended."""
    shifted = torch.from_numpy(shift_sigmas(distill_sigmas(num_inference_steps, num_train_timesteps,
                                                           num_distill_sample_steps), shift))
    sigmas = shifted.to(device=device, dtype=torch.float32)
    return sigmas * num_train_timesteps, torch.cat([sigmas, sigmas.new_zeros(1)])


def euler_step(model_output: torch.Tensor, sample: torch.Tensor, sigma: torch.Tensor,
               sigma_next: torch.Tensor) -> torch.Tensor:
    """One deterministic flow-matching Euler step ``x + (sigma_next - sigma) v``, in FP32, cast to the model
    output's dtype."""
    return (sample.float() + (sigma_next - sigma) * model_output).to(model_output.dtype)


def dit_timestep(t: torch.Tensor, batch: int, frames: int, dtype: torch.dtype) -> torch.Tensor:
    """The per-frame timestep tensor ``[batch, frames]`` the native DiT takes (``t`` in the DiT dtype)."""
    return t.reshape(()).to(dtype).expand(batch, frames).contiguous()


__all__ = ["continuation_schedule", "distill_sigmas", "dit_timestep", "euler_step", "shift_sigmas"]
