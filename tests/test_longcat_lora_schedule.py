"""LongCat LoRA branches (native state-dict format, additive branches evaluated beside the frozen weights) and the
distilled continuation schedule (checked against the installed reference module when present)."""

import importlib
import os
import sys

import numpy as np
import pytest
import torch

from .test_longcat import _inputs, _model

STEM = "lora___lorahyphen___blocks___lorahyphen___{layer}___lorahyphen___{path}"


def _lora_state(model, layer, path, rank, blocks, seed=0):
    g = torch.Generator().manual_seed(seed)
    from reelcache_b200.models.longcat_lora import NATIVE_TARGETS
    blk = model.blocks[layer]
    name = NATIVE_TARGETS[path]
    out_f, in_f = blk[f"{name}_w" if f"{name}_w" in blk else name].shape
    stem = STEM.format(layer=layer, path=path.replace(".", "___lorahyphen___"))
    state = {f"{stem}.lora_down.weight": torch.randn(rank, in_f, generator=g) * 0.1,
             f"{stem}.alpha_scale": torch.tensor(0.5)}
    if blocks == 1:
        state[f"{stem}.lora_up.weight"] = torch.randn(out_f, rank, generator=g) * 0.1
    else:
        for i in range(blocks):
            state[f"{stem}.lora_up.blocks.{i}.weight"] = torch.randn(out_f // blocks, rank // blocks, generator=g) * 0.1
    return state


def test_lora_parse_attach_and_forward_delta():
    from reelcache_b200.models import longcat_lora

    model = _model()
    latents, text = _inputs(model)
    base = model.forward(latents, 0.5, text)
    state = {**_lora_state(model, 0, "attn.qkv", 12, 3), **_lora_state(model, 1, "ffn.w2", 8, 1, seed=1),
             **_lora_state(model, 1, "cross_attn.kv_linear", 8, 2, seed=2)}
    parsed = longcat_lora.parse_state_dict(state)
    assert list(parsed) == ["blocks.0.attn.qkv", "blocks.1.cross_attn.kv_linear", "blocks.1.ffn.w2"]
    assert len(parsed["blocks.0.attn.qkv"][1]) == 3 and parsed["blocks.0.attn.qkv"][2] == 0.5
    assert sorted(model.attach_lora(state, multiplier=2.0)) == sorted(parsed)
    with pytest.raises(ValueError):
        model.attach_lora(state)                      # a target takes one branch
    # the branch is exactly multiplier * alpha * up(down(x)), split-up blocks on equal slices
    branch = model.blocks[0]["lora"]["qkv"][0]
    x = torch.randn(5, branch.in_features).to(torch.bfloat16)
    low = x.float() @ branch.down.float().t()
    expect = torch.cat([c @ u.float().t() for c, u in zip(low.to(torch.bfloat16).float().chunk(3, -1), branch.ups)], -1)
    got = branch.delta(x, model.ops.linear)
    assert torch.allclose(got, expect * 2.0 * 0.5, atol=1e-2, rtol=1e-2)
    with_lora = model.forward(latents, 0.5, text)
    assert not torch.allclose(with_lora, base)
    model.set_loras_enabled(False)
    assert torch.equal(model.forward(latents, 0.5, text), base)
    model.set_loras_enabled(True)
    assert model.detach_loras() == 3
    assert torch.equal(model.forward(latents, 0.5, text), base)


def test_lora_state_dict_errors():
    from reelcache_b200.models import longcat_lora

    model = _model()
    state = _lora_state(model, 0, "attn.proj", 4, 1)
    with pytest.raises(ValueError):
        longcat_lora.parse_state_dict({**state, "stray.weight": torch.zeros(1)})
    broken = dict(state)
    del broken[[k for k in broken if k.endswith("alpha_scale")][0]]
    with pytest.raises(ValueError):
        longcat_lora.parse_state_dict(broken)
    wrong = {k.replace("attn___lorahyphen___proj", "attn___lorahyphen___nothing"): v for k, v in state.items()}
    with pytest.raises(ValueError):
        model.attach_lora(wrong)


def test_distilled_schedule_values():
    from reelcache_b200.models.longcat_schedule import continuation_schedule, distill_sigmas, dit_timestep, euler_step

    sigmas = distill_sigmas(16)
    assert sigmas.dtype == torch.float32 and sigmas[0] == 1.0 and bool((sigmas[:-1] > sigmas[1:]).all())
    timesteps, shifted = continuation_schedule(16)
    assert timesteps.shape == (16,) and shifted.shape == (17,) and shifted[-1] == 0 and shifted[0] == 1.0
    s = 0.5
    assert distill_sigmas(2).tolist() == pytest.approx([1.0, 0.5])
    assert continuation_schedule(2)[1][1].item() == pytest.approx(12 * s / (1 + 11 * s))
    x = torch.ones(3)
    assert torch.equal(euler_step(torch.full((3,), 2.0), x, torch.tensor(1.0), torch.tensor(0.75)), torch.full((3,), 0.5))
    assert dit_timestep(torch.tensor(500.0), 2, 4, torch.bfloat16).shape == (2, 4)
    with pytest.raises(ValueError):
        distill_sigmas(51)


def test_distilled_schedule_matches_installed_reference():
    ref = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "baseline", "_ref")
    if not os.path.isdir(ref):
        pytest.skip("the reference is not installed under baseline/_ref")
    sys.path.insert(0, ref)
    try:
        theirs = importlib.import_module("reelcache_sglang_models.longcat_video.schedule")
    except Exception as error:  # noqa: BLE001
        pytest.skip(f"reference schedule not importable: {error}")
    finally:
        sys.path.remove(ref)
    from reelcache_b200.models import longcat_schedule as ours
    for steps in (1, 4, 7, 16, 33, 50):
        assert torch.equal(ours.distill_sigmas(steps), theirs.distill_sigmas(steps))
        for a, b in zip(ours.continuation_schedule(steps), theirs.continuation_schedule(steps)):
            assert torch.equal(a, b)
        assert np.array_equal(ours.shift_sigmas([0.1, 0.5]), theirs.shift_sigmas([0.1, 0.5]))
