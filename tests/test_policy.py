"""Online rank policies (prediction from anchors, guarded preparation, abstention, scalar state), static profile
selection and calibration registries, on CPU."""

import hashlib

import pytest
import torch

import reelcache_b200
from reelcache_b200.calibration import (Observation, configuration_fingerprint, fit_profile, load_rank_policy,
                                        load_registry, package_fingerprint, save_rank_policy, save_registry)
from reelcache_b200.errors import ConfigurationError, StateError
from reelcache_b200.online_rank import (RankAbstention, RankPolicy, RankPreparation, RankState, predict_rank)
from reelcache_b200.policy import Profile, QualityBudget, QualityEvidence, select_profile
from reelcache_b200.types import CodecSpec, MatrixKey

from .lineage_support import FRAMES, HEIGHT, MODEL, TOKENS, WIDTH, chunk

KEYS = [MatrixKey(layer, t) for layer in range(MODEL.layers) for t in ("K", "V")]


def _policy(**overrides):
    base = dict(policy_id="p", model=MODEL, geometry=(FRAMES, HEIGHT, WIDTH), energy_target=0.99,
                template_ranks={k: 8.0 for k in KEYS}, allowed_ranks={k: (4, 8, 12, 16, 24, 32) for k in KEYS},
                anchors=(MatrixKey(0, "K"), MatrixKey(0, "V")), anchor_mode="causal", history_max=4)
    base.update(overrides)
    return RankPolicy(**base)


def test_policy_round_trip_and_prediction():
    policy = _policy()
    assert RankPolicy.from_dict(policy.to_dict()) == policy
    assert reelcache_b200.RankPolicy is RankPolicy
    # an anchor at twice its template doubles the prediction of higher layers of the same target
    p = predict_rank(policy, MatrixKey(1, "K"), chunk_ordinal=1, current_anchors={MatrixKey(0, "K"): 16.0},
                     previous_anchors={}, previous_anchor_chunks={})
    assert p.predicted == pytest.approx(16.0) and p.initial_rank == 16
    p = predict_rank(policy, MatrixKey(1, "V"), chunk_ordinal=1, current_anchors={MatrixKey(0, "K"): 16.0},
                     previous_anchors={}, previous_anchor_chunks={})
    assert p.initial_rank == 8  # other target: template only
    with pytest.raises(ConfigurationError):
        predict_rank(policy, MatrixKey(1, "K"), chunk_ordinal=2, current_anchors={},
                     previous_anchors={MatrixKey(0, "K"): 3.0}, previous_anchor_chunks={MatrixKey(0, "K"): 2})
    with pytest.raises(ConfigurationError):
        _policy(anchor_mode="none")


def test_preparation_guards_and_advances_state():
    policy = _policy()
    matrices, contexts = chunk(0)
    with RankPreparation(policy, chunk_id="c0", parent_head=None, token_start=0) as prep:
        prepared = prep.prepare_staged(matrices, contexts)
        state = prep.next_state()
    for key, item in prepared.items():
        d = item.decision
        assert d.status == "accepted" and d.guard_relative_residual <= d.guard_threshold
        x = matrices[key]
        recon = item.factors.coefficients @ item.factors.basis.float()
        assert float((x - recon).norm() / x.norm()) <= d.guard_threshold + 1e-6
    assert state.completed_chunks == 1 and set(state.selected_ranks) == set(KEYS)
    assert RankState.from_dict(state.to_dict()) == state
    # the next chunk continues from the committed boundary
    matrices1, contexts1 = chunk(1)
    prep1 = RankPreparation(policy, state, chunk_id="c1", parent_head="node0", token_start=TOKENS)
    prep1.prepare_staged(matrices1, contexts1)
    assert prep1.next_state().completed_chunks == 2
    with pytest.raises(ConfigurationError):
        RankPreparation(policy, state, chunk_id="c1", parent_head="node0", token_start=0)


def test_abstention_when_no_allowed_rank_suffices():
    policy = _policy(allowed_ranks={k: (1, 2) for k in KEYS}, anchors=(), anchor_mode="none",
                     template_ranks={k: 1.0 for k in KEYS})
    matrices, contexts = chunk(0)
    prep = RankPreparation(policy, chunk_id="c0", parent_head=None, token_start=0)
    with pytest.raises(RankAbstention) as info:
        prep.prepare_matrix(matrices[KEYS[0]], contexts[KEYS[0]])
    assert info.value.decision.status == "abstained"
    with pytest.raises(StateError):
        prep.next_state()


def _profile(pid, size, evidence=None):
    specs = {k: CodecSpec("svd", 8) for k in KEYS}
    return Profile(pid, MODEL, specs, (FRAMES, HEIGHT, WIDTH), size, 0.01, 0.2, history_min=1, history_max=8,
                   feature_bounds={"K_residual_max": (0.0, 1.0)}, evidence=evidence)


def _evidence(ssim=0.97):
    sha = hashlib.sha256(b"x").hexdigest()
    prompts = tuple(f"p{i}" for i in range(6))
    return QualityEvidence("per_channel", ssim, ssim - 0.02, 0.01, prompts, tuple(f"v{i}" for i in range(6)),
                           tuple(f"c{i}" for i in range(6)), (sha,), held_out=True, native_validated=True)


def test_select_profile():
    budget = QualityBudget(min_mean_ssim=0.95, min_frame_ssim=0.9, max_mean_ssim_drop=0.05)
    profiles = [_profile("small-unqualified", 1000), _profile("qualified", 2000, _evidence()),
                _profile("bad-quality", 1500, _evidence(0.5))]
    kwargs = dict(model=MODEL, geometry=(FRAMES, HEIGHT, WIDTH), history_chunks=2,
                  features={"K_residual_max": 0.5}, raw_bytes=10_000)
    chosen = select_profile(profiles, budget=budget, **kwargs)
    assert chosen.profile_id == "qualified" and chosen.evidence_qualified
    assert set(chosen.rejected) == {"small-unqualified", "bad-quality"}
    raw = select_profile(profiles, **kwargs)  # no SSIM budget: nothing lossy qualifies
    assert raw.profile_id == "RAW"
    forced = select_profile(profiles, explicit_profile="small-unqualified", allow_experimental=True, **kwargs)
    assert forced.experimental and forced.profile_id == "small-unqualified"
    outside = select_profile(profiles, budget=budget, **{**kwargs, "features": {"K_residual_max": 3.0}})
    assert outside.profile_id == "RAW"


def test_calibration_registries(tmp_path):
    template = _profile("cal", 1)
    digest = configuration_fingerprint(template)
    sha = hashlib.sha256(b"s").hexdigest()
    rows = [Observation("cal", f"case{i}", f"p{i}", "calibration", digest, 2, 900 + i, 0.01, 0.1,
                        {"K_residual_max": 0.1 * i}) for i in range(6)]
    rows += [Observation("cal", f"val{i}", f"v{i}", "validation", digest, 2, 950, 0.01, 0.1, {}, 0.96, 0.93, 0.01,
                         sha) for i in range(6)]
    fitted = fit_profile(template, rows, native_validated=True)
    assert fitted.measured_stored_bytes == 905 and fitted.feature_bounds["K_residual_max"][1] == pytest.approx(0.5)
    assert fitted.evidence.held_out and fitted.evidence.mean_ssim == pytest.approx(0.96)
    path = tmp_path / "registry.json"
    checksum = save_registry(path, [fitted, _profile("other", 5)])
    assert save_registry(path, [fitted, _profile("other", 5)]) == checksum
    with pytest.raises(StateError):
        save_registry(path, [fitted])
    loaded = load_registry(path, expected_sha256=checksum)
    assert [p.profile_id for p in loaded] == ["cal", "other"] and loaded[0] == fitted
    policy_path = tmp_path / "policy.json"
    policy = _policy()
    save_rank_policy(policy_path, policy)
    assert load_rank_policy(policy_path) == policy
    assert len(package_fingerprint()) == 64
