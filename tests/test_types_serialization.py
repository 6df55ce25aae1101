"""Contracts round-trip through their JSON forms; the tensor container is bit-preserving."""

import pytest
import torch

from reelcache_b200 import serialization
from reelcache_b200.errors import ConfigurationError, IntegrityError
from reelcache_b200.types import (ActiveBasisBinding, BasisVersion, CacheEpoch, ChunkNode, CodecSpec, EnergyReport,
                                  MatrixKey, MatrixRecord, ModelIdentity, OnlineRidgeState, TensorContext,
                                  canonical_digest, energy_targets)

MODEL = ModelIdentity("tiny", "fp-1", 2, 256, "BTHD", "bfloat16")
H = "0" * 64


def test_model_and_context_roundtrip():
    ctx = TensorContext(MODEL, MatrixKey(1, "K"), 0, 3, 4, 5, "pre_rope")
    assert TensorContext.from_dict(ctx.to_dict()) == ctx
    assert ctx.shape == (60, 256)
    with pytest.raises(ConfigurationError):
        TensorContext(MODEL, MatrixKey(0, "V"), 0, 1, 1, 1, "pre_rope")


def test_codec_spec_versions():
    spec = CodecSpec("svd_hevc", 32)
    assert spec.to_dict()["inter_prediction"] is False
    legacy = CodecSpec.from_dict({k: v for k, v in spec.to_dict().items() if k != "inter_prediction"})
    assert legacy.legacy_gop


def test_record_node_epoch_roundtrip():
    ctx = TensorContext(MODEL, MatrixKey(0, "K"), 0, 1, 2, 2, "pre_rope")
    energy = EnergyReport(0.98, 0.99, 0.985, None, 30, 32, 32)
    record = MatrixRecord(ctx, CodecSpec("svd_hevc", 32), f"manifest:{H}", f"manifest:{'1' * 64}", 32, energy, None,
                          {"decision": "fresh"}, packet_tile=0)
    assert MatrixRecord.from_dict(record.to_dict()) == record
    epoch = CacheEpoch("e0", None, "initial", "global", (), {})
    assert CacheEpoch.from_dict(epoch.to_dict()) == epoch
    binding = ActiveBasisBinding(f"manifest:{'2' * 64}", 32, H, 30, "c0")
    node = ChunkNode("chunk", "c0", f"manifest:{'3' * 64}", "e0", f"manifest:{'4' * 64}", 0, 4, 1, 2, 2, 4,
                     ((MatrixKey(0, "K"), f"manifest:{'5' * 64}"),), ((MatrixKey(0, "K"), binding),))
    assert ChunkNode.from_dict(node.to_dict()) == node
    assert node.to_dict()["schema"] == "reelcache.chunk_node.v1"


def test_basis_version_rules():
    with pytest.raises(ConfigurationError):
        BasisVersion(None, f"basis:{H}", 4, 8, 256, H, MatrixKey(0, "K"), "fp", 0, H)
    v = BasisVersion(None, f"basis:{H}", 8, 8, 256, H, MatrixKey(0, "V"), "fp", 0, H)
    assert v.to_dict()["domain"] == "direct_v"
    assert BasisVersion.from_dict(v.to_dict()) == v


def test_ridge_state_update_and_predict():
    state = OnlineRidgeState.initial()
    assert abs(state.predict(0.0) - 32.0) < 1e-9
    state = state.updated(1.0, 64)
    assert state.observations == 1
    assert OnlineRidgeState.from_dict(state.to_dict()) == state


def test_energy_profiles_and_digest():
    assert energy_targets("causvid").key == 0.98
    assert canonical_digest({"b": 1, "a": [1, 2]}) == canonical_digest({"a": [1, 2], "b": 1})


def test_tensor_container_bitwise():
    tensors = {"rng": torch.arange(10, dtype=torch.int64), "lat": torch.randn(2, 3, dtype=torch.bfloat16)}
    data = serialization.serialize_tensors(tensors)
    assert data.startswith(b"REELCACHE_TENSORS\x00\x01")
    back = serialization.deserialize_tensors(data)
    assert torch.equal(back["rng"], tensors["rng"]) and torch.equal(back["lat"], tensors["lat"])
    corrupt = bytearray(data)
    corrupt[-1] ^= 1
    with pytest.raises(IntegrityError):
        serialization.deserialize_tensors(bytes(corrupt))


def test_parse_json_strict():
    with pytest.raises(IntegrityError):
        serialization.parse_json(b'{"a": 1, "a": 2}')
    with pytest.raises(IntegrityError):
        serialization.parse_json(b'{"a": NaN}')
