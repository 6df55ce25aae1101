"""Node packets on CPU: the canvas ladder, host finalization and mosaic round trips, pack-basis detachment."""

import numpy as np
import pytest
import torch

from reelcache_b200 import _hevc
from reelcache_b200.errors import ConfigurationError
from reelcache_b200.node_packets import (CANVAS_RANK_LADDER, assemble_canvas, attach_pack_bases, canvas_layout,
                                         canvas_rank, detach_pack_bases, finalize_tile, mosaic_host)


def test_ladder_and_layouts():
    assert canvas_rank(1) == 32 and canvas_rank(33) == 48 and canvas_rank(8192) == 8192
    with pytest.raises(ConfigurationError):
        canvas_rank(9000)
    a, b = canvas_layout(3, 30, 52, 57), canvas_layout(3, 30, 52, 60)
    assert (a["image_height"], a["image_width"]) == (b["image_height"], b["image_width"])  # same ladder canvas
    assert a["tile_rank"] == 57 and a["rank"] == 64
    assert list(CANVAS_RANK_LADDER) == sorted(CANVAS_RANK_LADDER)


def test_finalize_round_trip_host():
    g = torch.Generator().manual_seed(0)
    coefficients = torch.randn(2 * 6 * 10, 37, generator=g)
    tile = finalize_tile(coefficients, (2, 6, 10))
    pixels, affine, _ = _hevc.quantize_coefficients(coefficients.numpy(), "per_channel", 1.0)
    assert np.array_equal(tile.pixels(), pixels)
    assert tile.canvas.shape[1:] == (tile.layout["planes"], tile.layout["image_height"], tile.layout["image_width"])
    canvas, ranges = assemble_canvas([tile, tile])
    assert canvas.shape[0] == 2 * tile.canvas.shape[0] and ranges[1]["first_picture"] == tile.canvas.shape[0]
    layout = canvas_layout(2, 6, 10, 37)
    assert np.array_equal(mosaic_host(pixels, layout, 37), tile.canvas)


def test_pack_bases_detach_attach():
    meta = {"schema": "x", "tiles": [{"tile": 0, "basis": {"sha": "a"}}, {"tile": 1, "basis": {"sha": "b"}}]}
    detached, bases = detach_pack_bases(meta)
    assert all("basis" not in t for t in detached["tiles"]) and bases == [{"sha": "a"}, {"sha": "b"}]
    assert attach_pack_bases(detached, bases) == meta


def test_node_codec_api_packed_layer_groups_and_per_matrix():
    import torch
    from reelcache_b200.codecs import decode_packed, decode_tensor, encode_node, encode_packed
    from reelcache_b200.types import CodecSpec, MatrixKey, ModelIdentity, TensorContext
    model = ModelIdentity("tiny", "fp", 4, 64, "BTHD", "bfloat16")
    g = torch.Generator().manual_seed(0)
    matrices, contexts = {}, {}
    for layer in range(4):
        for target in "KV":
            key = MatrixKey(layer, target)
            rows = torch.randn(128, 6, generator=g) @ torch.linalg.qr(torch.randn(64, 6, generator=g))[0].t()
            matrices[key] = rows.to(torch.bfloat16)
            contexts[key] = TensorContext(model, key, 0, 2, 8, 8, "pre_rope" if target == "K" else "none")
    spec = CodecSpec("svd_hevc", 8)
    pack = encode_packed(matrices, contexts, spec, node_id="n0")
    decoded = decode_packed(pack)
    assert list(decoded) == sorted(matrices, key=lambda k: (k.layer, k.target))
    for key, value in decoded.items():
        source = matrices[key].float()
        assert float((value - source).norm() / source.norm()) < 0.02
    one = decode_packed(pack, keys=[MatrixKey(2, "V")])
    assert list(one) == [MatrixKey(2, "V")] and torch.equal(one[MatrixKey(2, "V")], decoded[MatrixKey(2, "V")])
    node = encode_node(matrices, contexts, spec)
    assert len(node.packets) == 1 and node.locations[MatrixKey(3, "V")] == (0, 7)
    groups = encode_node(matrices, contexts, spec, packing="layer_group", layer_group_size=2)
    assert len(groups.packets) == 2 and groups.locations[MatrixKey(2, "K")] == (1, 0)
    mixed = {k: (CodecSpec("raw") if k.layer == 0 else CodecSpec("svd", 8) if k.layer == 1 else spec)
             for k in matrices}
    per = encode_node(matrices, contexts, mixed, packing="per_matrix")
    assert len(per.packets) == 8 and all(tile is None for _, tile in per.locations.values())
    raw = decode_tensor(per.packets[per.locations[MatrixKey(0, "K")][0]])
    assert torch.equal(raw, matrices[MatrixKey(0, "K")])
    svd = decode_tensor(per.packets[per.locations[MatrixKey(1, "V")][0]])
    assert float((svd - matrices[MatrixKey(1, "V")].float()).norm() / matrices[MatrixKey(1, "V")].float().norm()) < 0.02
    mixed_node = encode_node(matrices, contexts, mixed)
    assert len(mixed_node.packets) == 4 + 1   # RAW and SVD single packets, the svd_hevc matrices in one pack


def test_factor_pack_validate_prepare_decode():
    import torch
    from reelcache_b200.codecs import descriptor, encode_factor_pack
    from reelcache_b200.errors import IntegrityError
    from reelcache_b200.factor_packs import (decode_factor_pack, factor_codec, is_factor_pack, prepare_factor_packet,
                                             validate_factor_pack)
    from reelcache_b200.types import CodecSpec, MatrixKey, ModelIdentity, TensorContext
    model = ModelIdentity("tiny", "fp", 2, 64, "BTHD", "bfloat16")
    g = torch.Generator().manual_seed(1)
    tiles, bases, sources = [], {}, {}
    for layer in range(2):
        key = MatrixKey(layer, "K")
        rows = torch.linalg.qr(torch.randn(64, 8, generator=g))[0].t().to(torch.float16)
        coeff = torch.randn(128, 8, generator=g)
        bases[key], sources[key] = rows, coeff.half().float() @ rows.float()
        tiles.append({"entry": {"key": key.to_dict()}, "context": TensorContext(model, key, 0, 2, 8, 8, "pre_rope"),
                      "coefficients": coeff.numpy(), "basis": descriptor(rows.numpy().tobytes(), 8, 64)})
    pack = encode_factor_pack(tiles)
    assert is_factor_pack(pack) and factor_codec(CodecSpec("svd", 8))["kind"] == "svd"
    assert len(validate_factor_pack(pack, verify=True)) == 2
    prepared = prepare_factor_packet(pack)
    assert prepared[1].entry == MatrixKey(1, "K") and prepared[1].values.shape == (128, 8)
    decoded = decode_factor_pack(pack, bases)
    for key, value in decoded.items():
        assert torch.allclose(value, sources[key], atol=1e-3)
    bad = type(pack)(pack.metadata, {"factors": pack.payloads["factors"][:-2]})
    with pytest.raises(IntegrityError):
        validate_factor_pack(bad)


def test_device_tile_pixels_inverts_the_mosaic_and_canvas_shapes():
    import numpy as np
    import torch
    from reelcache_b200 import _hevc
    from reelcache_b200.node_packets import canvas_layout, mosaic_host
    from reelcache_b200.packed_decode import canonical_canvas_shapes, device_tile_pixels

    frames, height, width, rank = 2, 6, 10, 45
    layout = canvas_layout(frames, height, width, rank)
    pixels = np.random.default_rng(0).integers(0, 256, (frames * height * width, rank), dtype=np.uint8)
    canvas = torch.from_numpy(mosaic_host(pixels, layout, rank))
    padded = torch.cat([torch.zeros((3,) + tuple(canvas.shape[1:]), dtype=torch.uint8), canvas])
    back = device_tile_pixels(padded, 3, layout)
    assert back.shape == (frames * height * width, rank) and np.array_equal(back.numpy(), pixels)
    shapes = canonical_canvas_shapes(frames, height, width, channels=256)
    assert shapes == sorted(shapes, key=lambda s: s[0] * s[1]) and len(shapes) == len(set(shapes))
    assert (layout["image_width"], layout["image_height"], "yuv444p") in shapes
    assert len(canonical_canvas_shapes(frames, height, width, channels=256, max_rank=32)) == 1
    assert _hevc.PIXEL_FORMATS[0] == "yuv444p"
