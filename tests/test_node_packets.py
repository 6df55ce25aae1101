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
