"""The C++ host fast paths against their Python readers: the NAL-unit table of Annex-B streams (same rows, same
integrity failures) and the channel-tile unmosaic (same coefficients for every layout shape: several segments,
one or three planes, padded pictures)."""

import numpy as np
import pytest

from reelcache_b200 import _hevc
from reelcache_b200.errors import IntegrityError


@pytest.fixture(scope="module")
def native():
    try:
        from reelcache_b200.ops._ext import ext
        module = ext()
    except Exception as error:  # noqa: BLE001 - an unbuilt extension skips the comparison
        pytest.skip(f"the native extension is not built: {error}")
    if not hasattr(module, "nal_units") or not hasattr(module, "unmosaic_all"):
        pytest.skip("the native extension predates the host fast paths")
    return module


def _stream(rng, units=40):
    out = bytearray()
    for i in range(units):
        out += b"\x00\x00\x00\x01" if i % 3 == 0 else b"\x00\x00\x01"
        kind = int(rng.integers(0, 40))
        payload = rng.integers(1, 255, size=int(rng.integers(2, 400)), dtype=np.uint8).tobytes()
        out += bytes([(kind << 1) & 0x7E, 1]) + payload.replace(b"\x00\x00", b"\x00\x03")
        if i % 5 == 4:
            out += b"\x00\x00"  # trailing zeros before the next start code
    return bytes(out)


def test_nal_table_matches_python(native):
    rng = np.random.default_rng(0)
    for seed in range(5):
        data = _stream(np.random.default_rng(seed), units=60)
        assert len(data) >= 4096
        assert _hevc.nal_units(data) == _hevc._nal_units_python(data)
    assert rng is not None


@pytest.mark.parametrize("bad", ["no_start", "forbidden", "short"])
def test_nal_table_integrity_failures_match(native, bad):
    data = bytearray(_stream(np.random.default_rng(9), units=60))
    if bad == "no_start":
        data = b"\x07" + data
    elif bad == "forbidden":
        data[4] |= 0x80
    else:
        data += b"\x00\x00\x01\x02"  # a final unit with a 1-byte header
    with pytest.raises(IntegrityError) as python_error:
        _hevc._nal_units_python(bytes(data))
    with pytest.raises(IntegrityError) as native_error:
        _hevc.nal_units(bytes(data))
    assert str(native_error.value) == str(python_error.value)


@pytest.mark.parametrize("frames,height,width,rank,pix_fmt", [(3, 30, 52, 64, "yuv444p"), (2, 8, 16, 7, "yuv444p"),
                                                              (4, 12, 10, 130, "yuv444p"), (1, 30, 52, 33, "yuv420p")])
def test_unmosaic_matches_python(native, frames, height, width, rank, pix_fmt):
    try:
        layout = _hevc.video_layout(frames, height, width, rank, pix_fmt)
    except Exception:  # noqa: BLE001 - a pixel format this build does not offer
        pytest.skip(f"no {pix_fmt} layout")
    rng = np.random.default_rng(rank)
    pixels = rng.integers(0, 256, size=(frames * height * width, rank), dtype=np.uint8)
    pictures = _hevc.mosaic_all(pixels, layout)
    assert np.array_equal(_hevc._unmosaic_all_python(pictures, layout), pixels)
    assert np.array_equal(_hevc.unmosaic_all(pictures, layout), pixels)
