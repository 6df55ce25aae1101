"""8-bit coefficient pictures and the HEVC stream contract (reference: reelcache/_hevc.py).

* Quantization: a per-column covering FP32 affine (``scale = (hi - lo) / 255`` nudged up with
  ``nextafter`` until ``255 * scale + lo`` covers ``hi``; ``offset = lo``) and FP64
  ``rint((v - offset) / scale)`` clipped to 0..255 (reference :400-474). ``global`` and
  ``leading_columns`` normalizations share one affine beyond the protected leading columns.
* Mosaic: the ``reelcache.channel_tiles.v1`` layout (reference :517-612): rank columns become
  ``height x width`` cells of a ``columns x rows`` grid on ``planes`` planes per picture
  (3 for yuv444p); a segment holds ``columns * rows * planes`` channels and every frame of a chunk is
  one picture per segment.
* Bitstreams: Annex-B NAL scanning and access-unit splitting (reference :686-820), and the pinned
  x265 all-intra QP-8 encoder contract ``reelcache.hevc_encoder.v2`` run through an FFmpeg child
  process when an ``ffmpeg`` with libx265 exists (``REELCACHE_FFMPEG_BIN`` or ``PATH``).
"""

from __future__ import annotations

import math
import os
import re
import shutil
import subprocess

import numpy as np

from .errors import ConfigurationError, IntegrityError, UnsupportedError

PIXEL_FORMATS = ("yuv444p", "yuv420p")
MAX_DIMENSION = 8192
CANVAS_ALIGNMENT = 32
NVDEC_MIN_DIMENSION = 144
MIN_CANVAS = -(-NVDEC_MIN_DIMENSION // CANVAS_ALIGNMENT) * CANVAS_ALIGNMENT
ENCODER_SCHEMA = "reelcache.hevc_encoder.v2"
_COMMON_X265 = (("ipratio", 1), ("pbratio", 1), ("info", 0))
_ALL_INTRA_GOP = (("keyint", 1), ("min-keyint", 1), ("bframes", 0), ("b-adapt", 0), ("scenecut", 0),
                  ("open-gop", 0))
_INTER_GOP = (("keyint", 250), ("min-keyint", 25), ("bframes", 3), ("b-adapt", 0), ("b-pyramid", 1), ("ref", 1),
              ("scenecut", 0), ("open-gop", 0))
_IRAP_TYPES = frozenset(range(16, 22))
_IDR_TYPES = frozenset((19, 20))
_PARAMETER_SET_TYPES = frozenset((32, 33, 34))
_AU_PREFIX_TYPES = frozenset((32, 33, 34, 35, 39, *range(41, 45), *range(48, 56)))
_START_CODE = re.compile(b"\x00\x00\x01")
_ENCODE_SECONDS_PER_MEGASAMPLE = 2.0


def size_scaled_timeout(samples, *, seconds_per_megasample=_ENCODE_SECONDS_PER_MEGASAMPLE):
    return max(300.0, samples / 1e6 * seconds_per_megasample)


def encoder_record(inter_prediction):
    """The portable x265 contract of a version-2 coefficient stream (recorded in packet metadata)."""
    if inter_prediction not in (True, False) or type(inter_prediction) is not bool:
        raise ConfigurationError(f"inter_prediction={inter_prediction!r}: expected True or False")
    gop = _INTER_GOP if inter_prediction else _ALL_INTRA_GOP
    return {
        "schema": ENCODER_SCHEMA, "encoder": "libx265", "preset": "ultrafast", "qp": 8,
        "inter_prediction": inter_prediction,
        "picture_structure": "closed_gop_b_pyramid" if inter_prediction else "all_intra_idr",
        "x265_params": {key: value for key, value in (*_COMMON_X265, *gop)},
    }


def x265_parameter_string(inter_prediction, threads, frames):
    gop = _INTER_GOP if inter_prediction else _ALL_INTRA_GOP
    params = [f"{k}={v}" for k, v in (("qp", 8), *_COMMON_X265, *gop)]
    params.append(x265_thread_params(threads, frames))
    return ":".join(params)


def x265_thread_params(threads, frames):
    """Thread-pool part of the x265 parameters: frame threading only with 4+ pool threads, at most 3."""
    if not (type(threads) is int and 0 < threads <= 64):
        raise ConfigurationError(f"x265 pool threads {threads!r}: expected an int from 1 to 64")
    return f"pools={threads}:frame-threads={min(3, max(1, frames)) if threads >= 4 else 1}"


def discover_ffmpeg(path=None) -> str:
    """Path of an FFmpeg binary (argument, ``REELCACHE_FFMPEG_BIN`` or ``PATH``) or UnsupportedError."""
    candidate = path or os.environ.get("REELCACHE_FFMPEG_BIN") or shutil.which("ffmpeg")
    if not candidate or not os.path.exists(candidate):
        raise UnsupportedError("no ffmpeg binary with libx265 is available (set REELCACHE_FFMPEG_BIN)")
    return candidate


def ffmpeg_available(path=None) -> bool:
    try:
        discover_ffmpeg(path)
        return True
    except UnsupportedError:
        return False


def validate_parameters(pix_fmt, qp=8, preset="ultrafast"):
    """The stream contract is pinned: a pixel format of ``PIXEL_FORMATS``, QP 8 and x265's ultrafast preset."""
    problems = []
    if pix_fmt not in PIXEL_FORMATS:
        problems.append(f"pixel format {pix_fmt!r} (supported: {', '.join(PIXEL_FORMATS)})")
    if not (type(qp) is int and qp == 8):
        problems.append(f"qp {qp!r} (pinned to 8)")
    if preset != "ultrafast":
        problems.append(f"preset {preset!r} (pinned to ultrafast)")
    if problems:
        raise UnsupportedError("HEVC coefficient streams cannot use " + ", ".join(problems))


# ---------------------------------------------------------------------------------------------
# Quantization
# ---------------------------------------------------------------------------------------------


def covering_affine(lo, hi):
    """``[2, n]`` little-endian FP32 (scale, offset) with ``255 * scale + offset >= hi`` in FP32."""
    lo = np.asarray(lo, dtype=np.float64)
    hi = np.asarray(hi, dtype=np.float64)
    span = hi - lo
    with np.errstate(over="ignore", invalid="ignore", under="ignore"):
        scale = (span / 255.0).astype(np.float32)
        scale = np.where(scale.astype(np.float64) * 255.0 < span, np.nextafter(scale, np.float32(np.inf)), scale)
        offset = lo.astype(np.float32)
        upper = np.float32(255) * scale + offset
        scale = np.where(upper.astype(np.float64) < hi, np.nextafter(scale, np.float32(np.inf)), scale)
        upper = np.float32(255) * scale + offset
    covered = np.isfinite(scale).all() and np.isfinite(upper).all() and not np.any(upper.astype(np.float64) < hi)
    if not covered:
        raise ConfigurationError("no finite FP32 (scale, offset) maps 0..255 over this coefficient range")
    return np.stack((scale, offset)).astype("<f4", copy=False)


_covering_affine = covering_affine


def normalization_layout(rank, normalization, protected_fraction):
    if not (type(rank) is int and rank > 0):
        raise ConfigurationError(f"coefficient rank {rank!r}: expected an int >= 1")
    if normalization not in ("per_channel", "global", "leading_columns"):
        raise UnsupportedError(f"normalization {normalization!r}: expected per_channel, global or leading_columns")
    fraction_ok = (isinstance(protected_fraction, (int, float)) and not isinstance(protected_fraction, bool)
                   and math.isfinite(protected_fraction) and 0 <= protected_fraction <= 1)
    if not fraction_ok:
        raise ConfigurationError(f"protected_fraction {protected_fraction!r}: expected a number in [0, 1]")
    if normalization == "per_channel":
        count, records = rank, rank
    elif normalization == "global":
        count, records = 0, 1
    else:
        count = int(math.ceil(rank * protected_fraction))
        records = count + 1
    return {"mode": normalization, "protected_count": count, "affine_shape": [2, records],
            "affine_order": ["scale", "offset"], "protected_columns": "leading"}


def expanded_affine(affine, layout, rank):
    if layout["mode"] == "per_channel":
        return affine[0], affine[1]
    scale = np.full(rank, affine[0, 0], dtype=np.float32)
    offset = np.full(rank, affine[1, 0], dtype=np.float32)
    count = layout["protected_count"]
    if count:
        scale[:count], offset[:count] = affine[0, 1:], affine[1, 1:]
    return scale, offset


_expanded_affine = expanded_affine


def affine_for(lo, hi, layout):
    """The packet affine of per-column extrema ``lo``/``hi`` under a normalization layout."""
    count = layout["protected_count"]
    if layout["mode"] == "per_channel":
        return covering_affine(lo, hi)
    affine = np.zeros(layout["affine_shape"], dtype="<f4")
    rank = len(lo)
    if count < rank:
        affine[:, 0] = covering_affine(np.min(lo[count:]), np.max(hi[count:]))
    if count:
        affine[:, 1:] = covering_affine(lo[:count], hi[:count])
    return affine


def quantize_coefficients(values, normalization, protected_fraction=1.0):
    """``(pixels uint8 [N, r], affine [2, records], layout)`` of FP32 coefficients."""
    values = np.asarray(values, dtype=np.float32)
    if not (values.ndim == 2 and values.size and np.isfinite(values).all()):
        raise ConfigurationError(f"quantize_coefficients takes a non-empty finite 2-D array, got shape {values.shape}")
    layout = normalization_layout(values.shape[1], normalization, protected_fraction)
    affine = affine_for(values.min(0), values.max(0), layout)
    scale, offset = expanded_affine(affine, layout, values.shape[1])
    ratios = np.zeros(values.shape, dtype=np.float64)
    np.divide(values.astype(np.float64) - offset.astype(np.float64), scale.astype(np.float64), out=ratios,
              where=scale > 0)
    return np.clip(np.rint(ratios), 0, 255).astype(np.uint8), affine, layout


def validate_affine(affine, layout, rank):
    affine = np.asarray(affine)
    shape_ok = affine.dtype == np.dtype("<f4") and list(affine.shape) == layout["affine_shape"]
    if not (shape_ok and np.isfinite(affine).all() and (affine[0] >= 0).all()):
        raise IntegrityError(f"affine payload {affine.dtype} {list(affine.shape)} is not a finite little-endian FP32 "
                             f"{layout['affine_shape']} with non-negative scales")
    everything_protected = layout["mode"] == "leading_columns" and layout["protected_count"] == rank
    if everything_protected and (affine[:, 0] != 0).any():
        raise IntegrityError("the shared affine column must be zero when every column has its own affine")
    with np.errstate(over="ignore", invalid="ignore"):
        top = np.float32(255) * affine[0] + affine[1]
    if not np.isfinite(top).all():
        raise IntegrityError("an affine maps pixel 255 to a non-finite value")
    return affine


def dequantize_coefficients(pixels, affine, layout):
    pixels = np.asarray(pixels)
    if not (pixels.dtype == np.uint8 and pixels.ndim == 2 and pixels.size):
        raise IntegrityError(f"coefficient pixels must be a non-empty 2-D uint8 array, got {pixels.dtype} "
                             f"{pixels.shape}")
    affine = validate_affine(affine, layout, pixels.shape[1])
    scale, offset = expanded_affine(affine, layout, pixels.shape[1])
    result = pixels.astype(np.float32) * scale + offset
    if not np.isfinite(result).all():
        raise IntegrityError("dequantized coefficients contain non-finite values")
    return np.ascontiguousarray(result)


# ---------------------------------------------------------------------------------------------
# Channel-tile mosaic
# ---------------------------------------------------------------------------------------------


def video_layout(frames, height, width, rank, pix_fmt="yuv444p"):
    validate_parameters(pix_fmt)
    dims = {"frames": frames, "height": height, "width": width, "rank": rank}
    bad = [name for name, value in dims.items() if not (type(value) is int and value > 0)]
    if bad:
        raise ConfigurationError(f"channel-tile layout: {', '.join(bad)} must be ints >= 1 ({dims})")
    if max(height, width) > MAX_DIMENSION:
        raise UnsupportedError(f"a {height}x{width} cell does not fit a {MAX_DIMENSION}-pixel picture")
    planes = 3 if pix_fmt == "yuv444p" else 1
    columns = min(MAX_DIMENSION // width, max(1, math.ceil(math.sqrt(rank / planes))))
    rows = min(MAX_DIMENSION // height, max(1, math.ceil(rank / (planes * columns))))
    image_width, image_height = max(16, columns * width), max(16, rows * height)
    if pix_fmt == "yuv420p":
        image_width += image_width % 2
        image_height += image_height % 2
    if max(image_width, image_height) > MAX_DIMENSION:
        raise UnsupportedError(f"the {image_width}x{image_height} mosaic picture exceeds {MAX_DIMENSION} pixels")
    slots = columns * rows * planes
    return {
        "schema": "reelcache.channel_tiles.v1", "frames": frames, "height": height, "width": width, "rank": rank,
        "pix_fmt": pix_fmt, "grid": [columns, rows], "planes": planes, "image_height": image_height,
        "image_width": image_width, "channels_per_segment": slots, "segments": math.ceil(rank / slots),
        "frame_padding": [image_height - rows * height, image_width - columns * width],
    }


def cells(layout, count):
    """``(index, plane, y, x)`` of the first ``count`` cells of a segment."""
    columns, _ = layout["grid"]
    for index in range(count):
        plane = index % layout["planes"]
        row, column = divmod(index // layout["planes"], columns)
        yield index, plane, row * layout["height"], column * layout["width"]


def segment_slots(layout, segment):
    slots = layout["channels_per_segment"]
    first = segment * slots
    return first, min(slots, layout["rank"] - first)


def mosaic(values, layout, segment):
    """One segment's channel tiles: ``[frames, planes, image_h, image_w]`` from ``[F, H, W, rank]``."""
    first, count = segment_slots(layout, segment)
    images = np.zeros((layout["frames"], layout["planes"], layout["image_height"], layout["image_width"]),
                      dtype=np.uint8)
    h, w = layout["height"], layout["width"]
    for index, plane, y, x in cells(layout, count):
        images[:, plane, y:y + h, x:x + w] = values[..., first + index]
    return images


def unmosaic(images, layout, segment, values):
    first, count = segment_slots(layout, segment)
    h, w = layout["height"], layout["width"]
    for index, plane, y, x in cells(layout, count):
        values[..., first + index] = images[:, plane, y:y + h, x:x + w]


def mosaic_all(pixels, layout):
    """All segments of ``pixels [N, rank]``: ``[segments * frames, planes, image_h, image_w]``
    (segment-major, then frame)."""
    values = np.asarray(pixels, dtype=np.uint8).reshape(layout["frames"], layout["height"], layout["width"],
                                                        layout["rank"])
    return np.concatenate([mosaic(values, layout, s) for s in range(layout["segments"])], axis=0)


def unmosaic_all(images, layout):
    """``[frames * height * width, rank]`` coefficients of a segment-major picture stack (native, without the
    GIL, when the extension is built)."""
    native = _native("unmosaic_all")
    if native is not None:
        import torch
        pictures = np.require(images, dtype=np.uint8, requirements=["C", "W"])
        columns, _ = layout["grid"]
        return native(torch.from_numpy(pictures), layout["frames"], layout["height"], layout["width"], layout["rank"],
                      columns, layout["planes"], layout["channels_per_segment"]).numpy()
    return _unmosaic_all_python(images, layout)


def _unmosaic_all_python(images, layout):
    values = np.empty((layout["frames"], layout["height"], layout["width"], layout["rank"]), dtype=np.uint8)
    frames = layout["frames"]
    for s in range(layout["segments"]):
        unmosaic(images[s * frames:(s + 1) * frames], layout, s, values)
    return values.reshape(-1, layout["rank"])


def align(value, alignment=CANVAS_ALIGNMENT):
    return -(-value // alignment) * alignment


# ---------------------------------------------------------------------------------------------
# Annex-B bitstreams
# ---------------------------------------------------------------------------------------------


def start_code_positions(stream):
    """Offsets of every ``00 00 01`` start code (the payload begins 3 bytes later); the native scanner
    (memchr over the stream, no Python-level copy of matches) when the extension is built."""
    data = bytes(stream)
    native = _native_scanner()
    if native is not None and len(data) >= 4096:
        import torch
        return native(torch.frombuffer(bytearray(data), dtype=torch.uint8))
    return [m.start() for m in _START_CODE.finditer(data)]


def _native_scanner():
    try:
        from .ops._ext import ext
        return ext().start_codes
    except Exception:  # noqa: BLE001 - the host fast path is optional
        return None


def _native(name):
    try:
        from .ops._ext import ext
        return getattr(ext(), name)
    except Exception:  # noqa: BLE001 - the host fast paths are optional
        return None


def nal_units(stream):
    """``[(offset, length, nal_type)]`` of an Annex-B HEVC stream, integrity-checked (in the native extension,
    without the GIL, when it is built; the same checks and table either way)."""
    data = bytes(stream)
    native = _native("nal_units") if len(data) >= 4096 else None
    if native is not None:
        import torch
        try:
            table = native(torch.frombuffer(bytearray(data), dtype=torch.uint8))
        except RuntimeError as error:
            message = str(error)
            if "integrity: " in message:
                raise IntegrityError(message.split("integrity: ", 1)[1].splitlines()[0]) from None
            raise
        return [tuple(row) for row in table.tolist()]
    return _nal_units_python(data)


def _nal_units_python(data: bytes):
    positions = start_code_positions(data)
    leading = positions[0] if positions else None
    if leading is None or leading > 1 or (leading == 1 and data[0] != 0):
        raise IntegrityError("an Annex-B HEVC stream must begin with a 3- or 4-byte start code")
    units = []
    for i, pos in enumerate(positions):
        begin = pos + 3
        end = positions[i + 1] if i + 1 < len(positions) else len(data)
        while end > begin and data[end - 1] == 0 and i + 1 < len(positions):
            end -= 1
        if end - begin < 2:
            raise IntegrityError(f"NAL unit at byte {begin} is shorter than its 2-byte header")
        header = data[begin]
        if header & 0x80:
            raise IntegrityError(f"NAL unit at byte {begin} sets the forbidden zero bit")
        units.append((begin, end - begin, (header >> 1) & 0x3F))
    return units


def access_units(stream):
    """Split into access units: a new unit begins at a prefix NAL after a picture's slices, or at the
    first slice segment of a picture."""
    data = bytes(stream)
    result = []
    current_start = None
    seen_vcl = False
    for begin, length, kind in nal_units(data):
        start = begin - 3
        if start > 0 and data[start - 1] == 0:
            start -= 1
        first_slice = kind < 32 and (data[begin + 2] & 0x80) != 0
        if current_start is None:
            current_start = start
        elif seen_vcl and (kind in _AU_PREFIX_TYPES or first_slice):
            result.append((current_start, start - current_start))
            current_start = start
            seen_vcl = False
        if kind < 32:
            seen_vcl = True
    if current_start is not None:
        result.append((current_start, len(data) - current_start))
    return result


def all_intra_access_units(stream, pictures):
    units = access_units(stream)
    if len(units) != pictures:
        raise IntegrityError(f"expected {pictures} access units, the stream has {len(units)}")
    for number, (offset, length) in enumerate(units):
        slices = {kind for _, _, kind in nal_units(stream[offset:offset + length]) if kind < 32}
        if not slices or not slices <= _IDR_TYPES:
            raise IntegrityError(f"picture {number} of an all-intra stream has slice types {sorted(slices)}, not IDR")
    return units


# ---------------------------------------------------------------------------------------------
# FFmpeg / libx265 child processes
# ---------------------------------------------------------------------------------------------


def _run(command, *, data=None, timeout=None):
    try:
        result = subprocess.run(command, input=data, capture_output=True, timeout=timeout, check=False)
    except FileNotFoundError as error:
        raise UnsupportedError(f"ffmpeg is unavailable: {error}") from error
    except subprocess.TimeoutExpired as error:
        raise UnsupportedError(f"ffmpeg timed out after {timeout} s") from error
    if result.returncode != 0:
        tail = result.stderr.decode(errors="replace")[-400:]
        raise UnsupportedError(f"ffmpeg exited with {result.returncode}: {tail}")
    return result


def encode_pictures(pictures, pix_fmt="yuv444p", *, ffmpeg_path=None, threads=1, inter_prediction=False):
    """HEVC-encode uint8 pictures ``[n, planes, H, W]`` (QP 8, ultrafast, pinned x265 parameters)."""
    binary = discover_ffmpeg(ffmpeg_path)
    pictures = np.ascontiguousarray(pictures, dtype=np.uint8)
    frames, planes, height, width = pictures.shape
    if pix_fmt == "yuv444p" and planes != 3:
        raise ConfigurationError(f"yuv444p pictures carry 3 planes, these carry {planes}")
    if pix_fmt == "yuv444p":
        raw = pictures.tobytes()
    else:
        chroma = np.full((frames, height * width // 2), 128, dtype=np.uint8)
        raw = np.concatenate((pictures[:, 0].reshape(frames, -1), chroma), axis=1).tobytes()
    command = [binary, "-hide_banner", "-loglevel", "error", "-nostdin", "-f", "rawvideo", "-pix_fmt", pix_fmt,
               "-s", f"{width}x{height}", "-framerate", "25", "-i", "pipe:0", "-an", "-c:v", "libx265",
               "-preset", "ultrafast", "-pix_fmt", f"+{pix_fmt}", "-threads", "1", "-x265-params",
               x265_parameter_string(inter_prediction, threads, frames), "-frames:v", str(frames), "-f", "hevc",
               "pipe:1"]
    result = _run(command, data=raw, timeout=size_scaled_timeout(pictures.size))
    if not result.stdout:
        raise UnsupportedError("ffmpeg returned no HEVC bytes")
    if not inter_prediction:
        all_intra_access_units(result.stdout, frames)
    return result.stdout


def decode_pictures(stream, *, pictures, height, width, pix_fmt="yuv444p", ffmpeg_path=None, timeout=None):
    """Software-decode an HEVC stream into uint8 ``[pictures, planes, height, width]``."""
    binary = discover_ffmpeg(ffmpeg_path)
    command = [binary, "-hide_banner", "-loglevel", "error", "-nostdin", "-f", "hevc", "-i", "pipe:0", "-f",
               "rawvideo", "-pix_fmt", pix_fmt, "pipe:1"]
    planes = 3 if pix_fmt == "yuv444p" else 1
    result = _run(command, data=bytes(stream), timeout=timeout or size_scaled_timeout(pictures * height * width))
    frame_bytes = height * width * (3 if pix_fmt == "yuv444p" else 1) if pix_fmt == "yuv444p" else height * width * 3 // 2
    data = np.frombuffer(result.stdout, dtype=np.uint8)
    if data.size != pictures * frame_bytes:
        raise IntegrityError(f"decoder returned {data.size} bytes for {pictures} pictures of {frame_bytes} bytes")
    if pix_fmt == "yuv444p":
        return data.reshape(pictures, planes, height, width).copy()
    return data.reshape(pictures, frame_bytes)[:, :height * width].reshape(pictures, 1, height, width).copy()
