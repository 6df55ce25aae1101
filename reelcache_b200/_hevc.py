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
    if type(inter_prediction) is not bool:
        raise ConfigurationError("inter_prediction must be a bool")
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
    if type(threads) is not int or not 1 <= threads <= 64:
        raise ConfigurationError("x265 threads must be an integer in [1, 64]")
    frame_threads = 1 if threads < 4 else max(1, min(3, frames))
    return f"pools={threads}:frame-threads={frame_threads}"


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
    if pix_fmt not in PIXEL_FORMATS:
        raise UnsupportedError(f"HEVC supports exactly {PIXEL_FORMATS}, not {pix_fmt!r}")
    if type(qp) is not int or qp != 8 or preset != "ultrafast":
        raise UnsupportedError("this HEVC provider supports only QP8 with preset='ultrafast'")


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
    if not np.isfinite(scale).all() or not np.isfinite(upper).all() or np.any(upper.astype(np.float64) < hi):
        raise ConfigurationError("coefficient range cannot use a finite covering FP32 affine")
    return np.stack((scale, offset)).astype("<f4", copy=False)


_covering_affine = covering_affine


def normalization_layout(rank, normalization, protected_fraction):
    if type(rank) is not int or rank < 1:
        raise ConfigurationError("coefficient rank must be a positive integer")
    if normalization not in {"per_channel", "global", "leading_columns"}:
        raise UnsupportedError("normalization must be per_channel, global, or leading_columns")
    if (isinstance(protected_fraction, bool) or not isinstance(protected_fraction, (int, float))
            or not math.isfinite(protected_fraction) or not 0 <= protected_fraction <= 1):
        raise ConfigurationError("protected_fraction must be in [0, 1]")
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
    if values.ndim != 2 or min(values.shape) < 1 or not np.isfinite(values).all():
        raise ConfigurationError("coefficients must be a nonempty finite FP32 matrix")
    layout = normalization_layout(values.shape[1], normalization, protected_fraction)
    affine = affine_for(values.min(0), values.max(0), layout)
    scale, offset = expanded_affine(affine, layout, values.shape[1])
    ratios = np.zeros(values.shape, dtype=np.float64)
    np.divide(values.astype(np.float64) - offset.astype(np.float64), scale.astype(np.float64), out=ratios,
              where=scale > 0)
    return np.clip(np.rint(ratios), 0, 255).astype(np.uint8), affine, layout


def validate_affine(affine, layout, rank):
    affine = np.asarray(affine)
    if (affine.dtype != np.dtype("<f4") or list(affine.shape) != layout["affine_shape"]
            or not np.isfinite(affine).all() or np.any(affine[0] < 0)):
        raise IntegrityError("invalid coefficient affine payload")
    if layout["mode"] == "leading_columns" and layout["protected_count"] == rank and np.any(affine[:, 0] != 0):
        raise IntegrityError("unused global affine must be zero when all columns are protected")
    with np.errstate(over="ignore", invalid="ignore"):
        upper = np.float32(255) * affine[0] + affine[1]
    if not np.isfinite(upper).all():
        raise IntegrityError("coefficient affine endpoints are nonfinite")
    return affine


def dequantize_coefficients(pixels, affine, layout):
    pixels = np.asarray(pixels)
    if pixels.dtype != np.uint8 or pixels.ndim != 2 or min(pixels.shape) < 1:
        raise IntegrityError("decoded coefficient pixels must be a nonempty uint8 matrix")
    affine = validate_affine(affine, layout, pixels.shape[1])
    scale, offset = expanded_affine(affine, layout, pixels.shape[1])
    result = pixels.astype(np.float32) * scale + offset
    if not np.isfinite(result).all():
        raise IntegrityError("decoded coefficients are nonfinite")
    return np.ascontiguousarray(result)


# ---------------------------------------------------------------------------------------------
# Channel-tile mosaic
# ---------------------------------------------------------------------------------------------


def video_layout(frames, height, width, rank, pix_fmt="yuv444p"):
    validate_parameters(pix_fmt)
    if any(type(v) is not int or v < 1 for v in (frames, height, width, rank)):
        raise ConfigurationError("HEVC dimensions must be positive integers")
    if height > MAX_DIMENSION or width > MAX_DIMENSION:
        raise UnsupportedError(f"coefficient tiles cannot exceed {MAX_DIMENSION}x{MAX_DIMENSION}")
    planes = 3 if pix_fmt == "yuv444p" else 1
    columns = min(MAX_DIMENSION // width, max(1, math.ceil(math.sqrt(rank / planes))))
    rows = min(MAX_DIMENSION // height, max(1, math.ceil(rank / (planes * columns))))
    image_width, image_height = max(16, columns * width), max(16, rows * height)
    if pix_fmt == "yuv420p":
        image_width += image_width % 2
        image_height += image_height % 2
    if image_width > MAX_DIMENSION or image_height > MAX_DIMENSION:
        raise UnsupportedError("padded HEVC frame dimensions exceed provider support")
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


def nal_units(stream):
    """``[(offset, length, nal_type)]`` of an Annex-B HEVC stream, integrity-checked."""
    data = bytes(stream)
    positions = start_code_positions(data)
    if not positions or positions[0] > 1 or (positions[0] == 1 and data[0] != 0):
        raise IntegrityError("HEVC stream does not start with a start code")
    units = []
    for i, pos in enumerate(positions):
        begin = pos + 3
        end = positions[i + 1] if i + 1 < len(positions) else len(data)
        while end > begin and data[end - 1] == 0 and i + 1 < len(positions):
            end -= 1
        if end - begin < 2:
            raise IntegrityError("truncated HEVC NAL unit header")
        header = data[begin]
        if header & 0x80:
            raise IntegrityError("HEVC forbidden_zero_bit is set")
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
        raise IntegrityError(f"HEVC stream holds {len(units)} pictures, expected {pictures}")
    for offset, length in units:
        kinds = {kind for _, _, kind in nal_units(stream[offset:offset + length]) if kind < 32}
        if not kinds or not kinds <= _IDR_TYPES:
            raise IntegrityError("all-intra HEVC stream contains a non-IDR picture")
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
        raise UnsupportedError(f"ffmpeg failed: {result.stderr.decode(errors='replace')[-400:]}")
    return result


def encode_pictures(pictures, pix_fmt="yuv444p", *, ffmpeg_path=None, threads=1, inter_prediction=False):
    """HEVC-encode uint8 pictures ``[n, planes, H, W]`` (QP 8, ultrafast, pinned x265 parameters)."""
    binary = discover_ffmpeg(ffmpeg_path)
    pictures = np.ascontiguousarray(pictures, dtype=np.uint8)
    frames, planes, height, width = pictures.shape
    if pix_fmt == "yuv444p" and planes != 3:
        raise ConfigurationError("yuv444p pictures have three planes")
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
        raise UnsupportedError("FFmpeg produced an empty HEVC stream")
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
        raise IntegrityError("decoded HEVC picture count or size differs from the packet")
    if pix_fmt == "yuv444p":
        return data.reshape(pictures, planes, height, width).copy()
    return data.reshape(pictures, frame_bytes)[:, :height * width].reshape(pictures, 1, height, width).copy()
