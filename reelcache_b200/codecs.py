"""Tensor codecs: RAW and factorized single-matrix packets and per-node coefficient packs
(reference: reelcache/codecs.py:56-60 for the schema names, :621-1187 for single packets, :1369-1608 for
node packs).

* ``reelcache.tensor.v1`` RAW packets hold a matrix bit for bit (``values`` payload).
* ``reelcache.tensor.v2`` factorized packets hold the 8-bit coefficients of ``A ~ P Q`` with their
  per-column FP32 affine and a descriptor (shape, view rank, SHA-256) binding the FP16 basis prefix
  they were encoded with; the basis bytes themselves live in the basis-version store.
* ``reelcache.tensor_pack.v2`` node packs hold every matrix of one committed node as tiles of one
  coefficient stream plus one affine payload. Tiles reference external basis versions.
* ``reelcache.factor_pack.v1`` packs hold FP16 factors (the SVD-only baseline).

Coefficient streams: ``hevc`` (all-intra QP-8 x265 through FFmpeg, the reference's contract; only
where an encoder exists) or ``raw8`` (the same 8-bit mosaic-free coefficient rows, uncompressed, or
``raw8+zlib``). Every stream decodes to the identical uint8 coefficients, so restores are bitwise
the same whichever stream a pack uses.
"""

from __future__ import annotations

import hashlib
import zlib
from dataclasses import dataclass
from typing import Any, Mapping, Sequence

import numpy as np
import torch

from . import _hevc
from .errors import ConfigurationError, IntegrityError, UnsupportedError
from .serialization import tensor_bytes, tensor_from_bytes
from .types import CodecSpec, EncodedTensor, TensorContext, entry_order, json_copy

TENSOR_V1 = "reelcache.tensor.v1"
TENSOR_V2 = "reelcache.tensor.v2"
PACK_SCHEMA = "reelcache.tensor_pack.v2"
FACTOR_PACK_SCHEMA = "reelcache.factor_pack.v1"
STREAM_CODECS = ("raw8", "raw8+zlib", "hevc")
REPRESENTATIONS = ("raw", "svd", "svd_hevc")


def descriptor(basis: bytes, rank_view: int, channels: int) -> dict[str, Any]:
    return {"shape": [rank_view, channels], "view_rank": rank_view, "dtype": "float16", "bytes": len(basis),
            "sha256": hashlib.sha256(basis).hexdigest()}


def default_stream_codec() -> str:
    """``hevc`` when an FFmpeg with libx265 is reachable, else ``raw8``."""
    return "hevc" if _hevc.ffmpeg_available() else "raw8"


# ---------------------------------------------------------------------------------------------
# Single-matrix packets
# ---------------------------------------------------------------------------------------------


_RAW_PAYLOAD = "tensor.bin"
_COEFFICIENT_PAYLOAD = "coefficients.f32"


def _payload_descriptor(payload: bytes, dtype: str, shape) -> dict[str, Any]:
    return {"bytes": len(payload), "dtype": dtype, "sha256": hashlib.sha256(payload).hexdigest(),
            "shape": [int(v) for v in shape]}


def encode_raw(matrix: torch.Tensor, context: TensorContext) -> EncodedTensor:
    """RAW packet: the canonical matrix bit for bit, in the ``reelcache.tensor.v1`` layout both implementations
    read (one ``tensor.bin`` payload described by its bytes, dtype, SHA-256 and shape; the factorization fields
    present and null)."""
    if tuple(matrix.shape) != context.shape:
        raise ConfigurationError("matrix shape differs from its context")
    payload = tensor_bytes(matrix)
    dtype = str(matrix.dtype).removeprefix("torch.")
    codec = _portable_codec(CodecSpec("raw"))
    metadata = {"schema": TENSOR_V1, "kind": "raw", "factorization_domain": "raw", "byte_order": "little",
                "codec": codec, "context": context.to_dict(), "dtype": dtype, "shape": list(matrix.shape),
                "payloads": {_RAW_PAYLOAD: _payload_descriptor(payload, dtype, matrix.shape)},
                "basis": None, "coefficient_shape": None, "normalization": None, "video": None,
                "decoded_coefficients_sha256": None}
    metrics = {"payload_bytes": len(payload), "source_bytes": len(payload), "basis_bytes": 0,
               "reuse_reason": "raw", "reuse_accepted": False}
    return EncodedTensor(metadata, {_RAW_PAYLOAD: payload}, metrics=metrics)


def _checked_payload(encoded: EncodedTensor, name: str) -> bytes:
    payload = encoded.payloads[name]
    described = encoded.metadata.get("payloads", {}).get(name)
    digest = encoded.metadata.get("sha256") if described is None else described["sha256"]
    if hashlib.sha256(payload).hexdigest() != digest:
        raise IntegrityError(f"packet payload {name} differs from its digest")
    return payload


def decode_v1(encoded: EncodedTensor, *, device: Any = "cpu") -> tuple[torch.Tensor, torch.Tensor | None]:
    """A ``reelcache.tensor.v1`` packet: ``(values, None)`` for RAW (``tensor.bin``, or the ``values`` payload of
    stores written before the layout was aligned), ``(coefficients FP32 [N, r], None)`` for a per-matrix SVD
    packet (``coefficients.f32``; its basis is the record's version prefix)."""
    meta = encoded.metadata
    kind = meta.get("kind", meta.get("representation", "raw"))
    if kind == "raw":
        name = _RAW_PAYLOAD if _RAW_PAYLOAD in encoded.payloads else "values"
        payload = _checked_payload(encoded, name)
        return tensor_from_bytes(payload, dtype=meta["dtype"], shape=meta["shape"], device=device), None
    if kind == "svd":
        payload = _checked_payload(encoded, _COEFFICIENT_PAYLOAD)
        shape = meta["payloads"][_COEFFICIENT_PAYLOAD]["shape"]
        values = np.frombuffer(payload, dtype="<f4").reshape(shape)
        return torch.from_numpy(values.copy()).to(device), None
    raise UnsupportedError(f"tensor.v1 packets of kind {kind!r} are not decoded here")


def quantize(coefficients: torch.Tensor, normalization: str = "per_channel", protected_fraction: float = 1.0):
    """(pixels uint8 [N, r] numpy, affine float32 [2, records], layout) of FP32 coefficients; device
    tensors are quantized on the device with the identical arithmetic (ops.quant)."""
    if coefficients.is_cuda:
        from .ops.quant import quantize_device
        return quantize_device(coefficients, normalization, protected_fraction)
    return _hevc.quantize_coefficients(coefficients.detach().float().cpu().numpy(), normalization,
                                       protected_fraction)


def encode_factorized(coefficients: torch.Tensor, basis_view: bytes, context: TensorContext, spec: CodecSpec, *,
                      stream_codec: str | None = None, metrics: Mapping[str, Any] | None = None) -> EncodedTensor:
    """``reelcache.tensor.v2`` packet of one matrix's coefficients (basis kept external)."""
    rank = coefficients.shape[1]
    if spec.kind not in ("svd", "svd_hevc") or spec.rank != rank:
        raise ConfigurationError("factorized packets need an svd/svd_hevc spec at the coefficient rank")
    if spec.kind == "svd":
        return _encode_svd_v1(coefficients, basis_view, context, spec, metrics)
    stream_codec = stream_codec or default_stream_codec()
    if stream_codec not in STREAM_CODECS:
        raise ConfigurationError(f"stream codec must be one of {STREAM_CODECS}")
    pixels, affine, layout = quantize(coefficients, spec.normalization, spec.protected_fraction)
    stream = _encode_stream(np.ascontiguousarray(pixels), context, stream_codec, spec)
    metadata = {"schema": TENSOR_V2, "representation": spec.kind, "context": context.to_dict(),
                "codec": spec.to_dict(), "rank": rank, "normalization": layout, "stream_codec": stream_codec,
                "basis": descriptor(basis_view, rank, context.channels),
                "coefficients": {"shape": [int(pixels.shape[0]), rank],
                                 "sha256": hashlib.sha256(np.ascontiguousarray(pixels).tobytes()).hexdigest()}}
    payloads = {"stream": stream, "affine": np.ascontiguousarray(affine, dtype="<f4").tobytes()}
    return EncodedTensor(metadata, payloads, basis=basis_view, metrics=dict(metrics or {}, bytes=len(stream)))


def _encode_svd_v1(coefficients: torch.Tensor, basis_view: bytes, context: TensorContext, spec: CodecSpec,
                   metrics: Mapping[str, Any] | None) -> EncodedTensor:
    """An SVD-only matrix: FP32 coefficients ``coefficients.f32`` in the ``reelcache.tensor.v1`` layout, the FP16
    basis view described (``basis``) and stored as the record's version prefix."""
    values = np.ascontiguousarray(coefficients.detach().to("cpu", torch.float32).numpy()).astype("<f4", copy=False)
    payload = values.tobytes()
    codec = _portable_codec(spec)
    metadata = {"schema": TENSOR_V1, "kind": "svd", "factorization_domain": _domain(context),
                "byte_order": "little", "codec": codec, "context": context.to_dict(),
                "dtype": context.dtype, "shape": list(context.shape), "coefficient_shape": list(values.shape),
                "payloads": {_COEFFICIENT_PAYLOAD: _payload_descriptor(payload, "float32", values.shape)},
                "basis": descriptor(basis_view, values.shape[1], context.channels), "normalization": None,
                "video": None, "decoded_coefficients_sha256": hashlib.sha256(payload).hexdigest()}
    return EncodedTensor(metadata, {_COEFFICIENT_PAYLOAD: payload}, basis=basis_view,
                         metrics=dict(metrics or {}, payload_bytes=len(payload)))


def _domain(context: TensorContext) -> str:
    """The factorization domain label of a matrix (factorized K is always the normalized pre-RoPE K)."""
    return "normalized_pre_rope_k" if context.key.target == "K" else "direct_v"


def _portable_codec(spec: CodecSpec) -> dict[str, Any]:
    """The codec header a tensor packet records: the spec without run-local fields (the encoder path)."""
    codec = spec.to_dict()
    codec.pop("ffmpeg_path", None)
    return codec


def _encode_stream(pixels: np.ndarray, context: TensorContext, stream_codec: str, spec: CodecSpec) -> bytes:
    if stream_codec == "raw8":
        return pixels.tobytes()
    if stream_codec == "raw8+zlib":
        return zlib.compress(pixels.tobytes(), 1)
    layout = _hevc.video_layout(context.frames, context.height, context.width, pixels.shape[1], spec.pix_fmt)
    pictures = _hevc.mosaic_all(pixels, layout)
    return _hevc.encode_pictures(pictures, spec.pix_fmt, ffmpeg_path=spec.ffmpeg_path,
                                 inter_prediction=bool(spec.inter_prediction))


def _decode_stream(stream: bytes, shape: Sequence[int], context: TensorContext, stream_codec: str,
                   spec: CodecSpec) -> np.ndarray:
    tokens, rank = shape
    if stream_codec == "raw8":
        data = stream
    elif stream_codec == "raw8+zlib":
        data = zlib.decompress(stream)
    elif stream_codec == "hevc":
        layout = _hevc.video_layout(context.frames, context.height, context.width, rank, spec.pix_fmt)
        pictures = _hevc.decode_pictures(stream, pictures=layout["segments"] * layout["frames"],
                                         height=layout["image_height"], width=layout["image_width"],
                                         pix_fmt=spec.pix_fmt, ffmpeg_path=spec.ffmpeg_path)
        return _hevc.unmosaic_all(pictures, layout)
    else:
        raise IntegrityError(f"unknown coefficient stream codec {stream_codec!r}")
    if len(data) != tokens * rank:
        raise IntegrityError("coefficient stream length differs from its shape")
    return np.frombuffer(data, dtype=np.uint8).reshape(tokens, rank)


def decode_coefficient_pixels(encoded: EncodedTensor) -> tuple[np.ndarray, np.ndarray, Mapping[str, Any]]:
    """(pixels uint8 [N, r], affine, normalization layout) of a factorized packet, hash-checked."""
    meta = encoded.metadata
    if meta.get("schema") != TENSOR_V2:
        raise IntegrityError("not a factorized tensor packet")
    context = TensorContext.from_dict(meta["context"])
    spec = CodecSpec.from_dict(meta["codec"])
    pixels = _decode_stream(encoded.payloads["stream"], meta["coefficients"]["shape"], context, meta["stream_codec"],
                            spec)
    if hashlib.sha256(np.ascontiguousarray(pixels).tobytes()).hexdigest() != meta["coefficients"]["sha256"]:
        raise IntegrityError("decoded coefficients differ from the packet digest")
    affine = np.frombuffer(encoded.payloads["affine"], dtype="<f4").reshape(meta["normalization"]["affine_shape"])
    return pixels, _hevc.validate_affine(affine.copy(), meta["normalization"], pixels.shape[1]), meta["normalization"]


def decode_tensor(encoded: EncodedTensor, *, device: Any = "cpu", dtype: torch.dtype = torch.float32) -> torch.Tensor:
    """The canonical matrix of a packet: RAW bitwise; factorized ``dequantize(P) @ Q`` (FP32)."""
    meta = encoded.metadata
    if meta.get("schema") == TENSOR_V1:
        values, _ = decode_v1(encoded, device=device)
        if meta.get("kind", "raw") == "svd":
            if encoded.basis is None:
                raise IntegrityError("factorized packets decode only with their attached basis view")
            rank, channels = meta["basis"]["shape"]
            basis = np.frombuffer(encoded.basis, dtype=np.float16).reshape(rank, channels)
            values = values @ torch.from_numpy(basis.copy()).to(device).float()
            return values.to(dtype)
        return values
    pixels, affine, layout = decode_coefficient_pixels(encoded)
    if encoded.basis is None:
        raise IntegrityError("factorized packets decode only with their attached basis view")
    rank = pixels.shape[1]
    channels = meta["basis"]["shape"][1]
    coefficients = torch.from_numpy(_hevc.dequantize_coefficients(pixels, affine, layout)).to(device)
    basis = torch.from_numpy(np.frombuffer(encoded.basis, dtype=np.float16).reshape(rank, channels).copy()).to(device)
    return (coefficients @ basis.float()).to(dtype)


def encode_tensor(matrix: torch.Tensor, context: TensorContext, spec: CodecSpec, *, basis: torch.Tensor | None = None,
                  stream_codec: str | None = None) -> EncodedTensor:
    """Encode one matrix: RAW, or factorized on ``basis`` (FP16 [r, C]) or on its own truncated
    eigenbasis at ``spec.rank``."""
    if spec.kind == "raw":
        return encode_raw(matrix, context)
    x = matrix.reshape(context.shape).float()
    if basis is None:
        g = x.t() @ x
        values, vectors = torch.linalg.eigh(g.double())
        order = torch.argsort(values, descending=True)[:spec.rank]
        basis = vectors[:, order].t().contiguous().to(torch.float16)
    basis = basis[:spec.rank].to(torch.float16)
    coefficients = x @ basis.float().t().to(x.device)
    view = basis.detach().cpu().numpy().tobytes()
    return encode_factorized(coefficients, view, context, spec, stream_codec=stream_codec)


# ---------------------------------------------------------------------------------------------
# Node packs
# ---------------------------------------------------------------------------------------------


def encode_node_pack(tiles: Sequence[Mapping[str, Any]], *, stream_codec: str = "raw8",
                     details: Mapping[str, Any] | None = None) -> EncodedTensor:
    """One ``reelcache.tensor_pack.v2`` pack from already-quantized tiles.

    Each tile: ``entry`` (JSON: key/stream), ``context`` (TensorContext), ``codec`` (CodecSpec),
    ``pixels`` (uint8 numpy [N, r]), ``affine`` (float32 [2, records]), ``normalization`` (layout),
    ``basis`` (descriptor dict, optionally with the version ref).
    """
    if stream_codec not in ("raw8", "raw8+zlib"):
        raise UnsupportedError("node packs are written as raw8 / raw8+zlib coefficient streams here; "
                               "HEVC packs need an HEVC encoder (ffmpeg/libx265 or NVENC), absent on this machine")
    chunks, affines, entries = [], [], []
    offset = 0
    affine_records = 0
    for index, tile in enumerate(tiles):
        pixels = np.ascontiguousarray(tile["pixels"], dtype=np.uint8)
        data = pixels.tobytes()
        affine = np.ascontiguousarray(tile["affine"], dtype="<f4")
        entries.append({
            "tile": index, "entry": json_copy(tile["entry"]), "context": tile["context"].to_dict(),
            "codec": tile["codec"].to_dict(), "rank": int(pixels.shape[1]), "normalization": tile["normalization"],
            "coefficients": {"offset": offset, "bytes": len(data), "shape": [int(pixels.shape[0]), int(pixels.shape[1])],
                             "sha256": hashlib.sha256(data).hexdigest()},
            "affine": {"record": affine_records, "records": int(affine.shape[1])},
            "basis": json_copy(tile["basis"]),
        })
        chunks.append(data)
        affines.append(affine)
        offset += len(data)
        affine_records += affine.shape[1]
    stream = b"".join(chunks)
    if stream_codec == "raw8+zlib":
        stream = zlib.compress(stream, 1)
    affine_payload = (np.concatenate(affines, axis=1) if affines else np.zeros((2, 0), "<f4")).astype("<f4").tobytes()
    metadata = {"schema": PACK_SCHEMA, "stream_codec": stream_codec, "tiles": entries,
                "stream_bytes": len(stream), "raw_bytes": offset, "details": json_copy(dict(details or {}))}
    return EncodedTensor(metadata, {"stream": stream, "affines": affine_payload},
                         metrics={"bytes": len(stream) + len(affine_payload)})


def validate_pack(metadata: Mapping[str, Any]) -> None:
    if metadata.get("schema") != PACK_SCHEMA or metadata.get("stream_codec") not in STREAM_CODECS:
        raise IntegrityError("unsupported node pack schema or stream codec")
    offset = 0
    for index, tile in enumerate(metadata["tiles"]):
        coeff = tile["coefficients"]
        if tile["tile"] != index or coeff["offset"] != offset or coeff["bytes"] != coeff["shape"][0] * coeff["shape"][1]:
            raise IntegrityError("node pack tile table is inconsistent")
        offset += coeff["bytes"]
    if offset != metadata["raw_bytes"]:
        raise IntegrityError("node pack byte count differs from its tiles")


class DecodedPack:
    """A node pack's decoded coefficient stream (uint8, host) and affines, with per-tile views."""

    def __init__(self, metadata: Mapping[str, Any], stream: bytes, affines: bytes, *, verify: bool = True):
        validate_pack(metadata)
        self.metadata = metadata
        data = zlib.decompress(stream) if metadata["stream_codec"] == "raw8+zlib" else stream
        if metadata["stream_codec"] == "hevc":
            raise UnsupportedError("HEVC node packs need an HEVC decoder (NVDEC or FFmpeg), absent on this machine")
        if len(data) != metadata["raw_bytes"]:
            raise IntegrityError("node pack stream length differs from its tiles")
        self.raw = np.frombuffer(data, dtype=np.uint8)
        total = sum(t["affine"]["records"] for t in metadata["tiles"])
        self.affines = np.frombuffer(affines, dtype="<f4").reshape(2, total)
        if verify:
            for tile in metadata["tiles"]:
                coeff = tile["coefficients"]
                chunk = self.raw[coeff["offset"]:coeff["offset"] + coeff["bytes"]]
                if hashlib.sha256(chunk.tobytes()).hexdigest() != coeff["sha256"]:
                    raise IntegrityError(f"node pack tile {tile['tile']} differs from its digest")

    @property
    def tiles(self):
        return self.metadata["tiles"]

    def pixels(self, index: int) -> np.ndarray:
        coeff = self.tiles[index]["coefficients"]
        return self.raw[coeff["offset"]:coeff["offset"] + coeff["bytes"]].reshape(coeff["shape"])

    def affine(self, index: int) -> np.ndarray:
        record = self.tiles[index]["affine"]
        return np.ascontiguousarray(self.affines[:, record["record"]:record["record"] + record["records"]])

    def scale_offset(self, index: int) -> tuple[np.ndarray, np.ndarray]:
        tile = self.tiles[index]
        scale, offset = _hevc.expanded_affine(self.affine(index), tile["normalization"], tile["rank"])
        return np.ascontiguousarray(scale, dtype=np.float32), np.ascontiguousarray(offset, dtype=np.float32)


def encode_factor_pack(tiles: Sequence[Mapping[str, Any]]) -> EncodedTensor:
    """``reelcache.factor_pack.v1``: FP16 coefficient matrices of the SVD-only baseline."""
    chunks, entries = [], []
    offset = 0
    for index, tile in enumerate(tiles):
        data = np.ascontiguousarray(tile["coefficients"], dtype=np.float16).tobytes()
        entries.append({"tile": index, "entry": json_copy(tile["entry"]), "context": tile["context"].to_dict(),
                        "rank": int(tile["coefficients"].shape[1]), "offset": offset, "bytes": len(data),
                        "sha256": hashlib.sha256(data).hexdigest(), "basis": json_copy(tile["basis"])})
        chunks.append(data)
        offset += len(data)
    return EncodedTensor({"schema": FACTOR_PACK_SCHEMA, "tiles": entries, "bytes": offset, "stream_bytes": offset,
                          "raw_bytes": offset // 2, "stream_codec": "fp16"},
                         {"factors": b"".join(chunks)}, metrics={"bytes": offset})


class FactorPack:
    """Decoded view of a ``reelcache.factor_pack.v1`` packet: per tile its FP16 ``[tokens, rank]`` factors."""

    def __init__(self, metadata: Mapping[str, Any], factors: bytes, *, verify: bool = True):
        if metadata.get("schema") != FACTOR_PACK_SCHEMA:
            raise IntegrityError("packet is not a factor pack")
        if len(factors) != int(metadata["bytes"]):
            raise IntegrityError("factor pack size differs from its manifest")
        self.metadata = metadata
        self.tiles = list(metadata["tiles"])
        self.raw = np.frombuffer(factors, dtype=np.uint8)
        if verify:
            for tile in self.tiles:
                chunk = factors[tile["offset"]:tile["offset"] + tile["bytes"]]
                if hashlib.sha256(chunk).hexdigest() != tile["sha256"]:
                    raise IntegrityError(f"factor pack tile {tile['tile']} fails its hash")

    def factors(self, index: int) -> np.ndarray:
        tile = self.tiles[index]
        rank = int(tile["rank"])
        view = self.raw[tile["offset"]:tile["offset"] + tile["bytes"]].view(np.float16)
        return view.reshape(-1, rank)


# ---------------------------------------------------------------------------------------------
# Node codec API: many matrices of one node, packed or per matrix
# ---------------------------------------------------------------------------------------------

PACKING_MODES = ("node", "layer_group", "per_matrix")


@dataclass(frozen=True)
class NodeEncoding:
    """The packets of one node and where each matrix went: ``locations[entry] = (packet index, tile index)``
    (tile index None: a single-matrix packet). Entries are ``MatrixKey`` or ``(MatrixKey, stream)``."""

    packets: tuple
    locations: Mapping[Any, tuple[int, int | None]]
    packing: str


def _entry_json(entry) -> dict:
    from .types import MatrixKey
    if isinstance(entry, MatrixKey):
        return {"key": entry.to_dict()}
    key, stream = entry
    return {"key": key.to_dict(), "stream": stream}


def _entry_of(record: Mapping[str, Any]):
    from .types import MatrixKey
    key = MatrixKey.from_dict(record["key"])
    return key if "stream" not in record else (key, record["stream"])


def _factor(matrix: torch.Tensor, context: TensorContext, spec: CodecSpec, basis: torch.Tensor | None):
    """(coefficients FP32 [N, r], FP16 basis rows [r, C]) of one matrix: on the given rows, or on its own
    truncated eigenbasis at ``spec.rank``."""
    x = matrix.reshape(context.shape).float()
    if basis is None:
        if spec.rank is None:
            raise ConfigurationError("a matrix without a basis needs a codec rank")
        g = x.t() @ x
        values, vectors = torch.linalg.eigh(g.double())
        order = torch.argsort(values, descending=True)[:spec.rank]
        basis = vectors[:, order].t().contiguous().to(torch.float16)
    basis = basis.to(torch.float16)
    if spec.rank is not None:
        basis = basis[:spec.rank]
    return x @ basis.float().t().to(x.device), basis.cpu()


def encode_packed(matrices: Mapping[Any, torch.Tensor], contexts: Mapping[Any, TensorContext],
                  specs: Mapping[Any, CodecSpec] | CodecSpec, *, bases: Mapping[Any, torch.Tensor] | None = None,
                  stream_codec: str = "raw8", node_id: str | None = None) -> EncodedTensor:
    """Several ``svd_hevc`` matrices of one node in ONE ``reelcache.tensor_pack.v2`` packet: each factorized on its
    FP16 basis rows (``bases``; default its own eigenbasis at the spec's rank), quantized with its covering affine
    and stored as one tile of the pack's coefficient stream. The packet is complete in memory: each tile's basis
    view travels as a ``basis.NNN.f16`` payload (a store keeps bases as versions instead)."""
    if not matrices or set(matrices) != set(contexts):
        raise ConfigurationError("encode_packed needs the same nonempty entries in matrices and contexts")
    tiles, payloads = [], {}
    for index, entry in enumerate(sorted(matrices, key=entry_order)):
        spec = specs if isinstance(specs, CodecSpec) else specs[entry]
        if spec.kind != "svd_hevc":
            raise ConfigurationError("node packs hold svd_hevc matrices (RAW and SVD travel as single packets)")
        context = contexts[entry]
        coefficients, basis = _factor(matrices[entry], context, spec, None if bases is None else bases.get(entry))
        pixels, affine, layout = quantize(coefficients, spec.normalization, spec.protected_fraction)
        view = basis.numpy().tobytes()
        name = f"basis.{index:03d}.f16"
        payloads[name] = view
        tiles.append({"entry": _entry_json(entry), "context": context, "pixels": pixels, "affine": affine,
                      "normalization": layout, "codec": CodecSpec(**{**spec.to_dict(), "rank": basis.shape[0]}),
                      "basis": {**descriptor(view, basis.shape[0], context.channels), "payload": name}})
    packed = encode_node_pack(tiles, stream_codec=stream_codec, details={"node_id": node_id} if node_id else None)
    return EncodedTensor(packed.metadata, {**packed.payloads, **payloads}, metrics=packed.metrics)


def encode_node(matrices: Mapping[Any, torch.Tensor], contexts: Mapping[Any, TensorContext],
                specs: Mapping[Any, CodecSpec] | CodecSpec, *, packing: str = "node",
                layer_group_size: int | None = None, bases: Mapping[Any, torch.Tensor] | None = None,
                stream_codec: str = "raw8") -> NodeEncoding:
    """Every matrix of one node under a packing mode: ``node`` (all ``svd_hevc`` matrices in one pack),
    ``layer_group`` (one pack per run of ``layer_group_size`` layers) or ``per_matrix`` (one packet each, as
    :func:`encode_tensor`). RAW and SVD-only matrices are always single packets."""
    if packing not in PACKING_MODES:
        raise ConfigurationError(f"packing must be one of {PACKING_MODES}")
    if (packing == "layer_group") != (layer_group_size is not None):
        raise ConfigurationError("layer_group_size goes with layer_group packing, and only with it")
    if layer_group_size is not None and (type(layer_group_size) is not int or layer_group_size < 1):
        raise ConfigurationError("layer_group_size must be a positive integer")
    spec_of = (lambda e: specs) if isinstance(specs, CodecSpec) else (lambda e: specs[e])
    packets, locations = [], {}
    grouped: dict[int, list] = {}
    for entry in sorted(matrices, key=entry_order):
        spec = spec_of(entry)
        if spec.kind != "svd_hevc" or packing == "per_matrix":
            basis = None if bases is None else bases.get(entry)
            if spec.kind == "raw":
                packets.append(encode_raw(matrices[entry].reshape(contexts[entry].shape), contexts[entry]))
            else:
                coefficients, rows = _factor(matrices[entry], contexts[entry], spec, basis)
                packets.append(encode_factorized(coefficients, rows.numpy().tobytes(), contexts[entry],
                                                 CodecSpec(**{**spec.to_dict(), "rank": rows.shape[0]}),
                                                 stream_codec=None if spec.kind == "svd" else stream_codec))
            locations[entry] = (len(packets) - 1, None)
            continue
        layer = (entry if not isinstance(entry, tuple) else entry[0]).layer
        group = 0 if packing == "node" else layer // layer_group_size
        grouped.setdefault(group, []).append(entry)
    for group in sorted(grouped):
        members = grouped[group]
        pack = encode_packed({e: matrices[e] for e in members}, {e: contexts[e] for e in members},
                             {e: spec_of(e) for e in members}, bases=bases, stream_codec=stream_codec)
        packets.append(pack)
        for tile, entry in enumerate(sorted(members, key=entry_order)):
            locations[entry] = (len(packets) - 1, tile)
    return NodeEncoding(tuple(packets), locations, packing)


def decode_packed(encoded: EncodedTensor, *, keys=None, device: Any = "cpu",
                  dtype: torch.dtype = torch.float32) -> dict:
    """The selected (default: all) matrices of an in-memory node pack, ``{entry: dequantize(P) @ Q}`` in tile
    order; the tiles' bases come from the packet's ``basis.NNN.f16`` payloads."""
    pack = DecodedPack(encoded.metadata, encoded.payloads["stream"], encoded.payloads["affines"])
    wanted = None if keys is None else set(keys)
    out = {}
    for index, tile in enumerate(pack.tiles):
        entry = _entry_of(tile["entry"])
        if wanted is not None and entry not in wanted:
            continue
        name = tile["basis"].get("payload")
        if name is None or name not in encoded.payloads:
            raise IntegrityError(f"tile {index} has no basis payload: decode it through its store record")
        rank, channels = tile["basis"]["shape"]
        view = encoded.payloads[name]
        if hashlib.sha256(view).hexdigest() != tile["basis"]["sha256"]:
            raise IntegrityError(f"basis of tile {index} differs from its digest")
        basis = torch.from_numpy(np.frombuffer(view, dtype=np.float16).reshape(rank, channels).copy()).to(device)
        scale, offset = pack.scale_offset(index)
        coefficients = torch.from_numpy(pack.pixels(index).astype(np.float32) * scale + offset).to(device)
        out[entry] = (coefficients @ basis.float()).to(dtype)
    if wanted is not None and set(out) != wanted:
        raise ConfigurationError(f"the pack holds none of {sorted(map(str, wanted - set(out)))}")
    return out
