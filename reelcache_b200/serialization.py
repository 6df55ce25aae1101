"""Canonical JSON and the pickle-free tensor-state container.

Byte layout of a container (shared with the reference implementation so that either can read the other's
execution-state blobs; reference reelcache/serialization.py:18,162-184)::

    MAGIC = b"REELCACHE_TENSORS\\x00\\x01"
    MAGIC | u64 little-endian header size | header (canonical JSON) | payloads

    header = {"version": 1, "byteorder": "little",
              "tensors": {name: {"dtype", "shape", "offset", "nbytes", "sha256"}}}

Payloads are the tensors' raw little-endian bytes, packed back to back in ascending name order; each
entry's ``offset`` is relative to the first payload byte. Reading is strict: the JSON must be UTF-8 with
unique keys and finite numbers, every entry must sit exactly where the previous one ended, its digest must
match, and no byte may be left over. Any violation raises :class:`~reelcache_b200.errors.IntegrityError`.
Nothing in this module unpickles.
"""

from __future__ import annotations

import hashlib
import json
import math
import struct
import sys
from typing import Any, Mapping, Sequence

import torch

from .errors import CapacityError, ConfigurationError, IntegrityError, UnsupportedError
from .types import json_copy

MAGIC = b"REELCACHE_TENSORS\x00\x01"
FORMAT_VERSION = 1
HEADER_LIMIT = 16 << 20
_LENGTH = struct.Struct("<Q")
_ENTRY_FIELDS = frozenset({"dtype", "shape", "offset", "nbytes", "sha256"})

# dtype name in the header -> torch dtype (names without the "torch." prefix)
_DTYPE_TABLE: dict[str, torch.dtype] = {}
for _name in ("bool", "uint8", "uint16", "uint32", "uint64", "int8", "int16", "int32", "int64", "float16",
              "bfloat16", "float32", "float64", "complex64", "complex128"):
    if hasattr(torch, _name):
        _DTYPE_TABLE[_name] = getattr(torch, _name)


def _require_little_endian() -> None:
    if sys.byteorder != "little":
        raise UnsupportedError("tensor containers are little-endian; this host is not")


# ------------------------------------------------------------------------------------------------- JSON

def canonical_json(value: Any) -> bytes:
    """UTF-8 JSON with sorted keys, no whitespace, non-ASCII kept and NaN/infinity refused."""
    text = json.dumps(json_copy(value), sort_keys=True, separators=(",", ":"), ensure_ascii=False,
                      allow_nan=False)
    return text.encode("utf-8")


class _StrictDecoder:
    """Hooks for :func:`json.loads` that turn the lenient corners of JSON into errors."""

    @staticmethod
    def pairs(items):
        keys = [key for key, _ in items]
        if len(set(keys)) != len(keys):
            raise IntegrityError("stored JSON repeats a key")
        return dict(items)

    @staticmethod
    def number(text: str) -> float:
        value = float(text)
        if math.isinf(value) or math.isnan(value):
            raise ValueError(f"stored JSON holds a non-finite number: {text}")
        return value

    @staticmethod
    def constant(name: str):
        raise ValueError(f"stored JSON holds the constant {name}")


def parse_json(data: bytes) -> Any:
    """Parse stored JSON strictly (see the module docstring)."""
    try:
        text = data.decode("utf-8")
        return json.loads(text, object_pairs_hook=_StrictDecoder.pairs, parse_float=_StrictDecoder.number,
                          parse_constant=_StrictDecoder.constant)
    except IntegrityError:
        raise
    except (ValueError, UnicodeError, TypeError, RecursionError) as exc:
        raise IntegrityError(f"stored JSON is malformed: {exc}") from exc


# ----------------------------------------------------------------------------------------------- dtypes

def resolve_dtype(dtype: str | torch.dtype) -> torch.dtype:
    label = str(dtype)
    if label.startswith("torch."):
        label = label[len("torch."):]
    found = _DTYPE_TABLE.get(label)
    if found is None:
        raise UnsupportedError(f"tensor containers do not hold dtype {dtype!r}")
    return found


def dtype_name(dtype: str | torch.dtype) -> str:
    return str(resolve_dtype(dtype))[len("torch."):]


def _itemsize(dtype: torch.dtype) -> int:
    return torch.empty((), dtype=dtype).element_size()


def tensor_nbytes(shape: Sequence[int], dtype: str | torch.dtype) -> int:
    """Storage bytes of a dense tensor of ``shape`` and ``dtype`` (validated)."""
    if not isinstance(shape, (list, tuple)):
        raise ConfigurationError("a tensor shape is a list of dimensions")
    if len(shape) > 64:
        raise ConfigurationError("tensor shapes have at most 64 dimensions")
    count = 1
    for size in shape:
        if type(size) is not int or size < 0 or size > sys.maxsize:
            raise ConfigurationError(f"tensor dimension {size!r} is not a nonnegative machine integer")
        count *= size
    total = count * _itemsize(resolve_dtype(dtype))
    if total > sys.maxsize:
        raise ConfigurationError("the tensor is larger than the host address space")
    return total


# ---------------------------------------------------------------------------------------------- tensors

def tensor_bytes(tensor: torch.Tensor) -> bytes:
    """The raw little-endian bytes of a dense tensor (copied to the host, contiguous)."""
    if not isinstance(tensor, torch.Tensor):
        raise ConfigurationError("tensor state holds torch.Tensor values only")
    resolve_dtype(tensor.dtype)
    dense = tensor.layout == torch.strided and not tensor.is_quantized and tensor.device.type != "meta"
    if not dense:
        raise UnsupportedError("only materialized dense (strided) tensors are serializable")
    _require_little_endian()
    host = tensor.detach().resolve_conj().resolve_neg().to("cpu").contiguous()
    return host.reshape(-1).view(torch.uint8).numpy().tobytes()


def tensor_from_bytes(data: bytes, *, dtype, shape: Sequence[int], device: Any = "cpu") -> torch.Tensor:
    """Rebuild a tensor from its raw bytes (validated against ``dtype`` and ``shape``)."""
    _require_little_endian()
    if not isinstance(data, bytes):
        raise IntegrityError("a tensor payload is an immutable bytes object")
    try:
        kind = resolve_dtype(dtype)
        size = tensor_nbytes(shape, kind)
    except (ConfigurationError, UnsupportedError) as exc:
        raise IntegrityError(f"stored tensor geometry is invalid: {exc}") from exc
    if len(data) != size:
        raise IntegrityError(f"stored tensor holds {len(data)} bytes, its geometry needs {size}")
    try:
        if size == 0:
            value = torch.empty(tuple(shape), dtype=kind)
        else:
            value = torch.frombuffer(bytearray(data), dtype=kind).reshape(tuple(shape))
    except (RuntimeError, TypeError, ValueError, OverflowError) as exc:
        raise IntegrityError(f"stored tensor cannot take its shape: {exc}") from exc
    try:
        return value.to(device=device)
    except (RuntimeError, TypeError, ValueError) as exc:
        raise ConfigurationError(f"device {device!r} cannot hold the restored tensor") from exc


# -------------------------------------------------------------------------------------------- container

def serialize_tensors(tensors: Mapping[str, torch.Tensor]) -> bytes:
    """Pack named tensors into one container (layout in the module docstring)."""
    if not isinstance(tensors, Mapping):
        raise ConfigurationError("tensor state is a mapping of names to tensors")
    for name in tensors:
        if not isinstance(name, str) or name == "":
            raise ConfigurationError(f"tensor state names are nonempty strings, not {name!r}")
    table: dict[str, dict[str, Any]] = {}
    body = bytearray()
    for name in sorted(tensors):
        value = tensors[name]
        raw = tensor_bytes(value)
        table[name] = {"dtype": dtype_name(value.dtype), "shape": list(value.shape), "offset": len(body),
                       "nbytes": len(raw), "sha256": hashlib.sha256(raw).hexdigest()}
        body += raw
    header = canonical_json({"version": FORMAT_VERSION, "byteorder": "little", "tensors": table})
    if len(header) > HEADER_LIMIT:
        raise CapacityError(f"a tensor state header is limited to {HEADER_LIMIT} bytes")
    return b"".join((MAGIC, _LENGTH.pack(len(header)), header, bytes(body)))


def _read_header(data: bytes) -> tuple[dict, memoryview]:
    if not isinstance(data, bytes) or data[:len(MAGIC)] != MAGIC:
        raise IntegrityError("the blob is not a tensor-state container")
    start = len(MAGIC) + _LENGTH.size
    if len(data) < start:
        raise IntegrityError("the container ends inside its header length")
    (size,) = _LENGTH.unpack_from(data, len(MAGIC))
    if size > HEADER_LIMIT or start + size > len(data):
        raise IntegrityError(f"the container declares an impossible header of {size} bytes")
    header = parse_json(data[start:start + size])
    valid = (isinstance(header, dict) and set(header) == {"version", "byteorder", "tensors"}
             and type(header["version"]) is int and header["version"] == FORMAT_VERSION
             and header["byteorder"] == "little" and isinstance(header["tensors"], dict))
    if not valid:
        raise IntegrityError("the container header has an unknown version or layout")
    return header, memoryview(data)[start + size:]


def deserialize_tensors(data: bytes, *, device: Any = "cpu", max_bytes: int | None = None) -> dict[str, torch.Tensor]:
    """Unpack a container; every entry is checked (position, size, digest) before any tensor is built."""
    header, body = _read_header(data)
    if max_bytes is not None:
        if type(max_bytes) is not int or max_bytes < 0:
            raise ConfigurationError("max_bytes is a nonnegative integer")
        if len(body) > max_bytes:
            raise CapacityError(f"the container's {len(body)} payload bytes exceed the budget of {max_bytes}")
    verified = []
    position = 0
    for name in sorted(header["tensors"]):
        entry = header["tensors"][name]
        if not name or not isinstance(entry, dict) or set(entry) != _ENTRY_FIELDS:
            raise IntegrityError(f"container entry {name!r} is malformed")
        if type(entry["offset"]) is not int or entry["offset"] != position:
            raise IntegrityError(f"container entry {name!r} does not start where the previous one ended")
        try:
            size = tensor_nbytes(entry["shape"], entry["dtype"])
        except (ConfigurationError, UnsupportedError) as exc:
            raise IntegrityError(f"container entry {name!r} has an invalid geometry: {exc}") from exc
        if type(entry["nbytes"]) is not int or entry["nbytes"] != size or position + size > len(body):
            raise IntegrityError(f"container entry {name!r} disagrees with its geometry or the container size")
        raw = bytes(body[position:position + size])
        if hashlib.sha256(raw).hexdigest() != entry["sha256"]:
            raise IntegrityError(f"container entry {name!r} fails its digest")
        verified.append((name, entry, raw))
        position += size
    if position != len(body):
        raise IntegrityError(f"the container has {len(body) - position} bytes no entry claims")
    return {name: tensor_from_bytes(raw, dtype=entry["dtype"], shape=entry["shape"], device=device)
            for name, entry, raw in verified}


__all__ = ["FORMAT_VERSION", "MAGIC", "canonical_json", "deserialize_tensors", "dtype_name", "parse_json",
           "resolve_dtype", "serialize_tensors", "tensor_bytes", "tensor_from_bytes", "tensor_nbytes"]
