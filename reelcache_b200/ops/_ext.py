"""Access to the native extension and the per-device kernel status words.

Every persistent kernel takes an int32 status word; a bounded wait that runs out writes a nonzero
code there and the kernel returns early instead of hanging. :func:`check_status` turns a nonzero
word into :class:`~reelcache_b200.errors.DeviceStatusError` (it synchronizes, so callers use it in
tests and at step boundaries, not inside hot loops).
"""

from __future__ import annotations

import threading

import torch

from .. import _native_build
from ..errors import DeviceStatusError, UnsupportedError

_status = {}
_lock = threading.Lock()

STATUS_NAMES = {
    0x101: "TMA producer wait timed out",
    0x102: "MMA issuer wait timed out",
    0x103: "epilogue wait timed out",
    0x104: "gather producer wait timed out",
    0x105: "drain wait timed out",
    0x201: "peer flag wait timed out",
    0x301: "bad kernel argument",
}


def ext():
    """The loaded extension module; raises UnsupportedError naming the missing library."""
    try:
        return _native_build.load()
    except ImportError as error:
        raise UnsupportedError(str(error)) from error


def available() -> bool:
    try:
        ext()
        return True
    except UnsupportedError:
        return False


def status_word(device) -> torch.Tensor:
    device = torch.device(device)
    if device.index is None:
        device = torch.device("cuda", torch.cuda.current_device())
    with _lock:
        word = _status.get(device.index)
        if word is None:
            word = torch.zeros(4, dtype=torch.int32, device=device)
            _status[device.index] = word
    return word


def check_status(device) -> None:
    """Raise DeviceStatusError if any kernel on ``device`` recorded a failure (synchronizes)."""
    word = status_word(device)
    code = int(word[0].item())
    if code:
        word.zero_()
        raise DeviceStatusError(f"kernel status 0x{code:x}: {STATUS_NAMES.get(code, 'unknown failure')}")


def require_cuda(tensor: torch.Tensor, what: str) -> None:
    if tensor.device.type != "cuda":
        raise UnsupportedError(f"{what} needs CUDA tensors")
