"""Typed failure modes of the runtime (mirrors reelcache/errors.py:4-33 of the reference).

Every declared failure derives from :class:`ReelCacheError`; callers distinguish configuration
mistakes, corrupt or missing immutable objects, bounded resources that refuse work, operations that
are invalid in the current state, and capabilities this machine lacks.
"""


class ReelCacheError(Exception):
    """Base class of every declared runtime failure."""


class ConfigurationError(ReelCacheError, ValueError):
    """A configuration, identity or argument is invalid or incompatible."""


class IntegrityError(ReelCacheError):
    """An immutable object is corrupt, missing or internally inconsistent."""


class QuarantinedError(IntegrityError):
    """A head found damaged when its store was opened (``on_open_error="quarantine"``) was used."""


class CapacityError(ReelCacheError):
    """A bounded resource cannot admit the requested operation."""


class StateError(ReelCacheError):
    """The operation is not valid in the current runtime state."""


class UnsupportedError(ReelCacheError):
    """A requested representation or capability is unavailable on this machine."""


class PendingError(StateError):
    """The requested state has not reached a committed clean boundary yet."""


class DeviceStatusError(ReelCacheError):
    """A kernel's bounded wait ran out and it returned early (its status word is nonzero)."""
