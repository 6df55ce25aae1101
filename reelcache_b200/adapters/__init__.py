"""Adapters that wrap a third-party model's own execution (its forward and cache stay native) to archive and
restore its clean history through this package: MAGI's Ulysses clean history (:mod:`.magi`)."""

from .magi import MagiAdapter, MagiGeometry

__all__ = ["MagiAdapter", "MagiGeometry"]
