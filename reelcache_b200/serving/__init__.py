"""HTTP serving layer over the bridge (``create_app``)."""

from .http import create_app

__all__ = ["create_app"]
