"""Neural-network helpers for imported models (``tynx.nn`` subset on CUDA)."""

from . import functional

__all__ = ["functional"]
