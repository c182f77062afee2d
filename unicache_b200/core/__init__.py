"""Contracts shared with the reference's plugin API (unicache/core)."""

from .decisions import PhysicalCacheRequest

__all__ = ["PhysicalCacheRequest"]
