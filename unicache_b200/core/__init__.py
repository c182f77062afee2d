"""Contracts shared with the reference's plugin API (unicache/core)."""

from .decisions import PhysicalCacheRequest
from .plugin import CapabilityDescriptor, ProcessingOperator

__all__ = ["CapabilityDescriptor", "PhysicalCacheRequest", "ProcessingOperator"]
