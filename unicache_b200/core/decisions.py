"""The physical-cache request contract between operators and the storage backend.

Same fields and validation as the reference's ``PhysicalCacheRequest``
(Superone77/UniCache, unicache/core/decisions.py:52-85), so operators and
adapters written against it work unchanged.
"""

from __future__ import annotations

from dataclasses import dataclass, field
from typing import Any

import torch


@dataclass
class PhysicalCacheRequest:
    """A one-way conversion of a dense KV segment into a physical layout."""

    operator: str
    segment_id: str
    token_count: int
    segment_mask: torch.Tensor
    params: dict[str, Any] = field(default_factory=dict)
    per_kv_head_scores: torch.Tensor | None = None
    metadata: dict[str, Any] = field(default_factory=dict)

    def __post_init__(self) -> None:
        if self.token_count < 0:
            raise ValueError("PhysicalCacheRequest token count must be non-negative")
        if (
            self.segment_mask.dtype != torch.bool
            or self.segment_mask.dim() != 1
            or int(self.segment_mask.numel()) != self.token_count
        ):
            raise ValueError("PhysicalCacheRequest segment_mask must be boolean and match token_count")
        if self.per_kv_head_scores is not None:
            if self.per_kv_head_scores.dim() != 2:
                raise ValueError("Physical per-KV-head scores must be [kv_heads, tokens]")
            if int(self.per_kv_head_scores.shape[-1]) != self.token_count:
                raise ValueError("Physical per-KV-head scores must match token_count")
